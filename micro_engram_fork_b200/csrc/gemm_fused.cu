// Projections with fused epilogues on the persistent tcgen05 GEMM (gemm_kernel.cuh): the
// gate|up GEMM with GeGLU, the down projection's dX with the GeGLU backward, and the tied head's
// logits with the softcapped cross-entropy partials.
#include "gemm_kernel.cuh"

using namespace me::gemm;

// m[M, F] = GeGLU(A . Wgu^T) with Wgu = [gate; up] [2F, K]; with save_gu also returns
// gu[M, 2F] = bf16(A . Wgu^T) for the backward.
std::vector<torch::Tensor> gemm_geglu(torch::Tensor A, torch::Tensor Wgu, bool save_gu) {
  check_operand(A, "A");
  check_operand(Wgu, "W");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1);
  TORCH_CHECK(Wgu.size(1) == K && Wgu.size(0) % 2 == 0, "gemm_geglu: W must be [2F, K]");
  const int F = (int)(Wgu.size(0) / 2);
  TORCH_CHECK(F % 8 == 0 && K % 8 == 0, "gemm_geglu: F and K must be multiples of 8");
  auto m = torch::empty({M, F}, A.options());
  torch::Tensor gu = save_gu ? torch::empty({M, 2 * F}, A.options()) : torch::Tensor();
  if (M == 0) return {m, gu};
  const int dev = A.get_device();
  GemmArgs a = base_args(M, F, K, (F + BN / 2 - 1) / (BN / 2), dev);
  a.D = reinterpret_cast<bf16*>(m.data_ptr());
  a.ldd = F;
  if (save_gu) {
    a.D2 = reinterpret_cast<bf16*>(gu.data_ptr());
    a.ldd2 = 2 * F;
  }
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BK, BM);
  const CUtensorMap tb = make_tmap(Wgu.data_ptr(), 2 * F, K, Wgu.stride(0), BK, BN / 2);
  launch<EPI_GEGLU, false>(ta, tb, a, dev, at::cuda::getCurrentCUDAStream());
  return {m, gu};
}

// d_gu[M, 2F] = GeGLU'(gu) applied to dm = dY . Wdown, with Wdown [d, F] (the down projection's
// weight: dm = dY[M, d] . Wdown, an N-major B operand) and gu [M, 2F] the forward's gate|up.
torch::Tensor gemm_dgeglu(torch::Tensor dY, torch::Tensor Wdown, torch::Tensor gu) {
  check_operand(dY, "dY");
  check_operand(Wdown, "W");
  check_operand(gu, "gu");
  const at::cuda::CUDAGuard guard(dY.device());
  const int M = (int)dY.size(0), K = (int)dY.size(1);
  TORCH_CHECK(Wdown.size(0) == K, "gemm_dgeglu: W must be [d, F]");
  const int F = (int)Wdown.size(1);
  TORCH_CHECK(gu.size(0) == M && gu.size(1) == 2 * F, "gemm_dgeglu: gu must be [M, 2F]");
  TORCH_CHECK(F % 8 == 0 && K % 8 == 0, "gemm_dgeglu: F and K must be multiples of 8");
  auto dgu = torch::empty({M, 2 * F}, dY.options());
  if (M == 0) return dgu;
  const int dev = dY.get_device();
  GemmArgs a = base_args(M, F, K, (F + BN - 1) / BN, dev);
  a.D = reinterpret_cast<bf16*>(dgu.data_ptr());
  a.ldd = 2 * F;
  a.aux = reinterpret_cast<const bf16*>(gu.data_ptr());
  a.ld_aux = gu.stride(0);
  const CUtensorMap ta = make_tmap(dY.data_ptr(), M, K, dY.stride(0), BK, BM);
  const CUtensorMap tb = make_tmap(Wdown.data_ptr(), K, F, Wdown.stride(0), 64, BK);
  launch<EPI_DGEGLU, true>(ta, tb, a, dev, at::cuda::getCurrentCUDAStream());
  return dgu;
}

// Softcapped cross-entropy partials of H[M, d] against this rank's vocab rows E[V, d]
// (labels in [lab_start, lab_start + n_valid) belong here; E may carry zero rows past n_valid so
// that V is a multiple of 8): returns (s_part [M, tiles], m_part [M, tiles] or empty when
// cap > 0 (every offset is the cap), tgt [M] (0 where the label is elsewhere), z [M, V] bf16
// logits when keep_logits (columns past n_valid hold the zero rows' logits), else empty).
std::vector<torch::Tensor> gemm_ce(torch::Tensor H, torch::Tensor E, torch::Tensor labels, int64_t lab_start,
                                   double cap, bool keep_logits, int64_t n_valid) {
  check_operand(H, "H");
  check_operand(E, "E");
  TORCH_CHECK(labels.is_cuda() && labels.scalar_type() == torch::kInt64 && labels.is_contiguous() &&
                  labels.numel() == H.size(0), "gemm_ce: labels must be int64 [M] on the GPU");
  const at::cuda::CUDAGuard guard(H.device());
  const int M = (int)H.size(0), K = (int)H.size(1), V = (int)E.size(0);
  TORCH_CHECK(E.size(1) == K && V % 8 == 0 && K % 8 == 0, "gemm_ce: E must be [V, d], V and d multiples of 8");
  TORCH_CHECK(n_valid > 0 && n_valid <= V, "gemm_ce: n_valid out of range");
  const int tiles_n = (V + BN - 1) / BN;
  auto fopt = H.options().dtype(torch::kFloat32);
  auto s_part = torch::empty({M, tiles_n}, fopt);
  auto m_part = cap > 0 ? torch::Tensor() : torch::empty({M, tiles_n}, fopt);
  auto tgt = torch::zeros({M}, fopt);
  auto z = keep_logits ? torch::empty({M, V}, H.options()) : torch::Tensor();
  if (M == 0) return {s_part, m_part, tgt, z};
  const int dev = H.get_device();
  GemmArgs a = base_args(M, (int)n_valid, K, tiles_n, dev);
  if (keep_logits) {
    a.D = reinterpret_cast<bf16*>(z.data_ptr());
    a.ldd = V;
  }
  a.labels = labels.data_ptr<int64_t>();
  a.lab_start = lab_start;
  a.cap = (float)cap;
  a.s_part = s_part.data_ptr<float>();
  a.m_part = cap > 0 ? nullptr : m_part.data_ptr<float>();
  a.tgt = tgt.data_ptr<float>();
  const CUtensorMap ta = make_tmap(H.data_ptr(), M, K, H.stride(0), BK, BM);
  const CUtensorMap tb = make_tmap(E.data_ptr(), V, K, E.stride(0), BK, BN / 2);
  launch<EPI_CE, false>(ta, tb, a, dev, at::cuda::getCurrentCUDAStream());
  return {s_part, m_part, tgt, z};
}

