// Projections of an NF4-stored frozen weight on the persistent tcgen05 GEMM: the kernel's B
// operand is dequantised inside the kernel by four extra warps per CTA (gemm_kernel.cuh, B_NF4),
// so the bf16 weight is never written to memory. Numerics equal the two-step path (nf4_dequant
// into bf16, then the bf16 GEMM): each weight becomes bf16(level * absmax) before the MMA.
//
// The weight W is [rows, cols] with cols % 64 == 0 (blocks of 64 along each row), stored as
// codes uint8 [rows * cols / 2] (low nibble first) and absmax fp32 [rows * cols / 64].
//
// Use: small M. Every 256-row M tile dequantises its B tiles again and the 16-level lookup costs
// several instructions per weight, so at training-size M (8192 tokens) the dequantising warps,
// not the tensor cores, set the pace; the decoder then expands a layer once into bf16 scratch
// (models/nf4.py) and runs the bf16 GEMM instead.
#include "gemm_kernel.cuh"

using namespace me::gemm;

namespace {

void check_nf4(const torch::Tensor& codes, const torch::Tensor& absmax, int64_t rows, int64_t cols,
               const char* who) {
  TORCH_CHECK(rows > 0 && cols > 0 && cols % 64 == 0, who, ": NF4 weight columns must be a multiple of 64");
  TORCH_CHECK(codes.is_cuda() && codes.scalar_type() == torch::kUInt8 && codes.is_contiguous() &&
                  codes.numel() == rows * cols / 2,
              who, ": codes must be contiguous uint8 [rows * cols / 2] on the GPU");
  TORCH_CHECK(absmax.is_cuda() && absmax.scalar_type() == torch::kFloat32 && absmax.is_contiguous() &&
                  absmax.numel() == rows * cols / 64,
              who, ": absmax must be contiguous fp32 [rows * cols / 64] on the GPU");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(codes.data_ptr()) % 16 == 0, who, ": codes must be 16-byte aligned");
}

void set_nf4(GemmArgs& a, const torch::Tensor& codes, const torch::Tensor& absmax, int64_t rows, int64_t cols) {
  a.q_codes = codes.data_ptr<uint8_t>();
  a.q_absmax = absmax.data_ptr<float>();
  a.q_rows = rows;
  a.q_cols = cols;
}

}  // namespace

// out[M, N] = A[M, K] . W^T with W [N, K] (b_kmajor, the forward), or A . W with W [K, N] (the
// input gradient). bf16 in and out, fp32 accumulation.
torch::Tensor gemm_nf4(torch::Tensor A, torch::Tensor codes, torch::Tensor absmax, int64_t rows, int64_t cols,
                       bool b_kmajor, c10::optional<torch::Tensor> out) {
  check_operand(A, "A");
  check_nf4(codes, absmax, rows, cols, "gemm_nf4");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1);
  const int N = (int)(b_kmajor ? rows : cols);
  TORCH_CHECK((b_kmajor ? cols : rows) == K, "gemm_nf4: inner dimensions differ");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "gemm_nf4: N and K must be multiples of 8");
  torch::Tensor D = out.has_value() ? *out : torch::empty({M, N}, A.options());
  check_operand(D, "out");
  TORCH_CHECK(D.size(0) == M && D.size(1) == N, "gemm_nf4: out shape");
  if (M == 0) return D;
  const int dev = A.get_device();
  GemmArgs a = base_args(M, N, K, (N + BN - 1) / BN, dev);
  a.D = reinterpret_cast<bf16*>(D.data_ptr());
  a.ldd = D.stride(0);
  set_nf4(a, codes, absmax, rows, cols);
  auto stream = at::cuda::getCurrentCUDAStream();
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BK, BM);
  if (b_kmajor) launch<EPI_STORE, false, false, true>(ta, ta, a, dev, stream);
  else launch<EPI_STORE, true, false, true>(ta, ta, a, dev, stream);
  return D;
}

// (m, gu) of the fused gate|up projection with an NF4 weight Wgu [2F, K] (see gemm_geglu).
std::vector<torch::Tensor> gemm_geglu_nf4(torch::Tensor A, torch::Tensor codes, torch::Tensor absmax, int64_t rows,
                                          int64_t cols, bool save_gu) {
  check_operand(A, "A");
  check_nf4(codes, absmax, rows, cols, "gemm_geglu_nf4");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1);
  TORCH_CHECK(cols == K && rows % 2 == 0, "gemm_geglu_nf4: W must be [2F, K]");
  const int F = (int)(rows / 2);
  TORCH_CHECK(F % 8 == 0, "gemm_geglu_nf4: F must be a multiple of 8");
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
  set_nf4(a, codes, absmax, rows, cols);
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BK, BM);
  launch<EPI_GEGLU, false, false, true>(ta, ta, a, dev, at::cuda::getCurrentCUDAStream());
  return {m, gu};
}

// d_gu of the down projection's input gradient with an NF4 weight Wdown [d, F] (see gemm_dgeglu).
torch::Tensor gemm_dgeglu_nf4(torch::Tensor dY, torch::Tensor codes, torch::Tensor absmax, int64_t rows,
                              int64_t cols, torch::Tensor gu) {
  check_operand(dY, "dY");
  check_operand(gu, "gu");
  check_nf4(codes, absmax, rows, cols, "gemm_dgeglu_nf4");
  const at::cuda::CUDAGuard guard(dY.device());
  const int M = (int)dY.size(0), K = (int)dY.size(1);
  TORCH_CHECK(rows == K, "gemm_dgeglu_nf4: W must be [d, F]");
  const int F = (int)cols;
  TORCH_CHECK(gu.size(0) == M && gu.size(1) == 2 * F, "gemm_dgeglu_nf4: gu must be [M, 2F]");
  auto dgu = torch::empty({M, 2 * F}, dY.options());
  if (M == 0) return dgu;
  const int dev = dY.get_device();
  GemmArgs a = base_args(M, F, K, (F + BN - 1) / BN, dev);
  a.D = reinterpret_cast<bf16*>(dgu.data_ptr());
  a.ldd = 2 * F;
  a.aux = reinterpret_cast<const bf16*>(gu.data_ptr());
  a.ld_aux = gu.stride(0);
  set_nf4(a, codes, absmax, rows, cols);
  const CUtensorMap ta = make_tmap(dY.data_ptr(), M, K, dY.stride(0), BK, BM);
  launch<EPI_DGEGLU, true, false, true>(ta, ta, a, dev, at::cuda::getCurrentCUDAStream());
  return dgu;
}
