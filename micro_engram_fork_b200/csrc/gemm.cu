// Plain projections on the persistent tcgen05 GEMM (kernel and its design: gemm_kernel.cuh):
// bf16 out for the decoder's forward and dX products, fp32 out for the LM head's dH.
#include "gemm_kernel.cuh"

using namespace me::gemm;

// out[M, N] = A[M, K] . W^T, where W is [N, K] (b_kmajor) or W is [K, N] (the transposed use:
// out = A . W). bf16 in, bf16 out, fp32 accumulation. `out` may be given (row stride >= N).
torch::Tensor gemm(torch::Tensor A, torch::Tensor W, bool b_kmajor, c10::optional<torch::Tensor> out) {
  check_operand(A, "A");
  check_operand(W, "W");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1);
  const int N = (int)(b_kmajor ? W.size(0) : W.size(1));
  TORCH_CHECK((b_kmajor ? W.size(1) : W.size(0)) == K, "gemm: inner dimensions differ");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "gemm: N and K must be multiples of 8");
  torch::Tensor D = out.has_value() ? *out : torch::empty({M, N}, A.options());
  check_operand(D, "out");
  TORCH_CHECK(D.size(0) == M && D.size(1) == N, "gemm: out shape");
  if (M == 0 || N == 0) return D;
  if (K == 0) return D.zero_();
  const int dev = A.get_device();
  GemmArgs a = base_args(M, N, K, (N + BN - 1) / BN, dev);
  a.D = reinterpret_cast<bf16*>(D.data_ptr());
  a.ldd = D.stride(0);
  auto stream = at::cuda::getCurrentCUDAStream();
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BK, BM);
  if (b_kmajor) {
    const CUtensorMap tb = make_tmap(W.data_ptr(), N, K, W.stride(0), BK, BN / 2);
    launch<EPI_STORE, false>(ta, tb, a, dev, stream);
  } else {
    const CUtensorMap tb = make_tmap(W.data_ptr(), K, N, W.stride(0), 64, BK);
    launch<EPI_STORE, true>(ta, tb, a, dev, stream);
  }
  return D;
}

// Rows scattered to their owners (the GEMM half of a fused GEMM -> reduce-scatter): rows
// [r * rows_per_rank, (r + 1) * rows_per_rank) of the fp32 product are stored into rank r's
// receive buffer recv_ptrs[r], in slot `slot` (slots of slot_elems floats; rows of N floats).
// The product is A . W with W [K, N] read N-major (the LM head's dH), or A . W^T with W [N, K]
// (b_kmajor: a row-parallel linear's partial). M may stop short of world * rows_per_rank: the
// missing rows are not stored. A product of one partial wave of tiles is split along K so that
// small-M calls (decode) keep every SM busy. The caller signals the peers after this launch
// (p2p_sum_slots) so the owners can sum their slots.
void gemm_f32_scatter(torch::Tensor A, torch::Tensor W, torch::Tensor recv_ptrs, int64_t rows_per_rank,
                      int64_t slot, int64_t slot_elems, bool b_kmajor) {
  check_operand(A, "A");
  check_operand(W, "W");
  TORCH_CHECK(recv_ptrs.is_cuda() && recv_ptrs.scalar_type() == torch::kInt64, "gemm_f32_scatter: recv_ptrs");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1);
  const int N = (int)(b_kmajor ? W.size(0) : W.size(1));
  TORCH_CHECK((b_kmajor ? W.size(1) : W.size(0)) == K && N % 8 == 0 && K % 8 == 0,
              "gemm_f32_scatter: inner dimensions differ, or N or K not a multiple of 8");
  TORCH_CHECK(rows_per_rank > 0 && M <= rows_per_rank * recv_ptrs.numel(), "gemm_f32_scatter: M > world * rows");
  TORCH_CHECK(slot_elems >= rows_per_rank * N && slot_elems % 4 == 0, "gemm_f32_scatter: slots too small");
  if (M == 0 || N == 0) return;
  TORCH_CHECK(K > 0, "gemm_f32_scatter: K == 0");
  const int dev = A.get_device();
  GemmArgs a = base_args(M, N, K, (N + BN - 1) / BN, dev);
  a.ldd = N;
  a.peer_out = recv_ptrs.data_ptr<int64_t>();
  a.peer_rows = (int)rows_per_rank;
  a.peer_slot = (int)slot;
  a.peer_slot_elems = slot_elems;
  a.split_one_wave = 1;
  auto stream = at::cuda::getCurrentCUDAStream();
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BK, BM);
  if (b_kmajor) {
    const CUtensorMap tb = make_tmap(W.data_ptr(), N, K, W.stride(0), BK, BN / 2);
    launch<EPI_F32, false>(ta, tb, a, dev, stream);
  } else {
    const CUtensorMap tb = make_tmap(W.data_ptr(), K, N, W.stride(0), 64, BK);
    launch<EPI_F32, true>(ta, tb, a, dev, stream);
  }
}

// out[M, N] (fp32) = A[M, K] . W, with W [K, N] read N-major (the LM head's dH = P . E).
torch::Tensor gemm_f32(torch::Tensor A, torch::Tensor W) {
  check_operand(A, "A");
  check_operand(W, "W");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), K = (int)A.size(1), N = (int)W.size(1);
  TORCH_CHECK(W.size(0) == K, "gemm_f32: inner dimensions differ");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "gemm_f32: N and K must be multiples of 8");
  auto D = torch::empty({M, N}, A.options().dtype(torch::kFloat32));
  if (M == 0 || N == 0) return D;
  if (K == 0) return D.zero_();
  const int dev = A.get_device();
  GemmArgs a = base_args(M, N, K, (N + BN - 1) / BN, dev);
  a.Df = D.data_ptr<float>();
  a.ldd = N;
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BK, BM);
  const CUtensorMap tb = make_tmap(W.data_ptr(), K, N, W.stride(0), 64, BK);
  launch<EPI_F32, true>(ta, tb, a, dev, at::cuda::getCurrentCUDAStream());
  return D;
}

// out[M, N] (fp32) = At^T . Bt with At [K, M] and Bt [K, N] (both read with the reduction
// dimension as rows): the weight gradient dW = dY^T . X of a projection y = x W^T.
torch::Tensor gemm_tn_f32(torch::Tensor At, torch::Tensor Bt) {
  check_operand(At, "At");
  check_operand(Bt, "Bt");
  const at::cuda::CUDAGuard guard(At.device());
  const int K = (int)At.size(0), M = (int)At.size(1), N = (int)Bt.size(1);
  TORCH_CHECK(Bt.size(0) == K, "gemm_tn_f32: At and Bt need the same number of rows");
  TORCH_CHECK(M % 8 == 0 && N % 8 == 0, "gemm_tn_f32: M and N must be multiples of 8 (16-byte rows)");
  auto D = torch::empty({M, N}, At.options().dtype(torch::kFloat32));
  if (M == 0 || N == 0) return D;
  if (K == 0) return D.zero_();
  const int dev = At.get_device();
  GemmArgs a = base_args(M, N, K, (N + BN - 1) / BN, dev);
  a.Df = D.data_ptr<float>();
  a.ldd = N;
  const CUtensorMap ta = make_tmap(At.data_ptr(), K, M, At.stride(0), 64, BK);
  const CUtensorMap tb = make_tmap(Bt.data_ptr(), K, N, Bt.stride(0), 64, BK);
  launch<EPI_F32, true, true>(ta, tb, a, dev, at::cuda::getCurrentCUDAStream());
  return D;
}

// The next GEMM launched on `device` also copies units [begin16, end16) of the segment table at
// `segs` (int64 [nsegs, 4] on the device: src, dst, start16, n16) in its side-copy warp.
void gemm_carry_copy(int64_t device, int64_t segs, int64_t nsegs, int64_t begin16, int64_t end16) {
  TORCH_CHECK(nsegs >= 0 && begin16 >= 0 && end16 >= begin16, "gemm_carry_copy: bad range");
  SideCopy& job = pending_copy((int)device);
  job.segs = reinterpret_cast<const me::GatherSeg*>(segs);
  job.nsegs = (int)nsegs;
  job.begin16 = begin16;
  job.end16 = end16;
}

torch::Tensor gemm_status(int64_t device) { return status_buffer((int)device); }
