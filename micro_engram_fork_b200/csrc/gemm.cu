// tcgen05 GEMM for sm_100a: D[M, N] = A[M, K] . B[N, K]^T, bf16 operands, fp32 accumulation
// in tensor memory, bf16 output.
//
// One CTA computes a 128 x BN tile with three warp roles (192 threads):
//   warp 0      TMA producer: one elected thread streams 64-wide K blocks of A and B into a
//               STAGES-deep ring of 128B-swizzled shared-memory stages (cp.async.bulk.tensor,
//               no multicast), each stage guarded by a full/empty mbarrier pair
//   warp 1      allocates the TMEM accumulator (BN fp32 columns x 128 lanes) and one elected
//               thread issues tcgen05.mma (M=128, N=BN, K=16; 4 per stage) and tcgen05.commit
//               to release each stage back to the producer and, at the end, to wake the epilogue
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns at a time (each warp owns the TMEM
//               lane quadrant warp%4), convert to bf16 and store
// Every mbarrier wait is bounded (%globaltimer, 2 s); on expiry the kernel records
// ME_ERR_TIMEOUT in the status word, the other roles stop, TMEM is freed and the kernel returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "tc_common.cuh"

using namespace me;
using namespace me::tc;

namespace {
using bf16 = __nv_bfloat16;
constexpr int BM = 128, BK = 64;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int TILE_BYTES = STAGES * (A_BYTES + B_BYTES);
  static constexpr int BYTES = TILE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, bf16* __restrict__ D,
                   int64_t ldd, int M, int N, int K, int* status) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort = 0;
    fence_barrier_init();
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES, r = kb / STAGES;
        if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, status, 1, abort)) break;
        mbar_expect_tx(&full[s], S::A_BYTES + S::B_BYTES);
        tma_load_2d(sA + s * S::A_BYTES, &ta, &full[s], kb * BK, m0);
        tma_load_2d(sB + s * S::B_BYTES, &tb, &full[s], kb * BK, n0);
      }
      // drain: make sure every issued copy has landed before the CTA can exit
      const int first = nk > STAGES ? nk - STAGES : 0;
      for (int kb = first; kb < nk; ++kb) mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1, status, 4, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(BM, BN);
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES, r = kb / STAGES;
        if (!mbar_wait(&full[s], r & 1, status, 2, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(sA + s * S::A_BYTES), b0 = smem_addr(sB + s * S::B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_bf16(tmem, desc_sw128(a0 + k * 32), desc_sw128(b0 + k * 32), idesc, (kb | k) != 0);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(done);
    }
  } else {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    if (mbar_wait(done, 0, status, 3, abort)) {
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + c * 32, v);
        const int col = n0 + c * 32;
        if (row < M) {
          bf16* dst = D + (int64_t)row * ldd + col;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (col + j * 8 < N) {
              BF16x8 o;
#pragma unroll
              for (int e = 0; e < 8; ++e) o.h[e] = f2bf(v[j * 8 + e]);
              *reinterpret_cast<uint4*>(dst + j * 8) = o.u;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host: tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 2-D K-major bf16 operand [rows, K] (row stride ld elements), box 64 x box_rows, 128B swizzle.
CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA operand base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return map;
}

torch::Tensor& status_buffer(int dev) {
  static std::unordered_map<int, torch::Tensor> bufs;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  auto it = bufs.find(dev);
  if (it == bufs.end())
    it = bufs.emplace(dev, torch::zeros({2}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev)))
             .first;
  return it->second;
}

template <int BN, int STAGES>
void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, bf16* D, int64_t ldd, int M, int N, int K, int* st,
                 cudaStream_t stream) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_tc_kernel<BN, STAGES>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES);
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  kern<<<grid, 192, S::BYTES, stream>>>(ta, tb, D, ldd, M, N, K, st);
}

}  // namespace

// D = A . B^T (A [M, K], B [N, K], bf16, row-major) on the tcgen05 kernel.
torch::Tensor gemm_tc(torch::Tensor A, torch::Tensor B, int64_t block_n) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "gemm_tc: CUDA tensors");
  TORCH_CHECK(A.scalar_type() == torch::kBFloat16 && B.scalar_type() == torch::kBFloat16, "gemm_tc: bf16");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_tc: A [M,K], B [N,K]");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_tc: K-major operands");
  const at::cuda::CUDAGuard guard(A.device());
  const int M = (int)A.size(0), N = (int)B.size(0), K = (int)A.size(1);
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gemm_tc: K and N must be multiples of 8");
  auto D = torch::empty({M, N}, A.options());
  if (M == 0 || N == 0) return D;
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status_buffer(A.get_device()).data_ptr<int>();
  auto* dp = reinterpret_cast<bf16*>(D.data_ptr());
  const CUtensorMap ta = make_tmap(A.data_ptr(), M, K, A.stride(0), BM);
  if (block_n == 128) {
    const CUtensorMap tb = make_tmap(B.data_ptr(), N, K, B.stride(0), 128);
    launch_gemm<128, 6>(ta, tb, dp, N, M, N, K, st, stream);
  } else {
    const CUtensorMap tb = make_tmap(B.data_ptr(), N, K, B.stride(0), 256);
    launch_gemm<256, 4>(ta, tb, dp, N, M, N, K, st, stream);
  }
  return D;
}

torch::Tensor gemm_status(int64_t device) { return status_buffer((int)device); }
