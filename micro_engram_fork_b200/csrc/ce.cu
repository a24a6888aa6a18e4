// Softcapped cross-entropy row kernels for the (vocab-parallel) tied head, sm_100a.
//
// Forward: for each row of a logits chunk against this rank's vocab rows, one pass gives
// the softcapped row max, the sum of exp relative to it (online rescaling), and the
// target logit when the label falls in this rank's rows. The ranks' partials (m, s) are
// combined as lse = M + log(sum_r s_r exp(m_r - M)), so full logits never exist anywhere.
// Backward: the logits buffer is overwritten in place with
//   (softmax - onehot) * w_row * softcap'(z)         (bf16)
// ready for the dH GEMM. Semantics follow micro_engram/train/head.py:76-165 (softcap as
// tanh(z/c)*c on the fp32 value of the bf16 GEMM output).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "act.cuh"
#include "common.cuh"

using namespace me;

namespace {
using bf16 = __nv_bfloat16;
constexpr int64_t kIgnore = -100;

// Same softcap evaluation as the tcgen05 head GEMM's CE epilogue (gemm.cu), so the backward's
// probabilities use exactly the logits the forward's log-sum-exp saw.
ME_DEVICE float capz(float z, float cap) { return cap > 0.f ? softcap_fast(z, cap) : z; }

ME_DEVICE void merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  const float mx = fmaxf(m, m2);
  s = s * exp2_fast((m - mx) * kLog2e) + s2 * exp2_fast((m2 - mx) * kLog2e);
  m = mx;
}

__global__ void ce_fwd_kernel(const bf16* __restrict__ z, int64_t M, int64_t V, const int64_t* __restrict__ labels,
                              int64_t start, float cap, float* __restrict__ mx_out, float* __restrict__ s_out,
                              float* __restrict__ tgt_out) {
  __shared__ float sm[32], ss[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    const bf16* row = z + r * V;
    float m = -INFINITY, s = 0.f;
    const int64_t nvec = V / 8;
    for (int64_t i = threadIdx.x; i < nvec; i += blockDim.x) {
      BF16x8 x;
      x.u = reinterpret_cast<const uint4*>(row)[i];
      float c[8];
      float lm = -INFINITY;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = capz(bf2f(x.h[e]), cap);
        lm = fmaxf(lm, c[e]);
      }
      float ls = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ls += exp2_fast((c[e] - lm) * kLog2e);
      merge(m, s, lm, ls);
    }
    for (int64_t j = nvec * 8 + threadIdx.x; j < V; j += blockDim.x) merge(m, s, capz(bf2f(row[j]), cap), 1.f);
    // warp then block merge
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge(m, s, m2, s2);
    }
    __syncthreads();
    if (lane == 0) {
      sm[wid] = m;
      ss[wid] = s;
    }
    __syncthreads();
    if (wid == 0) {
      m = lane < nw ? sm[lane] : -INFINITY;
      s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
        merge(m, s, m2, s2);
      }
      if (lane == 0) {
        mx_out[r] = m;
        s_out[r] = s;
        const int64_t lab = labels[r];
        const int64_t loc = lab - start;
        tgt_out[r] = (lab != kIgnore && loc >= 0 && loc < V) ? capz(bf2f(row[loc]), cap) : 0.f;
      }
    }
  }
}

// in place: z <- (exp(zc - lse) - [j == target]) * w_row * (1 - (zc/cap)^2)
__global__ void ce_bwd_kernel(bf16* __restrict__ z, int64_t M, int64_t V, const int64_t* __restrict__ labels,
                              int64_t start, float cap, const float* __restrict__ lse,
                              const float* __restrict__ w_row) {
  for (int64_t r = blockIdx.x; r < M; r += gridDim.x) {
    bf16* row = z + r * V;
    const float l = lse[r];
    const float w = w_row[r];
    const int64_t lab = labels[r];
    const int64_t loc = (lab != kIgnore) ? lab - start : -1;
    const int64_t nvec = V / 8;
    for (int64_t i = threadIdx.x; i < nvec; i += blockDim.x) {
      BF16x8 x;
      x.u = reinterpret_cast<const uint4*>(row)[i];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float zc = capz(bf2f(x.h[e]), cap);
        float p = exp2_fast((zc - l) * kLog2e);
        if (i * 8 + e == loc) p -= 1.f;
        float gr = p * w;
        if (cap > 0.f) {
          const float t = zc / cap;
          gr *= (1.f - t * t);
        }
        x.h[e] = f2bf(gr);
      }
      reinterpret_cast<uint4*>(row)[i] = x.u;
    }
    for (int64_t j = nvec * 8 + threadIdx.x; j < V; j += blockDim.x) {
      const float zc = capz(bf2f(row[j]), cap);
      float p = exp2_fast((zc - l) * kLog2e);
      if (j == loc) p -= 1.f;
      float gr = p * w;
      if (cap > 0.f) {
        const float t = zc / cap;
        gr *= (1.f - t * t);
      }
      row[j] = f2bf(gr);
    }
  }
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}
}  // namespace

// returns (row max, sum exp relative to it, target logit or 0), fp32 [M] each
std::vector<torch::Tensor> ce_fwd(torch::Tensor z, torch::Tensor labels, int64_t start, double softcap) {
  TORCH_CHECK(z.is_cuda() && z.is_contiguous() && z.scalar_type() == torch::kBFloat16, "logits: contiguous bf16");
  const at::cuda::CUDAGuard guard(z.device());
  const int64_t M = z.size(0), V = z.size(1);
  auto opts = z.options().dtype(torch::kFloat32);
  auto m = torch::empty({M}, opts), s = torch::empty({M}, opts), t = torch::empty({M}, opts);
  if (M == 0) return {m, s, t};
  auto lab = labels.to(torch::kLong).contiguous();
  const int grid = (int)std::min<int64_t>(M, (int64_t)sm_count() * 4);
  ce_fwd_kernel<<<grid, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(z.data_ptr()), M, V, lab.data_ptr<int64_t>(), start, (float)softcap,
      m.data_ptr<float>(), s.data_ptr<float>(), t.data_ptr<float>());
  return {m, s, t};
}

void ce_bwd_inplace(torch::Tensor z, torch::Tensor labels, int64_t start, double softcap, torch::Tensor lse,
                    torch::Tensor w_row) {
  TORCH_CHECK(z.is_cuda() && z.is_contiguous() && z.scalar_type() == torch::kBFloat16, "logits: contiguous bf16");
  const at::cuda::CUDAGuard guard(z.device());
  const int64_t M = z.size(0), V = z.size(1);
  if (M == 0) return;
  auto lab = labels.to(torch::kLong).contiguous();
  auto l = lse.to(torch::kFloat32).contiguous(), w = w_row.to(torch::kFloat32).contiguous();
  const int grid = (int)std::min<int64_t>(M, (int64_t)sm_count() * 4);
  ce_bwd_kernel<<<grid, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<bf16*>(z.data_ptr()), M, V, lab.data_ptr<int64_t>(), start, (float)softcap,
      l.data_ptr<float>(), w.data_ptr<float>());
}
