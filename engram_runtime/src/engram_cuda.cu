// sm_100a injection path of the engram runtime: the engram's tensors live on the GPU as bf16
// (norm scales fp32); one call runs
//   gather (rows -> mem, fp32)  ->  key / value (or down) projections for a few tokens at a time,
//   each weight row read once per token group  ->  gate + residual add (or gelu * mem -> up -> add).
// Decode batches are small, so the projections are weight-streaming GEMVs: one warp per
// output row, 16-byte weight loads, up to 8 tokens per pass with their inputs in shared memory.
// Large prefill batches run the same kernels over token groups (the weights stay in L2).
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <string>
#include <vector>

#include "engram_runtime.h"
#include "runtime.h"

namespace me {

struct GpuEngram {
  int device = -1;
  __nv_bfloat16* tables = nullptr;          // [total_rows, dim]
  __nv_bfloat16 *w_a = nullptr, *w_b = nullptr;  // key, value  (ple: down, up)
  float *qs = nullptr, *ks = nullptr;
  float* scratch = nullptr;  // mem, a, b, c  per token
  int64_t scratch_tokens = 0;
};

namespace {

constexpr int kTok = 8;  // tokens per projection pass
constexpr float kRmsEps = 1.1920928955078125e-07f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : 0.f;
  return warp_sum(v);
}

// mem[t, k*dim + c] = tables[rows[t*nt + k], c]
__global__ void gather_kernel(const __nv_bfloat16* __restrict__ tables, const int32_t* __restrict__ rows, int nt,
                              int dim, int64_t total_rows, float* __restrict__ mem, int* __restrict__ bad) {
  const int t = blockIdx.x;
  const int md = nt * dim;
  for (int i = threadIdx.x; i < md; i += blockDim.x) {
    const int k = i / dim, c = i - k * dim;
    const int64_t r = rows[(int64_t)t * nt + k];
    if (r < 0 || r >= total_rows) {  // never read outside the table; the host reports it
      if (c == 0) atomicExch(bad, 1);
      mem[(int64_t)t * md + i] = 0.f;
      continue;
    }
    mem[(int64_t)t * md + i] = __bfloat162float(tables[r * dim + c]);
  }
}

// y[t, r] = sum_i W[r, i] x[t, i] for t in [t0, t0+nt) (nt <= kTok); W bf16 [rows, cols] row-major.
// One warp per output row; x rows of the token group staged in shared memory.
template <bool VEC>
__global__ void gemv_kernel(const __nv_bfloat16* __restrict__ W, int64_t rows, int64_t cols,
                            const float* __restrict__ x, float* __restrict__ y, int ntok) {
  extern __shared__ float xs[];  // [ntok, cols]
  for (int64_t i = threadIdx.x; i < (int64_t)ntok * cols; i += blockDim.x) xs[i] = x[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const __nv_bfloat16* w = W + r * cols;
  float acc[kTok];
#pragma unroll
  for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
  if (VEC) {
    for (int64_t i0 = (int64_t)lane * 8; i0 < cols; i0 += 256) {
      const uint4 raw = *reinterpret_cast<const uint4*>(w + i0);
      const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&raw);
      float wf[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) wf[e] = __bfloat162float(wb[e]);
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        if (t < ntok) {
          const float* xr = xs + (int64_t)t * cols + i0;
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[t] += wf[e] * xr[e];
        }
      }
    }
  } else {
    for (int64_t i = lane; i < cols; i += 32) {
      const float wf = __bfloat162float(w[i]);
#pragma unroll
      for (int t = 0; t < kTok; ++t)
        if (t < ntok) acc[t] += wf * xs[(int64_t)t * cols + i];
    }
  }
#pragma unroll
  for (int t = 0; t < kTok; ++t) {
    if (t < ntok) {
      const float s = warp_sum(acc[t]);
      if (lane == 0) y[(int64_t)t * rows + r] = s;
    }
  }
}

// scalar / scalar_sqrt gate, one block per token: hidden += sigmoid(s) * v * keep
__global__ void gate_kernel(float* __restrict__ hidden, const float* __restrict__ k, const float* __restrict__ v,
                            const float* __restrict__ qs, const float* __restrict__ ks,
                            const float* __restrict__ keep, int d, int sqrt_gate) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  float* h = hidden + (int64_t)t * d;
  const float* kr = k + (int64_t)t * d;
  float sh = 0.f, sk = 0.f, dot = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float a = h[j], b = kr[j];
    sh += a * a;
    sk += b * b;
    dot += a * b * (qs ? qs[j] : 1.f) * (ks ? ks[j] : 1.f);
  }
  sh = block_sum(sh, red);
  sk = block_sum(sk, red);
  dot = block_sum(dot, red);
  const float rh = rsqrtf(sh / d + kRmsEps), rk = rsqrtf(sk / d + kRmsEps);
  float s = rh * rk * dot * rsqrtf((float)d);
  if (sqrt_gate) {
    const float sg = s > 0.f ? 1.f : (s < 0.f ? -1.f : 0.f);
    s = sg * sqrtf(fmaxf(fabsf(s), 1e-6f));
  }
  const float alpha = 1.f / (1.f + expf(-s)) * (keep ? keep[t] : 1.f);
  const float* vr = v + (int64_t)t * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) h[j] += alpha * vr[j];
}

// hn[t] = rms(hidden[t])  (ple gate input)
__global__ void rms_kernel(const float* __restrict__ hidden, float* __restrict__ hn, int d) {
  __shared__ float red[32];
  const float* h = hidden + (int64_t)blockIdx.x * d;
  float ss = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) ss += h[j] * h[j];
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / d + kRmsEps);
  for (int j = threadIdx.x; j < d; j += blockDim.x) hn[(int64_t)blockIdx.x * d + j] = h[j] * r;
}

// z <- gelu_tanh(z) * mem
__global__ void gelu_mul_kernel(float* __restrict__ z, const float* __restrict__ mem, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = z[i];
  z[i] = 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x))) * mem[i];
}

// hidden[t] += out[t] * keep[t]
__global__ void add_kernel(float* __restrict__ hidden, const float* __restrict__ out, const float* __restrict__ keep,
                           int d, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * d) return;
  hidden[i] += out[i] * (keep ? keep[i / d] : 1.f);
}

int ck(cudaError_t e, const char* what, std::string* err) {
  if (e == cudaSuccess) return ME_RT_OK;
  *err = std::string(what) + ": " + cudaGetErrorString(e);
  return ME_RT_ERR_CUDA;
}

template <typename T>
int upload(const std::vector<T>& host, T** dev, std::string* err) {
  if (int rc = ck(cudaMalloc(reinterpret_cast<void**>(dev), host.size() * sizeof(T)), "cudaMalloc", err)) return rc;
  return ck(cudaMemcpy(*dev, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice), "cudaMemcpy", err);
}

int bf16_of(const Tensor* t, __nv_bfloat16** dev, std::string* err) {
  std::vector<uint16_t> bits;
  if (!tensor_to_bf16(*t, &bits)) {
    *err = "tensor " + t->name + " has an unsupported type";
    return ME_RT_ERR_FORMAT;
  }
  return upload(bits, reinterpret_cast<uint16_t**>(dev), err);
}

void gemv(const __nv_bfloat16* W, int64_t rows, int64_t cols, const float* x, float* y, int64_t n,
          cudaStream_t s) {
  const int warps = 8;
  const bool vec = cols % 8 == 0 && (reinterpret_cast<uintptr_t>(W) % 16) == 0;
  const int64_t fit = std::max<int64_t>(1, std::min<int64_t>(kTok, (96 * 1024) / (cols * 4)));
  for (int64_t t0 = 0; t0 < n; t0 += fit) {
    const int nt = (int)std::min<int64_t>(fit, n - t0);
    const dim3 grid((unsigned)((rows + warps - 1) / warps));
    const size_t sm = (size_t)nt * cols * 4;
    if (vec)
      gemv_kernel<true><<<grid, warps * 32, sm, s>>>(W, rows, cols, x + t0 * cols, y + t0 * rows, nt);
    else
      gemv_kernel<false><<<grid, warps * 32, sm, s>>>(W, rows, cols, x + t0 * cols, y + t0 * rows, nt);
  }
}

}  // namespace

int cuda_available() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0 ? 1 : 0;
}

void cuda_release(Engram& e) {
  GpuEngram* g = e.gpu;
  if (!g) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  for (void* p : {(void*)g->tables, (void*)g->w_a, (void*)g->w_b, (void*)g->qs, (void*)g->ks, (void*)g->scratch})
    if (p) cudaFree(p);
  cudaSetDevice(prev);
  delete g;
  e.gpu = nullptr;
}

int cuda_upload(Engram& e, int64_t n_embd, int device, std::string* err) {
  if (!cuda_available()) {
    *err = "no CUDA device";
    return ME_RT_ERR_CUDA;
  }
  cuda_release(e);
  if (int rc = ck(cudaSetDevice(device), "cudaSetDevice", err)) return rc;
  static bool attr_set[2] = {false, false};
  if (!attr_set[0]) {  // allow the token group's inputs (up to 96 KB) in shared memory
    cudaFuncSetAttribute(gemv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024 + 1024);
    cudaFuncSetAttribute(gemv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024 + 1024);
    attr_set[0] = true;
  }
  auto* g = new GpuEngram();
  g->device = device;
  e.gpu = g;
  int rc = bf16_of(e.tables, &g->tables, err);
  if (!rc) rc = bf16_of(e.gate == ME_RT_GATE_PLE ? e.down : e.key, &g->w_a, err);
  if (!rc) rc = bf16_of(e.gate == ME_RT_GATE_PLE ? e.up : e.value, &g->w_b, err);
  if (!rc && e.q_scale) {
    std::vector<float> q, k;
    tensor_to_f32(*e.q_scale, &q);
    tensor_to_f32(*e.k_scale, &k);
    rc = upload(q, &g->qs, err);
    if (!rc) rc = upload(k, &g->ks, err);
  }
  (void)n_embd;
  if (rc) cuda_release(e);
  return rc;
}

int cuda_inject(Engram& e, int64_t d, float* d_hidden, const int32_t* d_rows, const float* d_keep, int64_t n,
                void* stream, std::string* err) {
  GpuEngram* g = e.gpu;
  if (!g) {
    *err = "engram not uploaded (call me_rt_cuda_upload first)";
    return ME_RT_ERR_CUDA;
  }
  if (n <= 0) return ME_RT_OK;
  if (!d_hidden || !d_rows) {
    *err = "null device pointer";
    return ME_RT_ERR_ARG;
  }
  if (int rc = ck(cudaSetDevice(g->device), "cudaSetDevice", err)) return rc;
  const int64_t md = e.mem_dim();
  const int64_t per_tok = md + 2 * std::max(d, md) + 1;
  if (g->scratch_tokens < n) {
    if (g->scratch) cudaFree(g->scratch);
    g->scratch = nullptr;
    g->scratch_tokens = 0;
    // an int flag for out-of-range rows sits after the per-token buffers
    if (int rc = ck(cudaMalloc(&g->scratch, (size_t)(n * per_tok + 4) * sizeof(float)), "cudaMalloc", err))
      return rc;
    g->scratch_tokens = n;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* mem = g->scratch;
  float* a = mem + n * md;
  float* b = a + n * std::max(d, md);
  int* bad = reinterpret_cast<int*>(g->scratch + (size_t)g->scratch_tokens * per_tok);
  if (int rc = ck(cudaMemsetAsync(bad, 0, 4, s), "cudaMemsetAsync", err)) return rc;
  gather_kernel<<<(unsigned)n, 256, 0, s>>>(g->tables, d_rows, (int)e.n_tables, (int)e.dim, (int64_t)e.total_rows,
                                             mem, bad);
  if (e.gate == ME_RT_GATE_PLE) {
    rms_kernel<<<(unsigned)n, 256, 0, s>>>(d_hidden, b, (int)d);
    gemv(g->w_a, md, d, b, a, n, s);  // down: [mem_dim, d]
    gelu_mul_kernel<<<(unsigned)((n * md + 255) / 256), 256, 0, s>>>(a, mem, n * md);
    gemv(g->w_b, d, md, a, b, n, s);  // up: [d, mem_dim]
    add_kernel<<<(unsigned)((n * d + 255) / 256), 256, 0, s>>>(d_hidden, b, d_keep, (int)d, n);
  } else {
    gemv(g->w_a, d, md, mem, a, n, s);  // key
    gemv(g->w_b, d, md, mem, b, n, s);  // value
    gate_kernel<<<(unsigned)n, 256, 0, s>>>(d_hidden, a, b, g->qs, g->ks, d_keep, (int)d,
                                            e.gate == ME_RT_GATE_SCALAR_SQRT ? 1 : 0);
  }
  if (int rc = ck(cudaGetLastError(), "kernel launch", err)) return rc;
  int h_bad = 0;
  if (int rc = ck(cudaMemcpyAsync(&h_bad, bad, 4, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync", err)) return rc;
  if (int rc = ck(cudaStreamSynchronize(s), "cudaStreamSynchronize", err)) return rc;
  if (h_bad) {
    *err = "row index out of range (those rows read as zero)";
    return ME_RT_ERR_ARG;
  }
  return ME_RT_OK;
}

}  // namespace me
