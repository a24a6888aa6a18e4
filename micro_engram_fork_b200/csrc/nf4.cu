// NF4 storage of the frozen base (4-bit NormalFloat, Dettmers et al. 2023, "QLoRA", sec. 3 and
// appendix: 16 levels, the quantiles of N(0,1) rescaled to [-1, 1] with an exact zero),
// one fp32 absmax per block of 64 consecutive weights, two codes per byte (low nibble first).
// The reference gets the same format from bitsandbytes (micro_engram/train/model.py:122-130:
// nf4, compute and storage bf16); here a layer's weights are expanded to bf16 just before use
// by a bandwidth-bound kernel, then the tensor-core GEMMs run on bf16 operands.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

using namespace me;

namespace {

// QLoRA appendix E, the NF4 data type
__constant__ float kNF4[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                               -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                               0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f,
                               0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f,
                               0.7229568362236023f, 1.0f};

constexpr int kBlock = 64;

// one thread per block of 64 weights: absmax, then the nearest level of w / absmax
__global__ void nf4_quantize_kernel(const __nv_bfloat16* __restrict__ w, int64_t n_blocks,
                                    uint8_t* __restrict__ codes, float* __restrict__ absmax) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  const __nv_bfloat16* src = w + b * kBlock;
  float m = 0.f;
  for (int i = 0; i < kBlock; ++i) m = fmaxf(m, fabsf(bf2f(src[i])));
  absmax[b] = m;
  const float inv = m > 0.f ? 1.f / m : 0.f;
  for (int i = 0; i < kBlock; i += 2) {
    uint8_t pair = 0;
    for (int h = 0; h < 2; ++h) {
      const float x = bf2f(src[i + h]) * inv;
      int best = 0;
      float bd = fabsf(x - kNF4[0]);
      for (int q = 1; q < 16; ++q) {
        const float dq = fabsf(x - kNF4[q]);
        if (dq < bd) {
          bd = dq;
          best = q;
        }
      }
      pair |= (uint8_t)(best << (4 * h));
    }
    codes[b * (kBlock / 2) + i / 2] = pair;
  }
}

// each thread expands 32 weights (16 code bytes, half a block) with 16-byte loads and stores
__global__ void nf4_dequant_kernel(const uint4* __restrict__ codes, const float* __restrict__ absmax,
                                   int64_t n_chunks, uint4* __restrict__ out) {
  __shared__ float lv[16];
  if (threadIdx.x < 16) lv[threadIdx.x] = kNF4[threadIdx.x];
  __syncthreads();
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n_chunks; c += (int64_t)gridDim.x * blockDim.x) {
    const uint4 raw = __ldcs(codes + c);
    const float s = __ldg(absmax + (c >> 1));
    const uint8_t* by = reinterpret_cast<const uint8_t*>(&raw);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      BF16x8 o;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint8_t v = by[q * 4 + j];
        o.h2[j] = __floats2bfloat162_rn(lv[v & 15] * s, lv[v >> 4] * s);
      }
      out[c * 4 + q] = o.u;
    }
  }
}

}  // namespace

// w [.., K] bf16 contiguous, numel % 64 == 0 -> (codes uint8 [numel/2], absmax fp32 [numel/64])
std::vector<torch::Tensor> nf4_quantize(torch::Tensor w) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kBFloat16 && w.is_contiguous(),
              "nf4_quantize: contiguous bf16 CUDA tensor expected");
  TORCH_CHECK(w.numel() % kBlock == 0, "nf4_quantize: the number of weights must be a multiple of 64");
  const at::cuda::CUDAGuard guard(w.device());
  const int64_t nb = w.numel() / kBlock;
  auto codes = torch::empty({w.numel() / 2}, w.options().dtype(torch::kUInt8));
  auto absmax = torch::empty({nb}, w.options().dtype(torch::kFloat32));
  if (nb) {
    nf4_quantize_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), nb, codes.data_ptr<uint8_t>(),
        absmax.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {codes, absmax};
}

// codes, absmax -> out (bf16, numel = 2 * codes.numel(), contiguous, 16-byte aligned)
void nf4_dequant(torch::Tensor codes, torch::Tensor absmax, torch::Tensor out) {
  TORCH_CHECK(codes.is_cuda() && codes.scalar_type() == torch::kUInt8 && codes.is_contiguous(), "nf4 codes");
  TORCH_CHECK(absmax.scalar_type() == torch::kFloat32 && absmax.numel() * 32 == codes.numel(), "nf4 absmax");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.numel() == 2 * codes.numel(),
              "nf4_dequant: out must be contiguous bf16 with 2 weights per code byte");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(codes.data_ptr()) % 16 == 0,
              "nf4_dequant: 16-byte aligned buffers expected");
  const at::cuda::CUDAGuard guard(codes.device());
  const int64_t chunks = codes.numel() / 16;
  if (!chunks) return;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>((chunks + 255) / 256, (int64_t)sms * 8);
  nf4_dequant_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(codes.data_ptr()), absmax.data_ptr<float>(), chunks,
      reinterpret_cast<uint4*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
