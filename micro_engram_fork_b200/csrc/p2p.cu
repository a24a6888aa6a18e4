// One-shot all-reduce (mean) of the replicated dense engram gradients over peer memory
// (CUDA IPC mappings of every rank's symmetric buffer, NVLink 5 / NVSwitch), in ONE kernel:
// signal, wait, reduce. It replaces the flat fp32 NCCL all_reduce / world of the reference
// (micro_engram/train/loop.py:316-327); the semantics (sum over ranks, then / world, in fp32)
// are the same.
//
// Buffer layout on every rank (same offsets everywhere):
//   flags  [world] u32 at offset 0: flags[r] = last call number rank r has staged
//   stage  [2][np] fp32 at offset `stage_off`, np = n rounded up to a multiple of 4 so both
//          halves start 16-byte aligned for the float4 loads: the caller packs its gradients into
//          stage[call & 1] before the kernel (double buffering: a rank can be at most one call
//          ahead of a peer that is still reading, since call c+1 cannot finish before every
//          peer has signalled c+1, which each does only after finishing call c)
// Every block of the kernel: (1) release-stores `call` into flags[rank] of every peer (idempotent,
// so no block depends on another block being scheduled), (2) waits with acquire loads until
// every flags[r] >= call, at most `timeout_ns` (then records ME_ERR_TIMEOUT and returns without
// writing), (3) sums its slice of stage[call & 1] over all ranks (L2-only loads: no stale L1
// lines from the call two steps back) and writes out = sum * scale.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gather.cuh"

using namespace me;

namespace {

constexpr int MAX_RANKS = 16;

__global__ void __launch_bounds__(256) p2p_allreduce_mean_kernel(const int64_t* __restrict__ bases, int world,
                                                                  int rank, int64_t stage_off, int64_t n,
                                                                  uint32_t call, float scale, uint64_t timeout_ns,
                                                                  float* __restrict__ out, int* status) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < world) {
    uint32_t* peer_flags = reinterpret_cast<uint32_t*>(bases[threadIdx.x]);
    st_release_sys(peer_flags + rank, call);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(bases[rank]) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if ((int32_t)(ld_acquire_sys(mine) - call) >= 0) break;
      if ((it & 63u) == 63u && globaltimer_ns() - t0 > timeout_ns) {
        report(status, ME_ERR_TIMEOUT, threadIdx.x);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (failed) return;
  const int64_t par = (int64_t)(call & 1u) * ((n + 3) / 4 * 4);  // half stride np: 16-byte aligned
  const float* src[MAX_RANKS];
#pragma unroll
  for (int r = 0; r < MAX_RANKS; ++r)
    src[r] = r < world ? reinterpret_cast<const float*>(bases[r] + stage_off) + par : nullptr;
  // UNR float4 per thread and iteration, all ranks' loads issued before any add: enough bytes in
  // flight to cover the NVLink round trip
  constexpr int UNR = 4;
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n4; i0 += stride * UNR) {
    float4 acc[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      float4 v[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int64_t i = i0 + u * stride;
        v[u] = i < n4 ? __ldcg(reinterpret_cast<const float4*>(src[r]) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) acc[u].x += v[u].x, acc[u].y += v[u].y, acc[u].z += v[u].z, acc[u].w += v[u].w;
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n4)
        reinterpret_cast<float4*>(out)[i] =
            make_float4(acc[u].x * scale, acc[u].y * scale, acc[u].z * scale, acc[u].w * scale);
    }
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < world; ++r) acc += __ldcg(src[r] + i);
    out[i] = acc * scale;
  }
}

// ------------------------------------------------------------------ exchanges of the vocab loss
// Every block signals `call` into flag[rank] of every peer and waits (acquire, bounded) until
// all flags have reached it: each rank's data staged before its launch is then readable.
ME_DEVICE bool flags_barrier(const int64_t* __restrict__ bases, int world, int rank, uint32_t call,
                             uint64_t timeout_ns, int* status) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < world) {
    st_release_sys(reinterpret_cast<uint32_t*>(bases[threadIdx.x]) + rank, call);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(bases[rank]) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if ((int32_t)(ld_acquire_sys(mine) - call) >= 0) break;
      if ((it & 63u) == 63u && globaltimer_ns() - t0 > timeout_ns) {
        report(status, ME_ERR_TIMEOUT, threadIdx.x);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  return failed == 0;
}

// out[r * n16 ...] = rank r's stage (n16 16-byte units at stage_off + parity * half) for every r.
// poison: when a wait ran out (here, or in an earlier kernel of this rank: status[0] set), every
// byte of out becomes 0xFF (NaN in fp32 and bf16) instead of stale data, so a consumer that does
// not read the status cannot silently use another call's values.
__global__ void __launch_bounds__(256) p2p_gather_kernel(const int64_t* __restrict__ bases, int world, int rank,
                                                         uint32_t call, int64_t stage_off, int64_t half_bytes,
                                                         int64_t n16, uint4* __restrict__ out, uint64_t timeout_ns,
                                                         int* status, bool poison) {
  const bool ok = flags_barrier(bases, world, rank, call, timeout_ns, status);
  const int64_t total = n16 * world;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (!ok || (poison && *reinterpret_cast<volatile int*>(status) != 0)) {
    if (poison)
      for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride)
        out[i] = make_uint4(~0u, ~0u, ~0u, ~0u);
    return;
  }
  const int64_t off = stage_off + (int64_t)(call & 1u) * half_bytes;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int r = (int)(i / n16);
    out[i] = __ldcg(reinterpret_cast<const uint4*>(bases[r] + off) + (i - (int64_t)r * n16));
  }
}

// out[i] = sum over slots s of this rank's recv[parity][s][i] (fp32), after every peer signalled
// that its scattered stores into those slots are done. OutT float4 (fp32 out) or uint2 (four
// bf16, rounded to nearest even: the reduce half of a row-parallel linear's all-reduce).
ME_DEVICE void put4(float4* out, int64_t i, const float4& v) { out[i] = v; }
ME_DEVICE void put4(uint2* out, int64_t i, const float4& v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

template <typename OutT>
__global__ void __launch_bounds__(256) p2p_sum_slots_kernel(const int64_t* __restrict__ bases, int world, int rank,
                                                            uint32_t call, int64_t recv_off, int64_t slot_elems,
                                                            int64_t n4, OutT* __restrict__ out, uint64_t timeout_ns,
                                                            int* status) {
  if (!flags_barrier(bases, world, rank, call, timeout_ns, status)) return;
  const float* recv = reinterpret_cast<const float*>(bases[rank] + recv_off) +
                      (int64_t)(call & 1u) * world * slot_elems;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sl = 0; sl < world; ++sl) {  // fixed order: the sum is the same on every run
      const float4 v = __ldcg(reinterpret_cast<const float4*>(recv + (int64_t)sl * slot_elems) + i);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
    }
    put4(out, i, acc);
  }
}

// The standalone form of a layer all-gather range: one warp per 32 threads, grid-strided.
__global__ void __launch_bounds__(256) layer_gather_kernel(const GatherSeg* __restrict__ segs, int nsegs,
                                                           int64_t begin16, int64_t end16) {
  const int warps = blockDim.x / 32;
  gather_range(segs, nsegs, begin16, end16, blockIdx.x * warps + threadIdx.x / 32, gridDim.x * warps,
               threadIdx.x & 31);
}

}  // namespace

// Copy units [begin16, end16) of a segment table (int64 [nsegs, 4] on the device: src, dst,
// start16, n16) as a kernel of its own (the first layer of a pass, or what no GEMM carried).
void layer_gather(torch::Tensor segs, int64_t begin16, int64_t end16) {
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == torch::kInt64 && segs.dim() == 2 && segs.size(1) == 4 &&
                  segs.is_contiguous(), "layer_gather: segs must be a contiguous int64 [n, 4] CUDA tensor");
  if (end16 <= begin16 || segs.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(segs.device());
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, segs.get_device());
  layer_gather_kernel<<<sms * 2, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const GatherSeg*>(segs.data_ptr<int64_t>()), (int)segs.size(0), begin16, end16);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int grid_for(int64_t units, int dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int)std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, (int64_t)sms * 4));
}

// Gather every rank's staged bytes (n16 16-byte units each) into out [world * n16 * 16 bytes].
void p2p_gather(torch::Tensor bases, int64_t rank, int64_t call, int64_t stage_off, int64_t half_bytes, int64_t n16,
                torch::Tensor out, double timeout_s, torch::Tensor status, bool poison) {
  const int world = (int)bases.numel();
  TORCH_CHECK(world >= 1 && world <= MAX_RANKS && out.is_cuda() && out.nbytes() >= (size_t)(world * n16 * 16),
              "p2p_gather: bad arguments");
  TORCH_CHECK(stage_off % 16 == 0 && half_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "p2p_gather: 16-byte alignment");
  const at::cuda::CUDAGuard guard(out.device());
  p2p_gather_kernel<<<grid_for(world * n16, out.get_device()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bases.data_ptr<int64_t>(), world, (int)rank, (uint32_t)call, stage_off, half_bytes, n16,
      reinterpret_cast<uint4*>(out.data_ptr()), (uint64_t)(timeout_s * 1e9), status.data_ptr<int>(), poison);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[n] (fp32, or bf16 rounded from the fp32 sum) = sum of this rank's `world` receive slots
// of the parity of `call`.
void p2p_sum_slots(torch::Tensor bases, int64_t rank, int64_t call, int64_t recv_off, int64_t slot_elems,
                   torch::Tensor out, double timeout_s, torch::Tensor status) {
  const int world = (int)bases.numel();
  const bool f32 = out.scalar_type() == torch::kFloat32;
  TORCH_CHECK(world >= 1 && world <= MAX_RANKS && out.is_cuda() && (f32 || out.scalar_type() == torch::kBFloat16) &&
                  out.is_contiguous() && out.numel() % 4 == 0 && out.numel() <= slot_elems,
              "p2p_sum_slots: bad arguments");
  TORCH_CHECK(recv_off % 16 == 0 && slot_elems % 4 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "p2p_sum_slots: 16-byte alignment");
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t n4 = out.numel() / 4;
  const int grid = grid_for(n4, out.get_device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (f32)
    p2p_sum_slots_kernel<float4><<<grid, 256, 0, stream>>>(
        bases.data_ptr<int64_t>(), world, (int)rank, (uint32_t)call, recv_off, slot_elems, n4,
        reinterpret_cast<float4*>(out.data_ptr()), (uint64_t)(timeout_s * 1e9), status.data_ptr<int>());
  else
    p2p_sum_slots_kernel<uint2><<<grid, 256, 0, stream>>>(
        bases.data_ptr<int64_t>(), world, (int)rank, (uint32_t)call, recv_off, slot_elems, n4,
        reinterpret_cast<uint2*>(out.data_ptr()), (uint64_t)(timeout_s * 1e9), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[n] fp32 = (sum over ranks of their stage[call & 1][:n]) * scale. `bases` [world] int64:
// every rank's symmetric-buffer base address (this rank's own at index `rank`).
void p2p_allreduce_mean(torch::Tensor bases, int64_t rank, int64_t stage_off, int64_t n, int64_t call, double scale,
                        double timeout_s, torch::Tensor out, torch::Tensor status) {
  TORCH_CHECK(bases.is_cuda() && bases.scalar_type() == torch::kInt64, "bases: int64 CUDA tensor");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.numel() >= n,
              "out: contiguous fp32 CUDA tensor of n elements");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "status: int32 CUDA tensor");
  const int world = (int)bases.numel();
  TORCH_CHECK(world >= 1 && world <= MAX_RANKS && rank >= 0 && rank < world, "p2p_allreduce: 1..16 ranks");
  TORCH_CHECK(stage_off % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "p2p_allreduce: 16-byte aligned stage and output");
  const at::cuda::CUDAGuard guard(out.device());
  if (n == 0) return;
  int dev = out.get_device(), sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)sms * 2);
  p2p_allreduce_mean_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bases.data_ptr<int64_t>(), world, (int)rank, stage_off, n, (uint32_t)call, (float)scale,
      (uint64_t)(timeout_s * 1e9), out.data_ptr<float>(), status.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
