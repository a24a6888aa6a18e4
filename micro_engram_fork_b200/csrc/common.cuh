// Shared device helpers for the sm_100a kernels of micro_engram_fork_b200.
//
// Everything here is written for Blackwell (sm_100a) only: 32-wide warps, 16-byte vector
// memory ops, fp32 atomics on float4 (sm_90+), and the device status word that every
// bounded wait reports into instead of trapping.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define ME_HOST_DEVICE __host__ __device__ __forceinline__
#define ME_DEVICE __device__ __forceinline__

namespace me {

// ---------------------------------------------------------------- device status word
// Kernels never trap or assert. A bounded wait that runs out, or an index that a
// bounds-checked build finds out of range, writes one of these codes (plus a detail
// word) into a status buffer the host reads after the step and raises on.
enum StatusCode : int {
  ME_OK = 0,
  ME_ERR_TIMEOUT = 1,      // a spin-wait on a peer flag / mbarrier ran past its limit
  ME_ERR_BOUNDS = 2,       // an index outside its table / buffer (bounds-checked builds)
  ME_ERR_CAPACITY = 3,     // a fixed-capacity buffer (touched-row list, hash set) overflowed
  ME_ERR_ALIGN = 4,        // a pointer or size broke a vector / TMA alignment rule
};

ME_DEVICE void report(int* status, int code, int detail) {
  if (status == nullptr) return;
  // first error wins; later ones are dropped
  if (atomicCAS(status, 0, code) == 0) status[1] = detail;
}

// ---------------------------------------------------------------- conversions
ME_DEVICE float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
ME_DEVICE __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

template <typename T>
ME_DEVICE float to_f(T x);
template <>
ME_DEVICE float to_f<float>(float x) { return x; }
template <>
ME_DEVICE float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
ME_DEVICE T from_f(float x);
template <>
ME_DEVICE float from_f<float>(float x) { return x; }
template <>
ME_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// 8 bf16 <-> one 16-byte vector
union BF16x8 {
  uint4 u;
  __nv_bfloat16 h[8];
  __nv_bfloat162 h2[4];
};

union F32x4 {
  float4 v;
  float f[4];
};

// ---------------------------------------------------------------- reductions
ME_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

ME_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over the whole block; `scratch` holds >= 32 floats of shared memory. All threads get
// the result. Blocks are multiples of 32 threads.
ME_DEVICE float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  float r = lane < nw ? scratch[lane] : 0.f;
  r = warp_sum(r);
  return r;
}

// Two sums at once (one barrier pair instead of two).
ME_DEVICE float2 block_sum2(float a, float b, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  __syncthreads();
  if (lane == 0) {
    scratch[wid] = a;
    scratch[32 + wid] = b;
  }
  __syncthreads();
  float ra = lane < nw ? scratch[lane] : 0.f;
  float rb = lane < nw ? scratch[32 + lane] : 0.f;
  return make_float2(warp_sum(ra), warp_sum(rb));
}

// ---------------------------------------------------------------- Philox4x32-10
// Counter-based RNG of Salmon, Moraes, Dror and Shaw, "Parallel Random Numbers: As Easy as
// 1, 2, 3" (SC'11): four 32-bit words of counter, two of key, ten rounds of the Philox
// S-box with the multipliers and Weyl key increments given in the paper.
struct Philox4 {
  uint32_t c[4];
};

ME_DEVICE void mulhilo32(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const uint64_t p = (uint64_t)a * (uint64_t)b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}

ME_DEVICE Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;   // round multipliers (paper, Table 2)
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;   // key schedule (golden ratio, sqrt(3)-1)
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, c0, hi0, lo0);
    mulhilo32(M1, c2, hi1, lo1);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
    c0 = n0;
    c1 = n1;
    c2 = n2;
    c3 = n3;
    k0 += W0;
    k1 += W1;
  }
  Philox4 out;
  out.c[0] = c0;
  out.c[1] = c1;
  out.c[2] = c2;
  out.c[3] = c3;
  return out;
}

// fp32 -> bf16 with stochastic rounding: add 16 random bits below the kept mantissa, cut.
// The sign is its own bit, so this rounds the magnitude and stays unbiased for both signs.
// Non-finite values keep their value (rounded to nearest, which keeps inf/nan).
ME_DEVICE __nv_bfloat16 sr_bf16(float x, uint32_t rnd16) {
  if (!isfinite(x)) return __float2bfloat16_rn(x);
  uint32_t bits = __float_as_uint(x);
  bits = (bits + (rnd16 & 0xFFFFu)) & 0xFFFF0000u;
  return __ushort_as_bfloat16((unsigned short)(bits >> 16));
}

// ---------------------------------------------------------------- globaltimer
ME_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- flags between GPUs
// A flag word in (possibly peer) global memory, published with release semantics at system
// scope and read with acquire semantics: everything written before the release store is
// visible to a reader that saw the value.
ME_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
ME_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spin (bounded) until the flag reaches `want` (wrap-around compare). False on timeout.
ME_DEVICE bool wait_flag_geq(const uint32_t* flag, uint32_t want, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if ((int32_t)(ld_acquire_sys(flag) - want) >= 0) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

}  // namespace me
