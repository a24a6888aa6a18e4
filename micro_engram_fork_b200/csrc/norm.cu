// Row-wise kernels of the Gemma-4-style decoder for sm_100a: RMSNorm (fp32 math, weight
// applied in fp32, cast back like Gemma4RMSNorm), the fused "post-norm + residual add (+
// layer scalar) + next pre-norm" of each sub-block, the q/k RMSNorm + partial RoPE and the
// v RMSNorm of attention (one warp per head row, cos/sin computed in-kernel from the
// per-layer inverse frequencies), and GeGLU. Forward and backward; the base is frozen, so
// no weight gradients are produced.
//
// Reference kernels these replace: micro_engram/train/vendor/gemma4_fused_rope.py:33-279
// (norm+RoPE), :446-582 (v-norm), and the Liger RMSNorm / GeGLU patches of
// micro_engram/train/model.py:71-98.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "act.cuh"
#include "common.cuh"

using namespace me;

namespace {

using bf16 = __nv_bfloat16;

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Loads / stores 8 bf16 at a time. VPT = 16-byte vectors per thread (d <= VPT*8*threads).
template <int VPT>
struct Row {
  float v[VPT][8];
  ME_DEVICE void load(const bf16* p, int nvec) {
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        BF16x8 x;
        x.u = reinterpret_cast<const uint4*>(p)[i];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[q][e] = bf2f(x.h[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[q][e] = 0.f;
      }
    }
  }
  ME_DEVICE float sumsq() const {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[q][e] * v[q][e];
    return s;
  }
};

ME_DEVICE void load_w(const float* w, int i, float out[8]) {
  const float4 a = reinterpret_cast<const float4*>(w)[2 * i];
  const float4 b = reinterpret_cast<const float4*>(w)[2 * i + 1];
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

ME_DEVICE void store8(bf16* p, int i, const float x[8]) {
  BF16x8 y;
#pragma unroll
  for (int e = 0; e < 8; ++e) y.h[e] = f2bf(x[e]);
  reinterpret_cast<uint4*>(p)[i] = y.u;
}

// y = bf16(x * rsqrt(mean(x^2) + eps) * w)
template <int VPT>
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, const float* __restrict__ w, int64_t N, int d,
                                   float eps, bf16* __restrict__ y, float* __restrict__ rstd) {
  __shared__ float scratch[64];
  const int nvec = d / 8;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    Row<VPT> r;
    r.load(x + n * d, nvec);
    const float rs = rsqrtf(block_sum(r.sumsq(), scratch) / d + eps);
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        float ww[8], o[8];
        if (w) load_w(w, i, ww);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = r.v[q][e] * rs * (w ? ww[e] : 1.f);
        store8(y + n * d, i, o);
      }
    }
    if (rstd && threadIdx.x == 0) rstd[n] = rs;
  }
}

// dx = rs * w * dy - rs^3/d * x * sum(x * w * dy)   (+ dx_add if given)
template <int VPT>
__global__ void rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                   const float* __restrict__ w, const float* __restrict__ rstd, int64_t N, int d,
                                   const bf16* __restrict__ dx_add, bf16* __restrict__ dx) {
  __shared__ float scratch[64];
  const int nvec = d / 8;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    Row<VPT> xr, gr;
    xr.load(x + n * d, nvec);
    gr.load(dy + n * d, nvec);
    const float rs = rstd[n];
    float dot = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        float ww[8];
        if (w) load_w(w, i, ww);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot += xr.v[q][e] * (w ? ww[e] : 1.f) * gr.v[q][e];
      }
    }
    const float c = rs * rs * rs * block_sum(dot, scratch) / d;
    Row<VPT> ar;
    if (dx_add) ar.load(dx_add + n * d, nvec);
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        float ww[8], o[8];
        if (w) load_w(w, i, ww);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          o[e] = rs * (w ? ww[e] : 1.f) * gr.v[q][e] - c * xr.v[q][e];
          if (dx_add) o[e] = bf2f(f2bf(o[e])) + ar.v[q][e];
        }
        store8(dx + n * d, i, o);
      }
    }
  }
}

// Sub-block epilogue of a Gemma-4 decoder layer:
//   x = bf16(bf16(r + bf16(rms(a) * w_post)) * ls)      (ls: the layer scalar, or 1)
//   h = bf16(rms(x) * w_next)                           (if w_next: the next pre-norm)
template <int VPT>
__global__ void __launch_bounds__(256, 4) post_norm_add_kernel(const bf16* __restrict__ r, const bf16* __restrict__ a,
                                     const float* __restrict__ w_post, const float* __restrict__ ls_ptr,
                                     const float* __restrict__ w_next, int64_t N, int d, float eps,
                                     bf16* __restrict__ x_out, bf16* __restrict__ h_out,
                                     float* __restrict__ rstd_a, float* __restrict__ rstd_x) {
  __shared__ float scratch[64];
  const int nvec = d / 8;
  const float ls = ls_ptr ? *ls_ptr : 1.f;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    Row<VPT> ar, rr;
    ar.load(a + n * d, nvec);
    rr.load(r + n * d, nvec);
    const float ra = rsqrtf(block_sum(ar.sumsq(), scratch) / d + eps);
    float sq = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        float ww[8];
        load_w(w_post, i, ww);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float nb = bf2f(f2bf(ar.v[q][e] * ra * ww[e]));
          float xv = bf2f(f2bf(rr.v[q][e] + nb));
          if (ls_ptr) xv = bf2f(f2bf(xv * ls));
          rr.v[q][e] = xv;  // reuse as x
          sq += xv * xv;
        }
        store8(x_out + n * d, i, rr.v[q]);
      }
    }
    if (w_next) {
      const float rx = rsqrtf(block_sum(sq, scratch) / d + eps);
#pragma unroll
      for (int q = 0; q < VPT; ++q) {
        const int i = threadIdx.x + q * blockDim.x;
        if (i < nvec) {
          float ww[8], o[8];
          load_w(w_next, i, ww);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = rr.v[q][e] * rx * ww[e];
          store8(h_out + n * d, i, o);
        }
      }
      if (threadIdx.x == 0) rstd_x[n] = rx;
    }
    if (threadIdx.x == 0) rstd_a[n] = ra;
  }
}

// Backward of post_norm_add. dxo: grad of x (may be null), dh: grad of h (may be null).
//   g  = dxo + rmsnorm_bwd(dh; x, w_next)        (grad of x)
//   gy = g * ls                                  (grad of r + n(a))
//   dr = gy ; da = rmsnorm_bwd(gy; a, w_post)
template <int VPT>
__global__ void __launch_bounds__(256, 3) post_norm_add_bwd_kernel(const bf16* __restrict__ dxo, const bf16* __restrict__ dh,
                                         const bf16* __restrict__ a, const bf16* __restrict__ x,
                                         const float* __restrict__ w_post, const float* __restrict__ ls_ptr,
                                         const float* __restrict__ w_next, const float* __restrict__ rstd_a,
                                         const float* __restrict__ rstd_x, int64_t N, int d,
                                         bf16* __restrict__ dr, bf16* __restrict__ da) {
  __shared__ float scratch[64];
  const int nvec = d / 8;
  const float ls = ls_ptr ? *ls_ptr : 1.f;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    Row<VPT> g;  // grad of x
    if (dxo) g.load(dxo + n * d, nvec);
    else {
#pragma unroll
      for (int q = 0; q < VPT; ++q)
#pragma unroll
        for (int e = 0; e < 8; ++e) g.v[q][e] = 0.f;
    }
    if (dh) {
      Row<VPT> xr, hr;
      xr.load(x + n * d, nvec);
      hr.load(dh + n * d, nvec);
      const float rx = rstd_x[n];
      float dot = 0.f;
#pragma unroll
      for (int q = 0; q < VPT; ++q) {
        const int i = threadIdx.x + q * blockDim.x;
        if (i < nvec) {
          float ww[8];
          load_w(w_next, i, ww);
#pragma unroll
          for (int e = 0; e < 8; ++e) dot += xr.v[q][e] * ww[e] * hr.v[q][e];
        }
      }
      const float c = rx * rx * rx * block_sum(dot, scratch) / d;
#pragma unroll
      for (int q = 0; q < VPT; ++q) {
        const int i = threadIdx.x + q * blockDim.x;
        if (i < nvec) {
          float ww[8];
          load_w(w_next, i, ww);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            g.v[q][e] = bf2f(f2bf(g.v[q][e] + bf2f(f2bf(rx * ww[e] * hr.v[q][e] - c * xr.v[q][e]))));
        }
      }
    }
    // gy = g * ls; dr = gy
    float dot = 0.f;
    Row<VPT> ar;
    ar.load(a + n * d, nvec);
    const float ra = rstd_a[n];
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        float ww[8];
        load_w(w_post, i, ww);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (ls_ptr) g.v[q][e] = bf2f(f2bf(g.v[q][e] * ls));
          dot += ar.v[q][e] * ww[e] * g.v[q][e];
        }
        store8(dr + n * d, i, g.v[q]);
      }
    }
    const float c = ra * ra * ra * block_sum(dot, scratch) / d;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int i = threadIdx.x + q * blockDim.x;
      if (i < nvec) {
        float ww[8], o[8];
        load_w(w_post, i, ww);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = ra * ww[e] * g.v[q][e] - c * ar.v[q][e];
        store8(da + n * d, i, o);
      }
    }
  }
}

// ---------------------------------------------------------------------------- q/k/v norm + RoPE
// qkv [N, (Hq + 2*Hk) * D] (the fused projection's output: q heads, then k heads, then v
// heads). A block takes QKV_TOK tokens at a time: it first fills a shared table of the
// tokens' rotary cos/sin (one sincos per (token, frequency), shared by every q/k head of the
// token), then one warp per (token, head) row. Each lane owns VH consecutive elements of each
// half of the head (RoPE pairs element j with j + D/2), loaded and stored as one vector.
// q/k: bf16(rms(x)*w) then the HF bf16 rotary formula bf16(bf16(x*cos) + bf16(rot(x)*sin))
// with cos/sin = bf16(cos/sin(pos * inv_freq)); v: bf16(rms(x)) with no weight.
constexpr int QKV_TOK = 4;

template <int VH>
ME_DEVICE void ld_bf(const bf16* __restrict__ p, float (&o)[VH]) {
  if constexpr (VH == 8) {
    BF16x8 t;
    t.u = *reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = bf2f(t.h[e]);
  } else if constexpr (VH == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    o[0] = __low2float(a), o[1] = __high2float(a), o[2] = __low2float(b), o[3] = __high2float(b);
  } else if constexpr (VH == 2) {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(p);
    o[0] = __low2float(a), o[1] = __high2float(a);
  } else {
    o[0] = bf2f(p[0]);
  }
}

template <int VH>
ME_DEVICE void st_bf(bf16* __restrict__ p, const float (&o)[VH]) {
  if constexpr (VH == 8) {
    BF16x8 t;
#pragma unroll
    for (int e = 0; e < 8; ++e) t.h[e] = f2bf(o[e]);
    *reinterpret_cast<uint4*>(p) = t.u;
  } else if constexpr (VH == 4) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]), b = __floats2bfloat162_rn(o[2], o[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  } else if constexpr (VH == 2) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(o[0], o[1]);
  } else {
    p[0] = f2bf(o[0]);
  }
}

// tab[t * HALF + e * 32 + lane] = (bf16(cos), bf16(sin)) of pos[n0 + t] * inv_freq[lane * VH + e]:
// the order in which a warp reads it, so each read of the table is 32 consecutive float2.
template <int VH>
ME_DEVICE void rope_table(float2* __restrict__ tab, const float* __restrict__ inv_freq,
                          const int64_t* __restrict__ pos, int64_t n0, int64_t N) {
  constexpr int HALF = VH * 32;
  for (int i = threadIdx.x; i < QKV_TOK * HALF; i += blockDim.x) {
    const int t = i / HALF, j = i % HALF;
    float sn = 0.f, cs = 1.f;
    if (n0 + t < N) sincosf((float)pos[n0 + t] * inv_freq[j], &sn, &cs);
    tab[t * HALF + (j % VH) * 32 + j / VH] = make_float2(bf2f(f2bf(cs)), bf2f(f2bf(sn)));
  }
}

template <int VH>
__global__ void __launch_bounds__(256) qkv_norm_rope_kernel(
    const bf16* __restrict__ qkv, const float* __restrict__ qw, const float* __restrict__ kw,
    const float* __restrict__ inv_freq, const int64_t* __restrict__ pos, int64_t N, int Hq, int Hk, int kv_shared,
    float eps, bf16* __restrict__ q, bf16* __restrict__ k, bf16* __restrict__ v, float* __restrict__ rstd) {
  constexpr int D = VH * 64, HALF = D / 2;
  __shared__ float2 tab[QKV_TOK * HALF];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int H = Hq + 2 * Hk;               // output heads (q, k, v)
  const int HI = kv_shared ? Hq + Hk : H;  // input heads per row (v = raw k when shared)
  const int base = lane * VH;
  const int64_t nblk = (N + QKV_TOK - 1) / QKV_TOK;
  for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const int64_t n0 = blk * QKV_TOK;
    __syncthreads();  // every warp is done with the previous tokens' table
    rope_table<VH>(tab, inv_freq, pos, n0, N);
    __syncthreads();
    const int rows = (int)(N - n0 < QKV_TOK ? N - n0 : QKV_TOK) * H;
    for (int r = warp; r < rows; r += nwarps) {
      const int t = r / H, hd = r % H;
      const int64_t n = n0 + t;
      const int src_hd = (kv_shared && hd >= Hq + Hk) ? hd - Hk : hd;
      const bf16* src = qkv + n * (int64_t)HI * D + (int64_t)src_hd * D;
      float lo[VH], hi[VH];
      ld_bf<VH>(src + base, lo);
      ld_bf<VH>(src + HALF + base, hi);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < VH; ++e) ss += lo[e] * lo[e] + hi[e] * hi[e];
      const float rs = rsqrtf(warp_sum(ss) / D + eps);
      if (lane == 0) rstd[n * H + hd] = rs;
      float ol[VH], oh[VH];
      bf16* dst;
      if (hd >= Hq + Hk) {  // v: plain rms norm
        dst = v + (n * Hk + (hd - Hq - Hk)) * (int64_t)D;
#pragma unroll
        for (int e = 0; e < VH; ++e) ol[e] = lo[e] * rs, oh[e] = hi[e] * rs;
      } else {
        const float* w = hd < Hq ? qw : kw;
        dst = hd < Hq ? q + (n * Hq + hd) * (int64_t)D : k + (n * Hk + (hd - Hq)) * (int64_t)D;
        const float2* cs = tab + t * HALF + lane;
#pragma unroll
        for (int e = 0; e < VH; ++e) {
          const int j = base + e;
          // the same bf16 roundings as below, two values per cvt.rn.bf16x2
          const float2 ab = __bfloat1622float2(__floats2bfloat162_rn(lo[e] * rs * w[j], hi[e] * rs * w[HALF + j]));
          const float a = ab.x, b = ab.y;
          const float2 c = cs[e * 32];
          // rotate_half: (-b, a); ol = bf16(a c) + bf16(-b s), oh = bf16(b c) + bf16(a s)
          const float2 t1 = __bfloat1622float2(__floats2bfloat162_rn(a * c.x, -b * c.y));
          const float2 t2 = __bfloat1622float2(__floats2bfloat162_rn(b * c.x, a * c.y));
          ol[e] = t1.x + t1.y;
          oh[e] = t2.x + t2.y;
        }
      }
      st_bf<VH>(dst + base, ol);
      st_bf<VH>(dst + HALF + base, oh);
    }
  }
}

// Backward: dq/dk/dv (attention layout) -> d_qkv (projection layout). Same token blocks and
// shared cos/sin table as the forward; one warp per input head; with kv_shared (v = raw k)
// the k head's warp adds the v path's gradient as well. cs == nullptr: the v path (no weight,
// no rotation).
template <int VH>
ME_DEVICE void norm_bwd_head(const float (&xl)[VH], const float (&xh)[VH], const bf16* __restrict__ gsrc,
                             const float* __restrict__ w, const float2* __restrict__ cs, float rs, int base,
                             float (&ol)[VH], float (&oh)[VH]) {
  constexpr int D = VH * 64, HALF = D / 2;
  float yl[VH], yh[VH], gl[VH], gh[VH], wl[VH], wh[VH];
  ld_bf<VH>(gsrc + base, yl);
  ld_bf<VH>(gsrc + HALF + base, yh);
#pragma unroll
  for (int e = 0; e < VH; ++e) {
    if (cs) {
      const float2 c = cs[e * 32];
      gl[e] = yl[e] * c.x + yh[e] * c.y;  // adjoint of (a, b) -> (a c - b s, b c + a s)
      gh[e] = yh[e] * c.x - yl[e] * c.y;
      wl[e] = w[base + e];
      wh[e] = w[HALF + base + e];
    } else {
      gl[e] = yl[e];
      gh[e] = yh[e];
      wl[e] = wh[e] = 1.f;
    }
  }
  float dot = 0.f;
#pragma unroll
  for (int e = 0; e < VH; ++e) dot += xl[e] * wl[e] * gl[e] + xh[e] * wh[e] * gh[e];
  const float c = rs * rs * rs * warp_sum(dot) / D;
#pragma unroll
  for (int e = 0; e < VH; ++e) {
    ol[e] += rs * wl[e] * gl[e] - c * xl[e];
    oh[e] += rs * wh[e] * gh[e] - c * xh[e];
  }
}

template <int VH>
__global__ void __launch_bounds__(256, 4) qkv_norm_rope_bwd_kernel(
    const bf16* __restrict__ dq, const bf16* __restrict__ dk, const bf16* __restrict__ dv,
    const bf16* __restrict__ qkv, const float* __restrict__ qw, const float* __restrict__ kw,
    const float* __restrict__ inv_freq, const int64_t* __restrict__ pos, const float* __restrict__ rstd, int64_t N,
    int Hq, int Hk, int kv_shared, bf16* __restrict__ dqkv) {
  constexpr int D = VH * 64, HALF = D / 2;
  __shared__ float2 tab[QKV_TOK * HALF];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int H = Hq + 2 * Hk;
  const int HI = kv_shared ? Hq + Hk : H;
  const int base = lane * VH;
  const int64_t nblk = (N + QKV_TOK - 1) / QKV_TOK;
  for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const int64_t n0 = blk * QKV_TOK;
    __syncthreads();
    rope_table<VH>(tab, inv_freq, pos, n0, N);
    __syncthreads();
    const int rows = (int)(N - n0 < QKV_TOK ? N - n0 : QKV_TOK) * HI;
    for (int r = warp; r < rows; r += nwarps) {
      const int t = r / HI, hd = r % HI;
      const int64_t n = n0 + t;
      const int64_t off = n * (int64_t)HI * D + (int64_t)hd * D;
      float xl[VH], xh[VH], ol[VH], oh[VH];
      ld_bf<VH>(qkv + off + base, xl);
      ld_bf<VH>(qkv + off + HALF + base, xh);
#pragma unroll
      for (int e = 0; e < VH; ++e) ol[e] = oh[e] = 0.f;
      const float2* cs = tab + t * HALF + lane;
      if (hd < Hq) {
        norm_bwd_head<VH>(xl, xh, dq + (n * Hq + hd) * (int64_t)D, qw, cs, rstd[n * H + hd], base, ol, oh);
      } else if (hd < Hq + Hk) {
        const int kh = hd - Hq;
        norm_bwd_head<VH>(xl, xh, dk + (n * Hk + kh) * (int64_t)D, kw, cs, rstd[n * H + hd], base, ol, oh);
        if (kv_shared)
          norm_bwd_head<VH>(xl, xh, dv + (n * Hk + kh) * (int64_t)D, nullptr, nullptr, rstd[n * H + Hq + Hk + kh],
                            base, ol, oh);
      } else {
        const int vh = hd - Hq - Hk;
        norm_bwd_head<VH>(xl, xh, dv + (n * Hk + vh) * (int64_t)D, nullptr, nullptr, rstd[n * H + hd], base, ol,
                          oh);
      }
      st_bf<VH>(dqkv + off + base, ol);
      st_bf<VH>(dqkv + off + HALF + base, oh);
    }
  }
}

// ---------------------------------------------------------------------------- GeGLU
// gu [N, 2F] = [gate | up]; m = bf16(bf16(gelu_tanh(gate)) * up).
// One block per row (grid-stride over rows), 16-byte vectors along the row: no index division.
__global__ void geglu_fwd_kernel(const bf16* __restrict__ gu, int64_t N, int F, bf16* __restrict__ m) {
  const int fv = F / 8;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    const uint4* gp = reinterpret_cast<const uint4*>(gu + n * 2 * F);
    const uint4* up = gp + fv;
    uint4* op = reinterpret_cast<uint4*>(m + n * F);
    for (int c = threadIdx.x; c < fv; c += blockDim.x) {
      BF16x8 g, u, o;
      g.u = gp[c];
      u.u = up[c];
#pragma unroll
      for (int e = 0; e < 8; ++e) o.h[e] = f2bf(bf2f(f2bf(gelu_tanh(bf2f(g.h[e])))) * bf2f(u.h[e]));
      op[c] = o.u;
    }
  }
}

__global__ void geglu_bwd_kernel(const bf16* __restrict__ dm, const bf16* __restrict__ gu, int64_t N, int F,
                                 bf16* __restrict__ dgu) {
  const int fv = F / 8;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    const uint4* gp = reinterpret_cast<const uint4*>(gu + n * 2 * F);
    const uint4* up = gp + fv;
    const uint4* dp = reinterpret_cast<const uint4*>(dm + n * F);
    uint4* ogp = reinterpret_cast<uint4*>(dgu + n * 2 * F);
    uint4* oup = ogp + fv;
    for (int c = threadIdx.x; c < fv; c += blockDim.x) {
      BF16x8 g, u, d, og, ou;
      g.u = gp[c];
      u.u = up[c];
      d.u = dp[c];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float x = bf2f(g.h[e]), upv = bf2f(u.h[e]), dd = bf2f(d.h[e]);
        og.h[e] = f2bf(dd * upv * gelu_tanh_grad(x));
        ou.h[e] = f2bf(dd * bf2f(f2bf(gelu_tanh(x))));
      }
      ogp[c] = og.u;
      oup[c] = ou.u;
    }
  }
}

template <typename F>
void dispatch_vpt(int d, int threads, F&& f) {
  const int nvec = d / 8;
  const int vpt = (nvec + threads - 1) / threads;
  TORCH_CHECK(vpt <= 8, "row width above 16384 is not supported");
  if (vpt <= 1) f(std::integral_constant<int, 1>{});
  else if (vpt <= 2) f(std::integral_constant<int, 2>{});
  else if (vpt <= 3) f(std::integral_constant<int, 3>{});
  else if (vpt <= 4) f(std::integral_constant<int, 4>{});
  else f(std::integral_constant<int, 8>{});
}

#define BFP(t) reinterpret_cast<bf16*>((t).data_ptr())
#define CBFP(t) reinterpret_cast<const bf16*>((t).data_ptr())

void check_row(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), name, " must be a contiguous CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bf16");
  TORCH_CHECK(t.size(-1) % 8 == 0, name, ": row width must be a multiple of 8");
}

}  // namespace

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> w, double eps) {
  check_row(x, "x");
  const at::cuda::CUDAGuard guard(x.device());
  const int d = (int)x.size(-1);
  const int64_t N = x.numel() / d;
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({N}, x.options().dtype(torch::kFloat32));
  if (N == 0) return {y, rstd};
  const int threads = d >= 2048 ? 256 : 128;
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 16);
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  dispatch_vpt(d, threads, [&](auto V) {
    rmsnorm_fwd_kernel<decltype(V)::value><<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
        CBFP(x), wp, N, d, (float)eps, BFP(y), rstd.data_ptr<float>());
  });
  return {y, rstd};
}

torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> w, torch::Tensor rstd,
                          c10::optional<torch::Tensor> dx_add) {
  check_row(x, "x");
  auto dyc = dy.contiguous();
  const at::cuda::CUDAGuard guard(x.device());
  const int d = (int)x.size(-1);
  const int64_t N = x.numel() / d;
  auto dx = torch::empty_like(x);
  if (N == 0) return dx;
  const int threads = d >= 2048 ? 256 : 128;
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 16);
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  const bf16* ap = dx_add.has_value() ? CBFP(*dx_add) : nullptr;
  dispatch_vpt(d, threads, [&](auto V) {
    rmsnorm_bwd_kernel<decltype(V)::value><<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
        CBFP(dyc), CBFP(x), wp, rstd.data_ptr<float>(), N, d, ap, BFP(dx));
  });
  return dx;
}

// returns x, h (or empty), rstd_a, rstd_x (or empty)
std::vector<torch::Tensor> post_norm_add(torch::Tensor r, torch::Tensor a, torch::Tensor w_post,
                                         c10::optional<torch::Tensor> ls, c10::optional<torch::Tensor> w_next,
                                         double eps) {
  check_row(r, "residual");
  check_row(a, "branch");
  const at::cuda::CUDAGuard guard(r.device());
  const int d = (int)r.size(-1);
  const int64_t N = r.numel() / d;
  auto x = torch::empty_like(r);
  auto ra = torch::empty({N}, r.options().dtype(torch::kFloat32));
  torch::Tensor h, rx;
  if (w_next.has_value()) {
    h = torch::empty_like(r);
    rx = torch::empty({N}, r.options().dtype(torch::kFloat32));
  }
  if (N == 0) return {x, h, ra, rx};
  const int threads = d >= 2048 ? 256 : 128;
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 16);
  dispatch_vpt(d, threads, [&](auto V) {
    post_norm_add_kernel<decltype(V)::value><<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
        CBFP(r), CBFP(a), w_post.data_ptr<float>(), ls.has_value() ? ls->data_ptr<float>() : nullptr,
        w_next.has_value() ? w_next->data_ptr<float>() : nullptr, N, d, (float)eps, BFP(x),
        w_next.has_value() ? BFP(h) : nullptr, ra.data_ptr<float>(), w_next.has_value() ? rx.data_ptr<float>() : nullptr);
  });
  return {x, h, ra, rx};
}

// returns dr, da
std::vector<torch::Tensor> post_norm_add_bwd(c10::optional<torch::Tensor> dxo, c10::optional<torch::Tensor> dh,
                                             torch::Tensor a, torch::Tensor x, torch::Tensor w_post,
                                             c10::optional<torch::Tensor> ls, c10::optional<torch::Tensor> w_next,
                                             torch::Tensor rstd_a, c10::optional<torch::Tensor> rstd_x) {
  check_row(a, "branch");
  const at::cuda::CUDAGuard guard(a.device());
  const int d = (int)a.size(-1);
  const int64_t N = a.numel() / d;
  auto dr = torch::empty_like(a), da = torch::empty_like(a);
  if (N == 0) return {dr, da};
  torch::Tensor dxoc, dhc;
  if (dxo.has_value()) dxoc = dxo->contiguous();
  if (dh.has_value()) dhc = dh->contiguous();
  const int threads = d >= 2048 ? 256 : 128;
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 16);
  dispatch_vpt(d, threads, [&](auto V) {
    post_norm_add_bwd_kernel<decltype(V)::value><<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
        dxo.has_value() ? CBFP(dxoc) : nullptr, dh.has_value() ? CBFP(dhc) : nullptr, CBFP(a), CBFP(x),
        w_post.data_ptr<float>(), ls.has_value() ? ls->data_ptr<float>() : nullptr,
        w_next.has_value() ? w_next->data_ptr<float>() : nullptr, rstd_a.data_ptr<float>(),
        rstd_x.has_value() ? rstd_x->data_ptr<float>() : nullptr, N, d, BFP(dr), BFP(da));
  });
  return {dr, da};
}

// returns q [N,Hq,D], k [N,Hk,D], v [N,Hk,D], rstd [N, Hq+2Hk]
std::vector<torch::Tensor> qkv_norm_rope(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw,
                                         torch::Tensor inv_freq, torch::Tensor pos, int64_t Hq, int64_t Hk,
                                         int64_t D, bool kv_shared, double eps) {
  check_row(qkv, "qkv");
  const at::cuda::CUDAGuard guard(qkv.device());
  const int64_t N = qkv.size(0);
  TORCH_CHECK(qkv.size(1) == (Hq + (kv_shared ? 1 : 2) * Hk) * D, "qkv width");
  auto opts = qkv.options();
  auto q = torch::empty({N, Hq, D}, opts), k = torch::empty({N, Hk, D}, opts), v = torch::empty({N, Hk, D}, opts);
  auto rstd = torch::empty({N, Hq + 2 * Hk}, opts.dtype(torch::kFloat32));
  if (N == 0) return {q, k, v, rstd};
  auto pos64 = pos.to(torch::kLong).contiguous();
  if (reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16) qkv = qkv.clone();  // the kernel's vector loads
  const int threads = 256;
  const int grid = (int)std::min<int64_t>((N + QKV_TOK - 1) / QKV_TOK, (int64_t)sm_count() * 8);
  auto stream = at::cuda::getCurrentCUDAStream();
#define ME_QKV(VH)                                                                                            \
  qkv_norm_rope_kernel<VH><<<grid, threads, 0, stream>>>(CBFP(qkv), qw.data_ptr<float>(), kw.data_ptr<float>(), \
                                                         inv_freq.data_ptr<float>(), pos64.data_ptr<int64_t>(), N, \
                                                         (int)Hq, (int)Hk, kv_shared ? 1 : 0, (float)eps, BFP(q),  \
                                                         BFP(k), BFP(v), rstd.data_ptr<float>())
  if (D == 64) ME_QKV(1);
  else if (D == 128) ME_QKV(2);
  else if (D == 256) ME_QKV(4);
  else if (D == 512) ME_QKV(8);
  else TORCH_CHECK(false, "head_dim must be 64, 128, 256 or 512");
#undef ME_QKV
  return {q, k, v, rstd};
}

torch::Tensor qkv_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                                torch::Tensor qw, torch::Tensor kw, torch::Tensor inv_freq, torch::Tensor pos,
                                torch::Tensor rstd, int64_t Hq, int64_t Hk, int64_t D, bool kv_shared) {
  const at::cuda::CUDAGuard guard(qkv.device());
  const int64_t N = qkv.size(0);
  auto dqkv = torch::empty(qkv.sizes(), qkv.options());
  if (N == 0) return dqkv;
  auto aligned = [](torch::Tensor t) {  // the kernel's vector loads want 16-byte aligned rows
    t = t.contiguous();
    return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 ? t.clone() : t;
  };
  auto dqc = aligned(dq), dkc = aligned(dk), dvc = aligned(dv);
  qkv = aligned(qkv);
  auto pos64 = pos.to(torch::kLong).contiguous();
  const int threads = 256;
  const int grid = (int)std::min<int64_t>((N + QKV_TOK - 1) / QKV_TOK, (int64_t)sm_count() * 8);
  auto stream = at::cuda::getCurrentCUDAStream();
#define ME_QKVB(VH)                                                                                           \
  qkv_norm_rope_bwd_kernel<VH><<<grid, threads, 0, stream>>>(                                                  \
      CBFP(dqc), CBFP(dkc), CBFP(dvc), CBFP(qkv), qw.data_ptr<float>(), kw.data_ptr<float>(),                  \
      inv_freq.data_ptr<float>(), pos64.data_ptr<int64_t>(), rstd.data_ptr<float>(), N, (int)Hq, (int)Hk,          \
      kv_shared ? 1 : 0, BFP(dqkv))
  if (D == 64) ME_QKVB(1);
  else if (D == 128) ME_QKVB(2);
  else if (D == 256) ME_QKVB(4);
  else if (D == 512) ME_QKVB(8);
  else TORCH_CHECK(false, "head_dim must be 64, 128, 256 or 512");
#undef ME_QKVB
  return dqkv;
}

torch::Tensor geglu_fwd(torch::Tensor gu) {
  check_row(gu, "gate_up");
  const at::cuda::CUDAGuard guard(gu.device());
  const int F = (int)(gu.size(-1) / 2);
  TORCH_CHECK(F % 8 == 0, "ffn width must be a multiple of 8");
  const int64_t N = gu.numel() / gu.size(-1);
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto m = torch::empty(sizes, gu.options());
  if (N == 0) return m;
  const int threads = 256;
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 8);
  geglu_fwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(CBFP(gu), N, F, BFP(m));
  return m;
}

torch::Tensor geglu_bwd(torch::Tensor dm, torch::Tensor gu) {
  check_row(gu, "gate_up");
  auto dmc = dm.contiguous();
  const at::cuda::CUDAGuard guard(gu.device());
  const int F = (int)(gu.size(-1) / 2);
  const int64_t N = gu.numel() / gu.size(-1);
  auto dgu = torch::empty_like(gu);
  if (N == 0) return dgu;
  const int threads = 256;
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 8);
  geglu_bwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(CBFP(dmc), CBFP(gu), N, F, BFP(dgu));
  return dgu;
}
