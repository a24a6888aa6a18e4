// Packed-varlen causal attention (optional sliding window, GQA) for sm_100a.
//
// Token-major layout q [T, Hq, D], k/v [T, Hk, D]; the document of token t starts at
// doc_start[t] and ends at doc_end[t]; t sees s iff doc_start[t] <= s <= t and (no window or
// s > t - window). Scale is applied to q.k before the softmax.
//
// This is the first-generation kernel set built on warp-level mma.sync (m16n8k16 bf16 ->
// fp32) with ldmatrix from XOR-swizzled shared memory and cp.async tile loads:
//   attn_fwd_kernel      one CTA = 64 queries of one head; online softmax; writes O and LSE.
//                        D=512 splits the O columns over gridDim.z (S recomputed per half).
//   attn_bwd_pre_kernel  delta = rowsum(dO * O)
//   attn_bwd_dkdv_kernel one CTA = BN keys of one kv head, looping over the query heads of
//                        its GQA group and the query tiles that can see the keys; P^T and
//                        dS^T go through shared memory; dK, dV accumulate in registers
//                        (no atomics).
//   attn_bwd_dq_kernel   one CTA = 64 queries of one head; dQ in registers (no atomics).
// Replaces the reference's Triton flash-d512 (micro_engram/train/vendor/flash_attn_d512.py)
// and the FA2/SDPA library calls; mask bounds come from doc_start/doc_end per tile, never an
// S x S mask.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

using namespace me;

namespace {
using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ PTX helpers
ME_DEVICE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

ME_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0: zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
ME_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
ME_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

ME_DEVICE void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
ME_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
ME_DEVICE void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
ME_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------------------ swizzled tiles
// A tile of ROWS x COLS bf16 in shared memory, 16-byte chunks XOR-swizzled by row so that
// the 8 row addresses of an ldmatrix hit different banks.
template <int COLS>
struct Tile {
  static constexpr int CHUNKS = COLS / 8;
  static constexpr int MASK = CHUNKS >= 8 ? 7 : CHUNKS - 1;
  ME_DEVICE static uint32_t off(int row, int chunk) {
    return (uint32_t)(row * COLS * 2 + ((chunk ^ (row & MASK)) << 4));
  }
};

// Async load of rows [row0, row0+ROWS) x cols [col0, col0+COLS) of a row-major global
// matrix with `ld` elements per row; rows >= nrows are zero-filled.
template <int ROWS, int COLS, int NT>
ME_DEVICE void load_tile(uint32_t sbase, const bf16* g, int64_t ld, int row0, int nrows, int col0) {
  constexpr int CH = COLS / 8;
  for (int i = threadIdx.x; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const int gr = row0 + r;
    const bool ok = gr < nrows && gr >= 0;
    const bf16* src = g + (int64_t)(ok ? gr : 0) * ld + col0 + c * 8;
    cp_async16(sbase + Tile<COLS>::off(r, c), src, ok);
  }
}

// One warp computes acc[MT][NT] (m16n8 tiles) += A[m0.., k] * B[k, n0..] over k in [0, K).
// A_T: A stored [k][m] (else [m][k]); B_T: B stored [k][n] (else [n][k]).
template <int MT, int NT, bool A_T, bool B_T, int A_COLS, int B_COLS>
ME_DEVICE void warp_gemm(float (&acc)[MT][NT][4], uint32_t sA, int m0, uint32_t sB, int n0, int K) {
  static_assert(NT % 2 == 0, "n tiles come in pairs");
  const int lane = threadIdx.x & 31;
  const int mi = lane >> 3;
#pragma unroll 2
  for (int k = 0; k < K; k += 16) {
    uint32_t a[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      const int m = m0 + i * 16;
      if (!A_T) {
        const int row = m + (lane & 15), ch = (k >> 3) + (lane >> 4);
        ldsm_x4(sA + Tile<A_COLS>::off(row, ch), a[i]);
      } else {
        const int row = k + (lane & 7) + ((mi >> 1) << 3), ch = (m >> 3) + (mi & 1);
        ldsm_x4_t(sA + Tile<A_COLS>::off(row, ch), a[i]);
      }
    }
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      const int n = n0 + j * 8;
      uint32_t b[4];
      if (!B_T) {
        const int row = n + (lane & 7) + ((mi >> 1) << 3), ch = (k >> 3) + (mi & 1);
        ldsm_x4(sB + Tile<B_COLS>::off(row, ch), b);
      } else {
        const int row = k + (lane & 7) + ((mi & 1) << 3), ch = (n >> 3) + (mi >> 1);
        ldsm_x4_t(sB + Tile<B_COLS>::off(row, ch), b);
      }
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        mma16816(acc[i][j], a[i], b[0], b[1]);
        mma16816(acc[i][j + 1], a[i], b[2], b[3]);
      }
    }
  }
}

template <int MT, int NT>
ME_DEVICE void zero(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
}

ME_DEVICE bool allowed(int t, int s, int ds_t, int window, int T) {
  return s <= t && s >= ds_t && (window <= 0 || s > t - window) && t < T && s < T;
}

// ------------------------------------------------------------------ forward
// grid (ceil(T/64), Hq, D/DV), 128 threads (4 warps x 16 query rows).
template <int D, int DV, int STAGES>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                       const bf16* __restrict__ v, const int* __restrict__ doc_start,
                                                       int T, int Hq, int Hk, int window, float scale,
                                                       bf16* __restrict__ o, float* __restrict__ lse) {
  constexpr int BM = 64, BN = 64, NT = 128;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BM * D * 2;
  const uint32_t sV0 = sK0 + STAGES * BN * D * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, hk = h / (Hq / Hk), dv0 = blockIdx.z * DV;
  const int64_t ldq = (int64_t)Hq * D, ldk = (int64_t)Hk * D;
  const bf16* qh = q + (int64_t)h * D;
  const bf16* kh = k + (int64_t)hk * D;
  const bf16* vh = v + (int64_t)hk * D;

  load_tile<BM, D, NT>(sQ, qh, ldq, q0, T, 0);
  const int qlast = min(q0 + BM - 1, T - 1);
  int kstart = doc_start[q0];
  if (window > 0) kstart = max(kstart, q0 - window + 1);
  const int kb_first = (kstart / BN) * BN;
  const int n_kb = (qlast - kb_first) / BN + 1;
  load_tile<BN, D, NT>(sK0, kh, ldk, kb_first, T, 0);
  load_tile<BN, DV, NT>(sV0, vh, ldk, kb_first, T, dv0);
  cp_async_commit();

  // the two rows this thread owns in the warp's 16-row slab
  const int r0 = q0 + warp * 16 + (lane >> 2), r1 = r0 + 8;
  const int ds0 = r0 < T ? doc_start[r0] : 0, ds1 = r1 < T ? doc_start[r1] : 0;
  const int ds_last = doc_start[qlast];
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc_o[1][DV / 8][4];
  zero(acc_o);

  for (int it = 0; it < n_kb; ++it) {
    const int kb = kb_first + it * BN;
    const int st = STAGES == 2 ? (it & 1) : 0;
    if (STAGES == 2 && it + 1 < n_kb) {  // prefetch the next tile into the other stage
      const int ns = (it + 1) & 1;
      load_tile<BN, D, NT>(sK0 + ns * BN * D * 2, kh, ldk, kb + BN, T, 0);
      load_tile<BN, DV, NT>(sV0 + ns * BN * DV * 2, vh, ldk, kb + BN, T, dv0);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + st * BN * D * 2, sV = sV0 + st * BN * DV * 2;
    float s[1][BN / 8][4];
    zero(s);
    warp_gemm<1, BN / 8, false, false, D, D>(s, sQ, warp * 16, sK, 0, D);
    // mask only where a tile straddles a bound
    const bool full = (kb + BN - 1 <= q0) && (kb >= ds_last) && (window <= 0 || kb > qlast - window) &&
                      (kb + BN <= T) && (q0 + BM <= T);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = e < 2 ? r0 : r1;
        const int sc = kb + j * 8 + (lane & 3) * 2 + (e & 1);
        float x = s[0][j][e] * scale;
        if (!full && !allowed(t, sc, e < 2 ? ds0 : ds1, window, T)) x = -INFINITY;
        s[0][j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m_run[r], mx[r]);
      alpha[r] = (m_run[r] == -INFINITY) ? 0.f : expf(m_run[r] - mn);
      m_run[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[BN / 16][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float p = (m_run[r] == -INFINITY) ? 0.f : expf(s[0][j][e] - m_run[r]);
        s[0][j][e] = p;
        rs[r] += p;
      }
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      pa[kk][0] = pack_bf16(s[0][2 * kk][0], s[0][2 * kk][1]);
      pa[kk][1] = pack_bf16(s[0][2 * kk][2], s[0][2 * kk][3]);
      pa[kk][2] = pack_bf16(s[0][2 * kk + 1][0], s[0][2 * kk + 1][1]);
      pa[kk][3] = pack_bf16(s[0][2 * kk + 1][2], s[0][2 * kk + 1][3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int j = 0; j < DV / 8; ++j) {
      acc_o[0][j][0] *= alpha[0];
      acc_o[0][j][1] *= alpha[0];
      acc_o[0][j][2] *= alpha[1];
      acc_o[0][j][3] *= alpha[1];
    }
    // O += P V  (V stored [key][dv]: B transposed)
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int j = 0; j < DV / 8; j += 2) {
        uint32_t b[4];
        const int mi = lane >> 3;
        const int row = kk * 16 + (lane & 7) + ((mi & 1) << 3), ch = (j * 8 >> 3) + (mi >> 1);
        ldsm_x4_t(sV + Tile<DV>::off(row, ch), b);
        mma16816(acc_o[0][j], pa[kk], b[0], b[1]);
        mma16816(acc_o[0][j + 1], pa[kk], b[2], b[3]);
      }
    }
    __syncthreads();
    if (STAGES == 1 && it + 1 < n_kb) {
      load_tile<BN, D, NT>(sK0, kh, ldk, kb + BN, T, 0);
      load_tile<BN, DV, NT>(sV0, vh, ldk, kb + BN, T, dv0);
      cp_async_commit();
    }
  }
  // epilogue
  const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f, inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
#pragma unroll
  for (int j = 0; j < DV / 8; ++j) {
    const int c = dv0 + j * 8 + (lane & 3) * 2;
    if (r0 < T)
      *reinterpret_cast<__nv_bfloat162*>(o + (int64_t)r0 * ldq + (int64_t)h * D + c) =
          __floats2bfloat162_rn(acc_o[0][j][0] * inv0, acc_o[0][j][1] * inv0);
    if (r1 < T)
      *reinterpret_cast<__nv_bfloat162*>(o + (int64_t)r1 * ldq + (int64_t)h * D + c) =
          __floats2bfloat162_rn(acc_o[0][j][2] * inv1, acc_o[0][j][3] * inv1);
  }
  if (blockIdx.z == 0 && (lane & 3) == 0) {
    if (r0 < T) lse[(int64_t)h * T + r0] = m_run[0] + logf(l_run[0]);
    if (r1 < T) lse[(int64_t)h * T + r1] = m_run[1] + logf(l_run[1]);
  }
}

// ------------------------------------------------------------------ backward: delta
__global__ void attn_bwd_pre_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout, int T, int Hq, int D,
                                    float* __restrict__ delta) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)T * Hq;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < rows;
       w += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int64_t t = w / Hq;
    const int h = (int)(w % Hq);
    const bf16* orow = o + w * D;
    const bf16* grow = dout + w * D;
    float s = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      BF16x8 a, b;
      a.u = *reinterpret_cast<const uint4*>(orow + c);
      b.u = *reinterpret_cast<const uint4*>(grow + c);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += bf2f(a.h[e]) * bf2f(b.h[e]);
    }
    s = warp_sum(s);
    if (lane == 0) delta[(int64_t)h * T + t] = s;
  }
}

// ------------------------------------------------------------------ backward: dK, dV
// grid (ceil(T/BN), Hk), 256 threads. Accumulates over the GQA group's query heads.
template <int D, int BN>
__global__ void __launch_bounds__(256) attn_bwd_dkdv_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, const bf16* __restrict__ dout,
    const float* __restrict__ lse, const float* __restrict__ delta, const int* __restrict__ doc_start,
    const int* __restrict__ doc_end, int T, int Hq, int Hk, int window, float scale, bf16* __restrict__ dk,
    bf16* __restrict__ dv) {
  constexpr int BM = 64, NTH = 256;
  // output tiling [BN x D] over 8 warps: WM x WN warps
  constexpr int WM = BN / 16 >= 2 ? 2 : 1;       // BN=64: 2 warp rows of 32; BN=32: 2 of 16
  constexpr int OM = BN / WM;                    // rows per warp
  constexpr int WN = 8 / WM;
  constexpr int ON = D / WN;                     // cols per warp
  constexpr int OMT = OM / 16, ONT = ON / 8;
  // S^T tiling [BN x BM] over 8 warps
  constexpr int SWM = BN / 16, SWN = 8 / SWM, SN = BM / SWN, SNT = SN / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BN * D * 2;
  const uint32_t sQ = sV + BN * D * 2;
  const uint32_t sO = sQ + BM * D * 2;        // dO
  const uint32_t sP = sO + BM * D * 2;        // P^T [BN][BM]
  const uint32_t sS = sP + BN * BM * 2;       // dS^T [BN][BM]
  float* sL = reinterpret_cast<float*>(smem + (size_t)(2 * BN * D + 2 * BM * D + 2 * BN * BM) * 2);
  float* sDl = sL + BM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb0 = blockIdx.x * BN, hk = blockIdx.y;
  const int rep = Hq / Hk;
  const int64_t ldq = (int64_t)Hq * D, ldk = (int64_t)Hk * D;
  const int klast = min(kb0 + BN - 1, T - 1);
  int qend = doc_end[klast];
  if (window > 0) qend = min(qend, klast + window - 1);
  qend = min(qend, T - 1);
  const int qb_first = (kb0 / BM) * BM;

  load_tile<BN, D, NTH>(sK, k + (int64_t)hk * D, ldk, kb0, T, 0);
  load_tile<BN, D, NTH>(sV, v + (int64_t)hk * D, ldk, kb0, T, 0);
  cp_async_commit();

  float acc_dk[OMT][ONT][4], acc_dv[OMT][ONT][4];
  zero(acc_dk);
  zero(acc_dv);
  const int wm = warp / WN, wn = warp % WN;
  const int swm = warp / SWN, swn = warp % SWN;

  for (int hh = 0; hh < rep; ++hh) {
    const int h = hk * rep + hh;
    for (int qb = qb_first; qb <= qend; qb += BM) {
      load_tile<BM, D, NTH>(sQ, q + (int64_t)h * D, ldq, qb, T, 0);
      load_tile<BM, D, NTH>(sO, dout + (int64_t)h * D, ldq, qb, T, 0);
      cp_async_commit();
      for (int i = threadIdx.x; i < BM; i += NTH) {
        const int t = qb + i;
        sL[i] = t < T ? lse[(int64_t)h * T + t] : 0.f;
        sDl[i] = t < T ? delta[(int64_t)h * T + t] : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();
      // S^T = K Q^T and dP^T = V dO^T for this warp's [16 x SN] slab
      float st[1][SNT][4], dpt[1][SNT][4];
      zero(st);
      zero(dpt);
      warp_gemm<1, SNT, false, false, D, D>(st, sK, swm * 16, sQ, swn * SN, D);
      warp_gemm<1, SNT, false, false, D, D>(dpt, sV, swm * 16, sO, swn * SN, D);
#pragma unroll
      for (int j = 0; j < SNT; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int krow = swm * 16 + (lane >> 2) + ((e >> 1) << 3);     // key index in tile
          const int qcol = swn * SN + j * 8 + (lane & 3) * 2 + (e & 1);  // query index in tile
          const int s_idx = kb0 + krow, t = qb + qcol;
          const bool ok = t < T && allowed(t, s_idx, doc_start[t], window, T);
          const float p = ok ? expf(st[0][j][e] * scale - sL[qcol]) : 0.f;
          st[0][j][e] = p;
          dpt[0][j][e] = p * (dpt[0][j][e] - sDl[qcol]);
        }
        // store P^T and dS^T (bf16) rows krow, cols qcol
        const int kr = swm * 16 + (lane >> 2);
        const int qc = swn * SN + j * 8 + (lane & 3) * 2;
        const uint32_t o0 = Tile<BM>::off(kr, qc >> 3) + (qc & 7) * 2;
        const uint32_t o1 = Tile<BM>::off(kr + 8, qc >> 3) + (qc & 7) * 2;
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(sP + o0), "r"(pack_bf16(st[0][j][0], st[0][j][1])));
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(sP + o1), "r"(pack_bf16(st[0][j][2], st[0][j][3])));
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(sS + o0), "r"(pack_bf16(dpt[0][j][0], dpt[0][j][1])));
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(sS + o1), "r"(pack_bf16(dpt[0][j][2], dpt[0][j][3])));
      }
      __syncthreads();
      // dV += P^T dO ; dK += dS^T Q   (A = [keys][q] as stored; B = [q][d] stored -> transposed)
      warp_gemm<OMT, ONT, false, true, BM, D>(acc_dv, sP, wm * OM, sO, wn * ON, BM);
      warp_gemm<OMT, ONT, false, true, BM, D>(acc_dk, sS, wm * OM, sQ, wn * ON, BM);
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < OMT; ++i) {
#pragma unroll
    for (int j = 0; j < ONT; ++j) {
      const int r = kb0 + wm * OM + i * 16 + (lane >> 2);
      const int c = wn * ON + j * 8 + (lane & 3) * 2;
      if (r < T) {
        *reinterpret_cast<__nv_bfloat162*>(dk + (int64_t)r * ldk + (int64_t)hk * D + c) =
            __floats2bfloat162_rn(acc_dk[i][j][0] * scale, acc_dk[i][j][1] * scale);
        *reinterpret_cast<__nv_bfloat162*>(dv + (int64_t)r * ldk + (int64_t)hk * D + c) =
            __floats2bfloat162_rn(acc_dv[i][j][0], acc_dv[i][j][1]);
      }
      if (r + 8 < T) {
        *reinterpret_cast<__nv_bfloat162*>(dk + (int64_t)(r + 8) * ldk + (int64_t)hk * D + c) =
            __floats2bfloat162_rn(acc_dk[i][j][2] * scale, acc_dk[i][j][3] * scale);
        *reinterpret_cast<__nv_bfloat162*>(dv + (int64_t)(r + 8) * ldk + (int64_t)hk * D + c) =
            __floats2bfloat162_rn(acc_dv[i][j][2], acc_dv[i][j][3]);
      }
    }
  }
}

// ------------------------------------------------------------------ backward: dQ
// grid (ceil(T/64), Hq), 256 threads.
template <int D, int BN>
__global__ void __launch_bounds__(256) attn_bwd_dq_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, const bf16* __restrict__ dout,
    const float* __restrict__ lse, const float* __restrict__ delta, const int* __restrict__ doc_start, int T, int Hq,
    int Hk, int window, float scale, bf16* __restrict__ dq) {
  constexpr int BM = 64, NTH = 256;
  constexpr int WM = 2, WN = 4, OM = BM / WM, ON = D / WN, OMT = OM / 16, ONT = ON / 8;
  constexpr int SWM = 4, SWN = 2, SN = BN / SWN, SNT = SN / 8;  // S tile [64 x BN]
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sO = sQ + BM * D * 2;
  const uint32_t sK = sO + BM * D * 2;
  const uint32_t sV = sK + BN * D * 2;
  const uint32_t sS = sV + BN * D * 2;  // dS [BM][BN]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, hk = h / (Hq / Hk);
  const int64_t ldq = (int64_t)Hq * D, ldk = (int64_t)Hk * D;
  load_tile<BM, D, NTH>(sQ, q + (int64_t)h * D, ldq, q0, T, 0);
  load_tile<BM, D, NTH>(sO, dout + (int64_t)h * D, ldq, q0, T, 0);
  cp_async_commit();
  const int qlast = min(q0 + BM - 1, T - 1);
  int kstart = doc_start[q0];
  if (window > 0) kstart = max(kstart, q0 - window + 1);
  const int kb_first = (kstart / BN) * BN;
  const int swm = warp / SWN, swn = warp % SWN;
  const int wm = warp / WN, wn = warp % WN;
  // this thread's rows in the S slab
  const int ra = q0 + swm * 16 + (lane >> 2), rb = ra + 8;
  const float lse_a = ra < T ? lse[(int64_t)h * T + ra] : 0.f, lse_b = rb < T ? lse[(int64_t)h * T + rb] : 0.f;
  const float dl_a = ra < T ? delta[(int64_t)h * T + ra] : 0.f, dl_b = rb < T ? delta[(int64_t)h * T + rb] : 0.f;
  const int ds_a = ra < T ? doc_start[ra] : 0, ds_b = rb < T ? doc_start[rb] : 0;
  float acc[OMT][ONT][4];
  zero(acc);
  for (int kb = kb_first; kb <= qlast; kb += BN) {
    load_tile<BN, D, NTH>(sK, k + (int64_t)hk * D, ldk, kb, T, 0);
    load_tile<BN, D, NTH>(sV, v + (int64_t)hk * D, ldk, kb, T, 0);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float s[1][SNT][4], dp[1][SNT][4];
    zero(s);
    zero(dp);
    warp_gemm<1, SNT, false, false, D, D>(s, sQ, swm * 16, sK, swn * SN, D);
    warp_gemm<1, SNT, false, false, D, D>(dp, sO, swm * 16, sV, swn * SN, D);
#pragma unroll
    for (int j = 0; j < SNT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool lo = e < 2;
        const int t = lo ? ra : rb;
        const int sc = kb + swn * SN + j * 8 + (lane & 3) * 2 + (e & 1);
        const bool ok = allowed(t, sc, lo ? ds_a : ds_b, window, T);
        const float p = ok ? expf(s[0][j][e] * scale - (lo ? lse_a : lse_b)) : 0.f;
        dp[0][j][e] = p * (dp[0][j][e] - (lo ? dl_a : dl_b));
      }
      const int qr = swm * 16 + (lane >> 2);
      const int kc = swn * SN + j * 8 + (lane & 3) * 2;
      const uint32_t o0 = Tile<BN>::off(qr, kc >> 3) + (kc & 7) * 2;
      const uint32_t o1 = Tile<BN>::off(qr + 8, kc >> 3) + (kc & 7) * 2;
      asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(sS + o0), "r"(pack_bf16(dp[0][j][0], dp[0][j][1])));
      asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(sS + o1), "r"(pack_bf16(dp[0][j][2], dp[0][j][3])));
    }
    __syncthreads();
    // dQ += dS K   (A = dS [q][keys]; B = K [keys][d] stored -> transposed)
    warp_gemm<OMT, ONT, false, true, BN, D>(acc, sS, wm * OM, sK, wn * ON, BN);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < OMT; ++i) {
#pragma unroll
    for (int j = 0; j < ONT; ++j) {
      const int r = q0 + wm * OM + i * 16 + (lane >> 2);
      const int c = wn * ON + j * 8 + (lane & 3) * 2;
      if (r < T)
        *reinterpret_cast<__nv_bfloat162*>(dq + (int64_t)r * ldq + (int64_t)h * D + c) =
            __floats2bfloat162_rn(acc[i][j][0] * scale, acc[i][j][1] * scale);
      if (r + 8 < T)
        *reinterpret_cast<__nv_bfloat162*>(dq + (int64_t)(r + 8) * ldq + (int64_t)h * D + c) =
            __floats2bfloat162_rn(acc[i][j][2] * scale, acc[i][j][3] * scale);
    }
  }
}

template <typename K>
void set_smem(K kernel, size_t bytes) {
  static_assert(true, "");
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int D>
void launch_fwd(const bf16* q, const bf16* k, const bf16* v, const int* ds, int T, int Hq, int Hk, int window,
                float scale, bf16* o, float* lse, cudaStream_t stream) {
  constexpr int DV = D > 256 ? 256 : D;
  constexpr int STAGES = D > 256 ? 1 : 2;
  const size_t smem = (size_t)(64 * D + STAGES * 64 * D + STAGES * 64 * DV) * 2;
  auto kern = attn_fwd_kernel<D, DV, STAGES>;
  set_smem(kern, smem);
  dim3 grid((T + 63) / 64, Hq, D / DV);
  kern<<<grid, 128, smem, stream>>>(q, k, v, ds, T, Hq, Hk, window, scale, o, lse);
}

template <int D>
void launch_bwd(const bf16* q, const bf16* k, const bf16* v, const bf16* dout, const float* lse, const float* delta,
                const int* ds, const int* de, int T, int Hq, int Hk, int window, float scale, bf16* dq, bf16* dk,
                bf16* dv, cudaStream_t stream) {
  constexpr int BN = D > 256 ? 32 : 64;
  {
    const size_t smem = (size_t)(2 * BN * D + 2 * 64 * D + 2 * BN * 64) * 2 + 2 * 64 * sizeof(float);
    auto kern = attn_bwd_dkdv_kernel<D, BN>;
    set_smem(kern, smem);
    dim3 grid((T + BN - 1) / BN, Hk);
    kern<<<grid, 256, smem, stream>>>(q, k, v, dout, lse, delta, ds, de, T, Hq, Hk, window, scale, dk, dv);
  }
  {
    const size_t smem = (size_t)(2 * 64 * D + 2 * BN * D + 64 * BN) * 2;
    auto kern = attn_bwd_dq_kernel<D, BN>;
    set_smem(kern, smem);
    dim3 grid((T + 63) / 64, Hq);
    kern<<<grid, 256, smem, stream>>>(q, k, v, dout, lse, delta, ds, T, Hq, Hk, window, scale, dq);
  }
}

void check_qkv(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "attention inputs must be CUDA tensors");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "attention inputs must be contiguous");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16,
              "attention runs on bf16");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "q/k/v must be [T, H, D]");
  TORCH_CHECK(q.size(1) % k.size(1) == 0, "query heads must be a multiple of kv heads");
}

#define ME_ATTN_DISPATCH(D, ...)                  \
  switch (D) {                                    \
    case 64: { constexpr int DD = 64; __VA_ARGS__; break; }   \
    case 128: { constexpr int DD = 128; __VA_ARGS__; break; } \
    case 256: { constexpr int DD = 256; __VA_ARGS__; break; } \
    case 512: { constexpr int DD = 512; __VA_ARGS__; break; } \
    default: TORCH_CHECK(false, "head_dim must be 64, 128, 256 or 512"); \
  }

}  // namespace

std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor doc_start,
                                    int64_t window, double scale) {
  check_qkv(q, k, v);
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hk = (int)k.size(1), D = (int)q.size(2);
  auto o = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(torch::kFloat32));
  if (T == 0) return {o, lse};
  auto ds = doc_start.to(torch::kInt32).contiguous();
  auto stream = at::cuda::getCurrentCUDAStream();
  ME_ATTN_DISPATCH(D, launch_fwd<DD>(reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
                                     reinterpret_cast<const bf16*>(v.data_ptr()), ds.data_ptr<int>(), T, Hq, Hk,
                                     (int)window, (float)scale, reinterpret_cast<bf16*>(o.data_ptr()),
                                     lse.data_ptr<float>(), stream));
  return {o, lse};
}

std::vector<torch::Tensor> attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                    torch::Tensor o, torch::Tensor lse, torch::Tensor doc_start, int64_t window,
                                    double scale) {
  check_qkv(q, k, v);
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hk = (int)k.size(1), D = (int)q.size(2);
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  if (T == 0) return {dq, dk, dv};
  auto doc = dout.contiguous();
  auto ds = doc_start.to(torch::kInt32).contiguous();
  // doc_end[t] = (start of the next document) - 1
  auto idx = torch::arange(T, ds.options());
  auto is_start = ds.eq(idx);
  auto nxt = torch::where(is_start, idx, torch::full_like(idx, T));
  // next start strictly after t: reverse cumulative min of the shifted starts
  auto shifted = torch::cat({nxt.slice(0, 1), torch::full({1}, T, ds.options())});
  auto de = (std::get<0>(torch::cummin(shifted.flip(0), 0)).flip(0) - 1).to(torch::kInt32).contiguous();
  auto delta = torch::empty({Hq, T}, q.options().dtype(torch::kFloat32));
  auto stream = at::cuda::getCurrentCUDAStream();
  {
    const int64_t rows = (int64_t)T * Hq;
    const int grid = (int)std::min<int64_t>((rows + 7) / 8, 148 * 32);
    attn_bwd_pre_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const bf16*>(o.data_ptr()),
                                                  reinterpret_cast<const bf16*>(doc.data_ptr()), T, Hq, D,
                                                  delta.data_ptr<float>());
  }
  ME_ATTN_DISPATCH(D, launch_bwd<DD>(reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()),
                                     reinterpret_cast<const bf16*>(v.data_ptr()), reinterpret_cast<const bf16*>(doc.data_ptr()),
                                     lse.data_ptr<float>(), delta.data_ptr<float>(), ds.data_ptr<int>(), de.data_ptr<int>(),
                                     T, Hq, Hk, (int)window, (float)scale, reinterpret_cast<bf16*>(dq.data_ptr()),
                                     reinterpret_cast<bf16*>(dk.data_ptr()), reinterpret_cast<bf16*>(dv.data_ptr()),
                                     stream));
  return {dq, dk, dv};
}

// =============================================================================== no-alloc entry
// Allocation-free variant of attn_bwd for callers that cannot allocate device memory (see
// noalloc.h). Its scratch is the file-scope array below; host code only ever passes the
// device address looked up with cudaGetSymbolAddress, never the array's name.
#include <mutex>

#include "noalloc.h"

namespace {

static __device__ __align__(256) unsigned char g_attn_bwd_scratch[ME_ATTN_BWD_NOALLOC_SCRATCH_BYTES];

constexpr int kNoAllocMaxDevices = 64;
void* g_scratch_addr[kNoAllocMaxDevices] = {nullptr};
std::mutex g_scratch_mu;
thread_local const char* g_noalloc_err = "no error";

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// doc_end[t] = last token of t's document. Document starts are non-decreasing along the packed
// row, so the end is the last position whose start equals ds[t]: one binary search per token
// (O(log T) work each, all tokens in parallel, whatever the document lengths).
__global__ void doc_end_from_start_kernel(const int* __restrict__ ds, int T, int* __restrict__ de) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    const int s = ds[t];
    int lo = t, hi = T - 1;  // invariant: ds[lo] == s; the answer lies in [lo, hi]
    while (lo < hi) {
      const int mid = lo + (hi - lo + 1) / 2;
      if (ds[mid] == s) lo = mid;
      else hi = mid - 1;
    }
    de[t] = lo;
  }
}

// launch_bwd with every step checked, for the allocation-free entry point: the shared-memory
// opt-in of each kernel and each launch report their own failure.
template <int D>
const char* launch_bwd_checked(const bf16* q, const bf16* k, const bf16* v, const bf16* dout, const float* lse,
                               const float* delta, const int* ds, const int* de, int T, int Hq, int Hk, int window,
                               float scale, bf16* dq, bf16* dk, bf16* dv, cudaStream_t stream) {
  constexpr int BN = D > 256 ? 32 : 64;
  const size_t smem_kv = (size_t)(2 * BN * D + 2 * 64 * D + 2 * BN * 64) * 2 + 2 * 64 * sizeof(float);
  const size_t smem_q = (size_t)(2 * 64 * D + 2 * BN * D + 64 * BN) * 2;
  auto kv = attn_bwd_dkdv_kernel<D, BN>;
  auto qk = attn_bwd_dq_kernel<D, BN>;
  if (cudaFuncSetAttribute(kv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv) != cudaSuccess)
    return "me_attn_bwd_noalloc: cudaFuncSetAttribute (shared memory) failed for the dK/dV kernel";
  if (cudaFuncSetAttribute(qk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_q) != cudaSuccess)
    return "me_attn_bwd_noalloc: cudaFuncSetAttribute (shared memory) failed for the dQ kernel";
  kv<<<dim3((T + BN - 1) / BN, Hk), 256, smem_kv, stream>>>(q, k, v, dout, lse, delta, ds, de, T, Hq, Hk, window,
                                                             scale, dk, dv);
  if (cudaGetLastError() != cudaSuccess) return "me_attn_bwd_noalloc: the dK/dV kernel failed to launch";
  qk<<<dim3((T + 63) / 64, Hq), 256, smem_q, stream>>>(q, k, v, dout, lse, delta, ds, T, Hq, Hk, window, scale, dq);
  if (cudaGetLastError() != cudaSuccess) return "me_attn_bwd_noalloc: the dQ kernel failed to launch";
  return nullptr;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Device address of the scratch array on the current device (looked up once per device).
void* scratch_on_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    *err = ME_NOALLOC_ERR_SETUP;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *err = ME_NOALLOC_ERR_SETUP;
      return nullptr;
    }
    g_scratch_addr[dev] = p;
  }
  return g_scratch_addr[dev];
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* me_noalloc_last_error(void) { return g_noalloc_err; }

extern "C" __attribute__((visibility("default"))) int me_attn_bwd_noalloc(
    const void* dout, const void* q, const void* k, const void* v, const void* o, const float* lse,
    const int* doc_start, int T, int Hq, int Hk, int D, int window, float scale, void* dq, void* dk, void* dv,
    cudaStream_t stream) {
  if (!dout || !q || !k || !v || !o || !lse || !doc_start || !dq || !dk || !dv || T <= 0 || Hq <= 0 || Hk <= 0 ||
      Hq % Hk != 0 || !(D == 64 || D == 128 || D == 256 || D == 512)) {
    g_noalloc_err = "me_attn_bwd_noalloc: null pointer, non-positive size, Hq not a multiple of Hk, or head_dim "
                    "not in {64, 128, 256, 512}";
    return ME_NOALLOC_ERR_ARGS;
  }
  // the kernels read and write the bf16 tensors 16 bytes at a time, lse and doc_start 4 at a time
  for (const void* p : {dout, q, k, v, o, (const void*)dq, (const void*)dk, (const void*)dv}) {
    if (!aligned(p, 16)) {
      g_noalloc_err = "me_attn_bwd_noalloc: dout, q, k, v, o, dq, dk and dv must start on 16-byte boundaries";
      return ME_NOALLOC_ERR_ARGS;
    }
  }
  if (!aligned(lse, 4) || !aligned(doc_start, 4)) {
    g_noalloc_err = "me_attn_bwd_noalloc: lse and doc_start must start on 4-byte boundaries";
    return ME_NOALLOC_ERR_ARGS;
  }
  if (cudaPeekAtLastError() != cudaSuccess) {
    // an earlier, unrelated launch left an error: report it as such and leave it pending for its owner
    g_noalloc_err = "me_attn_bwd_noalloc: a CUDA error from earlier work is pending (cudaPeekAtLastError); "
                    "nothing was launched";
    return ME_NOALLOC_ERR_LAUNCH;
  }
  const size_t delta_bytes = align256((size_t)Hq * (size_t)T * sizeof(float));
  const size_t need = delta_bytes + align256((size_t)T * sizeof(int));
  if (need > (size_t)ME_ATTN_BWD_NOALLOC_SCRATCH_BYTES) {
    g_noalloc_err = "me_attn_bwd_noalloc: Hq*T*4 + T*4 bytes of scratch exceed the fixed 8 MiB array "
                    "(ME_ATTN_BWD_NOALLOC_SCRATCH_BYTES); use attn_bwd for this size";
    return ME_NOALLOC_ERR_TOO_LARGE;
  }
  int err = ME_NOALLOC_OK;
  unsigned char* scratch = static_cast<unsigned char*>(scratch_on_current_device(&err));
  if (scratch == nullptr) {
    g_noalloc_err = "me_attn_bwd_noalloc: cudaGetSymbolAddress of the scratch array failed on this device";
    return err;
  }
  float* delta = reinterpret_cast<float*>(scratch);
  int* doc_end = reinterpret_cast<int*>(scratch + delta_bytes);
  {
    const int64_t rows = (int64_t)T * Hq;
    const int grid = (int)std::min<int64_t>((rows + 7) / 8, 148 * 32);
    attn_bwd_pre_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const bf16*>(o), reinterpret_cast<const bf16*>(dout),
                                                  T, Hq, D, delta);
    if (cudaGetLastError() != cudaSuccess) {
      g_noalloc_err = "me_attn_bwd_noalloc: the softmax-correction kernel failed to launch";
      return ME_NOALLOC_ERR_LAUNCH;
    }
    doc_end_from_start_kernel<<<(T + 255) / 256, 256, 0, stream>>>(doc_start, T, doc_end);
    if (cudaGetLastError() != cudaSuccess) {
      g_noalloc_err = "me_attn_bwd_noalloc: the document-end kernel failed to launch";
      return ME_NOALLOC_ERR_LAUNCH;
    }
  }
  const bf16* qp = reinterpret_cast<const bf16*>(q);
  const bf16* kp = reinterpret_cast<const bf16*>(k);
  const bf16* vp = reinterpret_cast<const bf16*>(v);
  const bf16* gp = reinterpret_cast<const bf16*>(dout);
  bf16* dqp = reinterpret_cast<bf16*>(dq);
  bf16* dkp = reinterpret_cast<bf16*>(dk);
  bf16* dvp = reinterpret_cast<bf16*>(dv);
  const char* failed = nullptr;
  switch (D) {
    case 64: failed = launch_bwd_checked<64>(qp, kp, vp, gp, lse, delta, doc_start, doc_end, T, Hq, Hk, window, scale, dqp, dkp, dvp, stream); break;
    case 128: failed = launch_bwd_checked<128>(qp, kp, vp, gp, lse, delta, doc_start, doc_end, T, Hq, Hk, window, scale, dqp, dkp, dvp, stream); break;
    case 256: failed = launch_bwd_checked<256>(qp, kp, vp, gp, lse, delta, doc_start, doc_end, T, Hq, Hk, window, scale, dqp, dkp, dvp, stream); break;
    default: failed = launch_bwd_checked<512>(qp, kp, vp, gp, lse, delta, doc_start, doc_end, T, Hq, Hk, window, scale, dqp, dkp, dvp, stream); break;
  }
  if (failed != nullptr) {
    g_noalloc_err = failed;
    return ME_NOALLOC_ERR_LAUNCH;
  }
  g_noalloc_err = "no error";
  return ME_NOALLOC_OK;
}
