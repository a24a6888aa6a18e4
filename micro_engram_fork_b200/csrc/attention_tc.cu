// tcgen05 (5th-gen tensor core) packed-varlen attention forward for sm_100a.
//
// One CTA = 128 queries of one head (M = 128 TMEM lanes) x DV output columns, looping over
// key blocks of 64. Warp roles (320 threads):
//   warp 0     TMA producer: Q once (D/64 chunks of 128x64, 128B swizzle), K in 64x64 chunks
//              through a KS-deep ring, V in 64-key x DV blocks through a VS-deep ring (3-D
//              tensor maps over [T, H, D]; no multicast)
//   warp 1     TMEM owner + single-thread MMA issuer:
//                S_j = Q K_j^T  into one of two 64-column S buffers  (A, B K-major)
//                O  += P_j V_j  into a DV-column O accumulator       (A = P_j from one of two
//                               shared-memory buffers, B = V, N-contiguous)
//              tcgen05.commit releases K/V stages and signals S-ready / P-free / PV-done
//   warps 2-9  softmax, two warps per TMEM lane quarter: each thread owns one query row and 32
//              of the block's 64 keys (tcgen05.ld), applies the document / causal / sliding-window
//              mask, agrees with its partner thread on the row max through shared memory and a
//              per-quarter mbarrier, keeps a running max with lazy rescaling (O in TMEM is
//              rescaled only when the max grows by more than 2^8, warp-uniformly, each warp its
//              half of the columns), writes its half of P (bf16) into the P buffer of the block's
//              parity (free once PV_{j-2} is done, so softmax j overlaps PV_{j-1}), and finally
//              normalises its half of O out of TMEM and writes O and the LSE.
// Every wait is bounded (2 s); a timeout records ME_ERR_TIMEOUT in the status word and the
// kernel frees TMEM and returns.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cudaTypedefs.h>

#include <mutex>

#include "tc_common.cuh"

using namespace me;
using namespace me::tc;

namespace {
using bf16 = __nv_bfloat16;

template <int D, int DV, int KS, int VS>
struct AttnLayout {
  static constexpr int BM = 128, BN = 64, NC = D / 64;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KCH_BYTES = BN * 64 * 2;
  static constexpr int V_BYTES = BN * DV * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + KS * KCH_BYTES;
  static constexpr int P_OFF = V_OFF + VS * V_BYTES;           // two P buffers
  static constexpr int RED_OFF = P_OFF + 2 * P_BYTES;          // [2 parity][2 half][128 rows] fp32
  static constexpr int BAR_OFF = RED_OFF + 2 * 2 * BM * 4;
  static constexpr int N_BARS = 1 + 2 * KS + 2 * VS + 2 + 2 + 2 + 2 + 1 + 4;
  static constexpr int BYTES = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = (128 + DV) <= 256 ? 256 : 512;
  static constexpr int O_COL = 128;
  static constexpr int THREADS = 320, NSOFT = 256;  // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
  static_assert(BYTES <= 232448, "shared memory");
};

template <int D, int DV, int KS, int VS>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const int* __restrict__ doc_start, int T, int Hq,
                       int Hk, int window, float scale, bf16* __restrict__ o, float* __restrict__ lse, int* status) {
  using L = AttnLayout<D, DV, KS, VS>;
  constexpr int BM = L::BM, BN = L::BN, NC = L::NC, HB = BN / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint8_t* sP = smem + L::P_OFF;
  float* red = reinterpret_cast<float*>(smem + L::RED_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + KS;
  uint64_t* v_full = k_empty + KS;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* o_final = pv_done + 2;
  uint64_t* pair = o_final + 1;  // per TMEM lane quarter: the two warps sharing its rows
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, hk = h / (Hq / Hk), dv0 = blockIdx.z * DV;
  const int qlast = min(q0 + BM - 1, T - 1);
  int kstart = doc_start[q0];
  if (window > 0) kstart = max(kstart, q0 - window + 1);
  const int kb_first = (kstart / BN) * BN;
  const int nkb = (qlast - kb_first) / BN + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], L::NSOFT);
      mbar_init(&p_full[i], L::NSOFT);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_final, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&pair[i], 64);
    *abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      mbar_expect_tx(q_full, L::Q_BYTES);
      for (int c = 0; c < NC; ++c) tma_load_3d(sQ + c * (BM * 128), &tq, q_full, c * 64, h, q0);
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      auto load_k = [&](int j) {
        for (int c = 0; c < NC && ok; ++c) {
          const int g = j * NC + c, st = g % KS, r = g / KS;
          if (r > 0 && !mbar_wait(&k_empty[st], (r - 1) & 1, status, 11, abort)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&k_full[st], L::KCH_BYTES);
          tma_load_3d(sK + st * L::KCH_BYTES, &tk, &k_full[st], c * 64, hk, kb_first + j * BN);
          issued_k = g + 1;
        }
      };
      auto load_v = [&](int j) {
        const int b = j % VS, r = j / VS;
        if (r > 0 && !mbar_wait(&v_empty[b], (r - 1) & 1, status, 12, abort)) {
          ok = false;
          return;
        }
        mbar_expect_tx(&v_full[b], L::V_BYTES);
        for (int vc = 0; vc < DV / 64; ++vc)
          tma_load_3d(sV + b * L::V_BYTES + vc * (BN * 128), &tv, &v_full[b], dv0 + vc * 64, hk, kb_first + j * BN);
        issued_v = j + 1;
      };
      load_k(0);
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb) load_k(j + 1);
        if (ok) load_v(j);
      }
      // drain every copy still in flight before the CTA may exit
      mbar_wait(q_full, 0, status, 19, nullptr);
      for (int g = max(0, issued_k - KS); g < issued_k; ++g) mbar_wait(&k_full[g % KS], (g / KS) & 1, status, 19, nullptr);
      for (int j = max(0, issued_v - VS); j < issued_v; ++j) mbar_wait(&v_full[j % VS], (j / VS) & 1, status, 19, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t id_s = idesc_bf16(BM, BN);
      const uint32_t id_o = idesc_bf16(BM, DV, true);
      const uint32_t aQ = smem_addr(sQ), aK = smem_addr(sK), aV = smem_addr(sV), aP = smem_addr(sP);
      bool ok = mbar_wait(q_full, 0, status, 20, abort);
      auto issue_pv = [&](int i) {
        if (!ok) return;
        const int vb = i % VS, pb = i & 1;
        if (!mbar_wait(&p_full[pb], (i >> 1) & 1, status, 21, abort) ||
            !mbar_wait(&v_full[vb], (i / VS) & 1, status, 22, abort)) {
          ok = false;
          return;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_bf16(tmem + L::O_COL, desc_sw128(aP + pb * L::P_BYTES + kk * 32),
                    desc_mn_sw128(aV + vb * L::V_BYTES + kk * 16 * 128, BN * 128, 1024), id_o, (i > 0 || kk > 0));
        umma_commit(&v_empty[vb]);
        umma_commit(&pv_done[pb]);
      };
      for (int j = 0; j < nkb && ok; ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&s_free[b], ((j - 2) >> 1) & 1, status, 23, abort)) {
          ok = false;
          break;
        }
        for (int c = 0; c < NC; ++c) {
          const int g = j * NC + c, st = g % KS;
          if (!mbar_wait(&k_full[st], (g / KS) & 1, status, 24, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + b * BN, desc_sw128(aQ + c * (BM * 128) + kk * 32),
                      desc_sw128(aK + st * L::KCH_BYTES + kk * 32), id_s, (c | kk) != 0);
          umma_commit(&k_empty[st]);
        }
        if (!ok) break;
        umma_commit(&s_full[b]);
        if (j >= 1) issue_pv(j - 1);
      }
      if (ok) issue_pv(nkb - 1);
      if (ok) umma_commit(o_final);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    // warps 2-9: TMEM lane quarter (warp & 3) and column half (warp - 2) / 4: the two warps of a
    // quarter share its 32 rows, each scoring 32 of the 64 keys of a block and owning half of O's
    // columns; they agree on the running max through `red` and their pair barrier every block.
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const int t = q0 + r;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int ds_t = t < T ? doc_start[t] : 0;
    const int lo = window > 0 ? max(ds_t, t - window + 1) : ds_t;
    // scores are kept in log2 units: p = 2^(s * scale * log2(e) - m), one FFMA + one ex2 per key
    const float sl2 = scale * 1.4426950408889634f;
    float m_used = -INFINITY, l = 0.f;  // m_used in log2 units; l: this half's share of the row sum
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int b = j & 1, kb = kb_first + j * BN + half * HB;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, status, 30, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[HB];
      tmem_ld32(tmem + lane_base + b * BN + half * HB, s);
      tc_fence_before();
      mbar_arrive(&s_free[b]);
      float mx = -INFINITY;
      if (t < T && kb >= lo && kb + HB - 1 <= t) {  // every key of this half-block is visible
#pragma unroll
        for (int c = 0; c < HB; ++c) mx = fmaxf(mx, s[c]);
      } else {
#pragma unroll
        for (int c = 0; c < HB; ++c) {
          const int sc = kb + c;
          if (t >= T || sc > t || sc < lo) s[c] = -INFINITY;  // sc <= t < T: the key exists
          mx = fmaxf(mx, s[c]);
        }
      }
      red[((j & 1) * 2 + half) * BM + r] = mx;
      mbar_arrive(&pair[q]);
      if (!mbar_wait(&pair[q], j & 1, status, 33, abort)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, red[((j & 1) * 2 + (half ^ 1)) * BM + r]) * sl2;  // raw max -> log2 units
      float m_new = m_used, alpha = 1.f;
      bool resc = false;
      if (mx > -INFINITY) {
        if (m_used == -INFINITY) {
          m_new = mx;
          alpha = 0.f;  // nothing accumulated yet (l = 0, O rows are zero)
        } else if (mx > m_used + 11.5415602f) {  // grew by more than e^8
          m_new = mx;
          alpha = ex2_approx(m_used - m_new);
          resc = true;
        }
      }
      float sum = 0.f;
      if (m_new == -INFINITY) {  // nothing visible yet on this row
#pragma unroll
        for (int c = 0; c < HB; ++c) s[c] = 0.f;
      } else {
#pragma unroll
        for (int c = 0; c < HB; ++c) {
          const float p = ex2_approx(fmaf(s[c], sl2, -m_new));  // masked keys: 2^-inf = 0
          s[c] = p;
          sum += p;
        }
      }
      l = l * alpha + sum;
      m_used = m_new;
      const int pb = j & 1;
      // O may be rescaled only once PV_{j-1} is done; P buffer pb is free once PV_{j-2} is
      const bool any_resc = j >= 1 && __any_sync(0xffffffffu, resc);
      if (any_resc) {
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, status, 31, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float f = resc ? alpha : 1.f;
#pragma unroll 1
        for (int cc = 0; cc < DV / 64; ++cc) {
          float v[32];
          const uint32_t col = L::O_COL + half * (DV / 2) + cc * 32;
          tmem_ld32(tmem + lane_base + col, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= f;
          tmem_st32(tmem + lane_base + col, v);
        }
        tmem_st_wait();
      }
      if (j >= 2 && !mbar_wait(&pv_done[pb], ((j - 2) >> 1) & 1, status, 34, abort)) {
        ok = false;
        break;
      }
      // P row r, this half's 32 keys: 4 swizzled 16-byte chunks of the 128-byte row
      const uint32_t prow = smem_addr(sP) + pb * L::P_BYTES + r * 128;
#pragma unroll
      for (int c8 = 0; c8 < HB / 8; ++c8) {
        BF16x8 pk;
#pragma unroll
        for (int e = 0; e < 4; ++e) pk.h2[e] = __floats2bfloat162_rn(s[c8 * 8 + 2 * e], s[c8 * 8 + 2 * e + 1]);
        const int chunk = half * (HB / 8) + c8;
        const uint32_t addr = prow + ((chunk ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk.u.x), "r"(pk.u.y), "r"(pk.u.z),
                     "r"(pk.u.w)
                     : "memory");
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
    }
    // row sum = both halves' shares (one more pair phase)
    if (ok) {
      red[((nkb & 1) * 2 + half) * BM + r] = l;
      mbar_arrive(&pair[q]);
      ok = mbar_wait(&pair[q], nkb & 1, status, 35, abort);
      if (ok) l += red[((nkb & 1) * 2 + (half ^ 1)) * BM + r];
    }
    if (ok && mbar_wait(o_final, 0, status, 32, abort)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t ldo = (int64_t)Hq * D;
#pragma unroll 1
      for (int cc = 0; cc < DV / 64; ++cc) {
        float v[32];
        const int c0 = half * (DV / 2) + cc * 32;
        tmem_ld32(tmem + lane_base + L::O_COL + c0, v);
        if (t < T) {
          bf16* dst = o + (int64_t)t * ldo + (int64_t)h * D + dv0 + c0;
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8) {
            BF16x8 ov;
#pragma unroll
            for (int e = 0; e < 8; ++e) ov.h[e] = f2bf(v[j8 * 8 + e] * inv);
            *reinterpret_cast<uint4*>(dst + j8 * 8) = ov.u;
          }
        }
      }
      if (blockIdx.z == 0 && half == 0 && t < T) lse[(int64_t)h * T + t] = (m_used + log2f(l)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

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

// [T, H, D] bf16 -> 3-D map with box {64 (D), 1 (head), rows (tokens)}, 128B swizzle.
CUtensorMap make_tmap_thd(const void* ptr, int64_t T, int64_t H, int64_t D, int rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "attention operand must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)(D * 2), (cuuint64_t)(H * D * 2)};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)rows};
  cuuint32_t estr[3] = {1, 1, 1};
  bind_primary_context();
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (attention) failed: ", (int)r);
  return map;
}

template <int D, int DV, int KS, int VS>
void launch_fwd_tc(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const int* ds, int window,
                   float scale, torch::Tensor& o, torch::Tensor& lse, int* status, cudaStream_t stream) {
  using L = AttnLayout<D, DV, KS, VS>;
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hk = (int)k.size(1);
  const CUtensorMap tq = make_tmap_thd(q.data_ptr(), T, Hq, D, 128);
  const CUtensorMap tk = make_tmap_thd(k.data_ptr(), T, Hk, D, 64);
  const CUtensorMap tv = make_tmap_thd(v.data_ptr(), T, Hk, D, 64);
  auto kern = attn_fwd_tc_kernel<D, DV, KS, VS>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
  dim3 grid((T + 127) / 128, Hq, D / DV);
  kern<<<grid, L::THREADS, L::BYTES, stream>>>(tq, tk, tv, ds, T, Hq, Hk, window, scale,
                                        reinterpret_cast<bf16*>(o.data_ptr()), lse.data_ptr<float>(), status);
}

torch::Tensor& attn_status(int dev) {
  static torch::Tensor bufs[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (!bufs[dev].defined())
    bufs[dev] = torch::zeros({2}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev));
  return bufs[dev];
}

}  // namespace

std::vector<torch::Tensor> attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor doc_start,
                                       int64_t window, double scale) {
  TORCH_CHECK(q.is_cuda() && q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "attn_fwd_tc: contiguous CUDA");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "attn_fwd_tc: bf16");
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), D = (int)q.size(2);
  auto o = torch::empty_like(q);
  auto lse = torch::empty({Hq, T}, q.options().dtype(torch::kFloat32));
  if (T == 0) return {o, lse};
  auto ds = doc_start.to(torch::kInt32).contiguous();
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = attn_status(q.get_device()).data_ptr<int>();
  switch (D) {
    case 64: launch_fwd_tc<64, 64, 8, 4>(q, k, v, ds.data_ptr<int>(), (int)window, (float)scale, o, lse, st, stream); break;
    case 128: launch_fwd_tc<128, 128, 8, 4>(q, k, v, ds.data_ptr<int>(), (int)window, (float)scale, o, lse, st, stream); break;
    case 256: launch_fwd_tc<256, 256, 4, 2>(q, k, v, ds.data_ptr<int>(), (int)window, (float)scale, o, lse, st, stream); break;
    case 512: launch_fwd_tc<512, 256, 3, 1>(q, k, v, ds.data_ptr<int>(), (int)window, (float)scale, o, lse, st, stream); break;
    default: TORCH_CHECK(false, "attn_fwd_tc: head_dim must be 64, 128, 256 or 512");
  }
  return {o, lse};
}

torch::Tensor attn_tc_status(int64_t device) { return attn_status((int)device); }

// =============================================================================== backward
// tcgen05 packed-varlen attention backward, three kernels from one template (head_dim <= 256):
//   MODE_DQ  one CTA = 128 queries of one head (resident Q and dO); per key block of BC keys:
//            S = Q K^T, dP = dO V^T (TMEM), dS = P * (dP - delta_row) -> smem, dQ += dS K
//   MODE_DK  one CTA = 128 keys of one kv head (resident K and V); per (query head of the GQA
//            group, block of BC queries): S^T = K Q^T, dP^T = V dO^T, dS^T = P^T * (dP^T - delta_col)
//            -> smem, dK += dS^T Q
//   MODE_DV  resident K; S^T = K Q^T, P^T -> smem, dV += P^T dO
// with P = exp(scale * S - LSE) from the forward's LSE. dK and dV sum over the GQA group inside
// the CTA (no atomics); dQ and dK carry the softmax scale. TMEM: two S buffers, two dP
// buffers, one D-column accumulator. Warp roles: warp 0 TMA producer (Q/K/V/dO tiles by 3-D
// tensor maps; per-query LSE, delta and document starts by untiled bulk copies), warp 1 TMEM
// owner + MMA issuer, warps 2-9 elementwise, two per TMEM lane quarter: one row (TMEM lane) per
// thread and half of each block's BC columns per warp. Every wait is bounded; a timeout records
// ME_ERR_TIMEOUT and the kernel frees TMEM and returns.
namespace {

enum { MODE_DQ = 0, MODE_DK = 1, MODE_DV = 2 };

// Streamed tiles live in two rings. Ring A holds the tile that is still needed by the
// accumulating MMA at the end of an iteration (DQ: K_j, DK: Q_j, DV: dO_j) plus the per-query
// columns the elementwise warps read; it is released only when that MMA completes, so it gets
// SA stages. Ring B holds the tile that only the S or dP product reads (DQ: V_j, DK: dO_j,
// DV: Q_j) and is released as soon as those MMAs complete.
template <int D, int BC, int MODE>
struct BwdLayout {
  static_assert(BC == 32, "W is double-buffered in the two 64-byte halves of 128-byte rows");
  static constexpr bool TWO = MODE != MODE_DV;    // a second product (dP) and resident R2
  static constexpr bool COLS = MODE != MODE_DQ;   // per-column (query) LSE / delta / doc start
  static constexpr int NC = D / 64;
  static constexpr int SA = MODE == MODE_DV ? 4 : 3, SB = 2;
  static constexpr int R_BYTES = 128 * D * 2;
  static constexpr int C_BYTES = BC * D * 2;      // one streamed tile (D/64 chunks of BC x 128 B)
  static constexpr int COL_FLOATS = 3 * BC;
  static constexpr int R_OFF = 0;
  static constexpr int R2_OFF = R_OFF + R_BYTES;
  static constexpr int A_OFF = R2_OFF + (TWO ? R_BYTES : 0);
  static constexpr int B_OFF = A_OFF + SA * C_BYTES;
  static constexpr int W_OFF = B_OFF + SB * C_BYTES;
  static constexpr int COL_OFF = W_OFF + 128 * 128;
  static constexpr int BAR_OFF = COL_OFF + (COLS ? SA * COL_FLOATS * 4 : 0);
  static constexpr int N_BARS = 1 + 2 * SA + 2 * SB + 2 + 2 + 2 + 2 + 1;
  static constexpr int BYTES = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static constexpr int S_COL = 0, DP_COL = 2 * BC, ACC_COL = TWO ? 4 * BC : 2 * BC;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int THREADS = 320;  // warp 0 producer, warp 1 MMA, warps 2-9 elementwise
  static constexpr int NCOMP = 256;
  static_assert(C_BYTES % 1024 == 0, "tiles keep the 1024-byte alignment of the swizzle atoms");
  static_assert(ACC_COL + D <= 512, "TMEM columns");
  static_assert(BYTES <= 232448, "shared memory");
};

template <int D, int BC, int MODE>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tr, const __grid_constant__ CUtensorMap tr2,
                       const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                       const float* __restrict__ lse, const float* __restrict__ delta, const int* __restrict__ ds,
                       const int* __restrict__ de, int T, int Tp, int Hq, int Hk, int window, float scale,
                       bf16* __restrict__ out, int* status) {
  using L = BwdLayout<D, BC, MODE>;
  constexpr int NC = L::NC, HB = BC / 2, SA = L::SA, SB = L::SB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sR = smem + L::R_OFF;
  uint8_t* sR2 = smem + L::R2_OFF;
  uint8_t* sW = smem + L::W_OFF;
  auto tile_a = [&](int st) { return smem + L::A_OFF + st * L::C_BYTES; };
  auto tile_b = [&](int st) { return smem + L::B_OFF + st * L::C_BYTES; };
  auto cols_of = [&](int st) { return reinterpret_cast<float*>(smem + L::COL_OFF) + st * L::COL_FLOATS; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* r_full = bars;
  uint64_t* a_full = r_full + 1;
  uint64_t* a_empty = a_full + SA;
  uint64_t* b_full = a_empty + SA;
  uint64_t* b_empty = b_full + SB;
  uint64_t* s_full = b_empty + SB;
  uint64_t* s_free = s_full + 2;
  uint64_t* w_full = s_free + 2;
  uint64_t* acc_done = w_full + 2;
  uint64_t* acc_final = acc_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_final + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = Hq / Hk;
  const int r0 = blockIdx.x * 128;  // first resident row (query for DQ, key otherwise)
  const int head = blockIdx.y;      // query head (DQ) or kv head
  const int rlast = min(r0 + 127, T - 1);
  int first, nblk, nit;
  if (MODE == MODE_DQ) {
    int kstart = ds[r0];
    if (window > 0) kstart = max(kstart, r0 - window + 1);
    first = (kstart / BC) * BC;
    nblk = (rlast - first) / BC + 1;
    nit = nblk;
  } else {
    int tmax = de[rlast];
    if (window > 0) tmax = min(tmax, rlast + window - 1);
    tmax = min(tmax, T - 1);
    first = (r0 / BC) * BC;
    nblk = (tmax - first) / BC + 1;
    nit = G * nblk;
  }

  if (threadIdx.x == 0) {
    mbar_init(r_full, 1);
    for (int i = 0; i < SA; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], L::NCOMP);
      mbar_init(&w_full[i], L::NCOMP);
      mbar_init(&acc_done[i], 1);
    }
    mbar_init(acc_final, 1);
    *abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tr);
    if (L::TWO) prefetch_tmap(&tr2);
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // streamed block of iteration i: (row start, head of the streamed operands)
  auto blk = [&](int i, int& start, int& shead) {
    if (MODE == MODE_DQ) {
      start = first + i * BC;
      shead = head / G;
    } else {
      start = first + (i % nblk) * BC;
      shead = head * G + i / nblk;
    }
  };

  if (warp == 0) {
    if (lane == 0 && nit > 0) {
      // ------------------------------------------------------------------ producer
      mbar_expect_tx(r_full, (L::TWO ? 2 : 1) * L::R_BYTES);
      for (int c = 0; c < NC; ++c) {
        tma_load_3d(sR + c * (128 * 128), &tr, r_full, c * 64, head, r0);
        if (L::TWO) tma_load_3d(sR2 + c * (128 * 128), &tr2, r_full, c * 64, head, r0);
      }
      int issued = 0;
      for (int i = 0; i < nit; ++i) {
        const int sa = i % SA, sb = i % SB;
        int start, shead;
        blk(i, start, shead);
        if (i >= SA && !mbar_wait(&a_empty[sa], ((i / SA) - 1) & 1, status, 41, abort)) break;
        mbar_expect_tx(&a_full[sa], L::C_BYTES + (L::COLS ? L::COL_FLOATS * 4 : 0));
        for (int c = 0; c < NC; ++c) tma_load_3d(tile_a(sa) + c * (BC * 128), &ta, &a_full[sa], c * 64, shead, start);
        if (L::COLS) {
          float* cols = cols_of(sa);
          bulk_load(cols, lse + (int64_t)shead * Tp + start, BC * 4, &a_full[sa]);
          bulk_load(cols + BC, delta + (int64_t)shead * Tp + start, BC * 4, &a_full[sa]);
          bulk_load(cols + 2 * BC, ds + start, BC * 4, &a_full[sa]);
        }
        if (i >= SB && !mbar_wait(&b_empty[sb], ((i / SB) - 1) & 1, status, 42, abort)) {
          issued = -(i + 1);  // A of iteration i is in flight, B is not
          break;
        }
        mbar_expect_tx(&b_full[sb], L::C_BYTES);
        for (int c = 0; c < NC; ++c) tma_load_3d(tile_b(sb) + c * (BC * 128), &tb, &b_full[sb], c * 64, shead, start);
        issued = i + 1;
      }
      // drain the copies in flight before the CTA may exit
      const int na = issued < 0 ? -issued : issued, nb = issued < 0 ? -issued - 1 : issued;
      mbar_wait(r_full, 0, status, 49, nullptr);
      for (int i = max(0, na - SA); i < na; ++i) mbar_wait(&a_full[i % SA], (i / SA) & 1, status, 49, nullptr);
      for (int i = max(0, nb - SB); i < nb; ++i) mbar_wait(&b_full[i % SB], (i / SB) & 1, status, 49, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && nit > 0) {
      // ------------------------------------------------------------------ MMA issuer
      const uint32_t id_s = idesc_bf16(128, BC);
      const uint32_t id_acc = idesc_bf16(128, D, true);
      const uint32_t aR = smem_addr(sR), aR2 = smem_addr(sR2), aW = smem_addr(sW);
      bool ok = mbar_wait(r_full, 0, status, 50, abort);
      auto issue_acc = [&](int i) {
        if (!ok) return;
        const int wb = i & 1;
        if (!mbar_wait(&w_full[wb], (i >> 1) & 1, status, 51, abort)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t aX = smem_addr(tile_a(i % SA));
#pragma unroll
        for (int kk = 0; kk < BC / 16; ++kk)
          umma_bf16(tmem + L::ACC_COL, desc_sw128(aW + wb * 64 + kk * 32),
                    desc_mn_sw128(aX + kk * 16 * 128, BC * 128, 1024), id_acc, (i > 0 || kk > 0));
        umma_commit(&a_empty[i % SA]);
        umma_commit(&acc_done[wb]);
      };
      for (int i = 0; i < nit && ok; ++i) {
        const int b = i & 1, sa = i % SA, sb = i % SB;
        if (i >= 2 && !mbar_wait(&s_free[b], ((i - 2) >> 1) & 1, status, 52, abort)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&a_full[sa], (i / SA) & 1, status, 53, abort) ||
            !mbar_wait(&b_full[sb], (i / SB) & 1, status, 54, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // S's streamed operand: Q_j / K_j in ring A (DQ, DK) or Q_j in ring B (DV); dP's is ring B
        const uint32_t aS = smem_addr(MODE == MODE_DV ? tile_b(sb) : tile_a(sa)), aP = smem_addr(tile_b(sb));
        for (int c = 0; c < NC; ++c) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_bf16(tmem + L::S_COL + b * BC, desc_sw128(aR + c * (128 * 128) + kk * 32),
                      desc_sw128(aS + c * (BC * 128) + kk * 32), id_s, (c | kk) != 0);
            if (L::TWO)
              umma_bf16(tmem + L::DP_COL + b * BC, desc_sw128(aR2 + c * (128 * 128) + kk * 32),
                        desc_sw128(aP + c * (BC * 128) + kk * 32), id_s, (c | kk) != 0);
          }
        }
        umma_commit(&s_full[b]);
        umma_commit(&b_empty[sb]);
        if (i >= 1) issue_acc(i - 1);
      }
      if (ok) issue_acc(nit - 1);
      if (ok) umma_commit(acc_final);
    }
  } else {
    // ------------------------------------------------------------------ elementwise + epilogue
    // warps 2-9: TMEM lane quarter (warp & 3), column half (warp - 2) / 4 of each BC block
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const int row = r0 + r;  // this thread's resident row
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float lse_r = 0.f, delta_r = 0.f;
    int lo_r = 0;
    if (MODE == MODE_DQ && row < T) {
      lse_r = lse[(int64_t)head * Tp + row];
      delta_r = delta[(int64_t)head * Tp + row];
      lo_r = ds[row];
      if (window > 0) lo_r = max(lo_r, row - window + 1);
    }
    bool ok = true;
    for (int i = 0; i < nit && ok; ++i) {
      const int b = i & 1, sa = i % SA;
      int start, shead;
      blk(i, start, shead);
      start += half * HB;
      if (!mbar_wait(&s_full[b], (i >> 1) & 1, status, 60, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[HB], dp[L::TWO ? HB : 1];
      tmem_ld16(tmem + lane_base + L::S_COL + b * BC + half * HB, s);
      if (L::TWO) tmem_ld16(tmem + lane_base + L::DP_COL + b * BC + half * HB, *reinterpret_cast<float(*)[16]>(dp));
      tc_fence_before();
      mbar_arrive(&s_free[b]);
      const float* cols = nullptr;
      if (L::COLS) {
        if (!mbar_wait(&a_full[sa], (i / SA) & 1, status, 61, abort)) {  // already complete: visibility
          ok = false;
          break;
        }
        cols = cols_of(sa) + half * HB;
      }
#pragma unroll
      for (int c = 0; c < HB; ++c) {
        float p;
        if (MODE == MODE_DQ) {
          const int key = start + c;
          const bool valid = row < T && key < T && key <= row && key >= lo_r;
          p = valid ? __expf(s[c] * scale - lse_r) : 0.f;
          s[c] = p * (dp[c] - delta_r);
        } else {
          const int t = start + c;
          const int dst = __float_as_int(cols[2 * BC + c]);
          const bool valid = row < T && t < T && t >= row && row >= dst && (window <= 0 || row > t - window);
          p = valid ? __expf(s[c] * scale - cols[c]) : 0.f;
          s[c] = MODE == MODE_DK ? p * (dp[L::TWO ? c : 0] - cols[BC + c]) : p;
        }
      }
      // W buffer b (64-byte half b of each 128-byte row) is free once ACC(i - 2) is done
      if (i >= 2 && !mbar_wait(&acc_done[b], ((i - 2) >> 1) & 1, status, 62, abort)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c8 = 0; c8 < HB / 8; ++c8) {
        BF16x8 pk;
#pragma unroll
        for (int e = 0; e < 8; ++e) pk.h[e] = f2bf(s[c8 * 8 + e]);
        const int chunk = b * 4 + half * (HB / 8) + c8;
        const uint32_t addr = smem_addr(sW) + r * 128 + ((chunk ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk.u.x), "r"(pk.u.y), "r"(pk.u.z),
                     "r"(pk.u.w)
                     : "memory");
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&w_full[b]);
    }
    const int64_t ld_out = (int64_t)(MODE == MODE_DQ ? Hq : Hk) * D;
    bf16* dst = out + (int64_t)row * ld_out + (int64_t)head * D + half * (D / 2);
    const float f = MODE == MODE_DV ? 1.f : scale;
    if (nit == 0) {
      if (row < T)
        for (int e = 0; e < D / 2; e += 8) *reinterpret_cast<uint4*>(dst + e) = make_uint4(0, 0, 0, 0);
    } else if (ok && mbar_wait(acc_final, 0, status, 63, abort)) {
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < D / 64; ++cc) {
        float v[32];
        tmem_ld32(tmem + lane_base + L::ACC_COL + half * (D / 2) + cc * 32, v);
        if (row < T) {
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8) {
            BF16x8 ov;
#pragma unroll
            for (int e = 0; e < 8; ++e) ov.h[e] = f2bf(v[j8 * 8 + e] * f);
            *reinterpret_cast<uint4*>(dst + cc * 32 + j8 * 8) = ov.u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// delta[h * Tp + t] = sum_d dO[t, h, d] * O[t, h, d]  (one warp per (t, h))
__global__ void attn_delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout, int T, int Hq, int D,
                                  int Tp, float* __restrict__ delta) {
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= (int64_t)T * Hq) return;
  const int t = (int)(w / Hq), h = (int)(w % Hq);
  const bf16* a = o + w * D;
  const bf16* b = dout + w * D;
  float acc = 0.f;
  for (int d = lane * 8; d < D; d += 256) {
    BF16x8 x, y;
    x.u = *reinterpret_cast<const uint4*>(a + d);
    y.u = *reinterpret_cast<const uint4*>(b + d);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += bf2f(x.h[e]) * bf2f(y.h[e]);
  }
  acc = warp_sum(acc);
  if (lane == 0) delta[(int64_t)h * Tp + t] = acc;
}

template <int D, int BC, int MODE>
void launch_bwd_tc(const CUtensorMap& tr, const CUtensorMap& tr2, const CUtensorMap& tc1, const CUtensorMap& tc2,
                   const float* lse, const float* delta, const int* ds, const int* de, int T, int Tp, int Hq, int Hk,
                   int window, float scale, bf16* out, int* status, cudaStream_t stream) {
  using L = BwdLayout<D, BC, MODE>;
  auto kern = attn_bwd_tc_kernel<D, BC, MODE>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
  dim3 grid((T + 127) / 128, MODE == MODE_DQ ? Hq : Hk, 1);
  kern<<<grid, L::THREADS, L::BYTES, stream>>>(tr, tr2, tc1, tc2, lse, delta, ds, de, T, Tp, Hq, Hk, window, scale,
                                               out, status);
}

template <int D>
void bwd_tc_all(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& dout,
                const float* lse, const float* delta, const int* ds, const int* de, int T, int Tp, int window,
                float scale, torch::Tensor& dq, torch::Tensor& dk, torch::Tensor& dv, int* status, cudaStream_t s) {
  const int Hq = (int)q.size(1), Hk = (int)k.size(1);
  constexpr int BC = 32;
  const CUtensorMap q128 = make_tmap_thd(q.data_ptr(), T, Hq, D, 128), o128 = make_tmap_thd(dout.data_ptr(), T, Hq, D, 128);
  const CUtensorMap k128 = make_tmap_thd(k.data_ptr(), T, Hk, D, 128), v128 = make_tmap_thd(v.data_ptr(), T, Hk, D, 128);
  const CUtensorMap qc = make_tmap_thd(q.data_ptr(), T, Hq, D, BC), oc = make_tmap_thd(dout.data_ptr(), T, Hq, D, BC);
  const CUtensorMap kc = make_tmap_thd(k.data_ptr(), T, Hk, D, BC), vc = make_tmap_thd(v.data_ptr(), T, Hk, D, BC);
  // dQ: resident Q, dO; ring A = K_j (S and the accumulation), ring B = V_j (dP)
  launch_bwd_tc<D, BC, MODE_DQ>(q128, o128, kc, vc, lse, delta, ds, de, T, Tp, Hq, Hk, window, scale,
                                reinterpret_cast<bf16*>(dq.data_ptr()), status, s);
  // dK: resident K, V; ring A = Q_j (S and the accumulation), ring B = dO_j (dP)
  launch_bwd_tc<D, BC, MODE_DK>(k128, v128, qc, oc, lse, delta, ds, de, T, Tp, Hq, Hk, window, scale,
                                reinterpret_cast<bf16*>(dk.data_ptr()), status, s);
  // dV: resident K; ring A = dO_j (the accumulation), ring B = Q_j (S)
  launch_bwd_tc<D, BC, MODE_DV>(k128, k128, oc, qc, lse, delta, ds, de, T, Tp, Hq, Hk, window, scale,
                                reinterpret_cast<bf16*>(dv.data_ptr()), status, s);
}

// Per-call inputs of both backward paths: document starts padded to Tp rows (value T), the
// forward's LSE and delta = rowsum(dO * O), both [Hq, Tp] fp32 (the bulk copies read whole blocks).
struct BwdPrep {
  torch::Tensor ds, lse, delta;
  int Tp;
};

BwdPrep bwd_prep(const torch::Tensor& o, const torch::Tensor& doc, const torch::Tensor& lse,
                 const torch::Tensor& doc_start, int T, int Hq, int D) {
  BwdPrep p;
  p.Tp = (T + 63) / 64 * 64 + 64;
  auto opts_i = doc_start.options().dtype(torch::kInt32);
  p.ds = torch::full({p.Tp}, T, opts_i);
  p.ds.slice(0, 0, T).copy_(doc_start.to(torch::kInt32));
  p.lse = torch::zeros({Hq, p.Tp}, lse.options());
  p.lse.slice(1, 0, T).copy_(lse);
  p.delta = torch::zeros({Hq, p.Tp}, lse.options());
  const int64_t warps = (int64_t)T * Hq;
  attn_delta_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(o.data_ptr()), reinterpret_cast<const bf16*>(doc.data_ptr()), T, Hq, D, p.Tp,
      p.delta.data_ptr<float>());
  return p;
}

}  // namespace

// dq, dk, dv of the packed-varlen attention (head_dim 64 / 128 / 256) from the forward's o, lse.
std::vector<torch::Tensor> attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                       torch::Tensor o, torch::Tensor lse, torch::Tensor doc_start, int64_t window,
                                       double scale) {
  TORCH_CHECK(q.is_cuda() && q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && o.is_contiguous(),
              "attn_bwd_tc: contiguous CUDA tensors");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16, "attn_bwd_tc: bf16");
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hk = (int)k.size(1), D = (int)q.size(2);
  TORCH_CHECK(Hq % Hk == 0 && v.size(1) == Hk && v.size(2) == D, "attn_bwd_tc: GQA shapes");
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  if (T == 0) return {dq, dk, dv};
  auto doc = dout.contiguous();
  BwdPrep prep = bwd_prep(o, doc, lse, doc_start, T, Hq, D);
  const int Tp = prep.Tp;
  auto opts_i = doc_start.options().dtype(torch::kInt32);
  auto ds32 = doc_start.to(torch::kInt32);
  // doc_end[t] = last token of t's document (reverse cumulative min of the next starts)
  auto idx = torch::arange(T, opts_i);
  auto nxt = torch::where(ds32.eq(idx), idx, torch::full_like(idx, T));
  auto shifted = torch::cat({nxt.slice(0, 1), torch::full({1}, T, opts_i)});
  auto de = (std::get<0>(torch::cummin(shifted.flip(0), 0)).flip(0) - 1).to(torch::kInt32).contiguous();
  auto ds = prep.ds, lse_p = prep.lse, delta = prep.delta;
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = attn_status(q.get_device()).data_ptr<int>();
  switch (D) {
    case 64: bwd_tc_all<64>(q, k, v, doc, lse_p.data_ptr<float>(), delta.data_ptr<float>(), ds.data_ptr<int>(), de.data_ptr<int>(), T, Tp, (int)window, (float)scale, dq, dk, dv, st, stream); break;
    case 128: bwd_tc_all<128>(q, k, v, doc, lse_p.data_ptr<float>(), delta.data_ptr<float>(), ds.data_ptr<int>(), de.data_ptr<int>(), T, Tp, (int)window, (float)scale, dq, dk, dv, st, stream); break;
    case 256: bwd_tc_all<256>(q, k, v, doc, lse_p.data_ptr<float>(), delta.data_ptr<float>(), ds.data_ptr<int>(), de.data_ptr<int>(), T, Tp, (int)window, (float)scale, dq, dk, dv, st, stream); break;
    default: TORCH_CHECK(false, "attn_bwd_tc: head_dim must be 64, 128 or 256");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv};
}

// =============================================================================== backward, tiles in HBM
// Backward for wide heads (head_dim 512: a 128x512 fp32 accumulator fills all of TMEM, and a
// resident 128-row Q + dO pair no longer fits shared memory, so the fused kernels above cannot
// hold it). The 128x128 tiles of P and dS are materialised in HBM as bf16 and the three
// gradients become block-sparse GEMMs without any recomputation:
//   1. attn_bwd_sdp_kernel  one CTA per (query block i, head): for each key block j the
//      document / window allows, S = Q_i K_j^T and dP = dO_i V_j^T (TMEM, double-buffered,
//      K = head_dim streamed in 64-column chunks), then P = exp(scale S - LSE) and
//      dS = P (dP - delta) are written as bf16 tiles in the UMMA K-major 128-byte-swizzled
//      layout (two 128 x 64 chunks per tile), so the next kernel copies them verbatim.
//   2. attn_bwd_acc_kernel  one CTA per (output block, head, 256-column half) of
//      dV = sum P^T dO, dK = scale sum dS^T Q (A operand M-major from the same tiles, summed
//      over the GQA group and every query block that sees the key block) and
//      dQ = scale sum dS K (A K-major); 64-row K slices through a 4-stage TMA / bulk-copy ring.
// Tiles of one head are indexed by off[i] + (j - jlo[i]) (attn_tiles_kernel). Heads are
// processed in passes of whole GQA groups so the tile buffers stay within a byte budget.
// FLOPs: 5 products per tile (the minimum), against 8 in the fused kernels' three passes.
namespace {

constexpr int MT = 128;               // tile rows (queries) = tile columns (keys)
constexpr int TILE_BYTES = MT * MT * 2;  // one bf16 tile: two 128-row x 64-column chunks

// jlo[i]: first key block of query block i; off[i]: index of tile (i, jlo[i]) among one head's
// tiles (exclusive prefix sum of i - jlo[i] + 1), off[nb] = tiles per head; ihi[j]: last query
// block that sees key block j. One block of 1024 threads.
__global__ void attn_tiles_kernel(const int* __restrict__ ds, int nb, int window, int* __restrict__ jlo,
                                  int* __restrict__ off, int* __restrict__ ihi) {
  __shared__ int wsum[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < nb; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int cnt = 0;
    if (i < nb) {
      int ks = ds[i * MT];
      if (window > 0) ks = max(ks, i * MT - window + 1);
      jlo[i] = ks / MT;
      cnt = i - ks / MT + 1;
    }
    int x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = lane < nw ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      wsum[lane] = w;
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? wsum[warp - 1] : 0) + x - cnt;
    if (i < nb) off[i] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + cnt;
    __syncthreads();
  }
  if (threadIdx.x == 0) off[nb] = carry;
  __syncthreads();
  for (int j = threadIdx.x; j < nb; j += blockDim.x) {  // jlo is non-decreasing and jlo[i] <= i
    int lo = j, hi = nb - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (jlo[mid] <= j) lo = mid;
      else hi = mid - 1;
    }
    ihi[j] = lo;
  }
}

template <int D>
struct SdpLayout {
  // head_dim <= 256: Q_i and dO_i stay resident (loaded once per CTA) and the ring streams only
  // K_j / V_j chunks; wider heads stream all four operands chunk by chunk.
  static constexpr bool RES = D <= 256;
  static constexpr int NC = D / 64, NS = 3;
  static constexpr int CH = MT * 128;  // one 128-row x 64-column chunk (16 KB)
  static constexpr int RES_BYTES = RES ? 2 * NC * CH : 0;  // resident Q_i, dO_i
  static constexpr int STAGE = (RES ? 2 : 4) * CH;         // [Q_i, dO_i,] K_j, V_j chunks
  static constexpr int RING_OFF = RES_BYTES;
  static constexpr int BAR_OFF = RING_OFF + NS * STAGE;
  static constexpr int N_BARS = 2 * NS + 2 + 2 + 1;
  static constexpr int BYTES = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static constexpr int THREADS = 320, NEPI = 256;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
  static_assert(BYTES <= 232448, "shared memory");
};

template <int D>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_sdp_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap to,
                        const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                        const float* __restrict__ lse, const float* __restrict__ delta, const int* __restrict__ ds,
                        const int* __restrict__ jlo_a, const int* __restrict__ off_a, int T, int Tp, int nb, int G,
                        int h0, int64_t ntmax, int window, float scale, uint8_t* __restrict__ pbuf,
                        uint8_t* __restrict__ dsbuf, int* status) {
  using L = SdpLayout<D>;
  constexpr int NC = L::NC, NS = L::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = full + NS;
  uint64_t* s_full = empty + NS;
  uint64_t* s_free = s_full + 2;
  uint64_t* r_full = s_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(r_full + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* ring = smem + L::RING_OFF;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x, hl = blockIdx.y, h = h0 + hl, g = h / G;
  const int jlo = jlo_a[i];
  int ntile = i - jlo + 1;
  const int64_t tbase = (int64_t)hl * ntmax + off_a[i];
  if (off_a[nb] > ntmax) {  // the host's bound on tiles per head does not hold: write nothing
    if (threadIdx.x == 0) report(status, ME_ERR_BOUNDS, 70);
    ntile = 0;
  }
  const int nit = ntile * NC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], L::NEPI);
    }
    mbar_init(r_full, 1);
    *abort = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&to);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nit > 0) {
      // ------------------------------------------------------------------ producer
      if (L::RES) {
        mbar_expect_tx(r_full, L::RES_BYTES);
        for (int c = 0; c < NC; ++c) {
          tma_load_3d(smem + c * L::CH, &tq, r_full, c * 64, h, i * MT);
          tma_load_3d(smem + (NC + c) * L::CH, &to, r_full, c * 64, h, i * MT);
        }
      }
      int issued = 0;
      for (int it = 0; it < nit; ++it) {
        const int s = it % NS, c = it % NC, j = jlo + it / NC;
        if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, status, 71, abort)) break;
        uint8_t* st = ring + s * L::STAGE;
        mbar_expect_tx(&full[s], L::STAGE);
        if (!L::RES) {
          tma_load_3d(st, &tq, &full[s], c * 64, h, i * MT);
          tma_load_3d(st + L::CH, &to, &full[s], c * 64, h, i * MT);
          st += 2 * L::CH;
        }
        tma_load_3d(st, &tk, &full[s], c * 64, g, j * MT);
        tma_load_3d(st + L::CH, &tv, &full[s], c * 64, g, j * MT);
        issued = it + 1;
      }
      if (L::RES) mbar_wait(r_full, 0, status, 79, nullptr);  // drain copies in flight
      for (int it = max(0, issued - NS); it < issued; ++it)
        mbar_wait(&full[it % NS], (it / NS) & 1, status, 79, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && nit > 0) {
      // ------------------------------------------------------------------ MMA issuer
      const uint32_t id = idesc_bf16(128, 128);
      bool ok = !L::RES || mbar_wait(r_full, 0, status, 75, abort);
      for (int it = 0; it < nit && ok; ++it) {
        const int s = it % NS, c = it % NC, tt = it / NC, b = tt & 1;
        if (c == 0 && tt >= 2 && !mbar_wait(&s_free[b], ((tt - 2) >> 1) & 1, status, 72, abort)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&full[s], (it / NS) & 1, status, 73, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // A operands: Q_i / dO_i chunk c (resident or in the stage); B operands: K_j / V_j chunk
        const uint32_t st = smem_addr(ring + s * L::STAGE);
        const uint32_t aq = L::RES ? smem_addr(smem + c * L::CH) : st;
        const uint32_t ao = L::RES ? smem_addr(smem + (NC + c) * L::CH) : st + L::CH;
        const uint32_t bk = L::RES ? st : st + 2 * L::CH;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + b * 256, desc_sw128(aq + kk * 32), desc_sw128(bk + kk * 32), id, (c | kk) != 0);
          umma_bf16(tmem + b * 256 + 128, desc_sw128(ao + kk * 32), desc_sw128(bk + L::CH + kk * 32), id,
                    (c | kk) != 0);
        }
        umma_commit(&empty[s]);
        if (c == NC - 1) umma_commit(&s_full[b]);
      }
    }
  } else {
    // ------------------------------------------------------------------ P / dS epilogue
    // warps 2-9: TMEM lane quarter (warp & 3), key half (warp - 2) / 4 = stored chunk
    const int qq = warp & 3, half = (warp - 2) >> 2;
    const int r = qq * 32 + lane, row = i * MT + r;
    const uint32_t lane_base = (uint32_t)(qq * 32) << 16;
    // p = 2^(s * scale * log2(e) - lse * log2(e)): one FFMA + one ex2 per element
    const float sl2 = scale * 1.4426950408889634f;
    float lse2 = INFINITY, delta_r = 0.f;  // rows past T: p = 2^-inf = 0
    int lo_r = 0;
    if (row < T) {
      lse2 = lse[(int64_t)h * Tp + row] * 1.4426950408889634f;
      delta_r = delta[(int64_t)h * Tp + row];
      lo_r = ds[row];
      if (window > 0) lo_r = max(lo_r, row - window + 1);
    }
    for (int tt = 0; tt < ntile; ++tt) {
      const int b = tt & 1, j = jlo + tt;
      if (!mbar_wait(&s_full[b], (tt >> 1) & 1, status, 74, abort)) break;
      tc_fence_after();
      const int64_t tile = tbase + tt;
      uint8_t* prow = pbuf + tile * TILE_BYTES + half * (TILE_BYTES / 2) + r * 128;
      uint8_t* drow = dsbuf + tile * TILE_BYTES + half * (TILE_BYTES / 2) + r * 128;
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        float sv[32], dp[32];
        tmem_ld32(tmem + lane_base + b * 256 + half * 64 + sub * 32, sv);
        tmem_ld32(tmem + lane_base + b * 256 + 128 + half * 64 + sub * 32, dp);
        const int k0 = j * MT + half * 64 + sub * 32;
        if (!(k0 >= lo_r && k0 + 31 <= row)) {  // not every key visible: mask (rows past T have lse2 = inf)
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (k0 + c > row || k0 + c < lo_r) sv[c] = -INFINITY;
        }
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          BF16x8 pk, dk;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c0 = u4 * 8 + 2 * e;
            const float p0 = ex2_approx(fmaf(sv[c0], sl2, -lse2));
            const float p1 = ex2_approx(fmaf(sv[c0 + 1], sl2, -lse2));
            pk.h2[e] = __floats2bfloat162_rn(p0, p1);
            dk.h2[e] = __floats2bfloat162_rn(p0 * (dp[c0] - delta_r), p1 * (dp[c0 + 1] - delta_r));
          }
          const int u = sub * 4 + u4;
          const int pos = (u ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + pos) = pk.u;
          *reinterpret_cast<uint4*>(drow + pos) = dk.u;
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
struct AccLayout {
  // two stages and two CTAs per SM (2 x 97 KB of shared memory, 2 x 256 TMEM columns): while one
  // CTA drains its accumulator the other keeps the tensor pipe fed
  static constexpr int DN = D < 256 ? D : 256, NH = D / DN, NS = 2;
  static constexpr int A_BYTES = 128 * 128;  // 128 M x 64 K (K-major) or 64 K x 128 M (two 8 KB pieces)
  static constexpr int B_BYTES = 64 * DN * 2;  // 64 K rows x DN columns: DN / 64 boxes of 8 KB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BAR_OFF = NS * STAGE;
  static constexpr int N_BARS = 2 * NS + 1;
  static constexpr int BYTES = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = DN;
  static constexpr int THREADS = 192;  // warp 0 loads, warp 1 MMA, warps 2-5 epilogue
  static_assert(STAGE % 1024 == 0, "stages keep the 1024-byte alignment of the swizzle atoms");
  static_assert(BYTES <= 232448, "shared memory");
};

// Job list of one pass: first the dV / dK blocks (kvh kv heads x key blocks x {dV, dK} x NH
// column halves; the longest jobs), then the dQ blocks (kvh * G query heads x query blocks x NH).
template <int D>
__global__ void __launch_bounds__(192, 2)
    attn_bwd_acc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap to,
                        const __grid_constant__ CUtensorMap tk, const int* __restrict__ jlo_a,
                        const int* __restrict__ off_a, const int* __restrict__ ihi_a, int T, int nb, int Hq, int Hk,
                        int G, int g0, int kvh, int64_t ntmax, float scale, const uint8_t* __restrict__ pbuf,
                        const uint8_t* __restrict__ dsbuf, bf16* __restrict__ dq, bf16* __restrict__ dk,
                        bf16* __restrict__ dv, int* status) {
  using L = AccLayout<D>;
  constexpr int NS = L::NS, DN = L::DN, NH = L::NH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = full + NS;
  uint64_t* acc_final = empty + NS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_final + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // ---- job
  int64_t x = blockIdx.x;
  const int64_t J1 = (int64_t)nb * kvh * 2 * NH;
  int kind, half, blk, hsel;  // kind 0 dV, 1 dK, 2 dQ; hsel: kv head (dV/dK) or query head (dQ) in the pass
  if (x < J1) {
    half = (int)(x % NH);
    x /= NH;
    kind = (int)(x % 2);
    x /= 2;
    hsel = (int)(x % kvh);
    blk = (int)(x / kvh);
  } else {
    x -= J1;
    half = (int)(x % NH);
    x /= NH;
    hsel = (int)(x % (kvh * G));
    blk = (int)(x / (kvh * G));
    kind = 2;
  }
  const int n_i = kind == 2 ? 0 : ihi_a[blk] - blk + 1;        // query blocks per head (dV / dK)
  const int jlo_b = kind == 2 ? jlo_a[blk] : 0;
  int ntile = kind == 2 ? blk - jlo_b + 1 : G * n_i;
  if (off_a[nb] > ntmax) {  // every tile index is below off[nb]; past the buffer: zeros out
    if (threadIdx.x == 0) report(status, ME_ERR_BOUNDS, 80);
    ntile = 0;
  }
  const int nit = 2 * ntile;  // two 64-row K slices per tile
  const uint8_t* abuf = kind == 0 ? pbuf : dsbuf;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_final, 1);
    *abort = 0;
    fence_barrier_init();
    prefetch_tmap(kind == 0 ? &to : kind == 1 ? &tq : &tk);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ loads
      int issued = 0;
      for (int it = 0; it < nit; ++it) {
        const int s = it % NS, sl = it & 1, t = it >> 1;
        int64_t tile;
        int brow, bhead;
        const CUtensorMap* bm;
        if (kind == 2) {  // dQ: tile (i = blk, j = jlo + t) of query head hsel; B = K_j rows
          const int j = jlo_b + t;
          tile = (int64_t)hsel * ntmax + off_a[blk] + t;
          brow = j * MT + sl * 64;
          bhead = g0 + hsel / G;
          bm = &tk;
        } else {  // dV / dK: tile (i, j = blk) of query head hl of the group; B = dO_i / Q_i rows
          const int hl = t / n_i, i = blk + t % n_i;
          const int qh = hsel * G + hl;
          tile = (int64_t)qh * ntmax + off_a[i] + (blk - jlo_a[i]);
          brow = i * MT + sl * 64;
          bhead = g0 * G + qh;
          bm = kind == 0 ? &to : &tq;
        }
        if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, status, 81, abort)) break;
        uint8_t* st = smem + s * L::STAGE;
        mbar_expect_tx(&full[s], L::STAGE);
        const uint8_t* src = abuf + tile * TILE_BYTES;
        if (kind == 2) {
          bulk_load(st, src + sl * (TILE_BYTES / 2), TILE_BYTES / 2, &full[s]);
        } else {
          bulk_load(st, src + sl * (TILE_BYTES / 4), TILE_BYTES / 4, &full[s]);
          bulk_load(st + TILE_BYTES / 4, src + TILE_BYTES / 2 + sl * (TILE_BYTES / 4), TILE_BYTES / 4, &full[s]);
        }
#pragma unroll
        for (int cb = 0; cb < DN / 64; ++cb)
          tma_load_3d(st + L::A_BYTES + cb * 8192, bm, &full[s], half * DN + cb * 64, bhead, brow);
        issued = it + 1;
      }
      for (int it = max(0, issued - NS); it < issued; ++it)
        mbar_wait(&full[it % NS], (it / NS) & 1, status, 89, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && nit > 0) {
      // ------------------------------------------------------------------ MMA issuer
      const uint32_t id = idesc_bf16(128, DN, true, kind != 2);
      bool ok = true;
      for (int it = 0; it < nit; ++it) {
        const int s = it % NS;
        if (!mbar_wait(&full[s], (it / NS) & 1, status, 82, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_addr(smem + s * L::STAGE), bq = a + L::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = kind == 2 ? desc_sw128(a + kk * 32) : desc_mn_sw128(a + kk * 2048, 8192, 1024);
          umma_bf16(tmem, ad, desc_mn_sw128(bq + kk * 2048, 8192, 1024), id, (it | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(acc_final);
    }
  } else {
    // ------------------------------------------------------------------ epilogue: one row per thread
    const int qq = warp & 3;
    const int r = qq * 32 + lane, row = blk * MT + r;
    const uint32_t lane_base = (uint32_t)(qq * 32) << 16;
    bf16* dst;
    if (kind == 2) dst = dq + (int64_t)row * Hq * D + (int64_t)(g0 * G + hsel) * D + half * DN;
    else dst = (kind == 0 ? dv : dk) + (int64_t)row * Hk * D + (int64_t)(g0 + hsel) * D + half * DN;
    const float f = kind == 0 ? 1.f : scale;
    if (nit == 0) {
      if (row < T)
        for (int e = 0; e < DN; e += 8) *reinterpret_cast<uint4*>(dst + e) = make_uint4(0, 0, 0, 0);
    } else if (mbar_wait(acc_final, 0, status, 83, abort)) {
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < DN / 32; ++cc) {
        float v[32];
        tmem_ld32(tmem + lane_base + cc * 32, v);
        if (row < T) {
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8) {
            BF16x8 ov;
#pragma unroll
            for (int e = 0; e < 8; ++e) ov.h[e] = f2bf(v[j8 * 8 + e] * f);
            *reinterpret_cast<uint4*>(dst + cc * 32 + j8 * 8) = ov.u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <int D>
void bwd_mat_all(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& dout,
                 const float* lse, const float* delta, const int* ds, int T, int Tp, int window, float scale,
                 int64_t budget, torch::Tensor& dq, torch::Tensor& dk, torch::Tensor& dv, int* status,
                 cudaStream_t stream) {
  const int Hq = (int)q.size(1), Hk = (int)k.size(1), G = Hq / Hk;
  const int nb = (T + MT - 1) / MT;
  auto opts_i = q.options().dtype(torch::kInt32);
  auto meta = torch::empty({3 * nb + 1}, opts_i);
  int* jlo = meta.data_ptr<int>();
  int* off = jlo + nb;  // nb + 1 entries
  int* ihi = off + nb + 1;
  attn_tiles_kernel<<<1, 1024, 0, stream>>>(ds, nb, window, jlo, off, ihi);
  // tiles per head, bounded on the host: every query block sees at most (window + 127) / 128 + 1
  // key blocks (all of 0..i without a window)
  const int64_t per_i = window > 0 ? std::min<int64_t>(nb, (window + MT - 1) / MT + 1) : nb;
  const int64_t ntmax = window > 0 ? nb * per_i : (int64_t)nb * (nb + 1) / 2;
  const int64_t group_bytes = (int64_t)G * ntmax * TILE_BYTES * 2;
  const int kvh = (int)std::max<int64_t>(1, std::min<int64_t>(Hk, budget / std::max<int64_t>(group_bytes, 1)));
  auto buf = torch::empty({(int64_t)kvh * G * ntmax * TILE_BYTES * 2}, q.options().dtype(torch::kUInt8));
  uint8_t* pbuf = buf.data_ptr<uint8_t>();
  uint8_t* dsbuf = pbuf + (int64_t)kvh * G * ntmax * TILE_BYTES;
  const CUtensorMap q128 = make_tmap_thd(q.data_ptr(), T, Hq, D, 128), o128 = make_tmap_thd(dout.data_ptr(), T, Hq, D, 128);
  const CUtensorMap k128 = make_tmap_thd(k.data_ptr(), T, Hk, D, 128), v128 = make_tmap_thd(v.data_ptr(), T, Hk, D, 128);
  const CUtensorMap q64 = make_tmap_thd(q.data_ptr(), T, Hq, D, 64), o64 = make_tmap_thd(dout.data_ptr(), T, Hq, D, 64);
  const CUtensorMap k64 = make_tmap_thd(k.data_ptr(), T, Hk, D, 64);
  using LS = SdpLayout<D>;
  using LA = AccLayout<D>;
  auto ks = attn_bwd_sdp_kernel<D>;
  auto ka = attn_bwd_acc_kernel<D>;
  cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, LS::BYTES);
  cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, LA::BYTES);
  bf16* pdq = reinterpret_cast<bf16*>(dq.data_ptr());
  bf16* pdk = reinterpret_cast<bf16*>(dk.data_ptr());
  bf16* pdv = reinterpret_cast<bf16*>(dv.data_ptr());
  for (int g0 = 0; g0 < Hk; g0 += kvh) {
    const int n = std::min(kvh, Hk - g0);
    ks<<<dim3(nb, n * G), LS::THREADS, LS::BYTES, stream>>>(q128, o128, k128, v128, lse, delta, ds, jlo, off, T, Tp,
                                                             nb, G, g0 * G, ntmax, window, scale, pbuf, dsbuf, status);
    const int64_t jobs = (int64_t)nb * n * 2 * LA::NH + (int64_t)nb * n * G * LA::NH;
    ka<<<(unsigned)jobs, LA::THREADS, LA::BYTES, stream>>>(q64, o64, k64, jlo, off, ihi, T, nb, Hq, Hk, G, g0, n,
                                                           ntmax, scale, pbuf, dsbuf, pdq, pdk, pdv, status);
  }
}

}  // namespace

// dq, dk, dv of the packed-varlen attention (head_dim 256 / 512) through P / dS tiles in HBM;
// `tile_budget_bytes` bounds the tile buffers (whole GQA groups per pass, at least one).
std::vector<torch::Tensor> attn_bwd_mat(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                        torch::Tensor o, torch::Tensor lse, torch::Tensor doc_start, int64_t window,
                                        double scale, int64_t tile_budget_bytes) {
  TORCH_CHECK(q.is_cuda() && q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && o.is_contiguous(),
              "attn_bwd_mat: contiguous CUDA tensors");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16, "attn_bwd_mat: bf16");
  const at::cuda::CUDAGuard guard(q.device());
  const int T = (int)q.size(0), Hq = (int)q.size(1), Hk = (int)k.size(1), D = (int)q.size(2);
  TORCH_CHECK(Hq % Hk == 0 && v.size(1) == Hk && v.size(2) == D, "attn_bwd_mat: GQA shapes");
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  if (T == 0) return {dq, dk, dv};
  auto doc = dout.contiguous();
  BwdPrep prep = bwd_prep(o, doc, lse, doc_start, T, Hq, D);
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = attn_status(q.get_device()).data_ptr<int>();
  switch (D) {
    case 256: bwd_mat_all<256>(q, k, v, doc, prep.lse.data_ptr<float>(), prep.delta.data_ptr<float>(), prep.ds.data_ptr<int>(), T, prep.Tp, (int)window, (float)scale, tile_budget_bytes, dq, dk, dv, st, stream); break;
    case 512: bwd_mat_all<512>(q, k, v, doc, prep.lse.data_ptr<float>(), prep.delta.data_ptr<float>(), prep.ds.data_ptr<int>(), T, prep.Tp, (int)window, (float)scale, tile_budget_bytes, dq, dk, dv, st, stream); break;
    default: TORCH_CHECK(false, "attn_bwd_mat: head_dim must be 256 or 512");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv};
}
