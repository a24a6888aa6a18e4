// Persistent tcgen05 GEMM for sm_100a on CTA pairs: D[M, N] = A[M, K] . B^T, bf16 operands,
// fp32 accumulation in tensor memory, with the epilogue fused for the decoder's projections.
//
// Shape of the work. A 2-CTA cluster owns one 256 x 256 output tile at a time: the even CTA
// (leader) issues tcgen05.mma.cta_group::2 with M=256, N=256, K=16; each CTA stages its own 128
// rows of A (K-major, or M-major for A^T . B products such as weight gradients) and its own 128
// rows of B (K-major or N-major) in a STAGES-deep ring of 128-byte-
// swizzled shared-memory stages, and each CTA's tensor memory receives its 128 rows of D. The
// grid is one cluster per pair of SMs that can be resident at once; clusters walk the tile list
// with a fixed stride (grouped raster: `group_m` M tiles side by side so that concurrently
// running tiles share A rows and B rows in L2).
//
// Warp roles (192 threads per CTA):
//   warp 0     TMA producer (one thread, both CTAs): per stage, wait until the stage is free
//              (the leader's MMA commit arrives on both CTAs' `empty` barriers), then load this
//              CTA's A and B halves; completion is counted on the LEADER's `full` barrier, which
//              the leader arms with the byte count of both halves. No multicast loads.
//   warp 1     TMEM owner in both CTAs (tcgen05.alloc.cta_group::2, 512 columns = two 256-column
//              accumulators); in the leader one thread issues the MMAs, releases stages with
//              tcgen05.commit to both CTAs, and signals `acc_full` on both CTAs per tile.
//   warp 6     side copy (optional): a range of a peer-to-local copy job (the next frozen layer's
//              all-gather under base_placement: sharded, gather.cuh) runs here while the tensor
//              cores work, so the layer's all-gather costs no separate kernel and no idle SMs
//   warps 7-10 NF4 B producer (B_NF4 only, 352 threads per CTA): the frozen weight stays in NF4
//              (4-bit codes, one fp32 absmax per 64 weights along its rows) and these 128 threads
//              dequantise this CTA's B half of every stage straight into the 128-byte-swizzled
//              layout the TMA would have written (one 128-byte row each: 32 code bytes + 1
//              absmax -> 64 bf16, bf16(level * absmax) exactly as the standalone dequant kernel
//              rounds), fence the generic-proxy stores for the tensor core, and arrive on the
//              leader's `full` barrier (which then counts 3 arrivals: the A expect_tx + one per
//              CTA). Loads run two stages ahead of the stores. So the bf16 weight never exists.
//   warps 2-5  epilogue (each warp owns the TMEM lane quarter warp % 4 = 32 rows): wait for
//              `acc_full`, tcgen05.ld 32 columns at a time, apply the epilogue, store, then
//              arrive on the leader's `acc_empty` so the next-but-one tile can reuse the
//              accumulator. Two accumulators let the epilogue of tile i overlap the MMAs of
//              tile i+1.
//
// Epilogues:
//   STORE    D = bf16(acc)
//   GEGLU    B = the fused [gate; up] weight [2F, K]; for a tile of 128 features the leader's
//            B half is gate rows f0.., the peer's is up rows F+f0.., so every thread holds both
//            for its row: m = bf16(bf16(gelu_tanh(g)) * u) with g, u rounded to bf16 first (the
//            numerics of the separate GEMM + GeGLU kernels); optionally also stores gu = [g | u]
//            for the backward.
//   DGEGLU   acc = dL/dm for 256 features; reads gu of the row and writes
//            d_gu = [bf16(dm * u * gelu'(g)) | bf16(dm * bf16(gelu(g)))].
//   F32      D = acc in fp32 (the LM head's dH, reduced across ranks in fp32); with peer_out set,
//            each row is stored straight into its token owner's receive slot on that GPU.
//   CE       logits of the tied head against this rank's vocab rows: z = bf16(acc) (stored only
//            when the backward needs it), zc = softcap(z); per (row, tile) the partial sum of
//            exp(zc - m) with m = the cap itself when softcapping (|zc| <= cap, so no running max
//            is needed and every tile and rank shares the offset) or the tile's max otherwise;
//            the target logit is written by the one tile that holds the row's label. Full-row
//            logits are never read back for the loss.
//
// Every mbarrier wait is bounded (%globaltimer, 2 s). On expiry the kernel records
// ME_ERR_TIMEOUT in the status word, every role of the CTA stops, in-flight copies and MMAs are
// waited for (again bounded), both CTAs meet at one cluster barrier, TMEM is freed and the
// kernel returns. No trap, no device assert.
#pragma once

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "act.cuh"
#include "gather.cuh"
#include "tc_common.cuh"

namespace me {
namespace gemm {
using namespace me::tc;
using bf16 = __nv_bfloat16;

constexpr int BM = 128;  // A rows per CTA (256 per pair)
constexpr int BN = 256;  // accumulator columns per tile
constexpr int BK = 64;   // K per stage (one 128-byte swizzle row of bf16)
constexpr int NTHREADS = 224;
constexpr int NTHREADS_NF4 = 352;  // + 4 warps dequantising the NF4 B operand
constexpr uint32_t TMEM_COLS = 512;  // two accumulators
constexpr int A_BYTES = BM * BK * 2;        // 16 KB
constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KB: this CTA's half of B
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;

enum Epi : int { EPI_STORE = 0, EPI_GEGLU = 1, EPI_DGEGLU = 2, EPI_F32 = 3, EPI_CE = 4 };
constexpr int64_t kIgnoreIndex = -100;

struct GemmArgs {
  bf16* D;              // STORE: [M, N]; GEGLU: m [M, F]; DGEGLU: d_gu [M, 2F]
  int64_t ldd;
  bf16* D2;             // GEGLU: gu [M, 2F] (may be null)
  int64_t ldd2;
  const bf16* aux;      // DGEGLU: gu [M, 2F]
  int64_t ld_aux;
  float* Df;            // F32: [M, N]
  // F32 with a peer-scattered output (the fused reduce-scatter of the LM head's dH): row r of D
  // belongs to rank r / peer_rows and goes to that rank's receive buffer peer_out[rank] at slot
  // `peer_slot` (this rank), row r % peer_rows; plain 16-byte stores over NVLink
  const int64_t* peer_out;
  int peer_rows;
  int64_t peer_slot_elems;
  int peer_slot;
  const int64_t* labels;  // CE: [M]
  int64_t lab_start;    // CE: first vocab id of this rank's rows
  float cap;            // CE: softcap (0 = none)
  float* s_part;        // CE: [M, tiles_n] partial sums of exp(zc - m)
  float* m_part;        // CE: [M, tiles_n] partial offsets m (only without softcap)
  float* tgt;           // CE: [M] softcapped target logit (left untouched when not in this shard)
  int M, N, K;          // N: output columns (GEGLU / DGEGLU: F)
  int tiles_m, tiles_n, group_m;
  // Split-K tail (STORE / F32): the first dp_tiles tiles run whole; the last (ntiles - dp_tiles)
  // tiles are cut into `splits` K ranges each (tail_units units, at most one per cluster). Each
  // unit writes its fp32 partial to its own slice ws[tail tile][split][256][256]; the last unit
  // to finish a 32-row slice (counted in `cnt`, which starts at zero) sums the splits in split
  // order and stores the result, so the tail is as deterministic as the rest of the GEMM.
  int dp_tiles, tail_units, splits;
  int split_one_wave;   // host only: also split a single partial wave (small-M F32 products)
  float* ws;
  int* cnt;
  // side copy carried by warp 6: units [gbegin16, gend16) of the segment table gsegs
  const GatherSeg* gsegs;
  int gnsegs;
  int64_t gbegin16, gend16;
  int* status;
  // B_NF4: the weight W [q_rows, q_cols] (row-major, two 4-bit codes per byte, low nibble first,
  // one fp32 absmax per 64 consecutive weights of a row; q_cols % 64 == 0). K-major B reads W's
  // rows as B rows (y = x . W^T); N-major B reads W's rows as the reduction dimension (dX = g . W).
  const uint8_t* q_codes;
  const float* q_absmax;
  int64_t q_rows, q_cols;
};

// The 16 NF4 levels (QLoRA, Dettmers et al. 2023, appendix E), the table nf4.cu quantises with.
static __constant__ float kNF4Levels[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                                     -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                                     0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f,
                                     0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f,
                                     0.7229568362236023f, 1.0f};

struct Unit {
  int tile, kb0, kb1, part;  // part < 0: the whole tile
};

// The w-th unit of work in the cluster-strided order (false past the end).
ME_DEVICE bool unit_at(int w, const GemmArgs& p, int nk, Unit& u) {
  if (w < p.dp_tiles) {
    u.tile = w;
    u.kb0 = 0;
    u.kb1 = nk;
    u.part = -1;
    return true;
  }
  const int x = w - p.dp_tiles;
  if (x >= p.tail_units) return false;
  u.tile = p.dp_tiles + x / p.splits;
  u.part = x % p.splits;
  u.kb0 = (int)((int64_t)nk * u.part / p.splits);
  u.kb1 = (int)((int64_t)nk * (u.part + 1) / p.splits);
  return true;
}

template <int STAGES>
struct Smem {
  static constexpr int TILES = STAGES * STAGE_BYTES;
  static constexpr int BYTES = TILES + 1024 /*alignment*/ + 512 /*barriers*/;
};

ME_DEVICE void tile_coords(int t, const GemmArgs& p, int& mb, int& nb) {
  const int per_group = p.group_m * p.tiles_n;
  const int g = t / per_group, first = g * p.group_m;
  const int gsz = min(p.tiles_m - first, p.group_m);
  const int r = t - g * per_group;
  mb = first + r % gsz;
  nb = r / gsz;
}

// Destination of row `row` of an fp32 output: local, or a peer's receive slot.
ME_DEVICE float* f32_row(const GemmArgs& p, int row) {
  if (p.peer_out == nullptr) return p.Df + (int64_t)row * p.ldd;
  const int owner = row / p.peer_rows;
  float* base = reinterpret_cast<float*>(p.peer_out[owner]) + (int64_t)p.peer_slot * p.peer_slot_elems;
  return base + (int64_t)(row - owner * p.peer_rows) * p.ldd;
}

ME_DEVICE void store_row32(bf16* dst, const float (&v)[32], int valid_cols) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (j * 8 < valid_cols) {
      BF16x8 o;
#pragma unroll
      for (int e = 0; e < 8; ++e) o.h[e] = f2bf(v[j * 8 + e]);
      *reinterpret_cast<uint4*>(dst + j * 8) = o.u;
    }
  }
}

// One 64-weight NF4 segment of a B row (32 code bytes and its absmax), fetched ahead of use.
struct Nf4Seg {
  uint4 lo, hi;
  float scale;
  bool valid;
};

// The k-block sequence of this cluster (same order as the producer and the MMA issuer).
struct KCursor {
  int w, kb;
  Unit u;
  bool have;
  ME_DEVICE void start(int cluster, const GemmArgs& p, int nk) {
    w = cluster;
    have = unit_at(w, p, nk, u);
    kb = have ? u.kb0 : 0;
  }
  ME_DEVICE void next(int nclusters, const GemmArgs& p, int nk) {
    if (++kb >= u.kb1) {
      w += nclusters;
      have = unit_at(w, p, nk, u);
      kb = have ? u.kb0 : 0;
    }
  }
};

template <int EPI, bool B_NMAJOR, bool A_MMAJOR, int STAGES, bool B_NF4 = false>
__global__ void __launch_bounds__(B_NF4 ? NTHREADS_NF4 : NTHREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     const GemmArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Smem<STAGES>::TILES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2], leader only
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* nf4_stop = reinterpret_cast<volatile int*>(tmem_slot + 2);
  float* nf4_lut = reinterpret_cast<float*>(smem + Smem<STAGES>::TILES + 256);  // 16 levels

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], B_NF4 ? 3 : 1);  // NF4: + one arrival per CTA's dequantising warps
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    fence_barrier_init();
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      const uint32_t full_leader = mapa_shared(smem_addr(full), 0);
      int it = 0;  // global k-block counter of this CTA
      bool ok = true;
      Unit u;
      for (int w = cluster; ok && unit_at(w, p, nk, u); w += nclusters) {
        int mb, nb;
        tile_coords(u.tile, p, mb, nb);
        const int a_row = mb * 2 * BM + (int)rank * BM;
        int b_row;  // K-major: first B row of this CTA's half; N-major: first output column
        if (EPI == EPI_GEGLU) b_row = (int)rank * p.N + nb * (BN / 2);
        else b_row = nb * BN + (int)rank * (BN / 2);
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
          const int s = it % STAGES, r = it / STAGES;
          if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, p.status, 10, abort)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full[s], B_NF4 ? 2 * A_BYTES : 2 * STAGE_BYTES);
          const uint32_t bar = full_leader + (uint32_t)(s * 8);
          if (A_MMAJOR) {  // A stored [K, M]: two 64-row (M) x 64 (K) boxes per half
            tma_load_2d_pair(sA + s * A_BYTES, &ta, bar, a_row, kb * BK);
            tma_load_2d_pair(sA + s * A_BYTES + A_BYTES / 2, &ta, bar, a_row + 64, kb * BK);
          } else {
            tma_load_2d_pair(sA + s * A_BYTES, &ta, bar, kb * BK, a_row);
          }
          if (B_NF4) {
            // B comes from the dequantising warps
          } else if (B_NMAJOR) {
            tma_load_2d_pair(sB + s * B_BYTES, &tb, bar, b_row, kb * BK);
            tma_load_2d_pair(sB + s * B_BYTES + B_BYTES / 2, &tb, bar, b_row + 64, kb * BK);
          } else {
            tma_load_2d_pair(sB + s * B_BYTES, &tb, bar, kb * BK, b_row);
          }
        }
      }
      // Drain: every stage this CTA filled is released again by the leader's commits (normal
      // path), so no copy or commit is still in flight towards this CTA when it exits.
      const int first = it > STAGES ? it - STAGES : 0;
      for (int j = first; j < it; ++j) {
        if (*abort && !leader) break;
        mbar_wait(&empty[j % STAGES], (j / STAGES) & 1, p.status, 11, abort, 500000000ull);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t idesc = idesc_bf16(2 * BM, BN, B_NMAJOR, A_MMAJOR);
      int it = 0, local = 0;
      bool ok = true;
      Unit u;
      for (int w = cluster; ok && unit_at(w, p, nk, u); w += nclusters, ++local) {
        const int acc = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait_cluster(&acc_empty[acc], (use - 1) & 1, p.status, 12, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
          const int s = it % STAGES, r = it / STAGES;
          if (!mbar_wait(&full[s], r & 1, p.status, 13, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + s * A_BYTES), b0 = smem_addr(sB + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t bd = B_NMAJOR ? desc_mn_sw128(b0 + k * 2048, B_BYTES / 2, 1024) : desc_sw128(b0 + k * 32);
            const uint64_t ad = A_MMAJOR ? desc_mn_sw128(a0 + k * 2048, A_BYTES / 2, 1024) : desc_sw128(a0 + k * 32);
            umma_bf16_pair(d, ad, bd, idesc, (kb != u.kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[s], 0x3);
        }
        if (ok) umma_commit_pair(&acc_full[acc], 0x3);
      }
      // every MMA issued has completed before TMEM can be freed
      umma_commit_pair(mma_done, 0x1);
      mbar_wait(mma_done, 0, p.status, 14, nullptr, 500000000ull);
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------------ side copy
    if (p.gnsegs > 0) gather_range(p.gsegs, p.gnsegs, p.gbegin16, p.gend16, blockIdx.x, gridDim.x, lane);
  } else if (B_NF4 && warp >= 7) {
    // ------------------------------------------------------------------ NF4 B producer
    const int t = threadIdx.x - 7 * 32;  // 0..127: one 128-byte row of this CTA's B half
    if (t < 16) nf4_lut[t] = kNF4Levels[t];
    if (t == 0) *nf4_stop = 0;
    named_sync(1, 128);
    const uint32_t full_leader = mapa_shared(smem_addr(full), 0);
    const int64_t cbytes = p.q_cols / 2, blocks = p.q_cols / 64;
    // where this thread's row of the stage comes from (W row, first column) and goes to
    int srow_in_atom;
    uint32_t dst_off;
    if (B_NMAJOR) {
      srow_in_atom = t & 63;
      dst_off = (uint32_t)((t >> 6) * (B_BYTES / 2) + (t & 63) * 128);
    } else {
      srow_in_atom = t;
      dst_off = (uint32_t)(t * 128);
    }
    auto fetch = [&](const KCursor& c, Nf4Seg& g) {
      int mb, nb;
      tile_coords(c.u.tile, p, mb, nb);
      int64_t row, col;
      if (B_NMAJOR) {
        row = (int64_t)c.kb * BK + (t & 63);
        col = (int64_t)nb * BN + (int64_t)rank * (BN / 2) + (t >> 6) * 64;
      } else {
        row = EPI == EPI_GEGLU ? (int64_t)rank * p.N + (int64_t)nb * (BN / 2) + t
                               : (int64_t)nb * BN + (int64_t)rank * (BN / 2) + t;
        col = (int64_t)c.kb * BK;
      }
      g.valid = row < p.q_rows && col < p.q_cols;
      if (g.valid) {
        const uint4* src = reinterpret_cast<const uint4*>(p.q_codes + row * cbytes + col / 2);
        g.lo = __ldg(src);
        g.hi = __ldg(src + 1);
        g.scale = __ldg(p.q_absmax + row * blocks + col / 64);
      }
    };
    KCursor ld, use;
    ld.start(cluster, p, nk);
    use.start(cluster, p, nk);
    Nf4Seg s0{}, s1{};
    if (ld.have) {
      fetch(ld, s0);
      ld.next(nclusters, p, nk);
    }
    if (ld.have) {
      fetch(ld, s1);
      ld.next(nclusters, p, nk);
    }
    for (int it = 0; use.have; use.next(nclusters, p, nk), ++it) {
      const Nf4Seg cur = s0;
      s0 = s1;
      if (ld.have) {
        fetch(ld, s1);
        ld.next(nclusters, p, nk);
      }
      const int s = it % STAGES, r = it / STAGES;
      if (t == 0 && r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, p.status, 16, abort)) *nf4_stop = 1;
      named_sync(1, 128);
      if (*nf4_stop) break;
      uint8_t* dst = sB + s * B_BYTES + dst_off;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (cur.valid) {
          const uint32_t w4 = c < 4 ? (&cur.lo.x)[c] : (&cur.hi.x)[c - 4];
          uint32_t packed[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t byte = (w4 >> (8 * j)) & 0xFFu;
            const __nv_bfloat162 two = __floats2bfloat162_rn(nf4_lut[byte & 15u] * cur.scale,
                                                             nf4_lut[byte >> 4] * cur.scale);
            packed[j] = *reinterpret_cast<const uint32_t*>(&two);
          }
          out = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
        *reinterpret_cast<uint4*>(dst + ((c ^ (srow_in_atom & 7)) * 16)) = out;
      }
      fence_async_smem();  // the tensor core reads these stores through the async proxy
      named_sync(1, 128);
      if (t == 0) mbar_arrive_cluster(full_leader + (uint32_t)(s * 8));
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const uint32_t acc_empty_leader = mapa_shared(smem_addr(acc_empty), 0);
    int local = 0;
    Unit u;
    for (int w = cluster; unit_at(w, p, nk, u); w += nclusters, ++local) {
      const int acc = local & 1, use = local >> 1;
      // every lane waits; the warp leaves together if any lane gave up (tcgen05.ld is .aligned)
      const bool ok = mbar_wait(&acc_full[acc], use & 1, p.status, 15, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(u.tile, p, mb, nb);
      const int row = mb * 2 * BM + (int)rank * BM + q * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const bool row_ok = row < p.M;
      if ((EPI == EPI_STORE || EPI == EPI_F32) && u.part >= 0) {
        // split-K tail unit: write this K range's partial to its own workspace slice; the last of
        // the `splits` units to finish these 32 rows sums all slices in order and stores them
        const int tt = u.tile - p.dp_tiles;
        const int64_t rowi = (int64_t)(int)rank * BM + q * 32 + lane;
        const int64_t slice = (int64_t)(2 * BM) * BN;
        float* mine = p.ws + ((int64_t)tt * p.splits + u.part) * slice + rowi * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(reinterpret_cast<float4*>(mine + c * 32 + j * 4),
                   make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]));
        }
        __threadfence();
        __syncwarp();
        int done = 0;
        if (lane == 0) done = atomicAdd(p.cnt + tt * 8 + (int)rank * 4 + q, 1);
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done == p.splits - 1) {
          __threadfence();
          const float* first = p.ws + (int64_t)tt * p.splits * slice + rowi * BN;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            const int col = nb * BN + c * 32;
            if (row_ok && col < p.N) {
              float v[32];
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = 0.f;
              for (int sp = 0; sp < p.splits; ++sp) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float4 f = __ldcg(reinterpret_cast<const float4*>(first + sp * slice + c * 32 + j * 4));
                  v[j * 4] += f.x;
                  v[j * 4 + 1] += f.y;
                  v[j * 4 + 2] += f.z;
                  v[j * 4 + 3] += f.w;
                }
              }
              if (EPI == EPI_STORE) {
                store_row32(p.D + (int64_t)row * p.ldd + col, v, p.N - col);
              } else {
                float* dst = f32_row(p, row) + col;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  if (col + j * 4 < p.N)
                    *reinterpret_cast<float4*>(dst + j * 4) =
                        make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
              }
            }
          }
        }
      } else if (EPI == EPI_STORE) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int col = nb * BN + c * 32;
          if (row_ok && col < p.N) store_row32(p.D + (int64_t)row * p.ldd + col, v, p.N - col);
        }
      } else if (EPI == EPI_GEGLU) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          float g[32], u[32];
          tmem_ld32(tbase + c * 32, g);
          tmem_ld32(tbase + BN / 2 + c * 32, u);
          const int f = nb * (BN / 2) + c * 32;
          if (row_ok && f < p.N) {
            float mv[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              g[e] = bf2f(f2bf(g[e]));
              u[e] = bf2f(f2bf(u[e]));
              mv[e] = bf2f(f2bf(gelu_tanh(g[e]))) * u[e];
            }
            store_row32(p.D + (int64_t)row * p.ldd + f, mv, p.N - f);
            if (p.D2 != nullptr) {
              store_row32(p.D2 + (int64_t)row * p.ldd2 + f, g, p.N - f);
              store_row32(p.D2 + (int64_t)row * p.ldd2 + p.N + f, u, p.N - f);
            }
          }
        }
      } else if (EPI == EPI_F32) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int col = nb * BN + c * 32;
          if (row_ok && col < p.N) {
            float* dst = f32_row(p, row) + col;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (col + j * 4 < p.N)
                *reinterpret_cast<float4*>(dst + j * 4) = make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
          }
        }
      } else if (EPI == EPI_CE) {
        const int64_t lab = row_ok ? p.labels[row] : kIgnoreIndex;
        const int64_t loc = lab != kIgnoreIndex ? lab - p.lab_start : -1;
        const int n0 = nb * BN;
        const bool capped = p.cap > 0.f;
        float m = capped ? p.cap : -INFINITY, s = 0.f, tv = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + c * 32, v);
          const int col = n0 + c * 32;
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = bf2f(f2bf(v[e]));
          if (p.D != nullptr && row_ok && col < p.N) store_row32(p.D + (int64_t)row * p.ldd + col, v, p.N - col);
          const int valid = p.N - col;
          if (capped) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (e < valid) {
                const float zc = softcap_fast(v[e], p.cap);
                s += exp2_fast((zc - p.cap) * kLog2e);
                if (col + e == loc) tv = zc;
              }
            }
          } else {
            float cm = -INFINITY;
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (e < valid) cm = fmaxf(cm, v[e]);
            if (cm > -INFINITY) {
              float cs = 0.f;
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                if (e < valid) cs += exp2_fast((v[e] - cm) * kLog2e);
                if (col + e == loc) tv = v[e];
              }
              const float mx = fmaxf(m, cm);
              s = s * exp2_fast((m - mx) * kLog2e) + cs * exp2_fast((cm - mx) * kLog2e);
              m = mx;
            }
          }
        }
        if (row_ok) {
          p.s_part[(int64_t)row * p.tiles_n + nb] = s;
          if (!capped) p.m_part[(int64_t)row * p.tiles_n + nb] = m;
          if (loc >= n0 && loc < n0 + BN && loc < p.N) p.tgt[row] = tv;
        }
      } else {  // EPI_DGEGLU
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float dm[32];
          tmem_ld32(tbase + c * 32, dm);
          const int f = nb * BN + c * 32;
          if (row_ok && f < p.N) {
            const bf16* gp = p.aux + (int64_t)row * p.ld_aux + f;
            float og[32], ou[32];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (f + j * 8 < p.N) {
                BF16x8 gv, uv;
                gv.u = *reinterpret_cast<const uint4*>(gp + j * 8);
                uv.u = *reinterpret_cast<const uint4*>(gp + p.N + j * 8);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const float x = bf2f(gv.h[e]), up = bf2f(uv.h[e]), dd = bf2f(f2bf(dm[j * 8 + e]));
                  og[j * 8 + e] = dd * up * gelu_tanh_grad(x);
                  ou[j * 8 + e] = dd * bf2f(f2bf(gelu_tanh(x)));
                }
              }
            }
            store_row32(p.D + (int64_t)row * p.ldd + f, og, p.N - f);
            store_row32(p.D + (int64_t)row * p.ldd + p.N + f, ou, p.N - f);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + (uint32_t)(acc * 8));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs done with every MMA, copy and remote arrive
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host: tensor maps
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  TORCH_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 2-D bf16 tensor [rows, cols] (row stride ld elements), box box_cols x box_rows, 128B swizzle.
inline CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA operand base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  bind_primary_context();
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return map;
}

inline torch::Tensor& status_buffer(int dev) {
  static std::unordered_map<int, torch::Tensor> bufs;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  auto it = bufs.find(dev);
  if (it == bufs.end())
    it = bufs.emplace(dev, torch::zeros({2}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev)))
             .first;
  return it->second;
}

constexpr int STAGES = 7;

// A side-copy job handed to the next GEMM launched on a device (gemm_carry_copy), then cleared.
struct SideCopy {
  const GatherSeg* segs = nullptr;
  int nsegs = 0;
  int64_t begin16 = 0, end16 = 0;
};
inline SideCopy& pending_copy(int dev) {
  static SideCopy jobs[64];
  return jobs[dev & 63];
}

template <int EPI, bool B_NMAJOR, bool A_MMAJOR = false, bool B_NF4 = false>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int dev, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<EPI, B_NMAJOR, A_MMAJOR, STAGES, B_NF4>;
  constexpr int nthreads = B_NF4 ? NTHREADS_NF4 : NTHREADS;
  constexpr int smem = Smem<STAGES>::BYTES;
  // max resident clusters of this kernel on this device, computed once per (kernel, device)
  static std::mutex mu;
  static std::unordered_map<int, int> resident;
  int nclusters;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = resident.find(dev);
    if (it == resident.end()) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      TORCH_CHECK(e == cudaSuccess, "gemm: cudaFuncSetAttribute failed: ", cudaGetErrorString(e));
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cfg.gridDim = dim3(sms & ~1);
      cfg.blockDim = dim3(nthreads);
      cfg.dynamicSmemBytes = smem;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = sms / 2;
      }
      it = resident.emplace(dev, n).first;
    }
    nclusters = it->second;
  }
  GemmArgs a = args;
  SideCopy& job = pending_copy(dev);
  a.gsegs = job.segs;
  a.gnsegs = job.nsegs;
  a.gbegin16 = job.begin16;
  a.gend16 = job.end16;
  job = SideCopy{};
  const int ntiles = a.tiles_m * a.tiles_n;
  const int nk = (a.K + BK - 1) / BK;
  a.dp_tiles = ntiles;
  a.tail_units = 0;
  a.splits = 1;
  torch::Tensor ws, cnt;
  const int rem = ntiles % nclusters;
  if ((EPI == EPI_STORE || EPI == EPI_F32) && (ntiles > nclusters || a.split_one_wave) && rem > 0 &&
      2 * rem <= nclusters) {
    // the last partial wave would leave most SMs idle: split its tiles along K instead
    const int splits = std::min(nclusters / rem, std::max(1, nk / 4));
    if (splits >= 2) {
      a.dp_tiles = ntiles - rem;
      a.splits = splits;
      a.tail_units = rem * splits;
      auto dev_opt = torch::TensorOptions().device(torch::kCUDA, dev);
      ws = torch::empty({(int64_t)rem * splits * 2 * BM * BN}, dev_opt.dtype(torch::kFloat32));
      cnt = torch::zeros({(int64_t)rem * 8}, dev_opt.dtype(torch::kInt32));
      a.ws = ws.data_ptr<float>();
      a.cnt = cnt.data_ptr<int>();
    }
  }
  const int grid_clusters = std::max(1, std::min(nclusters, a.dp_tiles + a.tail_units));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * grid_clusters);
  cfg.blockDim = dim3(nthreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, a);
  TORCH_CHECK(e == cudaSuccess, "gemm: launch failed: ", cudaGetErrorString(e));
}

inline void check_operand(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.dim() == 2, "gemm: ", name,
              " must be a 2-D bf16 CUDA tensor");
  TORCH_CHECK(t.stride(1) == 1, "gemm: ", name, " must have unit column stride");
  TORCH_CHECK(t.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "gemm: ", name,
              " rows must be 16-byte aligned");
}

inline int group_for(int tiles_m) {
  // About 74 tiles run at once. M tiles side by side in groups of `g` make a wave of about
  // g x (74 / g) tiles: every B tile of the wave is read by g tiles at the same time and stays
  // in L2 while they do; B is streamed from HBM tiles_m / g times in all. ME_GEMM_GROUP_M
  // overrides the default (for tuning).
  static const int forced = [] {
    const char* e = std::getenv("ME_GEMM_GROUP_M");
    return e ? std::atoi(e) : 0;
  }();
  const int g = forced > 0 ? forced : 16;
  return std::max(1, std::min(g, tiles_m));
}

inline GemmArgs base_args(int M, int N, int K, int tiles_n, int dev) {
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles_m = (M + 2 * BM - 1) / (2 * BM);
  a.tiles_n = tiles_n;
  a.group_m = group_for(a.tiles_m);
  a.status = status_buffer(dev).data_ptr<int>();
  return a;
}

}  // namespace gemm
}  // namespace me
