// Engram kernels for sm_100a: n-gram hashing, table-row gather from the row owners (local
// or NVLink peer memory), the gated residual injection (forward and backward), the push of
// row gradients into the owners' accumulators, and the touched-row AdamW with stochastic
// rounding.
//
// Behaviour mirrors the reference PyTorch engram (micro_engram/module.py:183-265 for hash
// and gate, micro_engram/rows.py:76-147 for the row exchange, micro_engram/optim.py:65-133
// for the optimizer); the B200 design replaces the all_to_all + host sync exchange with
// direct peer loads/stores/atomics through a table of per-rank base pointers, so no host
// round trip sits inside the step.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

using namespace me;

namespace {

constexpr int64_t kPrime = 2147483647LL;  // 2^31 - 1

ME_DEVICE int64_t floor_mod(int64_t x, int64_t m) {
  int64_t r = x % m;
  return r < 0 ? r + m : r;
}

// ------------------------------------------------------------------------------ hash
// ids [B, T]; pos [B, T] or null. out [n_tables, B*T].
// token t-i of the n-gram: canon[clamp(ids[t-i])], or the RAW pad id when t-i < 0 or the
// document started after it (pos[t] < i).
__global__ void hash_kernel(const int64_t* __restrict__ ids, const int64_t* __restrict__ pos,
                            int64_t B, int64_t T, const int64_t* __restrict__ canon, int64_t V,
                            const int64_t* __restrict__ mults, int n_tables, int max_order,
                            const int* __restrict__ orders, const int64_t* __restrict__ rows,
                            int64_t pad_id, int64_t* __restrict__ out) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= B * T) return;
  const int64_t b = n / T, t = n % T;
  int64_t tok[8];
  const int64_t p = pos ? pos[n] : INT64_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i >= max_order) break;
    if (t - i < 0 || (i > 0 && p < i)) {
      tok[i] = pad_id;
    } else {
      int64_t id = ids[b * T + t - i];
      id = id < 0 ? 0 : (id >= V ? V - 1 : id);
      tok[i] = canon[id];
    }
  }
  for (int k = 0; k < n_tables; ++k) {
    const int ord = orders[k];
    int64_t x = 0;
    for (int i = 0; i < ord; ++i) x += tok[i] * mults[k * max_order + i];
    out[(int64_t)k * B * T + n] = floor_mod(floor_mod(x, kPrime), rows[k]);
  }
}

// ids [N, max_order]: column i is the token at t-i, -1 where there is none.
__global__ void hash_prev_kernel(const int64_t* __restrict__ ids, int64_t N,
                                 const int64_t* __restrict__ canon, int64_t V,
                                 const int64_t* __restrict__ mults, int n_tables, int max_order,
                                 const int* __restrict__ orders, const int64_t* __restrict__ rows,
                                 int64_t pad_id, int64_t* __restrict__ out) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  int64_t tok[8];
  for (int i = 0; i < max_order && i < 8; ++i) {
    int64_t id = ids[n * max_order + i];
    if (id < 0) {
      tok[i] = pad_id;
    } else {
      id = id >= V ? V - 1 : id;
      tok[i] = canon[id];
    }
  }
  for (int k = 0; k < n_tables; ++k) {
    const int ord = orders[k];
    int64_t x = 0;
    for (int i = 0; i < ord; ++i) x += tok[i] * mults[k * max_order + i];
    out[(int64_t)k * N + n] = floor_mod(floor_mod(x, kPrime), rows[k]);
  }
}

// ------------------------------------------------------------------------------ gather
// mem[n, k*dim + c] = table_k[idx[k, n], c], read from the owner of the row:
// owner = row / per[k], local = row - owner*per[k], base = ptrs[owner*n_tables + k].
// One thread per 8 output elements (one 16-byte store).
template <typename Tin, typename Tout>
__global__ void gather_kernel(const int64_t* __restrict__ idx, int64_t N, int n_tables, int dim,
                              const int64_t* __restrict__ ptrs, const int64_t* __restrict__ per,
                              int world, Tout* __restrict__ mem, int* status) {
  const int chunks = dim / 8;
  const int64_t total = N * n_tables * chunks;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % chunks);
    const int64_t nk = i / chunks;
    const int k = (int)(nk % n_tables);
    const int64_t n = nk / n_tables;
    const int64_t row = idx[(int64_t)k * N + n];
    const int64_t pk = per[k];
    int owner = (int)(row / pk);
    const int64_t local = row - (int64_t)owner * pk;
#ifdef ME_BOUNDS_CHECK
    if (row < 0 || owner >= world) {
      report(status, ME_ERR_BOUNDS, (int)k);
      continue;
    }
#endif
    const Tin* src = reinterpret_cast<const Tin*>(ptrs[owner * n_tables + k]) + local * dim + c * 8;
    float v[8];
    if constexpr (sizeof(Tin) == 2) {
      BF16x8 x;
      x.u = *reinterpret_cast<const uint4*>(src);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = bf2f(x.h[j]);
    } else {
      F32x4 a, b;
      a.v = *reinterpret_cast<const float4*>(src);
      b.v = *reinterpret_cast<const float4*>(src + 4);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = a.f[j];
        v[4 + j] = b.f[j];
      }
    }
    Tout* dst = mem + n * (int64_t)n_tables * dim + (int64_t)k * dim + c * 8;
    if constexpr (sizeof(Tout) == 2) {
      BF16x8 y;
#pragma unroll
      for (int j = 0; j < 8; ++j) y.h[j] = f2bf(v[j]);
      *reinterpret_cast<uint4*>(dst) = y.u;
    } else {
      F32x4 a, b;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        a.f[j] = v[j];
        b.f[j] = v[4 + j];
      }
      *reinterpret_cast<float4*>(dst) = a.v;
      *reinterpret_cast<float4*>(dst + 4) = b.v;
    }
  }
}

// ------------------------------------------------------------------------------ row grads
// Backward of the gather: every looked-up row's gradient (scaled by `scale`, 1/world as the
// reference's owner-side average) is added into the owner's fp32 accumulator with float4
// atomics (peer memory over NVLink when the owner is another GPU). The accumulator is
// compact: a row's gradient lives in a slot of [cap, dim], cap = the rows one optimizer step
// can touch (tokens per step x ranks, at most the shard's rows). pos[row] = slot + 1 (0 =
// untouched); the first event on a row reserves a slot with one atomicAdd on the count and
// installs it with one atomicCAS on pos (a loser of that race leaves its reserved slot as a
// hole: list[slot] = -1, accumulator row zero). Each event reserves at most one slot, so
// cap = events per step can never be exceeded. One warp per (token, table) event; lane 0
// resolves the slot, all lanes add dim/32 floats. State pointer table layout, per
// (rank, table): acc [cap, dim] fp32, pos [per] i32, list [cap] i32, count [1] i32.
template <typename Tg>
__global__ void scatter_grad_kernel(const Tg* __restrict__ g, const int64_t* __restrict__ idx,
                                    int64_t N, int n_tables, int dim,
                                    const int64_t* __restrict__ acc_ptrs,
                                    const int64_t* __restrict__ pos_ptrs,
                                    const int64_t* __restrict__ list_ptrs,
                                    const int64_t* __restrict__ cnt_ptrs,
                                    const int64_t* __restrict__ per, const int64_t* __restrict__ caps, int world,
                                    float scale, int* status, int my_rank) {
  const int lane = threadIdx.x & 31;
  const int chunks = dim / 4;
  const int64_t total = N * n_tables;
  for (int64_t e = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; e < total;
       e += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int k = (int)(e % n_tables);
    const int64_t n = e / n_tables;
    const int64_t row = idx[(int64_t)k * N + n];
    const int64_t pk = per[k];
    const int owner = (int)(row / pk);
    const int64_t local = row - (int64_t)owner * pk;
#ifdef ME_BOUNDS_CHECK
    if (row < 0 || owner >= world) {
      if (lane == 0) report(status, ME_ERR_BOUNDS, (int)k);
      continue;
    }
#endif
    const int slot = owner * n_tables + k;
    int s = 0;
    if (lane == 0) {
      int* pos = reinterpret_cast<int*>(pos_ptrs[slot]) + local;
      s = *reinterpret_cast<volatile int*>(pos);
      if (s == 0) {
        const int t = atomicAdd(reinterpret_cast<int*>(cnt_ptrs[slot]), 1);
        if (t < caps[k]) {
          const int old = atomicCAS(pos, 0, t + 1);
          reinterpret_cast<int*>(list_ptrs[slot])[t] = old == 0 ? (int)local : -1;
          s = old == 0 ? t + 1 : old;
        } else {
          s = atomicAdd(pos, 0);  // another event may have installed a slot meanwhile
          if (s == 0) report(status, ME_ERR_CAPACITY, k);
        }
      }
    }
    s = __shfl_sync(0xffffffffu, s, 0);
    if (s <= 0) continue;
    float* acc = reinterpret_cast<float*>(acc_ptrs[slot]) + (int64_t)(s - 1) * dim;
    const Tg* src = g + n * (int64_t)n_tables * dim + (int64_t)k * dim;
    for (int c = lane; c < chunks; c += 32) {
      float4 v;
      if constexpr (sizeof(Tg) == 2) {
        const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(src + c * 4);
        const float2 a = __bfloat1622float2(s2[0]), b = __bfloat1622float2(s2[1]);
        v = make_float4(a.x * scale, a.y * scale, b.x * scale, b.y * scale);
      } else {
        const float4 a = *reinterpret_cast<const float4*>(src + c * 4);
        v = make_float4(a.x * scale, a.y * scale, a.z * scale, a.w * scale);
      }
      float* dst = acc + c * 4;
      if (owner == my_rank) {
        atomicAdd(reinterpret_cast<float4*>(dst), v);  // local memory: one 16-byte vector atomic
      } else {  // a peer's memory over NVLink: plain fp32 atomics
        atomicAdd(dst + 0, v.x);
        atomicAdd(dst + 1, v.y);
        atomicAdd(dst + 2, v.z);
        atomicAdd(dst + 3, v.w);
      }
    }
  }
}

// ------------------------------------------------------------------------------ row-grad exchange
// The multi-GPU return of row gradients without remote atomics, in two kernels per backward
// call (both on every rank, in the same order):
//
//   push        every (token, table) event whose row this rank owns is added into the local
//               compact accumulator at once (local float4 atomics). An event owned by rank o is
//               appended to o's inbox region for this rank: the entry index comes from a LOCAL
//               counter, the (table, local row) header and the bf16 row gradient go over NVLink
//               as plain 16-byte stores. The last block to finish publishes, per owner, the entry
//               count and then ready[this rank] = call (release, system scope).
//   accumulate  waits (bounded) until every peer's ready flag reached `call`, then adds every
//               entry of every inbox region into the local accumulator (local atomics), scaled.
//               Its last block tells each peer consumed[this rank] = call.
//
// A push writes into an owner's inbox only after that owner's accumulate of the previous call
// has finished (push waits, bounded, until consumed[o] >= call - 1), so one inbox per (owner,
// source) suffices. Exchange buffer, same offsets on every rank:
//   [0, 64)     ready[16]     u32    written by the sources
//   [64, 128)   consumed[16]  u32    written by the owners
//   [128, 192)  counts[16]    i32    entries source s wrote for the current call
//   [192, 256)  outcnt[16]    i32    this rank's entries per owner during a push
//   [256, 264)  done[2]       i32    blocks finished (push, accumulate)
//   [512, ...)  region[s] for every source s: hdr [cap_e] int2 (table, local row) at 0,
//               rows [cap_e, dim] bf16 at rows_off; regions region_bytes apart.
constexpr int kXReady = 0, kXConsumed = 64, kXCounts = 128, kXOut = 192, kXDone = 256, kXRegions = 512;

ME_DEVICE int claim_slot(int* pos, int* cnt, int* list, int64_t cap, int local, int* status, int k) {
  int s = *reinterpret_cast<volatile int*>(pos + local);
  if (s != 0) return s;
  const int t = atomicAdd(cnt, 1);
  if (t < cap) {
    const int old = atomicCAS(pos + local, 0, t + 1);
    list[t] = old == 0 ? local : -1;
    return old == 0 ? t + 1 : old;
  }
  s = atomicAdd(pos + local, 0);  // another event may have installed a slot meanwhile
  if (s == 0) report(status, ME_ERR_CAPACITY, k);
  return s;
}

// 8 bf16 (one 16-byte chunk) * scale added into acc[0..8) with two local float4 atomics.
ME_DEVICE void add_chunk(float* acc, uint4 raw, float scale) {
  BF16x8 x;
  x.u = raw;
  float f[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = bf2f(x.h[j]) * scale;
  atomicAdd(reinterpret_cast<float4*>(acc), make_float4(f[0], f[1], f[2], f[3]));
  atomicAdd(reinterpret_cast<float4*>(acc + 4), make_float4(f[4], f[5], f[6], f[7]));
}

struct RowTablesArgs {
  const int64_t* acc_ptrs;   // [world * n_tables]: (rank, table) -> accumulator base
  const int64_t* pos_ptrs;
  const int64_t* list_ptrs;
  const int64_t* cnt_ptrs;
  const int64_t* per;        // [n_tables] rows per shard
  const int64_t* caps;       // [n_tables] slots per accumulator
  const int64_t* xbases;     // [world] exchange buffer base of every rank
  int n_tables, dim, world, me;
  int64_t cap_e, region_bytes, rows_off;
  uint32_t call;
  uint64_t timeout_ns;
  int* status;
};

// Whether every block's stores are done: the last block to arrive on `done` returns true (and
// resets the counter for the next call).
ME_DEVICE bool last_block(int* done) {
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(done, 1) == (int)gridDim.x - 1;
    if (last) {
      __threadfence();
      *reinterpret_cast<volatile int*>(done) = 0;
    }
  }
  __syncthreads();
  return last;
}

// a warp takes 32 (token, table) events at a time; each is then handled by a group of 8 lanes
__global__ void __launch_bounds__(256) row_push_kernel(const __nv_bfloat16* __restrict__ g,
                                                       const int64_t* __restrict__ idx, int64_t N, RowTablesArgs a,
                                                       float scale) {
  __shared__ int failed;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.xbases[a.me]);
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < a.world && (int)threadIdx.x != a.me) {
    const uint32_t* consumed = reinterpret_cast<const uint32_t*>(mine + kXConsumed) + threadIdx.x;
    if (!wait_flag_geq(consumed, a.call - 1u, a.timeout_ns)) {
      report(a.status, ME_ERR_TIMEOUT, 100 + (int)threadIdx.x);
      failed = 1;
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
  const unsigned gmask = 0xFFu << (lane & 24);
  const int chunks = a.dim / 8;
  const int64_t events = N * a.n_tables;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int* outcnt = reinterpret_cast<int*>(mine + kXOut);
  for (int64_t base = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 32; !failed && base < events;
       base += warps * 32) {
    // one event per lane (table-major: the 32 row ids read are contiguous)
    const int64_t e = base + lane;
    int k = 0, owner = a.me, local = 0, slot = -1;
    int64_t n = 0;
    bool valid = e < events;
    if (valid) {
      k = (int)(e / N);
      n = e - (int64_t)k * N;
      const int64_t row = idx[e];
      const int64_t pk = a.per[k];
      owner = (int)(row / pk);
      local = (int)(row - (int64_t)owner * pk);
#ifdef ME_BOUNDS_CHECK
      if (row < 0 || owner >= a.world) {  // a row id outside every shard: dropped, reported
        report(a.status, ME_ERR_BOUNDS, k);
        valid = false;
        owner = a.me;
      }
#endif
    }
    // entries for other owners: one counter atomic per owner per warp, then each lane's place
    const bool remote = valid && owner != a.me;
    const unsigned rmask = __ballot_sync(0xffffffffu, remote);
    if (remote) {
      const unsigned same = __match_any_sync(rmask, owner);
      const int leader = __ffs(same) - 1;
      int first = 0;
      if (lane == leader) first = atomicAdd(outcnt + owner, __popc(same));
      first = __shfl_sync(same, first, leader);
      slot = first + __popc(same & ((1u << lane) - 1u));
    }
    // the 32 events, four at a time, 8 lanes each
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
      const int src_lane = j * 4 + grp;
      const bool v = __shfl_sync(0xffffffffu, valid, src_lane);
      const int kk = __shfl_sync(0xffffffffu, k, src_lane);
      const int oo = __shfl_sync(0xffffffffu, owner, src_lane);
      const int lo = __shfl_sync(0xffffffffu, local, src_lane);
      const int sl = __shfl_sync(0xffffffffu, slot, src_lane);
      const int64_t nn = __shfl_sync(0xffffffffu, n, src_lane);
      if (!v) continue;
      const __nv_bfloat16* src = g + nn * (int64_t)a.n_tables * a.dim + (int64_t)kk * a.dim;
      if (oo == a.me) {
        const int t = a.me * a.n_tables + kk;
        int s = 0;
        if (sub == 0)
          s = claim_slot(reinterpret_cast<int*>(a.pos_ptrs[t]), reinterpret_cast<int*>(a.cnt_ptrs[t]),
                         reinterpret_cast<int*>(a.list_ptrs[t]), a.caps[kk], lo, a.status, kk);
        s = __shfl_sync(gmask, s, 0, 8);
        if (s <= 0) continue;
        float* acc = reinterpret_cast<float*>(a.acc_ptrs[t]) + (int64_t)(s - 1) * a.dim;
        for (int c = sub; c < chunks; c += 8) add_chunk(acc + c * 8, *reinterpret_cast<const uint4*>(src + c * 8), scale);
      } else {
        if (sl >= a.cap_e) {
          if (sub == 0) report(a.status, ME_ERR_CAPACITY, 200 + oo);
          continue;
        }
        uint8_t* region = reinterpret_cast<uint8_t*>(a.xbases[oo]) + kXRegions + (int64_t)a.me * a.region_bytes;
        if (sub == 0) reinterpret_cast<int2*>(region)[sl] = make_int2(kk, lo);
        uint4* dst = reinterpret_cast<uint4*>(region + a.rows_off + (int64_t)sl * a.dim * 2);
        for (int c = sub; c < chunks; c += 8) dst[c] = *reinterpret_cast<const uint4*>(src + c * 8);
      }
    }
  }
  if (last_block(reinterpret_cast<int*>(mine + kXDone))) {
    if ((int)threadIdx.x < a.world && (int)threadIdx.x != a.me) {
      const int o = threadIdx.x;
      const int n_o = atomicExch(outcnt + o, 0);
      uint8_t* peer = reinterpret_cast<uint8_t*>(a.xbases[o]);
      reinterpret_cast<volatile int*>(peer + kXCounts)[a.me] = (int)min((int64_t)n_o, a.cap_e);
      st_release_sys(reinterpret_cast<uint32_t*>(peer + kXReady) + a.me, a.call);
    }
  }
}

__global__ void __launch_bounds__(256) row_accumulate_kernel(RowTablesArgs a, float scale) {
  __shared__ int failed;
  __shared__ int count[16];
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.xbases[a.me]);
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if ((int)threadIdx.x < a.world) {
    int c = 0;
    if ((int)threadIdx.x != a.me) {
      const uint32_t* ready = reinterpret_cast<const uint32_t*>(mine + kXReady) + threadIdx.x;
      if (wait_flag_geq(ready, a.call, a.timeout_ns)) {
        c = __ldcg(reinterpret_cast<const int*>(mine + kXCounts) + threadIdx.x);
      } else {
        report(a.status, ME_ERR_TIMEOUT, 300 + (int)threadIdx.x);
        failed = 1;
      }
    }
    count[threadIdx.x] = c;
  }
  __syncthreads();
  const int sub = threadIdx.x & 7;
  const unsigned gmask = 0xFFu << (threadIdx.x & 24);
  const int chunks = a.dim / 8;
  const int64_t groups = (int64_t)gridDim.x * (blockDim.x >> 3);
  const int64_t first = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
  for (int src = 0; !failed && src < a.world; ++src) {
    const uint8_t* region = mine + kXRegions + (int64_t)src * a.region_bytes;
    const int2* hdr = reinterpret_cast<const int2*>(region);
    for (int64_t i = first; i < count[src]; i += groups) {
      int s = 0, k = 0;
      if (sub == 0) {
        const int2 h = __ldcg(hdr + i);
        k = h.x;
#ifdef ME_BOUNDS_CHECK
        if (k < 0 || k >= a.n_tables || h.y < 0 || h.y >= a.per[k]) {  // a corrupt inbox entry
          report(a.status, ME_ERR_BOUNDS, 600 + src);
          k = 0;  // s stays 0: the entry is dropped
        } else
#endif
        {
          const int t = a.me * a.n_tables + k;
          s = claim_slot(reinterpret_cast<int*>(a.pos_ptrs[t]), reinterpret_cast<int*>(a.cnt_ptrs[t]),
                         reinterpret_cast<int*>(a.list_ptrs[t]), a.caps[k], h.y, a.status, k);
        }
      }
      s = __shfl_sync(gmask, s, 0, 8);
      k = __shfl_sync(gmask, k, 0, 8);
      if (s <= 0) continue;
      float* acc = reinterpret_cast<float*>(a.acc_ptrs[a.me * a.n_tables + k]) + (int64_t)(s - 1) * a.dim;
      const uint4* rowp = reinterpret_cast<const uint4*>(region + a.rows_off + i * a.dim * 2);
      for (int c = sub; c < chunks; c += 8) add_chunk(acc + c * 8, __ldcg(rowp + c), scale);
    }
  }
  if (last_block(reinterpret_cast<int*>(mine + kXDone) + 1)) {
    if ((int)threadIdx.x < a.world && (int)threadIdx.x != a.me)
      st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(a.xbases[threadIdx.x]) + kXConsumed) +
                         a.me,
                     a.call);
  }
}

// ------------------------------------------------------------------------------ owner-served fetch
// The multi-GPU forward fetch, inverted so that no GPU reads another GPU's tables: random reads
// of peer memory are bound by address translation (a measured 18 ms for 1.57M random 128-byte
// remote rows against 0.1 ms locally, 0.3 ms when the same rows sit in a small window). Each rank
// publishes its lookups; each OWNER reads the rows it holds from its own tables (random local
// reads) and writes them into the requester's receive buffer (one window of N x n_tables x dim
// bf16 per requester), then the requester copies the buffer out. Two kernels per call, on every
// rank, in the same order:
//
//   serve    prologue: this rank's lookups for `call` are in its fetch buffer and its receive
//            buffer is free, so it tells every owner (ntok, then ready = call, release). Then, for
//            every requester r (bounded wait for r's ready flag in this rank's buffer): scan r's
//            lookups 32 at a time (coalesced), and for those this rank owns, copy the row from the
//            local shard into r's receive buffer (16-byte stores, 8 lanes per row). The last block
//            tells every requester done = call.
//   collect  waits (bounded) until every owner's done flag reached `call`, then copies the
//            receive buffer into the output (the output outlives the next call).
//
// Fetch buffer layout (same offsets on every rank):
//   [0, 64)    ready[16] u32   requester r set it (at this owner) for the call it published
//   [64, 128)  ntok[16]  i32   that requester's token count
//   [128, 192) done[16]  u32   owner o set it (at this requester) when its rows are written
//   [192, 200) blocks finished (serve)
//   [256, ...) idx [n_tables, cap_tok] int64 of this rank's lookups, then recv [cap_tok, n_tables, row]
//              (rows as stored in the tables, row16 16-byte units each)
constexpr int kFReady = 0, kFNtok = 64, kFDone = 128, kFBlocks = 192, kFIdx = 256;

struct FetchArgs {
  const int64_t* fbases;  // [world] fetch buffer of every rank
  const int64_t* wptrs;   // [world * n_tables] table base of (rank, table); only this rank's are read
  const int64_t* per;     // [n_tables] rows per shard
  int n_tables, row16, world, me;  // row16: 16-byte units per table row (dim x element size / 16)
  int64_t cap_tok, recv_off;  // recv offset in the fetch buffer (16-byte aligned)
  uint32_t call;
  uint64_t timeout_ns;
  int* status;
};

__global__ void __launch_bounds__(256) rows_serve_kernel(FetchArgs a, int ntok_me) {
  __shared__ int failed;
  __shared__ int ntok[16];
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.fbases[a.me]);
  if (threadIdx.x == 0) failed = 0;
  if ((int)threadIdx.x < a.world) {  // publish: this rank's lookups are ready at every owner
    uint8_t* owner = reinterpret_cast<uint8_t*>(a.fbases[threadIdx.x]);
    reinterpret_cast<volatile int*>(owner + kFNtok)[a.me] = ntok_me;
    st_release_sys(reinterpret_cast<uint32_t*>(owner + kFReady) + a.me, a.call);
  }
  __syncthreads();
  if ((int)threadIdx.x < a.world) {
    const uint32_t* ready = reinterpret_cast<const uint32_t*>(mine + kFReady) + threadIdx.x;
    if (wait_flag_geq(ready, a.call, a.timeout_ns)) {
      ntok[threadIdx.x] = __ldcg(reinterpret_cast<const int*>(mine + kFNtok) + threadIdx.x);
    } else {
      report(a.status, ME_ERR_TIMEOUT, 400 + (int)threadIdx.x);
      failed = 1;
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
  const int chunks = a.row16;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  for (int r = 0; !failed && r < a.world; ++r) {
    int n = ntok[r];
#ifdef ME_BOUNDS_CHECK
    if (n < 0 || n > a.cap_tok) {  // a token count beyond the requester's lookup list
      if (threadIdx.x == 0) report(a.status, ME_ERR_BOUNDS, 700 + r);
      n = 0;
    }
#endif
    const int64_t events = (int64_t)n * a.n_tables;
    const uint8_t* req = reinterpret_cast<const uint8_t*>(a.fbases[r]);
    const int64_t* ridx = reinterpret_cast<const int64_t*>(req + kFIdx);
    uint4* recv = reinterpret_cast<uint4*>(const_cast<uint8_t*>(req) + a.recv_off);
    for (int64_t base = w0 * 32; base < events; base += warps * 32) {
      // one event per lane: table-major order, so the 32 lookups read are contiguous
      const int64_t e = base + lane;
      int k = 0, t = 0;
      int64_t local = -1;
      if (e < events) {
        k = (int)(e / n);
        t = (int)(e - (int64_t)k * n);
        const int64_t row = __ldcg(ridx + (int64_t)k * a.cap_tok + t);
        const int64_t pk = a.per[k];
#ifdef ME_BOUNDS_CHECK
        if (row < 0 || row / pk >= a.world) report(a.status, ME_ERR_BOUNDS, 800 + k);  // no owner serves it
#endif
        if (row >= 0 && row / pk == a.me) local = row - (int64_t)a.me * pk;
      }
      unsigned own = __ballot_sync(0xffffffffu, local >= 0);
      while (own) {  // four owned events at a time, 8 lanes each
        int pick = -1;
        unsigned rest = own;
        for (int q = 0; q <= grp && rest; ++q) {
          pick = __ffs(rest) - 1;
          rest &= rest - 1;
          if (q < grp) pick = -1;
        }
        const int64_t lo = __shfl_sync(0xffffffffu, local, pick < 0 ? 0 : pick);
        const int kk = __shfl_sync(0xffffffffu, k, pick < 0 ? 0 : pick);
        const int tt = __shfl_sync(0xffffffffu, t, pick < 0 ? 0 : pick);
        if (pick >= 0) {
          const uint4* src = reinterpret_cast<const uint4*>(a.wptrs[a.me * a.n_tables + kk]) + lo * chunks;
          uint4* dst = recv + ((int64_t)tt * a.n_tables + kk) * chunks;
          for (int c = sub; c < chunks; c += 8) dst[c] = src[c];
        }
        for (int q = 0; q < 4 && own; ++q) own &= own - 1;  // the four handled in this pass
      }
    }
  }
  if (last_block(reinterpret_cast<int*>(mine + kFBlocks))) {
    if ((int)threadIdx.x < a.world)
      st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(a.fbases[threadIdx.x]) + kFDone) + a.me,
                     a.call);
  }
}

// Wait until every owner wrote this call's rows, then copy n16 16-byte units of recv to out.
__global__ void __launch_bounds__(256) rows_collect_kernel(FetchArgs a, int64_t n16, uint4* __restrict__ out) {
  __shared__ int failed;
  const uint8_t* mine = reinterpret_cast<const uint8_t*>(a.fbases[a.me]);
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if ((int)threadIdx.x < a.world) {
    const uint32_t* done = reinterpret_cast<const uint32_t*>(mine + kFDone) + threadIdx.x;
    if (!wait_flag_geq(done, a.call, a.timeout_ns)) {
      report(a.status, ME_ERR_TIMEOUT, 500 + (int)threadIdx.x);
      failed = 1;
    }
  }
  __syncthreads();
  if (failed) return;
  const uint4* recv = reinterpret_cast<const uint4*>(mine + a.recv_off);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __ldcg(recv + i);
}

// Sum of squares of the touched rows' accumulated gradients (every row lives on exactly one
// rank, so the sum over ranks is the global table norm^2): the first min(count, cap) slots of
// each compact accumulator (holes are zero). counts are read on the device.
__global__ void __launch_bounds__(256) touched_sqnorm_kernel(const int64_t* __restrict__ acc_ptrs,
                                                              const int64_t* __restrict__ cnt_ptrs,
                                                              const int64_t* __restrict__ caps, int n_tables, int dim,
                                                              float* __restrict__ out) {
  // the used slots of a table are one contiguous [cnt, dim] block: a flat float4 reduction with
  // four loads in flight per thread
  __shared__ float scratch[64];
  float local_sum = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int k = 0; k < n_tables; ++k) {
    const int64_t cnt = min((int64_t)*reinterpret_cast<const int*>(cnt_ptrs[k]), caps[k]);
    const float4* acc = reinterpret_cast<const float4*>(acc_ptrs[k]);
    const int64_t n4 = cnt * dim / 4;
    int64_t i = t0;
    for (; i + 3 * stride < n4; i += 4 * stride) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = acc[i + u * stride];
#pragma unroll
      for (int u = 0; u < 4; ++u) local_sum += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
    }
    for (; i < n4; i += stride) {
      const float4 v = acc[i];
      local_sum += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  }
  const float s = block_sum(local_sum, scratch);
  if (threadIdx.x == 0) atomicAdd(out, s);
}

// coef = min(1, max_norm / (sqrt(sq) + 1e-6)); also stores the norm.
__global__ void clip_coef_kernel(const float* sq, float max_norm, float* coef, float* norm) {
  const float n = sqrtf(*sq);
  *norm = n;
  *coef = max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
}

// AdamW on the touched rows of one table shard (micro_engram/optim.py:65-133 semantics):
// rows whose gradient is all zero are left alone; rowwise keeps ONE fp32 second moment per
// row (mean of g^2 over the row); bf16 weights/moments are written back with stochastic
// rounding (Philox4x32-10 keyed by seed/step, counter = row, column block). The
// accumulator slot and the row's pos entry are cleared for the next step. One warp per slot
// of the compact accumulator (holes, list = -1, are only cleared).
// The touched-row AdamW of several tables in ONE launch (same semantics as adam_touched_kernel):
// a group of 8 lanes per touched row, each lane 8 consecutive values per 16-byte chunk, so a
// 64-wide bf16 row is one 16-byte load per lane of the weight and of the moment; 4 rows per warp
// are in flight at once. Rounding bits: Philox4x32-10 keyed by (seed, step), counter (row, table,
// chunk, 0/1): 16 bits per rounded value.
constexpr int kAdamMaxTables = 32;

struct AdamTable {
  void* p;          // weights [rows, dim] (bf16 or fp32)
  void* m;          // first moment, weight dtype (device or mapped pinned host memory)
  float* v_row;     // rowwise: fp32 [rows], else nullptr
  void* v_val;      // per-value second moment, weight dtype (when v_row is null)
  float* acc;       // compact fp32 accumulator [cap, dim]
  int* pos;         // row -> slot + 1
  const int* list;  // slot -> row (-1: hole)
  const int* cnt;   // slots handed out
  int cap;
  uint32_t table_id, step;
  float bc1, bc2_sqrt;
};

struct AdamTables {
  AdamTable t[kAdamMaxTables];
  int n;
};

ME_DEVICE float group8_sum(float x, unsigned mask) {
  x += __shfl_xor_sync(mask, x, 4, 8);
  x += __shfl_xor_sync(mask, x, 2, 8);
  x += __shfl_xor_sync(mask, x, 1, 8);
  return x;
}

template <typename T>
ME_DEVICE void load8(const T* src, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    BF16x8 x;
    x.u = *reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = bf2f(x.h[j]);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

// 8 values to T (stochastic rounding with 16 bits each of rnd[0..3] when sr and T is bf16)
template <typename T>
ME_DEVICE void store8(T* dst, const float (&v)[8], bool sr, const uint32_t (&rnd)[4]) {
  if constexpr (sizeof(T) == 2) {
    BF16x8 x;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t bits = (j & 1) ? (rnd[j >> 1] >> 16) : rnd[j >> 1];
      x.h[j] = sr ? sr_bf16(v[j], bits) : f2bf(v[j]);
    }
    *reinterpret_cast<uint4*>(dst) = x.u;
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// CPL: 16-byte chunks per lane (dim <= 64 * CPL). The (table, slot) pairs of all tables form one
// index space, split evenly over the groups of 8 lanes (prefix sums of the tables' counts).
template <typename T, int CPL>
__global__ void __launch_bounds__(256, CPL == 1 ? 4 : 2) adam_rows_kernel(const __grid_constant__ AdamTables tabs, int dim,
                                                        const float* coef_ptr, float lr, float beta1, float beta2,
                                                        float eps, float wd, int sr, uint32_t seed) {
  __shared__ int64_t first[kAdamMaxTables + 1];
  if (threadIdx.x == 0) {
    int64_t run = 0;
    for (int k = 0; k < tabs.n; ++k) {
      first[k] = run;
      run += min(*tabs.t[k].cnt, tabs.t[k].cap);
    }
    first[tabs.n] = run;
  }
  __syncthreads();
  const int sub = threadIdx.x & 7;
  const unsigned gmask = 0xFFu << (threadIdx.x & 24);
  const int64_t groups = (int64_t)gridDim.x * (blockDim.x >> 3);
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const int chunks = dim / 8;
  int k = 0;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3; i < first[tabs.n]; i += groups) {
    while (i >= first[k + 1]) ++k;  // i only grows, so the table index only moves forward
    const AdamTable& t = tabs.t[k];
    const int64_t r = i - first[k];
    const int row = t.list[r];
    float* a = t.acc + r * dim;
    T* P = reinterpret_cast<T*>(t.p);
    T* M = reinterpret_cast<T*>(t.m);
    T* VV = reinterpret_cast<T*>(t.v_val);
    // every load of the row first (accumulator slot, weights, moments), then the stores: the loads
    // are independent once the row is known, so they are in flight together
    float g[CPL][8], pw[CPL][8], mw[CPL][8], vv[CPL][8];
    float v_old = 0.f;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = sub + 8 * q;
      if (c < chunks) {
        const float4 x = *reinterpret_cast<const float4*>(a + c * 8), y = *reinterpret_cast<const float4*>(a + c * 8 + 4);
        g[q][0] = x.x, g[q][1] = x.y, g[q][2] = x.z, g[q][3] = x.w;
        g[q][4] = y.x, g[q][5] = y.y, g[q][6] = y.z, g[q][7] = y.w;
        if (row >= 0) {
          const int64_t o = (int64_t)row * dim + c * 8;
          load8(P + o, pw[q]);
          load8(M + o, mw[q]);
          if (!t.v_row) load8(VV + o, vv[q]);
        }
      }
    }
    if (row >= 0 && t.v_row) v_old = t.v_row[row];
    float gsq = 0.f;
    bool nz = false;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = sub + 8 * q;
      if (c < chunks) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          nz |= g[q][j] != 0.f;
          g[q][j] *= coef;
          gsq += g[q][j] * g[q][j];
        }
        *reinterpret_cast<float4*>(a + c * 8) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(a + c * 8 + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (row < 0) continue;  // a hole: only cleared
    if (sub == 0) t.pos[row] = 0;
    if (!__any_sync(gmask, nz)) continue;  // lazy: an all-zero row is left as it is
    float vr = 0.f;
    if (t.v_row) vr = v_old * beta2 + (1.f - beta2) * (group8_sum(gsq, gmask) / (float)dim);
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = sub + 8 * q;
      if (c >= chunks) break;
      const int64_t o = (int64_t)row * dim + c * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (wd != 0.f) pw[q][j] *= (1.f - lr * wd);
        mw[q][j] = mw[q][j] * beta1 + (1.f - beta1) * g[q][j];
        float denom;
        if (t.v_row) {
          denom = sqrtf(vr) / t.bc2_sqrt + eps;
        } else {
          vv[q][j] = vv[q][j] * beta2 + (1.f - beta2) * g[q][j] * g[q][j];
          denom = sqrtf(vv[q][j]) / t.bc2_sqrt + eps;
        }
        pw[q][j] = pw[q][j] + (-lr / t.bc1) * mw[q][j] / denom;
      }
      const Philox4 r0 = philox4x32_10((uint32_t)row, t.table_id, (uint32_t)c, 0u, seed, t.step);
      const Philox4 r1 = philox4x32_10((uint32_t)row, t.table_id, (uint32_t)c, 1u, seed, t.step);
      const uint32_t rp[4] = {r0.c[0], r0.c[1], r0.c[2], r0.c[3]};
      const uint32_t rm[4] = {r1.c[0], r1.c[1], r1.c[2], r1.c[3]};
      store8(P + o, pw[q], sr != 0, rp);
      store8(M + o, mw[q], sr != 0, rm);
      if (!t.v_row) {
        const uint32_t rv[4] = {rp[0] ^ rm[1], rp[1] ^ rm[2], rp[2] ^ rm[3], rp[3] ^ rm[0]};
        store8(VV + o, vv[q], sr != 0, rv);
      }
    }
    if (t.v_row && sub == 0) t.v_row[row] = vr;
  }
}

template <typename Tp, typename Tm>
__global__ void adam_touched_kernel(Tp* __restrict__ p, Tm* __restrict__ m, float* __restrict__ v_row,
                                    Tm* __restrict__ v_val, float* __restrict__ acc,
                                    int* __restrict__ pos, const int* __restrict__ list,
                                    const int* __restrict__ cnt_ptr, int cap, int dim, const float* coef_ptr,
                                    float lr, float beta1, float beta2, float eps, float wd, float bc1,
                                    float bc2_sqrt, int sr, uint32_t seed, uint32_t step,
                                    uint32_t table_id) {
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int cnt = min(*cnt_ptr, cap);
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < cnt; r += warps_total) {
    const int64_t row = list[r];
    float* a = acc + (int64_t)r * dim;
    if (row < 0) {
      for (int j = lane; j < dim; j += 32) a[j] = 0.f;
      continue;
    }
    // gradient of this row (dim <= 256: at most 8 per lane)
    float g[8];
    bool nz = false;
    float gsq = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = lane + q * 32;
      g[q] = 0.f;
      if (j < dim) {
        g[q] = a[j] * coef;
        nz |= (a[j] != 0.f);
        gsq += g[q] * g[q];
        a[j] = 0.f;
      }
    }
    if (lane == 0) pos[row] = 0;
    if (!__any_sync(0xffffffffu, nz)) continue;
    float vr = 0.f;
    if (v_row) {
      const float mean_g2 = warp_sum(gsq) / (float)dim;
      vr = v_row[row] * beta2 + (1.f - beta2) * mean_g2;
    }
    const Philox4 rnd0 = philox4x32_10((uint32_t)row, table_id, (uint32_t)lane, 0u, seed, step);
    const Philox4 rnd1 = philox4x32_10((uint32_t)row, table_id, (uint32_t)lane, 1u, seed, step);
    const uint32_t rbits[8] = {rnd0.c[0], rnd0.c[1], rnd0.c[2], rnd0.c[3],
                               rnd1.c[0], rnd1.c[1], rnd1.c[2], rnd1.c[3]};
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = lane + q * 32;
      if (j >= dim) break;
      const int64_t o = row * dim + j;
      float pw = to_f(p[o]);
      float mw = to_f(m[o]);
      if (wd != 0.f) pw *= (1.f - lr * wd);
      mw = mw * beta1 + (1.f - beta1) * g[q];
      float denom;
      float vv = 0.f;
      if (v_row) {
        denom = sqrtf(vr) / bc2_sqrt + eps;
      } else {
        vv = to_f(v_val[o]) * beta2 + (1.f - beta2) * g[q] * g[q];
        denom = sqrtf(vv) / bc2_sqrt + eps;
      }
      pw = pw + (-lr / bc1) * mw / denom;
      // write back (stochastic rounding for bf16 when enabled)
      const uint32_t rb = rbits[q];
      if constexpr (sizeof(Tp) == 2) {
        p[o] = sr ? sr_bf16(pw, rb) : f2bf(pw);
      } else {
        p[o] = pw;
      }
      if constexpr (sizeof(Tm) == 2) {
        m[o] = sr ? sr_bf16(mw, rb >> 16) : f2bf(mw);
        if (!v_row) v_val[o] = sr ? sr_bf16(vv, rb * 2654435761u) : f2bf(vv);
      } else {
        m[o] = mw;
        if (!v_row) v_val[o] = vv;
      }
    }
    if (v_row && lane == 0) v_row[row] = vr;
  }
}

// Plain AdamW over a whole tensor (the replicated dense engram parameters, and tables
// trained with the non-lazy optimizer). g is fp32 or the param dtype.
template <typename Tp, typename Tg>
__global__ void adam_dense_kernel(Tp* __restrict__ p, const Tg* __restrict__ g, Tp* __restrict__ m,
                                  Tp* __restrict__ v, int64_t n, float lr, float beta1, float beta2,
                                  float eps, float wd, float bc1, float bc2_sqrt, float gscale, int sr,
                                  uint32_t seed, uint32_t step) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gr = to_f(g[i]) * gscale;
    float pw = to_f(p[i]), mw = to_f(m[i]), vw = to_f(v[i]);
    if (wd != 0.f) pw *= (1.f - lr * wd);
    mw = mw * beta1 + (1.f - beta1) * gr;
    vw = vw * beta2 + (1.f - beta2) * gr * gr;
    pw = pw + (-lr / bc1) * mw / (sqrtf(vw) / bc2_sqrt + eps);
    if constexpr (sizeof(Tp) == 2) {
      const Philox4 r = philox4x32_10((uint32_t)i, (uint32_t)(i >> 32), 0x5eedu, 0u, seed, step);
      p[i] = sr ? sr_bf16(pw, r.c[0]) : f2bf(pw);
      m[i] = sr ? sr_bf16(mw, r.c[1]) : f2bf(mw);
      v[i] = sr ? sr_bf16(vw, r.c[2]) : f2bf(vw);
    } else {
      p[i] = pw;
      m[i] = mw;
      v[i] = vw;
    }
  }
}

// ------------------------------------------------------------------------------ gate
// The scalar / scalar_sqrt gate (micro_engram/module.py:239-261), one block per row:
//   hn = rms(h) * qs, kn = rms(k) * ks   (fp32, torch's default eps = FLT_EPSILON)
//   s  = <hn, kn> / sqrt(d);  sqrt gate: s = sign(s) sqrt(max(|s|, 1e-6))
//   a  = sigmoid(s);  out = h + bf16(a * v) * keep
// stats[n] = (rh, rk, s_raw, a) for the backward. gate_acc += (sum a, count, count a>0.99).
constexpr float kEps = 1.1920928955078125e-07f;

template <int VPT>
__global__ void gate_fwd_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ k,
                                const __nv_bfloat16* __restrict__ v, const float* __restrict__ qs,
                                const float* __restrict__ ks, const uint8_t* __restrict__ keep,
                                int64_t N, int d, int sqrt_gate, __nv_bfloat16* __restrict__ out,
                                float* __restrict__ stats, float* __restrict__ gate_acc) {
  __shared__ float scratch[64];
  const float inv_sqrt_d = rsqrtf((float)d);
  float acc_a = 0.f, acc_n = 0.f, acc_sat = 0.f;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    const __nv_bfloat16* hr = h + n * d;
    const __nv_bfloat16* kr = k + n * d;
    float hv[VPT], kv[VPT];
    float sh = 0.f, sk = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      hv[q] = j < d ? bf2f(hr[j]) : 0.f;
      kv[q] = j < d ? bf2f(kr[j]) : 0.f;
      sh += hv[q] * hv[q];
      sk += kv[q] * kv[q];
    }
    const float2 ss = block_sum2(sh, sk, scratch);
    const float rh = rsqrtf(ss.x / d + kEps), rk = rsqrtf(ss.y / d + kEps);
    float dot = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      if (j < d) {
        const float a = hv[q] * rh * (qs ? qs[j] : 1.f);
        const float b = kv[q] * rk * (ks ? ks[j] : 1.f);
        dot += a * b;
      }
    }
    const float s_raw = block_sum(dot, scratch) * inv_sqrt_d;
    float s = s_raw;
    if (sqrt_gate) {
      const float sg = s_raw > 0.f ? 1.f : (s_raw < 0.f ? -1.f : 0.f);
      s = sg * sqrtf(fmaxf(fabsf(s_raw), 1e-6f));
    }
    const float alpha = 1.f / (1.f + expf(-s));
    const float kp = keep ? (keep[n] ? 1.f : 0.f) : 1.f;
    const __nv_bfloat16* vr = v + n * d;
    __nv_bfloat16* orow = out + n * d;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      if (j < d) {
        const float add = bf2f(f2bf(alpha * bf2f(vr[j]) * kp));
        orow[j] = f2bf(hv[q] + add);
      }
    }
    if (threadIdx.x == 0) {
      stats[n * 4 + 0] = rh;
      stats[n * 4 + 1] = rk;
      stats[n * 4 + 2] = s_raw;
      stats[n * 4 + 3] = alpha;
      acc_a += alpha;
      acc_n += 1.f;
      acc_sat += alpha > 0.99f ? 1.f : 0.f;
    }
  }
  if (gate_acc && threadIdx.x == 0) {
    atomicAdd(gate_acc + 0, acc_a);
    atomicAdd(gate_acc + 1, acc_n);
    atomicAdd(gate_acc + 2, acc_sat);
  }
}

// Backward of the gate. g: grad of out. Produces dh (= g + the gate's grad through rms(h)),
// dk, dv (bf16, as autograd casts them back to the bf16 projections), and per-column
// partial sums for d(q_scale), d(k_scale) (fp32, atomically added once per block).
template <int VPT>
__global__ void gate_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ h,
                                const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                const float* __restrict__ qs, const float* __restrict__ ks,
                                const uint8_t* __restrict__ keep, const float* __restrict__ stats,
                                int64_t N, int d, int sqrt_gate, __nv_bfloat16* __restrict__ dh,
                                __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                                float* __restrict__ dqs, float* __restrict__ dks) {
  __shared__ float scratch[64];
  const float inv_sqrt_d = rsqrtf((float)d);
  float pq[VPT], pk[VPT];
#pragma unroll
  for (int q = 0; q < VPT; ++q) pq[q] = pk[q] = 0.f;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    const float rh = stats[n * 4 + 0], rk = stats[n * 4 + 1], s_raw = stats[n * 4 + 2],
                alpha = stats[n * 4 + 3];
    const float kp = keep ? (keep[n] ? 1.f : 0.f) : 1.f;
    float gv[VPT], hv[VPT], kv[VPT];
    float da = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      if (j < d) {
        gv[q] = bf2f(g[n * d + j]);
        hv[q] = bf2f(h[n * d + j]);
        kv[q] = bf2f(k[n * d + j]);
        const float vj = bf2f(v[n * d + j]);
        da += gv[q] * kp * vj;
        dv[n * d + j] = f2bf(alpha * gv[q] * kp);
      } else {
        gv[q] = hv[q] = kv[q] = 0.f;
      }
    }
    da = block_sum(da, scratch);
    // through sigmoid and the signed square root
    float ds = da * alpha * (1.f - alpha);
    if (sqrt_gate) {
      const float c = fabsf(s_raw);
      ds = (c >= 1e-6f && s_raw != 0.f) ? ds * 0.5f / sqrtf(c) : 0.f;
    }
    ds *= inv_sqrt_d;  // s = dot / sqrt(d)
    // dhn_j = ds * kn_j, dkn_j = ds * hn_j; rms-norm backward with weights qs / ks
    float sum_h = 0.f, sum_k = 0.f;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      if (j < d) {
        const float wq = qs ? qs[j] : 1.f, wk = ks ? ks[j] : 1.f;
        const float hn0 = hv[q] * rh, kn0 = kv[q] * rk;  // before the scales
        const float dhn = ds * kn0 * wk, dkn = ds * hn0 * wq;
        sum_h += hv[q] * wq * dhn;
        sum_k += kv[q] * wk * dkn;
        pq[q] += dhn * hn0;
        pk[q] += dkn * kn0;
      }
    }
    const float2 sums = block_sum2(sum_h, sum_k, scratch);
    const float ch = rh * rh * rh * sums.x / d, ck = rk * rk * rk * sums.y / d;
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      if (j < d) {
        const float wq = qs ? qs[j] : 1.f, wk = ks ? ks[j] : 1.f;
        const float hn0 = hv[q] * rh, kn0 = kv[q] * rk;
        const float dhn = ds * kn0 * wk, dkn = ds * hn0 * wq;
        const float dhg = rh * wq * dhn - ch * hv[q];
        const float dkg = rk * wk * dkn - ck * kv[q];
        dh[n * d + j] = f2bf(gv[q] + bf2f(f2bf(dhg)));
        dk[n * d + j] = f2bf(dkg);
      }
    }
  }
  if (dqs) {
#pragma unroll
    for (int q = 0; q < VPT; ++q) {
      const int j = threadIdx.x + q * blockDim.x;
      if (j < d) {
        atomicAdd(dqs + j, pq[q]);
        atomicAdd(dks + j, pk[q]);
      }
    }
  }
}

// Vectorised gate (16-byte loads, one block per row, NCH chunks of 8 bf16 per thread).
// The rms and dot products collapse into one pass: with D = sum_j h_j k_j qs_j ks_j,
//   s_raw = rh rk D / sqrt(d);   backward: sum_j h_j qs_j dhn_j = ds rk D, sum_j k_j ks_j dkn_j = ds rh D,
//   d qs_j = ks_j S_j, d ks_j = qs_j S_j with S_j = sum_n ds_n rh_n rk_n h_nj k_nj,
// so k is never held across a reduction in the forward and the column partials need one array.
// Requires d % 8 == 0 and 16-byte aligned rows; the scalar kernels above take the rest.
ME_DEVICE float3 block_sum3(float a, float b, float c, float* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  c = warp_sum(c);
  __syncthreads();
  if (lane == 0) {
    scratch[wid] = a;
    scratch[32 + wid] = b;
    scratch[64 + wid] = c;
  }
  __syncthreads();
  float ra = lane < nw ? scratch[lane] : 0.f, rb = lane < nw ? scratch[32 + lane] : 0.f,
        rc = lane < nw ? scratch[64 + lane] : 0.f;
  return make_float3(warp_sum(ra), warp_sum(rb), warp_sum(rc));
}

ME_DEVICE void load_scale8(const float* __restrict__ s, int c, float* out) {
  if (s) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(s) + 2 * c);
    const float4 b = __ldg(reinterpret_cast<const float4*>(s) + 2 * c + 1);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = 1.f;
  }
}

template <int NCH>
__global__ void __launch_bounds__(256) gate_fwd_vec_kernel(
    const uint4* __restrict__ h, const uint4* __restrict__ k, const uint4* __restrict__ v,
    const float* __restrict__ qs, const float* __restrict__ ks, const uint8_t* __restrict__ keep, int64_t N,
    int d, int sqrt_gate, uint4* __restrict__ out, float* __restrict__ stats, float* __restrict__ gate_acc) {
  __shared__ float scratch[96];
  const int nc = d >> 3;
  const float inv_sqrt_d = rsqrtf((float)d);
  float acc_a = 0.f, acc_n = 0.f, acc_sat = 0.f;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    BF16x8 hv[NCH];
    float sh = 0.f, sk = 0.f, dot = 0.f;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
      const int c = threadIdx.x + q * blockDim.x;
      BF16x8 kv;
      if (c < nc) {
        hv[q].u = __ldcs(h + n * nc + c);
        kv.u = __ldcs(k + n * nc + c);
        float w[8], u[8];
        load_scale8(qs, c, w);
        load_scale8(ks, c, u);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = bf2f(hv[q].h[e]), b = bf2f(kv.h[e]);
          sh += a * a;
          sk += b * b;
          dot += a * b * w[e] * u[e];
        }
      }
    }
    const float3 r3 = block_sum3(sh, sk, dot, scratch);
    const float rh = rsqrtf(r3.x / d + kEps), rk = rsqrtf(r3.y / d + kEps);
    const float s_raw = rh * rk * r3.z * inv_sqrt_d;
    float s = s_raw;
    if (sqrt_gate) {
      const float sg = s_raw > 0.f ? 1.f : (s_raw < 0.f ? -1.f : 0.f);
      s = sg * sqrtf(fmaxf(fabsf(s_raw), 1e-6f));
    }
    const float alpha = 1.f / (1.f + expf(-s));
    const float kp = keep ? (keep[n] ? 1.f : 0.f) : 1.f;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
      const int c = threadIdx.x + q * blockDim.x;
      if (c < nc) {
        BF16x8 vv, o;
        vv.u = __ldcs(v + n * nc + c);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float add = bf2f(f2bf(alpha * bf2f(vv.h[e]) * kp));
          o.h[e] = f2bf(bf2f(hv[q].h[e]) + add);
        }
        out[n * nc + c] = o.u;
      }
    }
    if (threadIdx.x == 0) {
      reinterpret_cast<float4*>(stats)[n] = make_float4(rh, rk, s_raw, alpha);
      acc_a += alpha;
      acc_n += 1.f;
      acc_sat += alpha > 0.99f ? 1.f : 0.f;
    }
  }
  if (gate_acc && threadIdx.x == 0) {
    atomicAdd(gate_acc + 0, acc_a);
    atomicAdd(gate_acc + 1, acc_n);
    atomicAdd(gate_acc + 2, acc_sat);
  }
}

template <int NCH>
__global__ void __launch_bounds__(256) gate_bwd_vec_kernel(
    const uint4* __restrict__ g, const uint4* __restrict__ h, const uint4* __restrict__ k,
    const uint4* __restrict__ v, const float* __restrict__ qs, const float* __restrict__ ks,
    const uint8_t* __restrict__ keep, const float* __restrict__ stats, int64_t N, int d, int sqrt_gate,
    uint4* __restrict__ dh, uint4* __restrict__ dk, uint4* __restrict__ dv, float* __restrict__ dqs,
    float* __restrict__ dks) {
  __shared__ float scratch[96];
  const int nc = d >> 3;
  const float inv_sqrt_d = rsqrtf((float)d);
  float S[NCH][8];
#pragma unroll
  for (int q = 0; q < NCH; ++q)
#pragma unroll
    for (int e = 0; e < 8; ++e) S[q][e] = 0.f;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    const float4 st = reinterpret_cast<const float4*>(stats)[n];
    const float rh = st.x, rk = st.y, s_raw = st.z, alpha = st.w;
    const float kp = keep ? (keep[n] ? 1.f : 0.f) : 1.f;
    BF16x8 gv[NCH], hv[NCH], kv[NCH];
    float da = 0.f, dot = 0.f;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
      const int c = threadIdx.x + q * blockDim.x;
      if (c < nc) {
        gv[q].u = __ldcs(g + n * nc + c);
        hv[q].u = __ldcs(h + n * nc + c);
        kv[q].u = __ldcs(k + n * nc + c);
        BF16x8 vv, o;
        vv.u = __ldcs(v + n * nc + c);
        float w[8], u[8];
        load_scale8(qs, c, w);
        load_scale8(ks, c, u);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float gg = bf2f(gv[q].h[e]);
          da += gg * kp * bf2f(vv.h[e]);
          dot += bf2f(hv[q].h[e]) * bf2f(kv[q].h[e]) * w[e] * u[e];
          o.h[e] = f2bf(alpha * gg * kp);
        }
        __stcs(dv + n * nc + c, o.u);
      }
    }
    const float2 r2 = block_sum2(da, dot, scratch);
    float ds = r2.x * alpha * (1.f - alpha);
    if (sqrt_gate) {
      const float c = fabsf(s_raw);
      ds = (c >= 1e-6f && s_raw != 0.f) ? ds * 0.5f / sqrtf(c) : 0.f;
    }
    ds *= inv_sqrt_d;
    const float ch = rh * rh * rh * ds * rk * r2.y / d, ck = rk * rk * rk * ds * rh * r2.y / d;
    const float cn = ds * rh * rk;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
      const int c = threadIdx.x + q * blockDim.x;
      if (c < nc) {
        float w[8], u[8];
        load_scale8(qs, c, w);
        load_scale8(ks, c, u);
        BF16x8 oh, ok;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float hh = bf2f(hv[q].h[e]), kk = bf2f(kv[q].h[e]);
          const float hk = cn * w[e] * u[e];
          const float dhg = hk * kk - ch * hh;
          const float dkg = hk * hh - ck * kk;
          oh.h[e] = f2bf(bf2f(gv[q].h[e]) + bf2f(f2bf(dhg)));
          ok.h[e] = f2bf(dkg);
          S[q][e] += cn * hh * kk;
        }
        __stcs(dh + n * nc + c, oh.u);
        __stcs(dk + n * nc + c, ok.u);
      }
    }
  }
  if (dqs) {
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
      const int c = threadIdx.x + q * blockDim.x;
      if (c < nc) {
        float w[8], u[8];
        load_scale8(qs, c, w);
        load_scale8(ks, c, u);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          atomicAdd(dqs + 8 * c + e, u[e] * S[q][e]);
          atomicAdd(dks + 8 * c + e, w[e] * S[q][e]);
        }
      }
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

int grid_for(int64_t work, int threads, int per_sm = 8) {
  const int64_t need = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)sm_count() * per_sm));
}

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace

// ================================================================================ bindings
torch::Tensor engram_hash(torch::Tensor ids, c10::optional<torch::Tensor> pos, torch::Tensor canon,
                          torch::Tensor mults, torch::Tensor orders, torch::Tensor rows,
                          int64_t pad_id) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.dim() == 2, "ids must be [B, T]");
  const at::cuda::CUDAGuard guard(ids.device());
  const int64_t B = ids.size(0), T = ids.size(1);
  const int nt = (int)mults.size(0), mo = (int)mults.size(1);
  TORCH_CHECK(mo <= 8, "n-gram orders above 8 are not supported");
  auto ids64 = ids.to(torch::kLong).contiguous();
  torch::Tensor pos64;
  if (pos.has_value()) pos64 = pos->to(torch::kLong).expand({B, T}).contiguous();
  auto out = torch::empty({nt, B, T}, ids.options().dtype(torch::kLong));
  const int threads = 256;
  const int64_t n = B * T;
  if (n == 0) return out;
  hash_kernel<<<(n + threads - 1) / threads, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids64.data_ptr<int64_t>(), pos.has_value() ? pos64.data_ptr<int64_t>() : nullptr, B, T,
      canon.data_ptr<int64_t>(), canon.numel(), mults.data_ptr<int64_t>(), nt, mo,
      orders.data_ptr<int>(), rows.data_ptr<int64_t>(), pad_id, out.data_ptr<int64_t>());
  return out;
}

torch::Tensor engram_hash_prev(torch::Tensor ids, torch::Tensor canon, torch::Tensor mults,
                               torch::Tensor orders, torch::Tensor rows, int64_t pad_id) {
  check_cuda(ids, "ids");
  const at::cuda::CUDAGuard guard(ids.device());
  const int nt = (int)mults.size(0), mo = (int)mults.size(1);
  TORCH_CHECK(ids.dim() == 2 && ids.size(1) == mo, "ids must be [N, max_order]");
  auto ids64 = ids.to(torch::kLong).contiguous();
  const int64_t N = ids.size(0);
  auto out = torch::empty({nt, N}, ids.options().dtype(torch::kLong));
  if (N == 0) return out;
  const int threads = 256;
  hash_prev_kernel<<<(N + threads - 1) / threads, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids64.data_ptr<int64_t>(), N, canon.data_ptr<int64_t>(), canon.numel(), mults.data_ptr<int64_t>(),
      nt, mo, orders.data_ptr<int>(), rows.data_ptr<int64_t>(), pad_id, out.data_ptr<int64_t>());
  return out;
}

// idx [n_tables, N] int64 (global rows per table); ptrs [world*n_tables] int64 device
// addresses (this rank's and its peers' shards); per [n_tables] rows per rank.
torch::Tensor engram_gather(torch::Tensor idx, torch::Tensor ptrs, torch::Tensor per, int64_t world,
                            int64_t dim, int64_t src_dtype, torch::ScalarType out_dtype,
                            c10::optional<torch::Tensor> status) {
  check_cuda(idx, "idx");
  const at::cuda::CUDAGuard guard(idx.device());
  const int nt = (int)idx.size(0);
  const int64_t N = idx.size(1);
  TORCH_CHECK(dim % 8 == 0, "engram dim must be a multiple of 8");
  auto mem = torch::empty({N, nt * dim}, idx.options().dtype(out_dtype));
  if (N == 0) return mem;
  const int threads = 256;
  const int64_t work = N * nt * (dim / 8);
  const int grid = grid_for(work, threads);
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  const int64_t* ip = idx.data_ptr<int64_t>();
  const int64_t* pp = ptrs.data_ptr<int64_t>();
  const int64_t* pe = per.data_ptr<int64_t>();
  const bool in_bf16 = src_dtype == 0;
  if (out_dtype == torch::kBFloat16) {
    auto* o = reinterpret_cast<__nv_bfloat16*>(mem.data_ptr());
    if (in_bf16)
      gather_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, threads, 0, stream>>>(ip, N, nt, dim, pp, pe, world, o, st);
    else
      gather_kernel<float, __nv_bfloat16><<<grid, threads, 0, stream>>>(ip, N, nt, dim, pp, pe, world, o, st);
  } else {
    TORCH_CHECK(out_dtype == torch::kFloat32, "gather output must be bf16 or fp32");
    auto* o = mem.data_ptr<float>();
    if (in_bf16)
      gather_kernel<__nv_bfloat16, float><<<grid, threads, 0, stream>>>(ip, N, nt, dim, pp, pe, world, o, st);
    else
      gather_kernel<float, float><<<grid, threads, 0, stream>>>(ip, N, nt, dim, pp, pe, world, o, st);
  }
  return mem;
}

void engram_scatter_grad(torch::Tensor g, torch::Tensor idx, torch::Tensor acc_ptrs, torch::Tensor pos_ptrs,
                         torch::Tensor list_ptrs, torch::Tensor cnt_ptrs, torch::Tensor per, torch::Tensor caps,
                         int64_t world, double scale, c10::optional<torch::Tensor> status, int64_t my_rank) {
  check_cuda(g, "g");
  check_cuda(idx, "idx");
  const at::cuda::CUDAGuard guard(g.device());
  const int nt = (int)idx.size(0);
  const int64_t N = idx.size(1);
  if (N == 0) return;
  const int dim = (int)(g.size(1) / nt);
  TORCH_CHECK(dim % 4 == 0, "engram dim must be a multiple of 4");
  const int threads = 256;
  const int grid = grid_for(N * nt * 32, threads);  // one warp per (token, table) event
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  if (g.scalar_type() == torch::kBFloat16) {
    scatter_grad_kernel<__nv_bfloat16><<<grid, threads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), idx.data_ptr<int64_t>(), N, nt, dim,
        acc_ptrs.data_ptr<int64_t>(), pos_ptrs.data_ptr<int64_t>(), list_ptrs.data_ptr<int64_t>(),
        cnt_ptrs.data_ptr<int64_t>(), per.data_ptr<int64_t>(), caps.data_ptr<int64_t>(), world, (float)scale, st,
        (int)my_rank);
  } else {
    TORCH_CHECK(g.scalar_type() == torch::kFloat32, "row grads must be bf16 or fp32");
    scatter_grad_kernel<float><<<grid, threads, 0, stream>>>(
        g.data_ptr<float>(), idx.data_ptr<int64_t>(), N, nt, dim, acc_ptrs.data_ptr<int64_t>(),
        pos_ptrs.data_ptr<int64_t>(), list_ptrs.data_ptr<int64_t>(), cnt_ptrs.data_ptr<int64_t>(),
        per.data_ptr<int64_t>(), caps.data_ptr<int64_t>(), world, (float)scale, st, (int)my_rank);
  }
}

// The exchange form of engram_scatter_grad for world > 1 (row_push_kernel, then
// row_accumulate_kernel; see the kernels). `x` holds the exchange layout: xbases [world] int64,
// and the sizes cap_e (entries per inbox region), region_bytes, rows_off.
static RowTablesArgs row_tables_args(const torch::Tensor& acc_ptrs, const torch::Tensor& pos_ptrs,
                              const torch::Tensor& list_ptrs, const torch::Tensor& cnt_ptrs,
                              const torch::Tensor& per, const torch::Tensor& caps, const torch::Tensor& xbases,
                              int64_t n_tables, int64_t dim, int64_t me, int64_t cap_e, int64_t region_bytes,
                              int64_t rows_off, int64_t call, double timeout_s, torch::Tensor& status) {
  const int world = (int)xbases.numel();
  TORCH_CHECK(world >= 2 && world <= 16, "row exchange: 2..16 ranks");
  TORCH_CHECK(dim % 8 == 0 && rows_off % 16 == 0 && region_bytes % 256 == 0, "row exchange: alignment");
  TORCH_CHECK(acc_ptrs.numel() == world * n_tables && per.numel() == n_tables && caps.numel() == n_tables,
              "row exchange: pointer tables");
  RowTablesArgs a;
  a.acc_ptrs = acc_ptrs.data_ptr<int64_t>();
  a.pos_ptrs = pos_ptrs.data_ptr<int64_t>();
  a.list_ptrs = list_ptrs.data_ptr<int64_t>();
  a.cnt_ptrs = cnt_ptrs.data_ptr<int64_t>();
  a.per = per.data_ptr<int64_t>();
  a.caps = caps.data_ptr<int64_t>();
  a.xbases = xbases.data_ptr<int64_t>();
  a.n_tables = (int)n_tables;
  a.dim = (int)dim;
  a.world = world;
  a.me = (int)me;
  a.cap_e = cap_e;
  a.region_bytes = region_bytes;
  a.rows_off = rows_off;
  a.call = (uint32_t)call;
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.status = status.data_ptr<int>();
  return a;
}

void engram_push_grads(torch::Tensor g, torch::Tensor idx, torch::Tensor acc_ptrs, torch::Tensor pos_ptrs,
                       torch::Tensor list_ptrs, torch::Tensor cnt_ptrs, torch::Tensor per, torch::Tensor caps,
                       torch::Tensor xbases, int64_t me, double scale, int64_t cap_e, int64_t region_bytes,
                       int64_t rows_off, int64_t call, double timeout_s, torch::Tensor status) {
  check_cuda(g, "g");
  check_cuda(idx, "idx");
  TORCH_CHECK(g.scalar_type() == torch::kBFloat16 && g.is_contiguous(), "row exchange: bf16 contiguous grads");
  const at::cuda::CUDAGuard guard(g.device());
  const int64_t nt = idx.size(0), N = idx.size(1);
  const int64_t dim = N ? g.size(1) / nt : 8;
  TORCH_CHECK(N == 0 || (g.size(0) == N && g.size(1) == nt * dim), "row exchange: g must be [N, n_tables * dim]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0, "row exchange: 16-byte aligned grads");
  RowTablesArgs a = row_tables_args(acc_ptrs, pos_ptrs, list_ptrs, cnt_ptrs, per, caps, xbases, nt, dim, me, cap_e,
                                    region_bytes, rows_off, call, timeout_s, status);
  // every launch signals its peers, also with no events (their accumulate waits for it)
  const int grid = grid_for(std::max<int64_t>(1, N * nt * 8), 256);
  row_push_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), idx.data_ptr<int64_t>(), N, a, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void engram_accumulate_grads(torch::Tensor acc_ptrs, torch::Tensor pos_ptrs, torch::Tensor list_ptrs,
                             torch::Tensor cnt_ptrs, torch::Tensor per, torch::Tensor caps, torch::Tensor xbases,
                             int64_t n_tables, int64_t dim, int64_t me, double scale, int64_t cap_e,
                             int64_t region_bytes, int64_t rows_off, int64_t call, double timeout_s,
                             torch::Tensor status) {
  const at::cuda::CUDAGuard guard(status.device());
  RowTablesArgs a = row_tables_args(acc_ptrs, pos_ptrs, list_ptrs, cnt_ptrs, per, caps, xbases, n_tables, dim, me,
                                    cap_e, region_bytes, rows_off, call, timeout_s, status);
  row_accumulate_kernel<<<sm_count() * 4, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, (float)scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// The owner-served fetch (rows_serve_kernel, then rows_collect_kernel; RowStore.gather calls both
// in turn): `idx` [n_tables, N] int64 must already be in this rank's fetch buffer (its idx
// region, row stride cap_tok); `out` receives the N x n_tables rows in the tables' dtype.
// Collective: every rank makes the same calls in the same order.
static FetchArgs fetch_args(const torch::Tensor& fbases, const torch::Tensor& wptrs, const torch::Tensor& per,
                            int64_t me, int64_t n_tables, int64_t row_bytes, int64_t cap_tok, int64_t recv_off,
                            int64_t call, double timeout_s, torch::Tensor& status) {
  const int world = (int)fbases.numel();
  TORCH_CHECK(world >= 2 && world <= 16, "engram_fetch: 2..16 ranks");
  TORCH_CHECK(row_bytes % 16 == 0 && recv_off % 16 == 0, "engram_fetch: 16-byte rows and receive buffer");
  TORCH_CHECK(wptrs.numel() == world * n_tables && per.numel() == n_tables, "engram_fetch: tables");
  FetchArgs a;
  a.fbases = fbases.data_ptr<int64_t>();
  a.wptrs = wptrs.data_ptr<int64_t>();
  a.per = per.data_ptr<int64_t>();
  a.n_tables = (int)n_tables;
  a.row16 = (int)(row_bytes / 16);
  a.world = world;
  a.me = (int)me;
  a.cap_tok = cap_tok;
  a.recv_off = recv_off;
  a.call = (uint32_t)call;
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.status = status.data_ptr<int>();
  return a;
}

void engram_fetch_serve(torch::Tensor fbases, torch::Tensor wptrs, torch::Tensor per, int64_t me, int64_t n_tables,
                        int64_t row_bytes, int64_t ntok, int64_t cap_tok, int64_t recv_off, int64_t call,
                        double timeout_s, torch::Tensor status) {
  TORCH_CHECK(ntok >= 0 && ntok <= cap_tok, "engram_fetch: more tokens than the fetch buffer holds");
  const at::cuda::CUDAGuard guard(status.device());
  FetchArgs a = fetch_args(fbases, wptrs, per, me, n_tables, row_bytes, cap_tok, recv_off, call, timeout_s, status);
  rows_serve_kernel<<<sm_count() * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a, (int)ntok);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void engram_fetch_collect(torch::Tensor fbases, torch::Tensor wptrs, torch::Tensor per, int64_t me, int64_t n_tables,
                          int64_t row_bytes, int64_t ntok, int64_t cap_tok, int64_t recv_off, int64_t call,
                          double timeout_s, torch::Tensor status, torch::Tensor out) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && (int64_t)out.nbytes() >= ntok * n_tables * row_bytes &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "engram_fetch: out must hold the rows (16-byte aligned)");
  const at::cuda::CUDAGuard guard(out.device());
  FetchArgs a = fetch_args(fbases, wptrs, per, me, n_tables, row_bytes, cap_tok, recv_off, call, timeout_s, status);
  const int64_t n16 = ntok * n_tables * (row_bytes / 16);
  rows_collect_kernel<<<grid_for(std::max<int64_t>(1, n16), 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, n16, reinterpret_cast<uint4*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// sq (fp32 [1], accumulated into) += sum over the local touched rows of acc^2.
void engram_touched_sqnorm(torch::Tensor acc_ptrs, torch::Tensor cnt_ptrs, torch::Tensor caps, int64_t dim,
                           torch::Tensor sq) {
  const at::cuda::CUDAGuard guard(sq.device());
  const int nt = (int)acc_ptrs.numel();
  TORCH_CHECK(dim % 4 == 0, "engram_touched_sqnorm: dim must be a multiple of 4");
  touched_sqnorm_kernel<<<sm_count() * 4, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      acc_ptrs.data_ptr<int64_t>(), cnt_ptrs.data_ptr<int64_t>(), caps.data_ptr<int64_t>(), nt, (int)dim,
      sq.data_ptr<float>());
}

void engram_clip_coef(torch::Tensor sq, double max_norm, torch::Tensor coef, torch::Tensor norm) {
  const at::cuda::CUDAGuard guard(sq.device());
  clip_coef_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(
      sq.data_ptr<float>(), (float)max_norm, coef.data_ptr<float>(), norm.data_ptr<float>());
}

// Touched-row AdamW of up to kAdamMaxTables tables of one row store in one launch per 32 tables.
// Per table: weights p, moments m and v (v fp32 [rows] when row-wise), compact accumulator acc,
// pos, list, cnt, and its own table id, bias corrections and step (rounding-bit key).
void engram_adam_rows(std::vector<torch::Tensor> p, std::vector<torch::Tensor> m, std::vector<torch::Tensor> v,
                      std::vector<torch::Tensor> acc, std::vector<torch::Tensor> pos, std::vector<torch::Tensor> list,
                      std::vector<torch::Tensor> cnt, std::vector<int64_t> table_ids, std::vector<double> bc1,
                      std::vector<double> bc2, std::vector<int64_t> steps, c10::optional<torch::Tensor> coef,
                      double lr, double beta1, double beta2, double eps, double wd, bool sr, int64_t seed) {
  const size_t n = p.size();
  TORCH_CHECK(m.size() == n && v.size() == n && acc.size() == n && pos.size() == n && list.size() == n &&
                  cnt.size() == n && table_ids.size() == n && bc1.size() == n && bc2.size() == n && steps.size() == n,
              "engram_adam_rows: one entry per table in every list");
  if (n == 0) return;
  check_cuda(p[0], "p");
  const at::cuda::CUDAGuard guard(p[0].device());
  const auto dtype = p[0].scalar_type();
  const int dim = (int)p[0].size(1);
  TORCH_CHECK(dim % 8 == 0 && dim <= 256, "engram_adam_rows: dim must be a multiple of 8, at most 256");
  TORCH_CHECK(dtype == torch::kBFloat16 || dtype == torch::kFloat32, "engram_adam_rows: bf16 or fp32 tables");
  auto device_view = [](const torch::Tensor& t, const char* name) -> void* {
    if (t.is_cuda()) return t.data_ptr();
    TORCH_CHECK(t.is_pinned(), name, " must live on the GPU or in pinned host memory");
    cudaPointerAttributes attr;
    C10_CUDA_CHECK(cudaPointerGetAttributes(&attr, t.data_ptr()));
    TORCH_CHECK(attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr, name,
                ": pinned host memory without a device mapping");
    return attr.devicePointer;
  };
  const float* cp = coef.has_value() ? coef->data_ptr<float>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  for (size_t a = 0; a < n; a += kAdamMaxTables) {
    AdamTables tabs{};
    tabs.n = (int)std::min<size_t>(kAdamMaxTables, n - a);
    for (int i = 0; i < tabs.n; ++i) {
      const size_t k = a + i;
      TORCH_CHECK(p[k].scalar_type() == dtype && p[k].size(1) == dim && p[k].is_contiguous(),
                  "engram_adam_rows: tables of one dtype and width");
      TORCH_CHECK(m[k].scalar_type() == dtype && m[k].numel() == p[k].numel(), "engram_adam_rows: exp_avg");
      TORCH_CHECK(acc[k].dim() == 2 && acc[k].size(1) == dim && pos[k].numel() >= p[k].size(0) &&
                      list[k].numel() >= acc[k].size(0),
                  "engram_adam_rows: compact accumulator shapes");
      const bool rowwise = v[k].dim() == 1;
      TORCH_CHECK(rowwise ? (v[k].is_cuda() && v[k].scalar_type() == torch::kFloat32) : v[k].scalar_type() == dtype,
                  "engram_adam_rows: exp_avg_sq");
      AdamTable& t = tabs.t[i];
      t.p = p[k].data_ptr();
      t.m = device_view(m[k], "exp_avg");
      t.v_row = rowwise ? v[k].data_ptr<float>() : nullptr;
      t.v_val = rowwise ? nullptr : device_view(v[k], "exp_avg_sq");
      t.acc = acc[k].data_ptr<float>();
      t.pos = pos[k].data_ptr<int>();
      t.list = list[k].data_ptr<int>();
      t.cnt = cnt[k].data_ptr<int>();
      t.cap = (int)acc[k].size(0);
      t.table_id = (uint32_t)table_ids[k];
      t.step = (uint32_t)steps[k];
      t.bc1 = (float)bc1[k];
      t.bc2_sqrt = (float)std::sqrt(bc2[k]);
    }
    const int grid = sm_count() * 8;
    auto run = [&](auto type_tag, auto cpl_tag) {
      using T = decltype(type_tag);
      constexpr int CPL = decltype(cpl_tag)::value;
      adam_rows_kernel<T, CPL><<<grid, 256, 0, stream>>>(tabs, dim, cp, (float)lr, (float)beta1, (float)beta2,
                                                          (float)eps, (float)wd, sr && sizeof(T) == 2 ? 1 : 0,
                                                          (uint32_t)seed);
    };
    auto by_width = [&](auto type_tag) {
      if (dim <= 64) run(type_tag, std::integral_constant<int, 1>{});
      else if (dim <= 128) run(type_tag, std::integral_constant<int, 2>{});
      else run(type_tag, std::integral_constant<int, 4>{});
    };
    if (dtype == torch::kBFloat16) by_width(__nv_bfloat16{});
    else by_width(float{});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void engram_adam_touched(torch::Tensor p, torch::Tensor m, torch::Tensor v, torch::Tensor acc,
                         torch::Tensor pos, torch::Tensor list, torch::Tensor cnt,
                         c10::optional<torch::Tensor> coef, double lr, double beta1, double beta2,
                         double eps, double wd, double bc1, double bc2, bool sr, int64_t seed,
                         int64_t step, int64_t table_id) {
  check_cuda(p, "p");
  const at::cuda::CUDAGuard guard(p.device());
  const int dim = (int)p.size(1);
  TORCH_CHECK(dim <= 256, "engram dim above 256 is not supported by the touched-row Adam");
  TORCH_CHECK(m.scalar_type() == p.scalar_type(), "exp_avg must have the weight dtype");
  TORCH_CHECK(m.is_contiguous() && m.numel() == p.numel(), "exp_avg must be contiguous and shaped like the table");
  // moments on this GPU, or in pinned host memory that the kernel reads and writes in place
  // through its device mapping (only the touched rows cross PCIe)
  auto device_view = [](const torch::Tensor& t, const char* name) -> void* {
    if (t.is_cuda()) return t.data_ptr();
    TORCH_CHECK(t.is_pinned(), name, " must live on the GPU or in pinned host memory");
    cudaPointerAttributes attr;
    C10_CUDA_CHECK(cudaPointerGetAttributes(&attr, t.data_ptr()));
    TORCH_CHECK(attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr, name,
                ": pinned host memory without a device mapping");
    return attr.devicePointer;
  };
  void* m_dev = device_view(m, "exp_avg");
  const bool rowwise = v.dim() == 1;
  TORCH_CHECK(rowwise ? v.scalar_type() == torch::kFloat32 : v.scalar_type() == p.scalar_type(),
              "exp_avg_sq dtype");
  TORCH_CHECK(acc.dim() == 2 && acc.size(1) == dim && pos.numel() >= p.size(0) && list.numel() >= acc.size(0),
              "compact accumulator shapes");
  const int cap = (int)acc.size(0);
  const int threads = 256;
  const int grid = sm_count() * 4;
  auto stream = at::cuda::getCurrentCUDAStream();
  const float* cp = coef.has_value() ? coef->data_ptr<float>() : nullptr;
  const float bc2s = (float)std::sqrt(bc2);
  TORCH_CHECK(!rowwise || v.is_cuda(), "a row-wise exp_avg_sq stays on the GPU");
  void* v_dev = device_view(v, "exp_avg_sq");
  float* vrow = rowwise ? reinterpret_cast<float*>(v_dev) : nullptr;
  if (p.scalar_type() == torch::kBFloat16) {
    adam_touched_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, threads, 0, stream>>>(
        reinterpret_cast<__nv_bfloat16*>(p.data_ptr()), reinterpret_cast<__nv_bfloat16*>(m_dev), vrow,
        rowwise ? nullptr : reinterpret_cast<__nv_bfloat16*>(v_dev), acc.data_ptr<float>(),
        pos.data_ptr<int>(), list.data_ptr<int>(), cnt.data_ptr<int>(), cap, dim, cp, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd, (float)bc1, bc2s, sr ? 1 : 0,
        (uint32_t)seed, (uint32_t)step, (uint32_t)table_id);
  } else {
    TORCH_CHECK(p.scalar_type() == torch::kFloat32, "tables must be bf16 or fp32");
    adam_touched_kernel<float, float><<<grid, threads, 0, stream>>>(
        p.data_ptr<float>(), reinterpret_cast<float*>(m_dev), vrow, rowwise ? nullptr : reinterpret_cast<float*>(v_dev),
        acc.data_ptr<float>(), pos.data_ptr<int>(), list.data_ptr<int>(), cnt.data_ptr<int>(), cap, dim, cp, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd,
        (float)bc1, bc2s, 0, (uint32_t)seed, (uint32_t)step, (uint32_t)table_id);
  }
}

void adam_dense(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr,
                double beta1, double beta2, double eps, double wd, double bc1, double bc2, double gscale,
                bool sr, int64_t seed, int64_t step) {
  check_cuda(p, "p");
  check_cuda(g, "g");
  const at::cuda::CUDAGuard guard(p.device());
  const int64_t n = p.numel();
  if (n == 0) return;
  const int threads = 256;
  const int grid = grid_for(n, threads, 4);
  auto stream = at::cuda::getCurrentCUDAStream();
  const float bc2s = (float)std::sqrt(bc2);
  TORCH_CHECK(m.scalar_type() == p.scalar_type() && v.scalar_type() == p.scalar_type(), "moment dtype");
  if (p.scalar_type() == torch::kBFloat16) {
    auto* pp = reinterpret_cast<__nv_bfloat16*>(p.data_ptr());
    auto* mp = reinterpret_cast<__nv_bfloat16*>(m.data_ptr());
    auto* vp = reinterpret_cast<__nv_bfloat16*>(v.data_ptr());
    if (g.scalar_type() == torch::kFloat32)
      adam_dense_kernel<__nv_bfloat16, float><<<grid, threads, 0, stream>>>(
          pp, g.data_ptr<float>(), mp, vp, n, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)wd,
          (float)bc1, bc2s, (float)gscale, sr ? 1 : 0, (uint32_t)seed, (uint32_t)step);
    else
      adam_dense_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, threads, 0, stream>>>(
          pp, reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), mp, vp, n, (float)lr, (float)beta1,
          (float)beta2, (float)eps, (float)wd, (float)bc1, bc2s, (float)gscale, sr ? 1 : 0, (uint32_t)seed,
          (uint32_t)step);
  } else {
    TORCH_CHECK(p.scalar_type() == torch::kFloat32 && g.scalar_type() == torch::kFloat32, "fp32 adam");
    adam_dense_kernel<float, float><<<grid, threads, 0, stream>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), n, (float)lr,
        (float)beta1, (float)beta2, (float)eps, (float)wd, (float)bc1, bc2s, (float)gscale, 0, (uint32_t)seed,
        (uint32_t)step);
  }
}

// A persistent grid: as many blocks as fit on every SM at once, at most one per row.
template <typename K>
static int occupancy_grid(K kernel, int threads, int64_t rows) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return (int)std::max<int64_t>(1, std::min<int64_t>(rows, (int64_t)sm_count() * per_sm));
}

// The vectorised gate wants 8-element (16-byte) chunks: d % 8 == 0, 16-byte aligned rows and
// scales, hidden size at most 8192 (4 chunks of 8 per thread at 256 threads).
static bool gate_vec_ok(int d, std::initializer_list<const void*> rows, const float* qs, const float* ks) {
  if (d % 8 != 0 || d > 8192) return false;
  for (const void* p : rows)
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return false;
  if ((qs && reinterpret_cast<uintptr_t>(qs) % 16) || (ks && reinterpret_cast<uintptr_t>(ks) % 16)) return false;
  return true;
}

// stats [N, 4] fp32 out; gate_acc [3] fp32 (accumulated) or None.
std::vector<torch::Tensor> engram_gate_fwd(torch::Tensor h, torch::Tensor k, torch::Tensor v,
                                           c10::optional<torch::Tensor> qs, c10::optional<torch::Tensor> ks,
                                           c10::optional<torch::Tensor> keep, bool sqrt_gate,
                                           c10::optional<torch::Tensor> gate_acc) {
  check_cuda(h, "hidden");
  check_cuda(k, "key");
  check_cuda(v, "value");
  TORCH_CHECK(h.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16,
              "the fused gate runs on bf16 hidden/key/value");
  const at::cuda::CUDAGuard guard(h.device());
  const int d = (int)h.size(-1);
  const int64_t N = h.numel() / d;
  auto out = torch::empty_like(h);
  auto stats = torch::empty({N, 4}, h.options().dtype(torch::kFloat32));
  if (N == 0) return {out, stats};
  const float* qsp0 = qs.has_value() ? qs->data_ptr<float>() : nullptr;
  const float* ksp0 = ks.has_value() ? ks->data_ptr<float>() : nullptr;
  if (gate_vec_ok(d, {h.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), stats.data_ptr()}, qsp0, ksp0)) {
    const int nch = (d / 8 + 255) / 256;
    const int threads = ((d / 8 + nch - 1) / nch + 31) / 32 * 32;
    auto stream = at::cuda::getCurrentCUDAStream();
    auto U = [](const torch::Tensor& t) { return reinterpret_cast<const uint4*>(t.data_ptr()); };
    const uint8_t* kpp0 = keep.has_value() ? keep->data_ptr<uint8_t>() : nullptr;
    float* gap0 = gate_acc.has_value() ? gate_acc->data_ptr<float>() : nullptr;
#define ME_GATE_FWD_VEC(C)                                                                                  \
  const int grid = occupancy_grid(gate_fwd_vec_kernel<C>, threads, N);                                      \
  gate_fwd_vec_kernel<C><<<grid, threads, 0, stream>>>(U(h), U(k), U(v), qsp0, ksp0, kpp0, N, d, sqrt_gate ? 1 : 0, \
                                                       reinterpret_cast<uint4*>(out.data_ptr()),            \
                                                       stats.data_ptr<float>(), gap0)
    if (nch == 1) { ME_GATE_FWD_VEC(1); }
    else if (nch == 2) { ME_GATE_FWD_VEC(2); }
    else if (nch == 3) { ME_GATE_FWD_VEC(3); }
    else { ME_GATE_FWD_VEC(4); }
#undef ME_GATE_FWD_VEC
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {out, stats};
  }
  const int threads = 256;
  const int vpt = (d + threads - 1) / threads;
  TORCH_CHECK(vpt <= 32, "hidden size above 8192 is not supported by the fused gate");
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 8);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  auto* kp = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  auto* vp = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  const float* qsp = qs.has_value() ? qs->data_ptr<float>() : nullptr;
  const float* ksp = ks.has_value() ? ks->data_ptr<float>() : nullptr;
  const uint8_t* kpp = keep.has_value() ? keep->data_ptr<uint8_t>() : nullptr;
  float* gap = gate_acc.has_value() ? gate_acc->data_ptr<float>() : nullptr;
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
#define ME_GATE_FWD(V)                                                                                  \
  gate_fwd_kernel<V><<<grid, threads, 0, stream>>>(hp, kp, vp, qsp, ksp, kpp, N, d, sqrt_gate ? 1 : 0, op, \
                                                   stats.data_ptr<float>(), gap)
  if (vpt <= 8) ME_GATE_FWD(8);
  else if (vpt <= 16) ME_GATE_FWD(16);
  else if (vpt <= 24) ME_GATE_FWD(24);
  else ME_GATE_FWD(32);
#undef ME_GATE_FWD
  return {out, stats};
}

std::vector<torch::Tensor> engram_gate_bwd(torch::Tensor g, torch::Tensor h, torch::Tensor k, torch::Tensor v,
                                           c10::optional<torch::Tensor> qs, c10::optional<torch::Tensor> ks,
                                           c10::optional<torch::Tensor> keep, torch::Tensor stats,
                                           bool sqrt_gate) {
  check_cuda(g, "grad");
  const at::cuda::CUDAGuard guard(h.device());
  auto gc = g.contiguous();
  const int d = (int)h.size(-1);
  const int64_t N = h.numel() / d;
  auto dh = torch::empty_like(h), dk = torch::empty_like(k), dv = torch::empty_like(v);
  torch::Tensor dqs, dks;
  if (qs.has_value()) {
    dqs = torch::zeros({d}, h.options().dtype(torch::kFloat32));
    dks = torch::zeros({d}, h.options().dtype(torch::kFloat32));
  }
  if (N == 0) return {dh, dk, dv, dqs, dks};
  {
    const float* qsp0 = qs.has_value() ? qs->data_ptr<float>() : nullptr;
    const float* ksp0 = ks.has_value() ? ks->data_ptr<float>() : nullptr;
    if (gate_vec_ok(d, {gc.data_ptr(), h.data_ptr(), k.data_ptr(), v.data_ptr(), dh.data_ptr(), dk.data_ptr(),
                        dv.data_ptr(), stats.data_ptr()}, qsp0, ksp0) &&
        stats.is_contiguous() && stats.scalar_type() == torch::kFloat32) {
      const int nch = (d / 8 + 255) / 256;
      const int threads = ((d / 8 + nch - 1) / nch + 31) / 32 * 32;
      auto stream = at::cuda::getCurrentCUDAStream();
      auto U = [](const torch::Tensor& t) { return reinterpret_cast<const uint4*>(t.data_ptr()); };
      auto W = [](torch::Tensor& t) { return reinterpret_cast<uint4*>(t.data_ptr()); };
      const uint8_t* kpp0 = keep.has_value() ? keep->data_ptr<uint8_t>() : nullptr;
      float* dq0 = qs.has_value() ? dqs.data_ptr<float>() : nullptr;
      float* dk0 = qs.has_value() ? dks.data_ptr<float>() : nullptr;
#define ME_GATE_BWD_VEC(C)                                                                                   \
  const int grid = occupancy_grid(gate_bwd_vec_kernel<C>, threads, N);                                       \
  gate_bwd_vec_kernel<C><<<grid, threads, 0, stream>>>(U(gc), U(h), U(k), U(v), qsp0, ksp0, kpp0,              \
                                                       stats.data_ptr<float>(), N, d, sqrt_gate ? 1 : 0, W(dh), \
                                                       W(dk), W(dv), dq0, dk0)
      if (nch == 1) { ME_GATE_BWD_VEC(1); }
      else if (nch == 2) { ME_GATE_BWD_VEC(2); }
      else if (nch == 3) { ME_GATE_BWD_VEC(3); }
      else { ME_GATE_BWD_VEC(4); }
#undef ME_GATE_BWD_VEC
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return {dh, dk, dv, dqs, dks};
    }
  }
  const int threads = 256;
  const int vpt = (d + threads - 1) / threads;
  TORCH_CHECK(vpt <= 32, "hidden size above 8192 is not supported by the fused gate");
  const int grid = (int)std::min<int64_t>(N, (int64_t)sm_count() * 4);
  auto stream = at::cuda::getCurrentCUDAStream();
  const float* qsp = qs.has_value() ? qs->data_ptr<float>() : nullptr;
  const float* ksp = ks.has_value() ? ks->data_ptr<float>() : nullptr;
  const uint8_t* kpp = keep.has_value() ? keep->data_ptr<uint8_t>() : nullptr;
#define BF(t) reinterpret_cast<__nv_bfloat16*>(t.data_ptr())
#define CBF(t) reinterpret_cast<const __nv_bfloat16*>(t.data_ptr())
#define ME_GATE_BWD(V)                                                                                   \
  gate_bwd_kernel<V><<<grid, threads, 0, stream>>>(CBF(gc), CBF(h), CBF(k), CBF(v), qsp, ksp, kpp,         \
                                                   stats.data_ptr<float>(), N, d, sqrt_gate ? 1 : 0, BF(dh), \
                                                   BF(dk), BF(dv), qs.has_value() ? dqs.data_ptr<float>() : nullptr, \
                                                   qs.has_value() ? dks.data_ptr<float>() : nullptr)
  if (vpt <= 8) ME_GATE_BWD(8);
  else if (vpt <= 16) ME_GATE_BWD(16);
  else if (vpt <= 24) ME_GATE_BWD(24);
  else ME_GATE_BWD(32);
#undef ME_GATE_BWD
#undef BF
#undef CBF
  return {dh, dk, dv, dqs, dks};
}

// ------------------------------------------------------------------------------ serving histories
// For every token a serving step runs, its n-gram history: out[t, i] = token at position p_t - i
// of the same request, -1 before the request's first token; rows [num_tokens, num_padded) = -1.
// Tokens from the step's own chunk come from input_ids (t - i), earlier ones from the request's
// row of all_ids (micro_engram_vllm/ids.py:10-59 of the reference states the same rule as torch
// ops). One thread per (token, i); the request of token t is found by binary search over the
// request offsets `qsl`. Index tensors may be int32 or int64 (is64 flags per tensor).
ME_DEVICE int64_t ld_index(const void* p, int is64, int64_t i) {
  return is64 ? reinterpret_cast<const int64_t*>(p)[i] : (int64_t)reinterpret_cast<const int32_t*>(p)[i];
}

__global__ void fill_ids_kernel(int32_t* __restrict__ out, int max_order, const void* input_ids, int ids64,
                                const void* positions, int pos64, const void* idx_mapping, int map64,
                                const void* qsl, int qsl64, const void* all_ids, int all64, int64_t all_stride,
                                int num_reqs, int num_tokens, int num_padded) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)num_padded * max_order) return;
  const int t = (int)(e / max_order), i = (int)(e % max_order);
  if (t >= num_tokens) {
    out[e] = -1;
    return;
  }
  int lo = 0, hi = num_reqs - 1;  // last request whose first token is <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ld_index(qsl, qsl64, mid) <= t) lo = mid;
    else hi = mid - 1;
  }
  const int64_t first = ld_index(qsl, qsl64, lo);
  const int64_t chunk_start = ld_index(positions, pos64, first);
  const int64_t q = ld_index(positions, pos64, t) - i;
  int64_t v;
  if (q < 0) v = -1;
  else if (q >= chunk_start) v = ld_index(input_ids, ids64, t - i);
  else v = ld_index(all_ids, all64, ld_index(idx_mapping, map64, lo) * all_stride + q);
  out[e] = (int32_t)v;
}

void engram_fill_ids(torch::Tensor out, torch::Tensor input_ids, torch::Tensor positions, torch::Tensor idx_mapping,
                     torch::Tensor qsl, torch::Tensor all_ids, int64_t num_reqs, int64_t num_tokens,
                     int64_t num_padded) {
  check_cuda(out, "out");
  TORCH_CHECK(out.scalar_type() == torch::kInt32 && out.dim() == 2 && out.is_contiguous(),
              "out must be a contiguous [max_tokens, max_order] int32 buffer");
  TORCH_CHECK(num_padded <= out.size(0) && num_tokens <= num_padded, "more tokens than the buffer holds");
  TORCH_CHECK(all_ids.dim() == 2 && all_ids.stride(1) == 1, "all_token_ids must be [max_reqs, max_len] row-major");
  auto is64 = [](const torch::Tensor& x) {
    TORCH_CHECK(x.scalar_type() == torch::kInt32 || x.scalar_type() == torch::kInt64, "index tensors are int32/int64");
    TORCH_CHECK(x.dim() == 2 || x.stride(0) == 1, "index vectors must be contiguous");
    return x.scalar_type() == torch::kInt64 ? 1 : 0;
  };
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t n = num_padded * out.size(1);
  if (n == 0) return;
  if (num_tokens > 0) TORCH_CHECK(num_reqs > 0, "tokens without requests");
  const int threads = 256;
  fill_ids_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      out.data_ptr<int32_t>(), (int)out.size(1), input_ids.data_ptr(), is64(input_ids), positions.data_ptr(),
      is64(positions), idx_mapping.data_ptr(), is64(idx_mapping), qsl.data_ptr(), is64(qsl), all_ids.data_ptr(),
      is64(all_ids), all_ids.stride(0), (int)num_reqs, (int)num_tokens, (int)num_padded);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
