// Copying a list of byte ranges from peer memory into this GPU's memory with plain 16-byte
// loads and stores: the all-gather of a row-sharded frozen layer. One copy job is a table of
// segments (one per weight matrix and owning rank); the job is addressed as the concatenation
// of its segments in 16-byte units, so it can be split into ranges and the ranges handed to
// different kernels (each tcgen05 GEMM of a layer carries a share of the next layer's gather in
// one extra warp per CTA; `layer_gather` runs a range as a kernel of its own).
//
// Loads go to L2 only (a peer's lines are never cached in this GPU's L1). Every warp keeps UNR
// 16-byte loads in flight per lane before storing, enough bytes per SM to cover an NVLink round
// trip.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace me {

struct GatherSeg {
  int64_t src;      // source address (a peer's mapping, or this GPU's own shard)
  int64_t dst;      // destination address on this GPU
  int64_t start16;  // first 16-byte unit of this segment in the job's concatenation
  int64_t n16;      // length in 16-byte units
};

// Copy units [begin16, end16) of the job, split over `nworkers` warps (this warp is `worker`).
ME_DEVICE void gather_range(const GatherSeg* __restrict__ segs, int nsegs, int64_t begin16, int64_t end16,
                            int worker, int nworkers, int lane) {
  constexpr int UNR = 16;
  constexpr int64_t CHUNK = 32 * UNR;  // units per warp iteration
  for (int s = 0; s < nsegs; ++s) {
    const GatherSeg g = segs[s];
    const int64_t lo = begin16 > g.start16 ? begin16 : g.start16;
    const int64_t hi = end16 < g.start16 + g.n16 ? end16 : g.start16 + g.n16;
    if (lo >= hi) continue;
    const uint4* src = reinterpret_cast<const uint4*>(g.src);
    uint4* dst = reinterpret_cast<uint4*>(g.dst);
    for (int64_t base = lo + (int64_t)worker * CHUNK; base < hi; base += (int64_t)nworkers * CHUNK) {
      uint4 v[UNR];
#pragma unroll
      for (int j = 0; j < UNR; ++j) {
        const int64_t e = base + j * 32 + lane;
        if (e < hi) v[j] = __ldcg(src + (e - g.start16));
      }
#pragma unroll
      for (int j = 0; j < UNR; ++j) {
        const int64_t e = base + j * 32 + lane;
        if (e < hi) dst[e - g.start16] = v[j];
      }
    }
  }
}

}  // namespace me
