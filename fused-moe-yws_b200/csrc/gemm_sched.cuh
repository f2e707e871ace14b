// gemm_sched.cuh -- work schedule shared by the grouped GEMM kernels: which tiles and
// K-step ranges each persistent CTA processes.
#pragma once

#include <cstdint>

namespace fmoe {

constexpr int kMaxKSteps = 128;  // H/128 and I/128 are validated <= 128

// Stream-K work split: the launch's work is num_tiles x KS K-steps, CTA c owns the
// contiguous global step range [start(c), start(c+1)). Ranges are cut at tile boundaries
// into segments; a segment that does not cover its whole tile is a partial.
struct StreamK {
  int64_t W;  // total K-steps
  int G;      // CTAs
  __device__ __forceinline__ int64_t start(int c) const { return (int64_t)c * W / G; }
  // the CTA whose range contains global step g
  __device__ __forceinline__ int cta_of(int64_t g) const {
    return (int)(((g + 1) * G + W - 1) / W) - 1;
  }
};

// Per-CTA work sequence: whole tiles round-robin over the CTAs for all but the last one
// to two waves ("data parallel": CTAs that run together work on neighbouring tiles, so an
// expert's weight tiles are shared through L2 by its chunks), then the remaining tiles
// split by stream-K in K-step units so every CTA ends at the same time. Every role of a
// CTA walks the same sequence. (Measured on B200: putting the split tiles first, or
// starting whole tiles at a CTA-dependent K step, is slower at every T.)
// A launch of G/2 .. G tiles runs them whole, one per CTA: the fix-up round trips of split
// tiles (partial stores, fences, counters: microseconds each while the other CTAs saturate
// HBM) cost more than the idle CTAs. Below G/2 tiles, splitting still wins: one CTA's
// per-K-step issue and promotion cost caps it far below its share of HBM bandwidth, so
// more CTAs must stream. (Decode calls on B200, graph-replayed device time: T = 1 66.8 ->
// 61.4 us, T = 4 81.5 -> 73.7, T = 8 82 -> 74.5; whole tiles for every launch of <= G tiles
// made T = 1 slower, its GEMM1 having 48 tiles.)
struct Schedule {
  int KS, G, cta;
  int dp_tiles;  // whole-tile prefix, a multiple of G
  StreamK sk;    // over the remaining tiles, in K-step units
  int64_t g, g_end;
  int dp_next;

  __device__ __forceinline__ Schedule(int num_tiles, int ks, int grid, int c) {
    KS = ks;
    G = grid;
    cta = c;
    dp_tiles = num_tiles <= G && 2 * num_tiles >= G ? num_tiles
               : num_tiles > 2 * G                      ? (num_tiles / G - 1) * G
                                                        : 0;
    sk.W = (int64_t)(num_tiles - dp_tiles) * KS;
    sk.G = G;
    g = sk.start(c);
    g_end = sk.start(c + 1);
    dp_next = c;
  }
  // next segment: tile index, K-step range [k0, k1); false when done
  __device__ __forceinline__ bool next(int& tile, int& k0, int& k1) {
    if (dp_next < dp_tiles) {
      tile = dp_next;
      k0 = 0;
      k1 = KS;
      dp_next += G;
      return true;
    }
    if (g < g_end) {
      const int64_t lt = g / KS;
      k0 = (int)(g % KS);
      k1 = (int)((int64_t)KS < k0 + (g_end - g) ? KS : k0 + (g_end - g));
      g += k1 - k0;
      tile = dp_tiles + (int)lt;
      return true;
    }
    return false;
  }
  __device__ __forceinline__ int64_t sk_begin() const { return sk.start(cta); }
  // Every CTA's stream-K range spans at least KS steps, so a split tile shared by two CTAs
  // has its tail done as the second CTA's first split segment, long before the first CTA
  // reaches the tile's head as its last segment.
  __device__ __forceinline__ bool ranges_cover_a_tile() const { return sk.W / G >= KS; }
  // first global stream-K step of a split tile
  __device__ __forceinline__ int64_t tile_begin(int tile) const {
    return (int64_t)(tile - dp_tiles) * KS;
  }
};

// How a segment takes part in the fix-up of a split tile. Contributors are the CTAs
// cf .. cl holding the tile's K steps in order.
//   pair: exactly two contributors and ranges_cover_a_tile(): the head owner cf finishes
//     the tile. The tail owner cl stores its fp32 partial (slot 0) and release-adds its
//     step count to counter[cf], without waiting; cf, at the start of its head segment,
//     waits for that count, loads the partial as its accumulator's starting value,
//     accumulates its own steps on top and finalizes -- no fix-up at the end of the run.
//   otherwise every contributor stores a partial and adds to counter[cf]; the one whose
//     add completes the K range sums all partials in K order and finalizes.
struct SplitRole {
  bool split;     // the segment does not cover the whole tile
  bool pair;      // two-contributor protocol
  bool head;      // this CTA holds the tile's first K step
  int cf, cl;     // contributor CTAs
  int slot;       // partial slot of this CTA for the tile
  int64_t tb;     // first stream-K step of the tile
};

__device__ __forceinline__ SplitRole split_role(const Schedule& sc, int tile, int k0, int k1) {
  SplitRole r{};
  r.split = k0 != 0 || k1 != sc.KS;
  if (!r.split) return r;
  r.tb = sc.tile_begin(tile);
  r.cf = sc.sk.cta_of(r.tb);
  r.cl = sc.sk.cta_of(r.tb + sc.KS - 1);
  r.slot = sc.sk_begin() >= r.tb ? 0 : 1;
  r.pair = r.cl == r.cf + 1 && sc.ranges_cover_a_tile();
  r.head = k0 == 0;
  return r;
}

}  // namespace fmoe
