// autotune_table.h -- token tile (MMA N, chunk size) of the grouped GEMMs per token count.
//
// Committed table, replacing the reference's fixed tiles and its T <= 512 path switch
// (solution/cuda/kernel.cu:41-51, :1781). A chunk is up to tile_n rows of one expert;
// each chunk re-reads the expert's weight tiles, so the tile should cover the typical
// rows per active expert (about T * top_k * E_local / E_global / active experts) while
// keeping the N side of the MMA busy. Entries are (largest T, tile_n), first match wins.
// The values come from a tile sweep of both GEMM families on one B200 (graph-replayed
// calls, L2 flushed between calls).
#pragma once

#include <cstdint>

namespace fmoe {

struct TileChoice {
  int64_t max_tokens;
  int tile_n;
};

constexpr TileChoice kAutotuneTable[] = {
    {256, 16},
    {768, 64},
    {INT64_MAX, 128},
};

inline int autotune_tile_n(int64_t num_tokens) {
  for (const TileChoice& c : kAutotuneTable)
    if (num_tokens <= c.max_tokens) return c.tile_n;
  return 128;
}

// Token tile of a call: the caller's choice (0 = the table); the throughput family (128)
// needs GEMM2's 256-row weight tiles to divide hidden_size, else 64 is used. Every entry
// point that plans chunks uses this, so they all launch the same plan for one problem.
inline int resolve_tile_n(int requested, int64_t num_tokens, int hidden_size) {
  const int bn = requested != 0 ? requested : autotune_tile_n(num_tokens);
  return bn == 128 && hidden_size % 256 != 0 ? 64 : bn;
}

}  // namespace fmoe
