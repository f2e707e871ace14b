// autotune_table.h -- token tile (MMA N, chunk size) of the grouped GEMMs per token count.
//
// Committed table, replacing the reference's fixed tiles and its T <= 512 path switch
// (solution/cuda/kernel.cu:41-51, :1781). A chunk is up to tile_n rows of one expert;
// each chunk re-reads the expert's weight tiles, so the tile should cover the typical
// rows per active expert (about T * top_k * E_local / E_global / active experts) while
// keeping the N side of the MMA busy. Entries are (largest T, tile_n), first match wins.
// The values come from the sweep recorded in profiles/autotune_sweep.md.
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

}  // namespace fmoe
