// autotune_table.h -- token tile (MMA N, chunk size) of the grouped GEMMs per expected
// number of routed rows per local expert.
//
// Committed table, replacing the reference's fixed tiles and its T <= 512 path switch
// (solution/cuda/kernel.cu:41-51, :1781). A chunk is up to tile_n rows of one expert; each
// chunk re-reads the expert's weight tiles, so the tile should cover the typical rows per
// expert while keeping the N side of the MMA busy. What the GEMMs see is rows per local
// expert, not tokens: with the top_k routes of T tokens spread over E_global experts, a
// local expert expects T * top_k / E_global rows, whatever the slice (32 experts of a
// DeepSeek-V3 rank, all 256 on one GPU, or the 16-expert contest geometry). Entries are
// (largest expected rows per local expert, tile_n), first match wins: tile 16 (the decode
// family) up to 8 rows, 64 up to 24 rows, then 128 (the throughput family). The values
// come from a tile sweep of both families on one B200 (graph-replayed calls, L2 flushed
// between calls); for DeepSeek-V3 routing (top_k 8 of 256) the bounds are T = 256 and 768.
#pragma once

#include <cstdint>

namespace fmoe {

struct TileChoice {
  int64_t max_rows_per_expert;
  int tile_n;
};

constexpr TileChoice kAutotuneTable[] = {
    {8, 16},
    {24, 64},
    {INT64_MAX, 128},
};

inline int autotune_tile_n(int64_t num_tokens, int top_k, int num_experts) {
  const int64_t routes = num_tokens * top_k;  // rows per local expert = routes / num_experts
  for (const TileChoice& c : kAutotuneTable)
    if (c.max_rows_per_expert == INT64_MAX || routes <= c.max_rows_per_expert * num_experts)
      return c.tile_n;
  return 128;
}

// Token tile of a call: the caller's choice (0 = the table); the throughput family (128)
// needs GEMM2's 256-row weight tiles to divide hidden_size, else 64 is used. Every entry
// point that plans chunks uses this, so they all launch the same plan for one problem.
inline int resolve_tile_n(int requested, int64_t num_tokens, int top_k, int num_experts,
                          int hidden_size) {
  const int bn = requested != 0 ? requested : autotune_tile_n(num_tokens, top_k, num_experts);
  return bn == 128 && hidden_size % 256 != 0 ? 64 : bn;
}

}  // namespace fmoe
