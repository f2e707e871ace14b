// fmoe_kernels.cuh -- argument blocks and launch entry points of the fused MoE kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>
#include <utility>

#include "fmoe_common.cuh"

namespace fmoe {

struct RouteArgs {
  const float* logits;     // [T, E]
  const uint16_t* bias;    // [E] bf16 bits
  const int* in_idx;       // routed mode: given [T, K] expert ids (logits unused); else null
  const float* in_w;       // routed mode: given [T, K] weights
  const int* t_dev;        // routed mode, or null: tokens actually present (<= T), read on the
                           // device; tokens [*t_dev, T) get no route
  int64_t T;
  int E, n_group, topk_group, top_k, E_local, local_offset;
  float rsf;
  int bn;                  // token tile of the grouped GEMMs (chunk size, a power of two)
  int bn_log2;
  int64_t row_cap, max_chunks;
  int* topk_idx;           // [T, K]
  float* topk_w;           // [T, K]
  int* cta_counts;         // [n_ctas, E_local]
  int* cta_base;           // [n_ctas, E_local]
  int* expert_cnt;         // [E_local]
  int* expert_off;         // [E_local + 1]
  int* meta;               // [kMetaWords]
  Chunk* chunks;           // [max_chunks]
  int inject_err;          // test hook: DeviceError bits CTA 0 ORs into the error word (0: none)
};

struct ScatterArgs {
  const uint8_t* hidden;        // [T, H] e4m3
  const float* hidden_scale;    // [H/128, T]
  int64_t T;
  int H, top_k, E_local, local_offset;
  int64_t row_cap;
  const int* topk_idx;
  const float* topk_w;
  const int* cta_base;
  const int* expert_cnt;
  const int* expert_off;
  int* token_row;               // [T, K]
  int* row_token;               // [row_cap]
  float* row_w;                 // [row_cap]
  uint8_t* a_perm;              // [row_cap, H]
  float* a_scale;               // [H/128, row_cap]
  int* meta;
};

struct GemmArgs {
  const Chunk* chunks;
  const int* meta;
  const int* expert_cnt;   // routed rows per local expert
  int m_tiles;             // weight-row tiles per expert (I/128 for GEMM1, H/128 for GEMM2)
  int k_steps;             // 128-wide K steps: H/128 (GEMM1) or I/128 (GEMM2)
  int H, I;
  int64_t row_cap;         // leading dimension of the activation scale arrays
  const float* w_scale;    // [E_local, rows/128, cols/128]
  const float* act_scale;  // GEMM1: a_scale [H/128, row_cap]; GEMM2: c_scale [I/128, row_cap]
  // GEMM1 outputs
  uint8_t* cq;             // [row_cap, 2I]: per 128-column block j, 128 hi bytes then 128 lo
  float* c_scale;          // [I/128, row_cap]
  // GEMM2 inputs / outputs
  const float* row_w;      // [row_cap]
  __nv_bfloat16* ow;       // [row_cap, H] weighted expert outputs
  int* err;                // device error word
  // Weights laid out ahead of time (fmoe_prelayout_weights), or null: every K step's 32 KB
  // weight tile of (expert, m tile) stored as the swizzled shared-memory image, tiles
  // [expert][m tile][k step] back to back, so one contiguous bulk copy fetches it.
  const uint8_t* w_pre;
  float* partials;         // stream-K partial tiles, [CTA][2 slots]
  int* tile_counters;      // stream-K arrival counters by first contributor CTA (self-resetting)
};

struct CombineArgs {
  const int* token_row;         // [T, K]
  const __nv_bfloat16* ow;      // [row_cap, H]
  __nv_bfloat16* out;           // [T, H]
  int64_t T;
  int H, top_k;
  const int* err_word;          // the call's device error word (meta[kMetaError])
  unsigned* err_sink;           // host-mapped {bits, count} of the device, or null
  const int* t_dev;             // or null: output rows [*t_dev, T) are not written
  // Expert-parallel return, or null: row t goes to rank s's buffer peer_out[s] at row
  // t + row_shift[s], s the source with src_start[s] <= t < src_start[s + 1] (rows outside
  // [0, capacity) are dropped and set bit 1 of *xerr), instead of to out.
  __nv_bfloat16* const* peer_out;
  const int64_t* src_start;     // [world + 1]
  const int64_t* row_shift;     // [world]
  int world;
  int64_t capacity;
  int* xerr;
};

// Host-mapped error sink, one per device: the combine kernel (the last kernel of every
// call) adds a non-zero error word of its call to it with plain system-scope stores --
// sink[0] |= bits, then sink[1] += 1 -- and the host polls it without synchronising.
// Only the error path writes host memory; a clean call reads one word of its workspace.
__device__ __forceinline__ void report_device_error(unsigned* sink, int bits) {
  volatile unsigned* v = sink;
  v[0] = v[0] | (unsigned)bits;
  __threadfence_system();
  v[1] = v[1] + 1u;
  __threadfence_system();
}

// Launch with programmatic stream serialization (see pdl_wait / pdl_trigger).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__global__ void route_plan_kernel(RouteArgs a);
__global__ void scatter_gather_kernel(ScatterArgs a);
// combine_kernel<V>: grid (T, ceil(H / 8 / (128 * V))), 128 threads; each thread sums V
// 16-byte vectors of its token's row. V = 1 below kCombineWideTokens tokens (latency-bound:
// more CTAs), V = 2 from there on (more loads in flight per thread).
constexpr int64_t kCombineWideTokens = 512;
template <int V>
__global__ void combine_kernel(CombineArgs a);

// Grouped GEMM launchers (gemm_sm100.cu). `bn` selects the token tile; returns a CUDA error.
cudaError_t launch_gemm1(int bn, const CUtensorMap& w13_map, const CUtensorMap& a_map,
                         const GemmArgs& args, int grid, cudaStream_t stream);
cudaError_t launch_gemm2(int bn, const CUtensorMap& w2_map, const CUtensorMap& cq_map,
                         const GemmArgs& args, int grid, cudaStream_t stream);
// Throughput family (gemm_sm100_tm.cu): 128 token rows on the MMA M side; tile_n 128.
cudaError_t launch_gemm1_tm(const CUtensorMap& a_map, const CUtensorMap& w13_map,
                            const GemmArgs& args, int grid, cudaStream_t stream);
cudaError_t launch_gemm2_tm(const CUtensorMap& cq_map, const CUtensorMap& w2_map,
                            const GemmArgs& args, int grid, cudaStream_t stream);
bool gemm_bn_supported(int bn);
// Tile images of fmoe_prelayout_weights (gemm_sm100.cu).
constexpr int kPrelaidTileBytes = 256 * 128;
cudaError_t launch_prelayout(const uint8_t* w13, const uint8_t* w2, uint8_t* w13_out,
                             uint8_t* w2_out, int E_local, int H, int I, cudaStream_t stream);
void set_last_error(const std::string& msg);  // message returned by fmoe_last_error()
size_t gemm_partial_bytes();

}  // namespace fmoe
