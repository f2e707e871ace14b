// ep.cu -- device side of the expert-parallel exchange around the fused operator.
//
// The reference operator computes one expert slice (local_expert_offset,
// solution/cuda/kernel.cu:540-544) and leaves the movement of tokens and partial outputs
// between GPUs to its caller. The caller here (fmoe_b200/ep.py) moves them with NCCL
// all-to-all; these kernels build what it sends and consume what it receives, so no step of
// the exchange runs as a chain of framework ops:
//
//   fmoe_ep_plan     per-destination send lists from the routing (stable in token order);
//                    fmoe_ep_plan_placed first maps expert ids to placement positions
//   fmoe_ep_pack     one payload row per (token, destination): FP8 row | block scales |
//                    expert ids | weights
//   fmoe_ep_unpack   received rows -> the operator's inputs (row-major FP8, [H/128, R]
//                    scales, ids, weights)
//   fmoe_ep_combine  each token's returned partial outputs summed in rank order in fp32,
//                    cast to bf16 (tokens with no route get zeros)
//
// Rank d owns experts [d * e_per_rank, (d + 1) * e_per_rank) (ids, or placement positions
// after fmoe_ep_plan_placed); a token goes to every rank owning at least one of its selected
// experts, once.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "fmoe.h"
#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"

namespace fmoe {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxWorld = 32;

// destinations of token t as a bit mask
__device__ __forceinline__ uint32_t dest_mask(const int* idx, int64_t t, int K, int e_per_rank,
                                              int world) {
  uint32_t m = 0;
  for (int k = 0; k < K; ++k) {
    const int e = idx[t * K + k];
    if (e >= 0) {
      const int d = e / e_per_rank;
      if (d < world) m |= 1u << d;
    }
  }
  return m;
}

// One CTA. Pass 1 counts each destination's tokens; pass 2 gives every (token, destination)
// its row in the send buffer: the destinations' segments in rank order, tokens ascending
// inside a segment (a block-wide exclusive scan per destination and chunk of tokens).
// With an expert placement (expert_pos != null), every selected expert id is first
// replaced in place by its position expert_pos[e]; ranks own ranges of positions.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(int* idx, int64_t T, int K,
                                                               int e_per_rank, int world,
                                                               const int* expert_pos,
                                                               int num_experts, int* pos,
                                                               int* tokens, int* counts) {
  __shared__ int s_cnt[kMaxWorld];
  __shared__ int s_base[kMaxWorld];
  __shared__ int s_warp[kPlanThreads / 32][kMaxWorld];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < kMaxWorld) s_cnt[tid] = 0;
  if (expert_pos) {
    for (int64_t i = tid; i < T * K; i += kPlanThreads) {
      const int e = idx[i];
      if (e >= 0 && e < num_experts) idx[i] = __ldg(expert_pos + e);
    }
  }
  __syncthreads();
  // pass 1: per-destination totals
  for (int d = 0; d < world; ++d) {
    int v = 0;
    for (int64_t t = tid; t < T; t += kPlanThreads)
      v += (dest_mask(idx, t, K, e_per_rank, world) >> d) & 1u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && v) atomicAdd(&s_cnt[d], v);
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int d = 0; d < world; ++d) {
      s_base[d] = run;
      counts[d] = s_cnt[d];
      run += s_cnt[d];
    }
  }
  __syncthreads();
  // pass 2: rows, chunk by chunk of kPlanThreads tokens (token order = thread order)
  for (int64_t c0 = 0; c0 < T; c0 += kPlanThreads) {
    const int64_t t = c0 + tid;
    const uint32_t m = t < T ? dest_mask(idx, t, K, e_per_rank, world) : 0u;
    for (int d = 0; d < world; ++d) {
      const bool on = (m >> d) & 1u;
      const uint32_t b = __ballot_sync(0xffffffffu, on);
      if (lane == 0) s_warp[warp][d] = __popc(b);
    }
    __syncthreads();
    for (int d = 0; d < world; ++d) {
      const bool on = (m >> d) & 1u;  // false past T (m = 0 there)
      const uint32_t b = __ballot_sync(0xffffffffu, on);
      int r = -1;
      if (on) {
        r = __popc(b & ((1u << lane) - 1u)) + s_base[d];
        for (int w = 0; w < warp; ++w) r += s_warp[w][d];
        tokens[r] = (int)t;
      }
      if (t < T) pos[(int64_t)d * T + t] = r;
    }
    __syncthreads();
    if (tid < world) {
      int n = 0;
      for (int w = 0; w < kPlanThreads / 32; ++w) n += s_warp[w][tid];
      s_base[tid] += n;
    }
    __syncthreads();
  }
}

// One CTA per token: its payload row for every destination it goes to.
__global__ void __launch_bounds__(256) ep_pack_kernel(const uint8_t* hidden, const float* hscale,
                                                      const int* idx, const float* w,
                                                      const int* pos, int64_t T, int H, int K,
                                                      int world, uint8_t* send) {
  const int64_t t = blockIdx.x;
  const int kb = H / kBlock;
  const int64_t row_bytes = (int64_t)H + 4 * kb + 8 * K;  // a multiple of 4
  const int nv = H / 16;
  for (int d = 0; d < world; ++d) {
    const int r = pos[(int64_t)d * T + t];
    if (r < 0) continue;
    uint8_t* dst = send + (int64_t)r * row_bytes;
    if (row_bytes % 16 == 0) {
      for (int v = threadIdx.x; v < nv; v += blockDim.x)
        reinterpret_cast<uint4*>(dst)[v] =
            __ldg(reinterpret_cast<const uint4*>(hidden + t * H) + v);
    } else {  // rows only 4-byte aligned (small geometries)
      for (int v = threadIdx.x; v < H / 4; v += blockDim.x)
        reinterpret_cast<uint32_t*>(dst)[v] =
            __ldg(reinterpret_cast<const uint32_t*>(hidden + t * H) + v);
    }
    float* ds = reinterpret_cast<float*>(dst + H);
    for (int b = threadIdx.x; b < kb; b += blockDim.x) ds[b] = __ldg(hscale + (int64_t)b * T + t);
    int* di = reinterpret_cast<int*>(dst + H + 4 * kb);
    float* dw = reinterpret_cast<float*>(dst + H + 4 * kb + 4 * K);
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      di[k] = __ldg(idx + t * K + k);
      dw[k] = __ldg(w + t * K + k);
    }
  }
}

// One CTA per received row. R is the row capacity (the scale array's leading dimension);
// with rows_dev, rows at or past *rows_dev are not copied.
__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* recv, int64_t R, int H,
                                                        int K, uint8_t* hs, float* sc, int* idx,
                                                        float* w, const int* rows_dev) {
  const int64_t r = blockIdx.x;
  if (rows_dev && r >= (int64_t)*rows_dev) return;
  const int kb = H / kBlock;
  const int64_t row_bytes = (int64_t)H + 4 * kb + 8 * K;
  const uint8_t* src = recv + r * row_bytes;
  if (row_bytes % 16 == 0) {
    for (int v = threadIdx.x; v < H / 16; v += blockDim.x)
      reinterpret_cast<uint4*>(hs + r * H)[v] = reinterpret_cast<const uint4*>(src)[v];
  } else {  // rows only 4-byte aligned (small geometries)
    for (int v = threadIdx.x; v < H / 4; v += blockDim.x)
      reinterpret_cast<uint32_t*>(hs + r * H)[v] = reinterpret_cast<const uint32_t*>(src)[v];
  }
  const float* ss = reinterpret_cast<const float*>(src + H);
  for (int b = threadIdx.x; b < kb; b += blockDim.x) sc[(int64_t)b * R + r] = ss[b];
  const int* si = reinterpret_cast<const int*>(src + H + 4 * kb);
  const float* sw = reinterpret_cast<const float*>(src + H + 4 * kb + 4 * K);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    idx[r * K + k] = si[k];
    w[r * K + k] = sw[k];
  }
}

// One CTA per token: out[t] = bf16(0 + back[pos(0, t)] + back[pos(1, t)] + ...), fp32 adds
// in rank order.
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* back,
                                                         const int* pos, int64_t T, int H,
                                                         int world, __nv_bfloat16* out) {
  __shared__ int s_pos[kMaxWorld];
  const int64_t t = blockIdx.x;
  if (threadIdx.x < world) s_pos[threadIdx.x] = pos[(int64_t)threadIdx.x * T + t];
  __syncthreads();
  // 8 bf16 per 16-byte vector
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    for (int d = 0; d < world; ++d) {
      const int r = s_pos[d];
      if (r < 0) continue;
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(back + (int64_t)r * H) + v);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) oh[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
    reinterpret_cast<uint4*>(out + t * H)[v] = o;
  }
}


// P2P dispatch: the payload row of (token t, rank d) goes straight into rank d's receive
// buffer at row pos[d, t] + shift[d] (peer memory over NVLink; plain stores, no multicast).
// Rows outside [0, capacity) are dropped and flagged. A system fence makes the rows visible
// to the peers once the kernel has completed.
__global__ void __launch_bounds__(256) ep_pack_p2p_kernel(
    const uint8_t* hidden, const float* hscale, const int* idx, const float* w, const int* pos,
    int64_t T, int H, int K, int world, uint8_t* const* peer_recv, const int64_t* shift,
    int64_t capacity, int* err) {
  const int64_t t = blockIdx.x;
  const int kb = H / kBlock;
  const int64_t row_bytes = (int64_t)H + 4 * kb + 8 * K;
  for (int d = 0; d < world; ++d) {
    const int r0 = pos[(int64_t)d * T + t];
    if (r0 < 0) continue;
    const int64_t r = r0 + shift[d];
    if (r < 0 || r >= capacity) {
      if (threadIdx.x == 0) atomicOr(err, 1);
      continue;
    }
    uint8_t* dst = peer_recv[d] + r * row_bytes;
    if (row_bytes % 16 == 0) {
      for (int v = threadIdx.x; v < H / 16; v += blockDim.x)
        reinterpret_cast<uint4*>(dst)[v] =
            __ldg(reinterpret_cast<const uint4*>(hidden + t * H) + v);
    } else {
      for (int v = threadIdx.x; v < H / 4; v += blockDim.x)
        reinterpret_cast<uint32_t*>(dst)[v] =
            __ldg(reinterpret_cast<const uint32_t*>(hidden + t * H) + v);
    }
    float* ds = reinterpret_cast<float*>(dst + H);
    for (int b = threadIdx.x; b < kb; b += blockDim.x) ds[b] = __ldg(hscale + (int64_t)b * T + t);
    int* di = reinterpret_cast<int*>(dst + H + 4 * kb);
    float* dw = reinterpret_cast<float*>(dst + H + 4 * kb + 4 * K);
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      di[k] = __ldg(idx + t * K + k);
      dw[k] = __ldg(w + t * K + k);
    }
  }
  __threadfence_system();
}

// P2P return: received row r (from source rank s, rows [src_start[s], src_start[s + 1]))
// goes back into rank s's buffer at row r + shift[s], as bf16 [H].
__global__ void __launch_bounds__(256) ep_return_p2p_kernel(
    const __nv_bfloat16* part, int64_t R, int H, int world, const int64_t* src_start,
    __nv_bfloat16* const* peer_back, const int64_t* shift, int64_t capacity, int* err) {
  const int64_t r = blockIdx.x;
  if (r >= src_start[world]) return;  // past the received rows (grid sized by a capacity)
  int s = 0;
  while (s + 1 < world && r >= src_start[s + 1]) ++s;
  const int64_t q = r + shift[s];
  if (q < 0 || q >= capacity) {
    if (threadIdx.x == 0) atomicOr(err, 2);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(part + r * H);
  uint4* dst = reinterpret_cast<uint4*>(peer_back[s] + q * H);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = __ldg(src + v);
  __threadfence_system();
}

// Row offsets of the P2P exchange from every rank's per-destination counts, on the device
// (no host round trip): m[s][d] = rows rank s sends to rank d (an int64 [world][world + 1]
// all-gather of each rank's counts; the last column is not used). Writes tables =
// {shift_pack[world], starts[world + 1], shift_ret[world]} and rows = starts[world]:
//   starts[s]     = sum_{q < s} m[q][me]       (first row of source s in my receive buffer)
//   shift_pack[d] = sum_{q < me} m[q][d] - sum_{q < d} m[me][q]
//   shift_ret[s]  = sum_{q < me} m[s][q] - starts[s]
__global__ void ep_offsets_kernel(const int64_t* m, int world, int me, int64_t* tables,
                                  int* rows) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int W1 = world + 1;
  int64_t* shift_pack = tables;
  int64_t* starts = tables + world;
  int64_t* shift_ret = tables + 2 * world + 1;
  int64_t run = 0;
  for (int s = 0; s < world; ++s) {
    starts[s] = run;
    run += m[(int64_t)s * W1 + me];
  }
  starts[world] = run;
  *rows = (int)run;
  int64_t seg = 0;  // sum_{q < d} m[me][q]
  for (int d = 0; d < world; ++d) {
    int64_t src = 0;
    for (int q = 0; q < me; ++q) src += m[(int64_t)q * W1 + d];
    shift_pack[d] = src - seg;
    seg += m[(int64_t)me * W1 + d];
  }
  for (int s = 0; s < world; ++s) {
    int64_t base = 0;
    for (int q = 0; q < me; ++q) base += m[(int64_t)s * W1 + q];
    shift_ret[s] = base - starts[s];
  }
}

int ep_fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

int ep_check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return ep_fail(FMOE_ERR_RUNTIME, std::string(what) + ": " + cudaGetErrorString(e));
  return FMOE_OK;
}

bool ep_geometry_ok(int64_t T, int H, int K, int world) {
  return T >= 0 && H > 0 && H % kBlock == 0 && K > 0 && K <= 32 && world > 0 &&
         world <= kMaxWorld;
}

}  // namespace
}  // namespace fmoe

using namespace fmoe;

static int ep_plan_impl(int* topk_idx, int64_t num_tokens, int top_k, int world,
                        int experts_per_rank, const int* expert_pos, int num_experts, int* pos,
                        int* tokens, int* counts, void* stream, const char* name) {
  if (!ep_geometry_ok(num_tokens, kBlock, top_k, world) || experts_per_rank <= 0)
    return ep_fail(FMOE_ERR_VALUE, std::string(name) + ": bad geometry");
  if (expert_pos && num_experts != world * experts_per_rank)
    return ep_fail(FMOE_ERR_VALUE,
                   std::string(name) + ": num_experts != world * experts_per_rank");
  if (!counts) return ep_fail(FMOE_ERR_VALUE, std::string(name) + ": NULL pointer");
  if (num_tokens == 0) {  // empty tensors may have NULL data: only the counts are written
    const cudaError_t e =
        cudaMemsetAsync(counts, 0, sizeof(int) * world, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return ep_fail(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
    return FMOE_OK;
  }
  if (!topk_idx || !pos || !tokens)
    return ep_fail(FMOE_ERR_VALUE, std::string(name) + ": NULL pointer");
  ep_plan_kernel<<<1, kPlanThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      topk_idx, num_tokens, top_k, experts_per_rank, world, expert_pos, num_experts, pos,
      tokens, counts);
  return ep_check_launch(name);
}

extern "C" int fmoe_ep_plan(const int* topk_idx, int64_t num_tokens, int top_k, int world,
                            int experts_per_rank, int* pos, int* tokens, int* counts,
                            void* stream) {
  // the kernel writes topk_idx only when given a placement
  return ep_plan_impl(const_cast<int*>(topk_idx), num_tokens, top_k, world, experts_per_rank,
                      nullptr, 0, pos, tokens, counts, stream, "fmoe_ep_plan");
}

extern "C" int fmoe_ep_plan_placed(int* topk_idx, int64_t num_tokens, int top_k, int world,
                                   int experts_per_rank, const int* expert_pos, int num_experts,
                                   int* pos, int* tokens, int* counts, void* stream) {
  if (!expert_pos) return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_plan_placed: NULL pointer");
  return ep_plan_impl(topk_idx, num_tokens, top_k, world, experts_per_rank, expert_pos,
                      num_experts, pos, tokens, counts, stream, "fmoe_ep_plan_placed");
}

extern "C" int fmoe_ep_pack(const void* hidden_states, const float* hidden_states_scale,
                            const int* topk_idx, const float* topk_w, const int* pos,
                            int64_t num_tokens, int hidden_size, int top_k, int world,
                            void* send, void* stream) {
  if (!ep_geometry_ok(num_tokens, hidden_size, top_k, world))
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_pack: bad geometry");
  if (num_tokens == 0) return FMOE_OK;
  if (!hidden_states || !hidden_states_scale || !topk_idx || !topk_w || !pos || !send)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_pack: NULL pointer");
  if (reinterpret_cast<uintptr_t>(hidden_states) % 16 || reinterpret_cast<uintptr_t>(send) % 16)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_pack: hidden_states and send must be 16-byte aligned");
  ep_pack_kernel<<<(unsigned)num_tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(hidden_states), hidden_states_scale, topk_idx, topk_w, pos,
      num_tokens, hidden_size, top_k, world, static_cast<uint8_t*>(send));
  return ep_check_launch("fmoe_ep_pack");
}

extern "C" int fmoe_ep_unpack(const void* recv, int64_t rows, int hidden_size, int top_k,
                              void* hidden_states, float* hidden_states_scale, int* topk_idx,
                              float* topk_w, void* stream) {
  if (!ep_geometry_ok(rows, hidden_size, top_k, 1))
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_unpack: bad geometry");
  if (rows == 0) return FMOE_OK;
  if (!recv || !hidden_states || !hidden_states_scale || !topk_idx || !topk_w)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_unpack: NULL pointer");
  if (reinterpret_cast<uintptr_t>(recv) % 16 || reinterpret_cast<uintptr_t>(hidden_states) % 16)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_unpack: recv and hidden_states must be 16-byte aligned");
  ep_unpack_kernel<<<(unsigned)rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(recv), rows, hidden_size, top_k,
      static_cast<uint8_t*>(hidden_states), hidden_states_scale, topk_idx, topk_w, nullptr);
  return ep_check_launch("fmoe_ep_unpack");
}

extern "C" int fmoe_ep_unpack_count(const void* recv, int64_t capacity_rows,
                                    const int* rows_dev, int hidden_size, int top_k,
                                    void* hidden_states, float* hidden_states_scale,
                                    int* topk_idx, float* topk_w, void* stream) {
  if (!ep_geometry_ok(capacity_rows, hidden_size, top_k, 1))
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_unpack_count: bad geometry");
  if (capacity_rows == 0) return FMOE_OK;
  if (!recv || !rows_dev || !hidden_states || !hidden_states_scale || !topk_idx || !topk_w)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_unpack_count: NULL pointer");
  if (reinterpret_cast<uintptr_t>(recv) % 16 || reinterpret_cast<uintptr_t>(hidden_states) % 16)
    return ep_fail(FMOE_ERR_VALUE,
                   "fmoe_ep_unpack_count: recv and hidden_states must be 16-byte aligned");
  ep_unpack_kernel<<<(unsigned)capacity_rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(recv), capacity_rows, hidden_size, top_k,
      static_cast<uint8_t*>(hidden_states), hidden_states_scale, topk_idx, topk_w, rows_dev);
  return ep_check_launch("fmoe_ep_unpack_count");
}

extern "C" int fmoe_ep_offsets(const int64_t* counts_all, int world, int rank, int64_t* tables,
                               int* rows, void* stream) {
  if (world <= 0 || world > kMaxWorld || rank < 0 || rank >= world)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_offsets: bad world / rank");
  if (!counts_all || !tables || !rows)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_offsets: NULL pointer");
  ep_offsets_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(counts_all, world, rank,
                                                                     tables, rows);
  return ep_check_launch("fmoe_ep_offsets");
}

extern "C" int fmoe_ep_combine(const void* back, const int* pos, int64_t num_tokens,
                               int hidden_size, int world, void* output, void* stream) {
  if (!ep_geometry_ok(num_tokens, hidden_size, 1, world))
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_combine: bad geometry");
  if (num_tokens == 0) return FMOE_OK;
  if (!back || !pos || !output) return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_combine: NULL pointer");
  if (reinterpret_cast<uintptr_t>(back) % 16 || reinterpret_cast<uintptr_t>(output) % 16)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_combine: back and output must be 16-byte aligned");
  ep_combine_kernel<<<(unsigned)num_tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(back), pos, num_tokens, hidden_size, world,
      static_cast<__nv_bfloat16*>(output));
  return ep_check_launch("fmoe_ep_combine");
}

// ---- peer buffers (CUDA IPC) and the P2P exchange ------------------------------------------
extern "C" int fmoe_ep_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_ipc_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return ep_fail(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
  e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return ep_fail(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
  }
  return FMOE_OK;
}

extern "C" int fmoe_ep_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ep_fail(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
  return FMOE_OK;
}

extern "C" int fmoe_ep_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? FMOE_OK : ep_fail(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
}

extern "C" int fmoe_ep_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? FMOE_OK : ep_fail(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
}

extern "C" int fmoe_ep_pack_p2p(const void* hidden_states, const float* hidden_states_scale,
                                const int* topk_idx, const float* topk_w, const int* pos,
                                int64_t num_tokens, int hidden_size, int top_k, int world,
                                void* const* peer_recv, const int64_t* row_shift,
                                int64_t capacity_rows, int* err, void* stream) {
  if (!ep_geometry_ok(num_tokens, hidden_size, top_k, world))
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_pack_p2p: bad geometry");
  if (num_tokens == 0) return FMOE_OK;
  if (!hidden_states || !hidden_states_scale || !topk_idx || !topk_w || !pos || !peer_recv ||
      !row_shift || !err)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_pack_p2p: NULL pointer");
  if (reinterpret_cast<uintptr_t>(hidden_states) % 16)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_pack_p2p: hidden_states must be 16-byte aligned");
  ep_pack_p2p_kernel<<<(unsigned)num_tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(hidden_states), hidden_states_scale, topk_idx, topk_w, pos,
      num_tokens, hidden_size, top_k, world, reinterpret_cast<uint8_t* const*>(peer_recv),
      row_shift, capacity_rows, err);
  return ep_check_launch("fmoe_ep_pack_p2p");
}

extern "C" int fmoe_ep_return_p2p(const void* partial, int64_t rows, int hidden_size, int world,
                                  const int64_t* src_start, void* const* peer_back,
                                  const int64_t* row_shift, int64_t capacity_rows, int* err,
                                  void* stream) {
  if (!ep_geometry_ok(rows, hidden_size, 1, world))
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_return_p2p: bad geometry");
  if (rows == 0) return FMOE_OK;
  if (!partial || !src_start || !peer_back || !row_shift || !err)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_return_p2p: NULL pointer");
  if (reinterpret_cast<uintptr_t>(partial) % 16)
    return ep_fail(FMOE_ERR_VALUE, "fmoe_ep_return_p2p: partial must be 16-byte aligned");
  ep_return_p2p_kernel<<<(unsigned)rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(partial), rows, hidden_size, world, src_start,
      reinterpret_cast<__nv_bfloat16* const*>(peer_back), row_shift, capacity_rows, err);
  return ep_check_launch("fmoe_ep_return_p2p");
}
