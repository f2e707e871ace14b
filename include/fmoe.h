/*
 * fmoe.h -- C ABI of the B200-native fused FP8 block-scaled MoE operator.
 *
 * This is the drop-in boundary for the reference operator
 *   ffi::Tensor kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale,
 *                      gemm1_weights, gemm1_weights_scale, gemm2_weights,
 *                      gemm2_weights_scale, int32_t local_expert_offset,
 *                      float routed_scaling_factor)
 * of YuWei-CH/Fused-MoE-YWS solution/cuda/kernel.cu:1727-1734 (exported through TVM-FFI
 * at kernel.cu:1839). The TVM-FFI binding in fused-moe-yws_b200/csrc/tvm_ffi_kernel.cc and
 * the Python mirror in fused-moe-yws_b200/fmoe_b200 both call these functions.
 *
 * Conventions: plain device pointers and sizes, no framework types. Every function
 * returns FMOE_OK or an error code; fmoe_last_error() gives the message of the most
 * recent failure on the calling thread. The value/type/runtime split mirrors the
 * reference's ValueError / TypeError / RuntimeError (kernel.cu:121-168, :53-62).
 * Launches are asynchronous on the given stream; nothing synchronises the host.
 */
#ifndef FMOE_H_
#define FMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FMOE_ABI_VERSION 1

enum fmoe_status {
  FMOE_OK = 0,
  FMOE_ERR_VALUE = 1,     /* bad shape, geometry, size or alignment (reference: ValueError) */
  FMOE_ERR_TYPE = 2,      /* bad dtype code (reference: TypeError) */
  FMOE_ERR_RUNTIME = 3,   /* CUDA launch / driver failure (reference: RuntimeError) */
  FMOE_ERR_WORKSPACE = 4, /* workspace missing or too small */
  FMOE_ERR_DEVICE = 5     /* a kernel reported an error word (timeout, overflow) */
};

/* Problem geometry. The reference hard-codes the DeepSeek-V3 values
 * (kernel.cu:32-40); here they are runtime fields so the tiny contest geometry
 * (H=256, I=128, 16 experts, 4 groups) runs through the same kernels. */
typedef struct fmoe_problem {
  int64_t num_tokens;          /* T: routing_logits.shape[0] */
  int32_t num_experts;         /* E_global: routing_logits.shape[1] (<= 256, multiple of n_group) */
  int32_t num_local_experts;   /* E_local: gemm1_weights.shape[0] (<= 256) */
  int32_t hidden_size;         /* H: multiple of 128, <= 16384 */
  int32_t intermediate_size;   /* I: multiple of 128, <= 16384 */
  int32_t top_k;               /* experts per token (<= 32) */
  int32_t n_group;             /* routing groups (<= 32) */
  int32_t topk_group;          /* groups kept per token */
  int32_t local_expert_offset; /* first global expert of this slice (kernel.cu:541) */
  float routed_scaling_factor; /* multiplies the renormalised weights (kernel.cu:512) */
  int32_t tile_n;              /* token tile of the grouped GEMMs; 0 = autotune table */
} fmoe_problem;

/* Device pointers, all contiguous, all on the current device; shapes as in
 * kernel.cu:1746-1769. 8-bit float buffers hold E4M3 bytes; bf16 buffers hold raw bits.
 * Base addresses must be 16-byte aligned (TMA). */
typedef struct fmoe_tensors {
  const float* routing_logits;      /* [T, E_global] fp32 */
  const void* routing_bias;         /* [E_global] bf16 */
  const void* hidden_states;        /* [T, H] e4m3 */
  const float* hidden_states_scale; /* [H/128, T] fp32 (block-major, transposed) */
  const void* gemm1_weights;        /* [E_local, 2I, H] e4m3 (rows [0,I) gate, [I,2I) up) */
  const float* gemm1_weights_scale; /* [E_local, 2I/128, H/128] fp32 */
  const void* gemm2_weights;        /* [E_local, H, I] e4m3 */
  const float* gemm2_weights_scale; /* [E_local, H/128, I/128] fp32 */
  void* output;                     /* [T, H] bf16, written completely */
} fmoe_tensors;

/* Routing outputs (device pointers) for fmoe_route(). */
typedef struct fmoe_route_out {
  int32_t* topk_idx; /* [T, top_k] global expert ids in selection order, -1 if unfilled */
  float* topk_w;     /* [T, top_k] routed weights */
} fmoe_route_out;

/* Returns FMOE_ABI_VERSION. */
int fmoe_abi_version(void);

/* Message of the last failure on this thread ("" if none). */
const char* fmoe_last_error(void);

/* Geometry and argument checks without touching the device
 * (replaces CheckTensor / CheckScalarVector, kernel.cu:121-168, for the size fields). */
int fmoe_validate(const fmoe_problem* p);

/* Scratch bytes fmoe_forward() needs for this problem. The reference keeps
 * process-lifetime thread_local scratch caches instead (kernel.cu:234-270, :1784-1797);
 * here the caller owns the workspace, so the library itself never allocates. */
int fmoe_workspace_size(const fmoe_problem* p, size_t* bytes);

/* Token tile (MMA N) the committed autotune table picks for num_tokens tokens of
 * DeepSeek-V3 routing (top_k 8 of 256 experts). The table is keyed by the expected routed
 * rows per local expert, num_tokens * top_k / num_experts (the reference's fixed tiles and
 * T <= 512 switch, kernel.cu:41-51, :1781, have no such key). */
int fmoe_autotune_tile_n(int64_t num_tokens);

/* Token tile a call with this problem uses (its tile_n, or the table's choice for its
 * tokens, top_k and experts; 64 where 128 would not divide hidden_size), or the negated
 * status code if the problem is invalid. */
int fmoe_tile_n(const fmoe_problem* p);

/* The whole operator: routing -> permute/gather -> GEMM1+SwiGLU -> GEMM2 -> combine,
 * writing bf16 [T, H] into t->output. Replaces kernel() at kernel.cu:1727-1837, minus its
 * final cudaStreamSynchronize (kernel.cu:1834): everything is enqueued on `stream`
 * (a cudaStream_t; NULL = legacy default stream). One call at a time per workspace. */
int fmoe_forward(const fmoe_problem* p, const fmoe_tensors* t, void* workspace,
                 size_t workspace_bytes, void* stream);

/* The operator on routing decided elsewhere: topk_idx/topk_w ([T, top_k] global expert ids
 * and weights, device pointers, 16-byte aligned) replace routing_logits/routing_bias, which
 * are ignored. Used by the expert-parallel layer, where the rank that owns a token routes it
 * once and ships (ids, weights) with the token to the ranks that own those experts. It
 * replaces the reference's local-slice hook (local_expert_offset, kernel.cu:540-544,
 * :572-586, :857-859) for tokens arriving from other ranks. */
int fmoe_forward_routed(const fmoe_problem* p, const int32_t* topk_idx, const float* topk_w,
                        const fmoe_tensors* t, void* workspace, size_t workspace_bytes,
                        void* stream);
/* fmoe_forward_routed with the token count on the device: p->num_tokens is a capacity (the
 * sizes of every tensor and of the workspace), *num_tokens_dev (device int, 0 <=
 * *num_tokens_dev <= p->num_tokens, written earlier on `stream`) the tokens present. Tokens
 * past it get no route and their output rows are not written. Lets an expert-parallel step
 * run without a host round trip for the received token count; repeated calls with the same
 * buffers replay one cached graph. */
int fmoe_forward_routed_count(const fmoe_problem* p, const int32_t* topk_idx,
                              const float* topk_w, const int32_t* num_tokens_dev,
                              const fmoe_tensors* t, void* workspace, size_t workspace_bytes,
                              void* stream);
/* fmoe_forward_routed_count whose combine writes each output row straight back to the rank
 * its token came from (expert-parallel return over peer memory, replacing fmoe_ep_return_p2p
 * after the operator): row r, from the source s with src_start[s] <= r < src_start[s + 1],
 * goes to peer_out[s] at row r + row_shift[s] (peer_out: device array of `world` buffer
 * addresses; src_start / row_shift as for fmoe_ep_return_p2p). Rows outside
 * [0, capacity_rows) are not written and set bit 1 of *err. t->output must still be a valid
 * 16-byte aligned pointer; it is not written. The caller orders the ranks with a barrier
 * after the call, as after fmoe_ep_return_p2p. */
int fmoe_forward_routed_count_p2p(const fmoe_problem* p, const int32_t* topk_idx,
                                  const float* topk_w, const int32_t* num_tokens_dev,
                                  const fmoe_tensors* t, void* workspace, size_t workspace_bytes,
                                  void* const* peer_out, const int64_t* src_start,
                                  const int64_t* row_shift, int world, int64_t capacity_rows,
                                  int* err, void* stream);

/* Weight pre-layout (the weight side of the reference's per-call dequantise passes,
 * kernel.cu:924-1003, done once instead): writes every 32 KB weight tile the GEMMs load per
 * 128-K step -- GEMM1: 128 gate rows then the matching 128 up rows of W13; GEMM2: 256 rows
 * of W2 -- as the swizzled shared-memory image the GEMMs consume, tiles ordered [expert]
 * [row tile][K step], into gemm1_out / gemm2_out (each the size of its input, 16-byte
 * aligned, not overlapping the inputs). The values are unchanged (FP8 bytes moved, scales
 * untouched), so the prelaid entry points below give the same output bits, with each
 * weight tile fetched by one contiguous bulk copy. Needs hidden_size % 256 == 0.
 * Asynchronous on `stream`. */
int fmoe_prelayout_weights(const fmoe_problem* p, const void* gemm1_weights,
                           const void* gemm2_weights, void* gemm1_out, void* gemm2_out,
                           void* stream);

/* fmoe_forward / fmoe_forward_routed with t->gemm1_weights and t->gemm2_weights pointing at
 * fmoe_prelayout_weights outputs (scales as usual). */
int fmoe_forward_prelaid(const fmoe_problem* p, const fmoe_tensors* t, void* workspace,
                         size_t workspace_bytes, void* stream);
int fmoe_forward_routed_prelaid(const fmoe_problem* p, const int32_t* topk_idx,
                                const float* topk_w, const fmoe_tensors* t, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Routing only (replaces sigmoid_bias_kernel + routing_select_kernel,
 * kernel.cu:388-516), for parity tests and the expert-parallel dispatch.
 * Needs the same workspace as fmoe_forward. */
int fmoe_route(const fmoe_problem* p, const float* routing_logits, const void* routing_bias,
               const fmoe_route_out* out, void* workspace, size_t workspace_bytes,
               void* stream);

/* Synchronises `stream`, then reads and clears the device error word the kernels of the
 * last call on this workspace wrote (bitmask of timeouts / overflow; 0 = clean). */
int fmoe_read_device_error(const fmoe_problem* p, void* workspace, void* stream,
                           int32_t* device_error);

/* Device errors without a synchronisation. The last kernel of every fmoe_forward() /
 * fmoe_forward_routed() passes a non-zero device error word of its call (a bounded wait
 * that ran out: that call's output is invalid) to a host-mapped word of the library, one
 * per device. This reads it for the current device: *device_error = the error bits
 * reported by calls that finished since the previous poll (0: none), without waiting for
 * calls still running. The reference raises RuntimeError for every CUDA error
 * (kernel.cu:53-62) after a full stream synchronisation (kernel.cu:1834); the TVM-FFI
 * binding and the Python mirror poll at the start of every call and raise then. The word
 * is allocated (8 bytes of pinned host memory) by a device's first call or poll that is not
 * inside a stream capture; calls captured into a graph before that report nothing. */
int fmoe_poll_device_error(int32_t* device_error);

/* Test hook for the error path above (no fault, no hang): the next fmoe_forward() or
 * fmoe_forward_routed() on the calling thread runs eagerly and its routing kernel ORs
 * `bits` into the call's device error word, as an expired wait would; the call's output is
 * still computed normally. The reference has no such hook. */
int fmoe_selftest_inject_device_error(int32_t bits);

/* Stage timing: when `events` is non-NULL, every later fmoe_forward() on this thread
 * records events[0..5] (cudaEvent_t handles owned by the caller) on its stream at the
 * stage boundaries: start, after routing, after permute/gather, after GEMM1+SwiGLU,
 * after GEMM2, after combine. NULL turns recording off. The reference's profiling hook
 * (FUSED_MOE_PROFILE, set by scripts/run_modal.py:106-116) is never read by kernel.cu;
 * this one is live. */
int fmoe_set_stage_events(void* const* events);

/* Failure-detection self-test (no fault, trap or hang): runs a one-CTA kernel whose two
 * bounded waits -- the mbarrier wait and the global-flag wait every GEMM kernel uses
 * (the reference has no bounded waits; its failures surface as CUDA errors through
 * kernel.cu:53-62) -- can never complete, with the limit set to timeout_ns (<= 1e8).
 * Synchronises `stream`, then writes result[0] = bitmask of the waits that expired
 * (bit 0 mbarrier, bit 1 flag; 3 when the limits work), result[1..2] = ns each waited. */
int fmoe_selftest_wait_timeout(uint64_t timeout_ns, uint64_t* result, void* stream);

/* Dense FP8 tensor-core rate of the current GPU, measured (no counterpart in the
 * reference, which quotes no peak): one CTA per SM issues mmas_per_cta back-to-back
 * tcgen05.mma.kind::f8f6f4 M128 x N256 x K32 instructions (the throughput GEMMs'
 * instruction shape) on operands resident in shared memory; one untimed launch, then one
 * timed with events on `stream`, which is synchronised. Writes *tflops (dense, 2 FLOP per
 * multiply-add) and *ms. mmas_per_cta in [64, 2^22]; 16384 takes about 1 ms. */
int fmoe_probe_fp8_mma_rate(int64_t mmas_per_cta, double* tflops, double* ms, void* stream);

/* Debug view of the permutation of the last call (device pointers into the workspace):
 * expert counts [E_local], expert offsets [E_local+1], row->token [row_cap],
 * (token,k)->row [T*top_k], and row_cap. For parity tests of the permute kernel. */
typedef struct fmoe_plan_view {
  const int32_t* expert_cnt;
  const int32_t* expert_off;
  const int32_t* row_token;
  const int32_t* token_row;
  const int32_t* meta;
  int64_t row_cap;
} fmoe_plan_view;
int fmoe_plan_view_get(const fmoe_problem* p, void* workspace, fmoe_plan_view* view);

/* Routing that takes no workspace and allocates nothing. This entry point has no
 * counterpart in the reference operator. It exists for callers that cannot hand the
 * library scratch memory: plugin interfaces that pass only the call's tensors, or engines
 * that reserve all device memory at start-up and forbid later allocation (cudaMalloc would
 * also synchronise the device and break stream capture). It computes what fmoe_route()
 * computes, with its scratch in a fixed device array of about 0.53 MB per GPU that stays
 * allocated until the process exits. Limits: num_tokens <= 8192, num_local_experts <= 64,
 * top_k <= 32; larger problems fail with FMOE_ERR_VALUE. The first call on a device looks up
 * the array's address there, so make it before any stream capture. All calls share the
 * array: calls that overlap on the GPU race and must be ordered by the caller. */
int fmoe_route_static(const fmoe_problem* p, const float* routing_logits,
                      const void* routing_bias, const fmoe_route_out* out, void* stream);
/* (fmoe_route_static reports no device error word: within its limits the routing plan
 * cannot overflow, which is the routing kernel's only device-side error. Its array's
 * address is looked up again when the device's context changes, e.g. after a reset.) */

/* Expert-parallel exchange, device side. The reference operator computes one expert slice
 * (local_expert_offset, kernel.cu:540-544) and leaves the exchange of tokens and partial
 * outputs between GPUs to its caller; these entry points build what that caller sends and
 * consume what it receives (the collectives themselves are the caller's, e.g. NCCL
 * all-to-all). Rank d owns experts [d * experts_per_rank, (d + 1) * experts_per_rank); a
 * token goes once to every rank owning one of its selected experts. All pointers are device
 * pointers; work is queued on `stream`.
 *
 * Payload row (bytes): FP8 hidden row [H] | block scales fp32 [H/128] | expert ids int32
 * [top_k] | weights fp32 [top_k]; rows are packed back to back.
 *
 * fmoe_ep_plan: pos [world, T] = send-buffer row of (token, rank) or -1; tokens [sum counts]
 *   = token of each send row; counts [world] = rows per rank. Rows are grouped by rank in
 *   rank order, tokens ascending inside a group. */
int fmoe_ep_plan(const int* topk_idx, int64_t num_tokens, int top_k, int world,
                 int experts_per_rank, int* pos, int* tokens, int* counts, void* stream);
/* fmoe_ep_plan_placed: fmoe_ep_plan under an expert placement. expert_pos [num_experts]
 * (num_experts = world * experts_per_rank) gives each expert's position in the placement
 * (rank r owns positions [r * experts_per_rank, (r + 1) * experts_per_rank)); every
 * selected id in topk_idx is replaced IN PLACE by its position first, so the payload rows
 * and the receiving rank's fmoe_forward_routed (local_expert_offset = r * experts_per_rank,
 * weights stacked in placement order) see positions. Ids < 0 are left as they are. */
int fmoe_ep_plan_placed(int* topk_idx, int64_t num_tokens, int top_k, int world,
                        int experts_per_rank, const int* expert_pos, int num_experts, int* pos,
                        int* tokens, int* counts, void* stream);
/* fmoe_ep_pack: one payload row per (token, rank) at the row pos[rank, token] of `send`.
 * hidden_states [T, H] FP8, hidden_states_scale [H/128, T]; both hidden_states and send
 * 16-byte aligned. */
int fmoe_ep_pack(const void* hidden_states, const float* hidden_states_scale,
                 const int* topk_idx, const float* topk_w, const int* pos, int64_t num_tokens,
                 int hidden_size, int top_k, int world, void* send, void* stream);
/* fmoe_ep_unpack: `rows` received payload rows -> hidden_states [rows, H] FP8,
 * hidden_states_scale [H/128, rows], topk_idx / topk_w [rows, top_k] (the inputs of
 * fmoe_forward_routed). recv and hidden_states 16-byte aligned. */
int fmoe_ep_unpack(const void* recv, int64_t rows, int hidden_size, int top_k,
                   void* hidden_states, float* hidden_states_scale, int* topk_idx,
                   float* topk_w, void* stream);
/* fmoe_ep_unpack_count: the same for *rows_dev rows (a device int) into arrays sized for
 * capacity_rows rows (hidden_states_scale [H/128, capacity_rows]); rows past the count are
 * not written. */
int fmoe_ep_unpack_count(const void* recv, int64_t capacity_rows, const int* rows_dev,
                         int hidden_size, int top_k, void* hidden_states,
                         float* hidden_states_scale, int* topk_idx, float* topk_w, void* stream);
/* fmoe_ep_offsets: the P2P row offsets on the device from counts_all, the int64
 * [world][world + 1] all-gather of every rank's per-destination counts (the last column is
 * free for the caller): tables = {row_shift for fmoe_ep_pack_p2p [world], src_start for
 * fmoe_ep_return_p2p [world + 1], row_shift for fmoe_ep_return_p2p [world]} (int64), and
 * *rows = rows this rank receives (int32, for fmoe_ep_unpack_count and
 * fmoe_forward_routed_count). */
int fmoe_ep_offsets(const int64_t* counts_all, int world, int rank, int64_t* tables, int* rows,
                    void* stream);
/* fmoe_ep_combine: output [T, H] bf16 = per token, the bf16 partial rows back[pos[r, t]]
 * (rows in send order, as returned by the ranks) summed in fp32 in rank order starting from
 * 0, then rounded to bf16; tokens with no route get zeros. back and output 16-byte aligned. */
int fmoe_ep_combine(const void* back, const int* pos, int64_t num_tokens, int hidden_size,
                    int world, void* output, void* stream);

/* Exchange over peer memory instead of a collective library: each rank's receive buffer
 * and return buffer are device allocations shared with the other ranks by CUDA IPC
 * (fmoe_ep_ipc_alloc returns the 64-byte cudaIpcMemHandle_t, fmoe_ep_ipc_open maps a peer's
 * buffer into this process). The P2P kernels write with plain stores over NVLink (no
 * multicast) and end with a system-scope fence; the caller orders the ranks with a barrier
 * after each of them (e.g. a one-element all-reduce on the stream).
 *
 * fmoe_ep_pack_p2p: the payload row of (token t, rank d) goes to peer_recv[d] at row
 *   pos[d, t] + row_shift[d]; peer_recv and row_shift are device arrays of world entries.
 * fmoe_ep_return_p2p: received row r, from the source rank s with
 *   src_start[s] <= r < src_start[s + 1] (device array of world + 1), goes to peer_back[s] at
 *   row r + row_shift[s], as H bf16. `rows` may be an upper bound: rows at or past
 *   src_start[world] are skipped.
 * Rows outside [0, capacity_rows) are not written; they set bit 0 (pack) or 1 (return) of *err
 * (a device int the caller clears and reads). */
int fmoe_ep_ipc_alloc(size_t bytes, void** ptr, void* handle);
int fmoe_ep_ipc_open(const void* handle, void** ptr);
int fmoe_ep_ipc_close(void* ptr);
int fmoe_ep_ipc_free(void* ptr);
int fmoe_ep_pack_p2p(const void* hidden_states, const float* hidden_states_scale,
                     const int* topk_idx, const float* topk_w, const int* pos, int64_t num_tokens,
                     int hidden_size, int top_k, int world, void* const* peer_recv,
                     const int64_t* row_shift, int64_t capacity_rows, int* err, void* stream);
int fmoe_ep_return_p2p(const void* partial, int64_t rows, int hidden_size, int world,
                       const int64_t* src_start, void* const* peer_back, const int64_t* row_shift,
                       int64_t capacity_rows, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FMOE_H_ */
