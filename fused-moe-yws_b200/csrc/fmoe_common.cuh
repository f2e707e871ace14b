// fmoe_common.cuh -- definitions shared by the host orchestration and the kernels of
// the fused FP8 block-scaled MoE operator: geometry, workspace layout, error codes and
// the exactly reproducible sigmoid used by routing.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace fmoe {

// Error bits written to the device error word (meta[kMetaError]).
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutProducer = 1 << 0,  // TMA producer gave up waiting for a free stage
  kErrTimeoutMma = 1 << 1,       // MMA issuer gave up waiting for data / accumulator space
  kErrTimeoutEpilogue = 1 << 2,  // epilogue gave up waiting for an accumulator
  kErrRowOverflow = 1 << 3,      // more routed rows than the workspace was sized for
  kErrBadExpert = 1 << 4,        // routing produced an id outside [0, E_global)
};

// meta[] word indices inside the workspace.
enum MetaSlot : int {
  kMetaNumChunks = 0,  // chunks (expert, row range) for the grouped GEMMs
  kMetaTotalRows = 1,  // padded routed rows
  kMetaTicket = 2,     // last-block ticket of the routing kernel (self-resetting)
  kMetaError = 3,      // DeviceError bits (sticky until cleared by the host)
  kMetaWords = 16,
};

constexpr int kBlock = 128;        // FP8 block-scale granularity
constexpr int kRowAlign = 16;      // expert row segments padded to the MMA N granularity
constexpr int kRouteTokensPerCta = 16;  // one warp per token in the routing kernel
constexpr int kMaxBN = 128;        // largest token tile (rows per chunk) the GEMMs use
constexpr int kMaxLocalExperts = 256;  // experts one call may own (all 8 DS-V3 slices)
constexpr int kMaxSms = 160;       // upper bound on SMs per GPU for split-K scratch sizing
constexpr int kTileCounters = kMaxSms;  // stream-K arrival counters, one per CTA

struct Geometry {
  int64_t T;          // tokens
  int E;              // global experts
  int E_local;        // local experts in this slice
  int H;              // hidden size
  int I;              // intermediate size
  int top_k;
  int n_group;
  int topk_group;
};

// One chunk = a run of up to BN rows of one local expert.
struct Chunk {
  int expert;  // local expert id
  int row0;    // first row in the permuted row space
  int rows;    // real rows in this chunk (<= BN)
  int ncols;   // rows rounded up to 16 (MMA N)
};

// Byte offsets of every scratch array inside one caller-provided workspace buffer.
struct WorkspaceLayout {
  int64_t row_cap;      // capacity of the permuted row space
  int64_t max_chunks;
  int64_t n_route_ctas;
  size_t topk_idx, topk_w, token_row, cta_counts, cta_base, expert_cnt, expert_off, meta, chunks,
      row_token, row_w, a_perm, a_scale, cq, c_scale, ow, counters, partials;
  size_t total;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline WorkspaceLayout make_layout(const Geometry& g) {
  WorkspaceLayout L{};
  // Every (token, k) pair makes at most one routed row, and padding adds fewer than
  // kRowAlign rows per expert, so the plan can never overflow row_cap or max_chunks, even
  // when a caller's routing (fmoe_forward_routed) names one expert several times per token.
  L.row_cap = (int64_t)align_up((size_t)(g.T * g.top_k + (int64_t)kRowAlign * g.E_local), 256);
  L.max_chunks = g.E_local + (g.T * g.top_k) / kRowAlign + 1;
  L.n_route_ctas = (g.T + kRouteTokensPerCta - 1) / kRouteTokensPerCta;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t TK = (size_t)g.T * g.top_k;
  L.topk_idx = take(TK * 4);
  L.topk_w = take(TK * 4);
  L.token_row = take(TK * 4);
  L.cta_counts = take((size_t)L.n_route_ctas * g.E_local * 4);
  L.cta_base = take((size_t)L.n_route_ctas * g.E_local * 4);
  L.expert_cnt = take((size_t)g.E_local * 4);
  L.expert_off = take((size_t)(g.E_local + 1) * 4);
  L.meta = take(kMetaWords * 4);
  L.counters = take((size_t)kTileCounters * 4);  // right after meta: zeroed together
  L.chunks = take((size_t)L.max_chunks * sizeof(Chunk));
  L.row_token = take((size_t)L.row_cap * 4);
  L.row_w = take((size_t)L.row_cap * 4);
  L.a_perm = take((size_t)L.row_cap * g.H);
  L.a_scale = take((size_t)(g.H / kBlock) * L.row_cap * 4);
  L.cq = take((size_t)L.row_cap * 2 * g.I);
  L.c_scale = take((size_t)(g.I / kBlock) * L.row_cap * 4);
  L.ow = take((size_t)L.row_cap * g.H * 2);
  L.partials = take((size_t)2 * kMaxSms * 2 * 128 * kMaxBN * 4);  // 2 slots per CTA
  L.total = off;
  return L;
}

// ----------------------------------------------------------------------------- PDL
// Programmatic dependent launch: every kernel of the operator is launched with
// programmatic stream serialization. pdl_wait() blocks until the preceding kernel in
// the stream has completed and its writes are visible; it must come before the first
// global-memory access to the workspace. pdl_trigger() lets the next kernel start
// launching (its CTAs then run their own prologue and wait in pdl_wait()).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------------------- sigmoid
// exp(x) by Cody-Waite reduction (ln2 = hi + lo), a degree-7 Taylor polynomial on
// |r| <= ln2/2 and an exact two-step scaling by 2^n. Only IEEE round-to-nearest
// single-precision adds, multiplies, fmas and divides are used (explicit _rn
// intrinsics, so nvcc cannot contract or approximate them), which makes the result
// identical to the same algorithm on the host.
__device__ __forceinline__ float pow2i_dev(int n) { return __int_as_float((n + 127) << 23); }

__device__ __forceinline__ float exact_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208404541015625f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.428606765330187045e-06f, r);
  float p = 1.98412701138295233249664306640625e-04f;
  p = __fmaf_rn(p, r, 1.388888922519981861114501953125e-03f);
  p = __fmaf_rn(p, r, 8.333333767950534820556640625e-03f);
  p = __fmaf_rn(p, r, 4.1666667908430099487304687500e-02f);
  p = __fmaf_rn(p, r, 1.6666667163372039794921875e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni / 2;
  const int n2 = ni - n1;
  return __fmul_rn(__fmul_rn(p, pow2i_dev(n1)), pow2i_dev(n2));
}

// 1 / (1 + e) correctly rounded: __frcp_rn(d) is the IEEE quotient 1 / d, so it equals
// the host's 1.0f / d bit for bit.
__device__ __forceinline__ float exact_sigmoid(float x) {
  return __frcp_rn(__fadd_rn(1.0f, exact_expf(-x)));
}

}  // namespace fmoe
