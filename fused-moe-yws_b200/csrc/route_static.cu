// route_static.cu -- routing entry point that needs no caller workspace and allocates
// nothing.
//
// Some hosts cannot give this library scratch memory: a plugin interface that passes only
// the tensors of the call (no allocator, no workspace argument), or a serving engine that
// reserves all device memory at start-up and forbids allocation later. Calling cudaMalloc
// from such a host would also synchronise the device and break stream capture.
// fmoe_route_static() serves them. It runs the same routing kernel as fmoe_route(), but
// its scratch (per-CTA counts and bases, the expert plan, the chunk list and the small
// meta block) lives in the file-scope device array below. That array has a fixed size and
// is held by every GPU that loads the library, until the process exits.
//
// Limits and rules:
//   * num_tokens <= kStaticRouteMaxTokens (8192) and num_local_experts <= 64; larger
//     problems are rejected with FMOE_ERR_VALUE before anything is launched.
//   * The first call on a device looks up the array's device address there
//     (cudaGetSymbolAddress). Make that first call before any stream capture. The address
//     is looked up again if the device's context has changed since (a device reset).
//   * No device-side error word can be read back: within these limits the plan cannot
//     overflow (at most num_tokens * top_k routed rows), which is the routing kernel's only
//     error.
//   * All calls share the one array and it keeps the last call's contents. The call
//     clears the words that must start at zero. Calls that overlap on the GPU (different
//     streams, or different host threads, without ordering between them) race on the
//     array, so order them.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "fmoe.h"
#include "autotune_table.h"
#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"

namespace fmoe {
namespace {

constexpr int64_t kStaticRouteMaxTokens = 8192;
constexpr int kStaticRouteMaxLocal = 64;
constexpr int kStaticRouteMaxK = 32;
constexpr int64_t kStaticCtas =
    (kStaticRouteMaxTokens + kRouteTokensPerCta - 1) / kRouteTokensPerCta;
constexpr int64_t kStaticMaxChunks =
    kStaticRouteMaxLocal + kStaticRouteMaxTokens * kStaticRouteMaxK / kRowAlign + 1;

// Byte offsets inside the static scratch (each 256-byte aligned).
constexpr size_t kOffMeta = 0;
constexpr size_t kOffExpertCnt = 256;
constexpr size_t kOffExpertOff = kOffExpertCnt + 512;
constexpr size_t kOffCtaCounts = kOffExpertOff + 512;
constexpr size_t kOffCtaBase = kOffCtaCounts + (size_t)kStaticCtas * kStaticRouteMaxLocal * 4;
constexpr size_t kOffChunks = kOffCtaBase + (size_t)kStaticCtas * kStaticRouteMaxLocal * 4;
constexpr size_t kStaticScratchBytes = kOffChunks + (size_t)kStaticMaxChunks * sizeof(Chunk);

// The scratch itself: about 0.53 MB per device.
static __device__ __align__(256) unsigned char g_route_scratch[kStaticScratchBytes];

int fail_static(int code, const std::string& msg) {
  set_last_error(msg);  // reported by fmoe_last_error(), like every other entry point
  return code;
}

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The driver context current on this thread (nullptr if the entry point is unavailable).
CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(ptr);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  CUcontext ctx = nullptr;
  if (fn) fn(&ctx);
  return ctx;
}

// Per-device address of g_route_scratch, looked up once per device with that device current.
// The address belongs to the device's context: if that context was destroyed and a new one
// created (cudaDeviceReset, for one), the address is looked up again in the new context.
int scratch_address(unsigned char** out) {
  static std::mutex mu;
  static unsigned char* addr[64] = {nullptr};
  static CUcontext ctx_of[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_static(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail_static(FMOE_ERR_RUNTIME, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev] || ctx_of[dev] != current_context()) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess)
      return fail_static(FMOE_ERR_RUNTIME,
                         std::string("cudaGetSymbolAddress(g_route_scratch) failed: ") +
                             cudaGetErrorString(e));
    addr[dev] = static_cast<unsigned char*>(p);
    ctx_of[dev] = current_context();  // the lookup made the device's context current
  }
  *out = addr[dev];
  return FMOE_OK;
}

}  // namespace
}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_route_static(const fmoe_problem* p, const float* routing_logits,
                                 const void* routing_bias, const fmoe_route_out* out,
                                 void* stream_ptr) {
  const int v = fmoe_validate(p);
  if (v != FMOE_OK) return v;
  if (p->num_tokens > kStaticRouteMaxTokens)
    return fail_static(FMOE_ERR_VALUE,
                       "fmoe_route_static: num_tokens " + std::to_string(p->num_tokens) +
                           " exceeds the static scratch limit of " +
                           std::to_string(kStaticRouteMaxTokens));
  if (p->num_local_experts > kStaticRouteMaxLocal || p->top_k > kStaticRouteMaxK)
    return fail_static(FMOE_ERR_VALUE, "fmoe_route_static: geometry beyond the static limits");
  if (p->num_tokens == 0) return FMOE_OK;
  if (!routing_logits || !routing_bias || !out || !out->topk_idx || !out->topk_w)
    return fail_static(FMOE_ERR_VALUE, "fmoe_route_static: pointers must not be NULL");
  unsigned char* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != FMOE_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  // the last-CTA ticket and the error word must start at zero
  cudaError_t e = cudaMemsetAsync(scratch + kOffMeta, 0, kMetaWords * sizeof(int), stream);
  if (e != cudaSuccess) return fail_static(FMOE_ERR_RUNTIME, cudaGetErrorString(e));

  const int bn =
      resolve_tile_n(p->tile_n, p->num_tokens, p->top_k, p->num_experts, p->hidden_size);
  RouteArgs a;
  a.in_idx = nullptr;
  a.in_w = nullptr;
  a.t_dev = nullptr;
  a.inject_err = 0;
  a.logits = routing_logits;
  a.bias = static_cast<const uint16_t*>(routing_bias);
  a.T = p->num_tokens;
  a.E = p->num_experts;
  a.n_group = p->n_group;
  a.topk_group = p->topk_group;
  a.top_k = p->top_k;
  a.E_local = p->num_local_experts;
  a.local_offset = p->local_expert_offset;
  a.rsf = p->routed_scaling_factor;
  a.bn = bn;
  a.bn_log2 = 0;
  while ((1 << a.bn_log2) < bn) ++a.bn_log2;
  // T * top_k routed rows at most (the same bound as make_layout), so the plan never
  // overflows and the routing kernel sets no device error word here; this entry point has
  // no way to report one.
  a.row_cap = p->num_tokens * p->top_k + (int64_t)kRowAlign * p->num_local_experts;
  a.max_chunks = kStaticMaxChunks;
  a.topk_idx = out->topk_idx;  // results go straight to the caller's buffers
  a.topk_w = out->topk_w;
  a.cta_counts = reinterpret_cast<int*>(scratch + kOffCtaCounts);
  a.cta_base = reinterpret_cast<int*>(scratch + kOffCtaBase);
  a.expert_cnt = reinterpret_cast<int*>(scratch + kOffExpertCnt);
  a.expert_off = reinterpret_cast<int*>(scratch + kOffExpertOff);
  a.meta = reinterpret_cast<int*>(scratch + kOffMeta);
  a.chunks = reinterpret_cast<Chunk*>(scratch + kOffChunks);
  const unsigned ctas = (unsigned)((p->num_tokens + kRouteTokensPerCta - 1) / kRouteTokensPerCta);
  e = launch_pdl(route_plan_kernel, dim3(ctas), dim3(kRouteTokensPerCta * 32), 0, stream, a);
  if (e != cudaSuccess) return fail_static(FMOE_ERR_RUNTIME, cudaGetErrorString(e));
  return FMOE_OK;
}
