// fmoe_api.cu -- host side of the C ABI declared in include/fmoe.h.
//
// Restates the reference's host orchestration (solution/cuda/kernel.cu:1727-1837 and
// the two pipelines at :1447-1720) for the B200 kernels:
//   * argument checks mirror CheckTensor / CheckSameDevice (kernel.cu:121-168) for
//     what a pointer ABI can check (sizes, geometry, alignment);
//   * no per-call allocation, no host round trip and no stream synchronisation: the
//     reference's cudaStreamSynchronize (kernel.cu:1544, :1834), pinned-host count copy
//     and per-call cudaMallocAsync (kernel.cu:1532-1546, :1290-1310) are replaced by
//     device-side planning in route_plan_kernel and a caller-owned workspace;
//   * one pipeline for every T; the token tile comes from the autotune table instead of
//     the reference's fixed T <= 512 switch (kernel.cu:47, :1781).
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "fmoe.h"
#include "autotune_table.h"
#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"

namespace fmoe {
namespace {

thread_local std::string g_last_error;
thread_local cudaEvent_t g_stage_events[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
thread_local bool g_stage_on = false;
thread_local int g_inject_err = 0;  // fmoe_selftest_inject_device_error, next forward call

int mark_stage(int i, cudaStream_t s);

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

#define FMOE_CUDA_TRY(expr)                                                              \
  do {                                                                                   \
    cudaError_t err__ = (expr);                                                          \
    if (err__ != cudaSuccess)                                                            \
      return fail(FMOE_ERR_RUNTIME, std::string("CUDA error at ") + __FILE__ + ":" +      \
                                        std::to_string(__LINE__) + ": " +                \
                                        cudaGetErrorString(err__));                      \
  } while (0)

Geometry to_geometry(const fmoe_problem& p) {
  Geometry g;
  g.T = p.num_tokens;
  g.E = p.num_experts;
  g.E_local = p.num_local_experts;
  g.H = p.hidden_size;
  g.I = p.intermediate_size;
  g.top_k = p.top_k;
  g.n_group = p.n_group;
  g.topk_group = p.topk_group;
  return g;
}

int validate(const fmoe_problem* p) {
  if (!p) return fail(FMOE_ERR_VALUE, "problem must not be NULL");
  if (p->num_tokens < 0) return fail(FMOE_ERR_VALUE, "num_tokens must be >= 0");
  if (p->num_tokens > (int64_t)1 << 24)
    return fail(FMOE_ERR_VALUE, "num_tokens exceeds 2^24");
  if (p->num_experts < 1 || p->num_experts > 256)
    return fail(FMOE_ERR_VALUE, "num_experts must be in [1, 256]");
  if (p->n_group < 1 || p->n_group > 32 || p->num_experts % p->n_group != 0)
    return fail(FMOE_ERR_VALUE, "n_group must be in [1, 32] and divide num_experts");
  if (p->topk_group < 1 || p->topk_group > p->n_group)
    return fail(FMOE_ERR_VALUE, "topk_group must be in [1, n_group]");
  if (p->top_k < 1 || p->top_k > 32 ||
      p->top_k > p->topk_group * (p->num_experts / p->n_group))
    return fail(FMOE_ERR_VALUE, "top_k must be in [1, 32] and fit in the kept groups");
  if (p->num_local_experts < 1 || p->num_local_experts > kMaxLocalExperts)
    return fail(FMOE_ERR_VALUE, "num_local_experts must be in [1, 256]");
  if (p->hidden_size < 128 || p->hidden_size % 128 != 0 || p->hidden_size > 16384)
    return fail(FMOE_ERR_VALUE, "hidden_size must be a positive multiple of 128 (<= 16384)");
  if (p->intermediate_size < 128 || p->intermediate_size % 128 != 0 ||
      p->intermediate_size > 16384)
    return fail(FMOE_ERR_VALUE,
                "intermediate_size must be a positive multiple of 128 (<= 16384)");
  if (p->tile_n != 0 && !gemm_bn_supported(p->tile_n))
    return fail(FMOE_ERR_VALUE, "tile_n must be 0 or one of 16, 32, 64, 128");
  if (p->tile_n == 128 && p->hidden_size % 256 != 0)
    return fail(FMOE_ERR_VALUE, "tile_n 128 needs hidden_size to be a multiple of 256");
  const WorkspaceLayout L = make_layout(to_geometry(*p));
  if (L.row_cap * (int64_t)p->hidden_size >= ((int64_t)1 << 40))
    return fail(FMOE_ERR_VALUE, "problem too large for the row-permuted workspace");
  return FMOE_OK;
}

int tile_n_of(const fmoe_problem* p) {
  return resolve_tile_n(p->tile_n, p->num_tokens, p->top_k, p->num_experts, p->hidden_size);
}

bool aligned(const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Byte tensor of rank 2 or 3: dims[0] is the contiguous one, strides[i] is the byte
// distance between consecutive indices of dims[i + 1]; box[i] elements per dimension.
int encode_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
               const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
               const char* what) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(FMOE_ERR_RUNTIME, "cuTensorMapEncodeTiled unavailable");
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank,
                         const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FMOE_ERR_RUNTIME, std::string("tensor map encode failed for ") + what +
                                      " (CUresult " + std::to_string((int)r) + ")");
  return FMOE_OK;
}

// 2D byte tensor [outer, inner] with row pitch `pitch` bytes; box [box_outer, box_inner].
int make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch,
             uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz, const char* what) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_inner, box_outer};
  return encode_map(map, base, 2, dims, strides, box, swz, what);
}

int num_sms_current() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// ---------------------------------------------------------------------- error sink
// One host-mapped pinned pair {error bits, report count} per device. The combine kernel of
// every call adds its call's device error word to it (report_device_error), so a timeout
// inside a GEMM reaches the host without a synchronisation: fmoe_poll_device_error() reads
// the pair. It is allocated on a device's first call that is not being captured into a
// graph (a capturing stream cannot allocate); calls captured before that report nothing.
struct ErrorSink {
  unsigned* host = nullptr;  // [0] bits, [1] count
  unsigned* dev = nullptr;
  unsigned seen = 0;         // count at the last poll
};
std::mutex g_sink_mu;
ErrorSink g_sinks[64];

unsigned* error_sink_for(int dev, cudaStream_t stream) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_sink_mu);
  ErrorSink& s = g_sinks[dev];
  if (s.dev) return s.dev;
  if (stream) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
      return nullptr;
  }
  void* h = nullptr;
  if (cudaHostAlloc(&h, 2 * sizeof(unsigned), cudaHostAllocMapped | cudaHostAllocPortable) !=
      cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
    cudaGetLastError();
    cudaFreeHost(h);
    return nullptr;
  }
  s.host = static_cast<unsigned*>(h);
  s.host[0] = 0;
  s.host[1] = 0;
  s.dev = static_cast<unsigned*>(d);
  return s.dev;
}

int mark_stage(int i, cudaStream_t s) {
  if (!g_stage_on) return FMOE_OK;
  FMOE_CUDA_TRY(cudaEventRecord(g_stage_events[i], s));
  return FMOE_OK;
}

struct Carved {
  WorkspaceLayout L;
  uint8_t* base;
  template <typename T>
  T* at(size_t off) const {
    return reinterpret_cast<T*>(base + off);
  }
};

int carve(const fmoe_problem* p, void* ws, size_t ws_bytes, Carved* c) {
  c->L = make_layout(to_geometry(*p));
  if (!ws) return fail(FMOE_ERR_WORKSPACE, "workspace must not be NULL");
  if (!aligned(ws, 256)) return fail(FMOE_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (ws_bytes < c->L.total)
    return fail(FMOE_ERR_WORKSPACE, "workspace too small: need " + std::to_string(c->L.total) +
                                        " bytes, got " + std::to_string(ws_bytes));
  c->base = static_cast<uint8_t*>(ws);
  return FMOE_OK;
}

RouteArgs route_args(const fmoe_problem* p, const Carved& c, const float* logits,
                     const void* bias, int bn) {
  RouteArgs a;
  a.in_idx = nullptr;
  a.in_w = nullptr;
  a.t_dev = nullptr;
  a.inject_err = 0;
  a.logits = logits;
  a.bias = static_cast<const uint16_t*>(bias);
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
  a.row_cap = c.L.row_cap;
  a.max_chunks = c.L.max_chunks;
  a.topk_idx = c.at<int>(c.L.topk_idx);
  a.topk_w = c.at<float>(c.L.topk_w);
  a.cta_counts = c.at<int>(c.L.cta_counts);
  a.cta_base = c.at<int>(c.L.cta_base);
  a.expert_cnt = c.at<int>(c.L.expert_cnt);
  a.expert_off = c.at<int>(c.L.expert_off);
  a.meta = c.at<int>(c.L.meta);
  a.chunks = c.at<Chunk>(c.L.chunks);
  return a;
}

int launch_route(const fmoe_problem* p, const Carved& c, const float* logits, const void* bias,
                 int bn, cudaStream_t stream, const int* in_idx = nullptr,
                 const float* in_w = nullptr, int inject_err = 0,
                 const int* t_dev = nullptr) {
  // meta words and the stream-K counters are contiguous: one small memset per call
  FMOE_CUDA_TRY(cudaMemsetAsync(c.at<int>(c.L.meta), 0, c.L.counters - c.L.meta +
                                kTileCounters * sizeof(int), stream));
  RouteArgs ra = route_args(p, c, logits, bias, bn);
  ra.in_idx = in_idx;
  ra.in_w = in_w;
  ra.inject_err = inject_err;
  ra.t_dev = t_dev;
  FMOE_CUDA_TRY(launch_pdl(route_plan_kernel, dim3((unsigned)c.L.n_route_ctas),
                           dim3(kRouteTokensPerCta * 32), 0, stream, ra));
  return FMOE_OK;
}

}  // namespace
}  // namespace fmoe

void fmoe::set_last_error(const std::string& msg) { g_last_error = msg; }

using namespace fmoe;

extern "C" int fmoe_abi_version(void) { return FMOE_ABI_VERSION; }

extern "C" const char* fmoe_last_error(void) { return g_last_error.c_str(); }

extern "C" int fmoe_validate(const fmoe_problem* p) { return validate(p); }

extern "C" int fmoe_autotune_tile_n(int64_t num_tokens) {
  return autotune_tile_n(num_tokens, 8, 256);  // DeepSeek-V3 routing: top_k 8 of 256
}

extern "C" int fmoe_tile_n(const fmoe_problem* p) {
  const int v = validate(p);
  if (v != FMOE_OK) return -v;
  return tile_n_of(p);
}

extern "C" int fmoe_workspace_size(const fmoe_problem* p, size_t* bytes) {
  const int v = validate(p);
  if (v != FMOE_OK) return v;
  if (!bytes) return fail(FMOE_ERR_VALUE, "bytes must not be NULL");
  *bytes = make_layout(to_geometry(*p)).total;
  return FMOE_OK;
}

namespace fmoe {
namespace {
// Expert-parallel return of the combine's rows to their source ranks (peer memory), or none.
struct EpReturn {
  void* const* peer_out;
  const int64_t* src_start;
  const int64_t* row_shift;
  int world;
  int64_t capacity;
  int* err;
};

int run_forward(const fmoe_problem* p, const fmoe_tensors* t, const int32_t* in_idx,
                const float* in_w, const int32_t* t_dev, void* workspace,
                size_t workspace_bytes, void* stream_ptr, bool prelaid,
                const EpReturn* ret = nullptr) {
  int v = validate(p);
  if (v != FMOE_OK) return v;
  if (prelaid && p->hidden_size % 256 != 0)
    return fail(FMOE_ERR_VALUE, "pre-laid-out weights need hidden_size to be a multiple of 256");
  if (!t) return fail(FMOE_ERR_VALUE, "tensors must not be NULL");
  if (p->num_tokens == 0) return FMOE_OK;  // empty batch: nothing to write
  if (in_idx && (!in_w || !aligned(in_idx, 16) || !aligned(in_w, 16)))
    return fail(FMOE_ERR_VALUE, "topk_idx / topk_w must be non-NULL and 16-byte aligned");
  const void* ptrs[] = {in_idx ? (const void*)in_idx : t->routing_logits,
                        in_idx ? (const void*)in_w : t->routing_bias, t->hidden_states,
                        t->hidden_states_scale, t->gemm1_weights, t->gemm1_weights_scale,
                        t->gemm2_weights, t->gemm2_weights_scale, t->output};
  const char* names[] = {in_idx ? "topk_idx" : "routing_logits",
                         in_idx ? "topk_w" : "routing_bias", "hidden_states",
                         "hidden_states_scale", "gemm1_weights", "gemm1_weights_scale",
                         "gemm2_weights", "gemm2_weights_scale", "output"};
  for (int i = 0; i < 9; ++i) {
    if (!ptrs[i]) return fail(FMOE_ERR_VALUE, std::string(names[i]) + " must not be NULL");
    if (!aligned(ptrs[i], 16))
      return fail(FMOE_ERR_VALUE, std::string(names[i]) + " must be 16-byte aligned");
  }
  Carved c;
  v = carve(p, workspace, workspace_bytes, &c);
  if (v != FMOE_OK) return v;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int bn = tile_n_of(p);
  const bool tm = bn == 128;  // throughput family: token rows on the MMA M side
  const int64_t T = p->num_tokens;
  const int H = p->hidden_size, I = p->intermediate_size, EL = p->num_local_experts;

  int dev = 0;
  FMOE_CUDA_TRY(cudaGetDevice(&dev));
  unsigned* sink = error_sink_for(dev, stream);
  const int inject = g_inject_err;
  g_inject_err = 0;
  if ((v = mark_stage(0, stream)) != FMOE_OK) return v;
  v = launch_route(p, c, t->routing_logits, t->routing_bias, bn, stream, in_idx, in_w, inject,
                   t_dev);
  if (v != FMOE_OK) return v;
  if ((v = mark_stage(1, stream)) != FMOE_OK) return v;

  ScatterArgs sa;
  sa.hidden = static_cast<const uint8_t*>(t->hidden_states);
  sa.hidden_scale = t->hidden_states_scale;
  sa.T = T;
  sa.H = H;
  sa.top_k = p->top_k;
  sa.E_local = EL;
  sa.local_offset = p->local_expert_offset;
  sa.row_cap = c.L.row_cap;
  sa.topk_idx = c.at<int>(c.L.topk_idx);
  sa.topk_w = c.at<float>(c.L.topk_w);
  sa.cta_base = c.at<int>(c.L.cta_base);
  sa.expert_cnt = c.at<int>(c.L.expert_cnt);
  sa.expert_off = c.at<int>(c.L.expert_off);
  sa.token_row = c.at<int>(c.L.token_row);
  sa.row_token = c.at<int>(c.L.row_token);
  sa.row_w = c.at<float>(c.L.row_w);
  sa.a_perm = c.at<uint8_t>(c.L.a_perm);
  sa.a_scale = c.at<float>(c.L.a_scale);
  sa.meta = c.at<int>(c.L.meta);
  int permute_ctas = 0;
  {
    // split each row's columns over enough CTAs to cover the SMs at small T
    const int sms = num_sms_current();
    int parts = (int)((2 * sms + c.L.n_route_ctas - 1) / c.L.n_route_ctas);
    parts = parts < 1 ? 1 : (parts > 28 ? 28 : parts);
    permute_ctas = (int)c.L.n_route_ctas * parts;
    FMOE_CUDA_TRY(launch_pdl(scatter_gather_kernel,
                             dim3((unsigned)c.L.n_route_ctas, (unsigned)parts), dim3(256), 0,
                             stream, sa));
  }
  if ((v = mark_stage(2, stream)) != FMOE_OK) return v;

  // Tensor maps. Throughput family: token rows on the MMA M side (128-row boxes of tokens
  // and of weights). Decode family: 32 KB of weights per box -- W13 as {K, row in half,
  // (expert, gate|up)} with box {128, 128, 2}, W2 with 256-row boxes -- and the hi / lo
  // token tiles of one C block as {byte in block, row, 128-byte block} with box {128, BN, 2}.
  CUtensorMap m_w13, m_a, m_w2, m_cq;
  uint8_t* cq = c.at<uint8_t>(c.L.cq);
  if ((v = make_map(&m_a, sa.a_perm, H, c.L.row_cap, H, 128, bn, CU_TENSOR_MAP_SWIZZLE_128B,
                    "permuted activations")) != FMOE_OK)
    return v;
  if (tm) {
    if ((v = make_map(&m_w13, t->gemm1_weights, H, (uint64_t)EL * 2 * I, H, 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B, "gemm1_weights")) != FMOE_OK)
      return v;
    if ((v = make_map(&m_w2, t->gemm2_weights, I, (uint64_t)EL * H, I, 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B, "gemm2_weights")) != FMOE_OK)
      return v;
    if ((v = make_map(&m_cq, cq, 2 * (uint64_t)I, c.L.row_cap, 2 * (uint64_t)I, 128, bn,
                      CU_TENSOR_MAP_SWIZZLE_128B, "quantised intermediate")) != FMOE_OK)
      return v;
  } else {
    const cuuint64_t d13[3] = {(cuuint64_t)H, (cuuint64_t)I, 2 * (cuuint64_t)EL};
    const cuuint64_t s13[2] = {(cuuint64_t)H, (cuuint64_t)I * H};
    const cuuint32_t b13[3] = {128, 128, 2};
    if ((v = encode_map(&m_w13, t->gemm1_weights, 3, d13, s13, b13, CU_TENSOR_MAP_SWIZZLE_128B,
                        "gemm1_weights")) != FMOE_OK)
      return v;
    if ((v = make_map(&m_w2, t->gemm2_weights, I, (uint64_t)EL * H, I, 128, 256,
                      CU_TENSOR_MAP_SWIZZLE_128B, "gemm2_weights")) != FMOE_OK)
      return v;
    const cuuint64_t dq[3] = {128, (cuuint64_t)c.L.row_cap, 2 * (cuuint64_t)I / 128};
    const cuuint64_t sq[2] = {2 * (cuuint64_t)I, 128};
    const cuuint32_t bq[3] = {128, (cuuint32_t)bn, 2};
    if ((v = encode_map(&m_cq, cq, 3, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B,
                        "quantised intermediate")) != FMOE_OK)
      return v;
  }

  GemmArgs g;
  g.chunks = c.at<Chunk>(c.L.chunks);
  g.meta = c.at<int>(c.L.meta);
  g.expert_cnt = c.at<int>(c.L.expert_cnt);
  g.H = H;
  g.I = I;
  g.row_cap = c.L.row_cap;
  g.cq = cq;
  g.c_scale = c.at<float>(c.L.c_scale);
  g.row_w = c.at<float>(c.L.row_w);
  g.ow = c.at<__nv_bfloat16>(c.L.ow);
  g.err = c.at<int>(c.L.meta) + kMetaError;
  g.w_pre = prelaid ? static_cast<const uint8_t*>(t->gemm1_weights) : nullptr;
  g.partials = c.at<float>(c.L.partials);
  g.tile_counters = c.at<int>(c.L.counters);
  const int sms = num_sms_current() < kMaxSms ? num_sms_current() : kMaxSms;

  g.m_tiles = I / kBlock;
  g.k_steps = H / kBlock;
  g.w_scale = t->gemm1_weights_scale;
  g.act_scale = sa.a_scale;
  int64_t bound = c.L.max_chunks * (int64_t)g.m_tiles;
  // Decode family with a small permute grid (T <= 16: 28 CTAs): GEMM1 leaves the permute's
  // SMs free. Its CTAs then all start while the permute runs and issue their first weight
  // stages, instead of a quarter of them starting only when the permute has finished and
  // ending last (T = 1: GEMM1's span after its wait 29 -> 26.7 us on B200).
  int sms1 = sms;
  if (!tm && permute_ctas * 4 <= sms) sms1 = sms - permute_ctas;
  const int grid1 = (int)(bound < sms1 ? bound : sms1);
  if (tm)
    FMOE_CUDA_TRY(launch_gemm1_tm(m_a, m_w13, g, grid1, stream));
  else
    FMOE_CUDA_TRY(launch_gemm1(bn, m_w13, m_a, g, grid1, stream));
  if ((v = mark_stage(3, stream)) != FMOE_OK) return v;

  g.m_tiles = tm ? H / 256 : (H + 255) / 256;
  g.k_steps = I / kBlock;
  g.w_scale = t->gemm2_weights_scale;
  g.w_pre = prelaid ? static_cast<const uint8_t*>(t->gemm2_weights) : nullptr;
  g.act_scale = g.c_scale;
  bound = c.L.max_chunks * (int64_t)g.m_tiles;
  const int grid2 = (int)(bound < sms ? bound : sms);
  if (tm)
    FMOE_CUDA_TRY(launch_gemm2_tm(m_cq, m_w2, g, grid2, stream));
  else
    FMOE_CUDA_TRY(launch_gemm2(bn, m_w2, m_cq, g, grid2, stream));
  if ((v = mark_stage(4, stream)) != FMOE_OK) return v;

  CombineArgs ca;
  ca.token_row = sa.token_row;
  ca.ow = g.ow;
  ca.out = static_cast<__nv_bfloat16*>(t->output);
  ca.T = T;
  ca.H = H;
  ca.top_k = p->top_k;
  ca.err_word = g.err;
  ca.err_sink = sink;
  ca.t_dev = t_dev;
  ca.peer_out = ret ? reinterpret_cast<__nv_bfloat16* const*>(ret->peer_out) : nullptr;
  ca.src_start = ret ? ret->src_start : nullptr;
  ca.row_shift = ret ? ret->row_shift : nullptr;
  ca.world = ret ? ret->world : 0;
  ca.capacity = ret ? ret->capacity : 0;
  ca.xerr = ret ? ret->err : nullptr;
  if (T >= kCombineWideTokens)
    FMOE_CUDA_TRY(launch_pdl(combine_kernel<2>,
                             dim3((unsigned)T, (unsigned)((H / 8 + 255) / 256)), dim3(128), 0,
                             stream, ca));
  else
    FMOE_CUDA_TRY(launch_pdl(combine_kernel<1>,
                             dim3((unsigned)T, (unsigned)((H / 8 + 127) / 128)), dim3(128), 0,
                             stream, ca));
  return mark_stage(5, stream);
}
}  // namespace
}  // namespace fmoe

namespace fmoe {
namespace {

// ---------------------------------------------------------------------- graph cache
// A call whose arguments (problem, every pointer, workspace, device, stream) repeat is
// replayed from a CUDA graph: the second identical call captures the operator (memset and
// the five PDL-linked kernels) on a library-owned stream and every later one launches the
// instantiated graph on the caller's stream, so the per-call cost is one graph launch
// instead of six launches. The graph reads the buffers' current contents; only the
// addresses and sizes are frozen, and they are the key. Calls whose stream is itself being
// captured, calls with stage events on, and FMOE_GRAPH_CACHE=0 run eagerly.
struct GraphKey {
  fmoe_problem p;
  int prelaid;
  fmoe_tensors t;
  const void* in_idx;
  const void* in_w;
  const void* t_dev;
  EpReturn ret;
  void* ws;
  size_t ws_bytes;
  void* stream;
  int device;
};

struct GraphEntry {
  GraphKey key;
  cudaGraphExec_t exec;  // null until the key has been seen twice
  uint64_t last_use;
};

constexpr size_t kGraphCacheSize = 16;
std::mutex g_graph_mu;
std::vector<GraphEntry> g_graphs;
uint64_t g_graph_clock = 0;

bool graph_cache_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("FMOE_GRAPH_CACHE");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool same_key(const GraphKey& a, const GraphKey& b) {
  return std::memcmp(&a, &b, sizeof(GraphKey)) == 0;
}

cudaStream_t capture_stream(int device) {
  static std::mutex mu;
  static std::vector<cudaStream_t> streams;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)streams.size() <= device) streams.resize(device + 1, nullptr);
  if (!streams[device]) {
    cudaStream_t st = nullptr;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    streams[device] = st;
  }
  return streams[device];
}

int forward_cached(const fmoe_problem* p, const fmoe_tensors* t, const int32_t* in_idx,
                   const float* in_w, void* workspace, size_t workspace_bytes,
                   void* stream_ptr, bool prelaid = false, const int32_t* t_dev = nullptr,
                   const EpReturn* ret = nullptr) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (!graph_cache_enabled() || g_stage_on || g_inject_err != 0 || !p || !t ||
      p->num_tokens <= 0 ||
      cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
    return run_forward(p, t, in_idx, in_w, t_dev, workspace, workspace_bytes, stream_ptr,
                       prelaid, ret);
  GraphKey key;
  std::memset(&key, 0, sizeof(key));  // padding bytes take part in the comparison
  key.p = *p;
  key.prelaid = prelaid;
  key.t = *t;
  key.in_idx = in_idx;
  key.in_w = in_w;
  key.t_dev = t_dev;
  if (ret) std::memcpy(&key.ret, ret, sizeof(EpReturn));  // callers zero its padding
  key.ws = workspace;
  key.ws_bytes = workspace_bytes;
  key.stream = stream_ptr;
  FMOE_CUDA_TRY(cudaGetDevice(&key.device));

  std::unique_lock<std::mutex> lock(g_graph_mu);
  GraphEntry* hit = nullptr;
  for (GraphEntry& e : g_graphs)
    if (same_key(e.key, key)) hit = &e;
  if (hit && hit->exec) {
    hit->last_use = ++g_graph_clock;
    cudaGraphExec_t exec = hit->exec;
    lock.unlock();
    FMOE_CUDA_TRY(cudaGraphLaunch(exec, stream));
    return FMOE_OK;
  }
  if (!hit) {
    // first sighting: remember the key (evicting the least recently used), run eagerly
    if (g_graphs.size() >= kGraphCacheSize) {
      size_t old = 0;
      for (size_t i = 1; i < g_graphs.size(); ++i)
        if (g_graphs[i].last_use < g_graphs[old].last_use) old = i;
      if (g_graphs[old].exec) cudaGraphExecDestroy(g_graphs[old].exec);
      g_graphs.erase(g_graphs.begin() + (std::ptrdiff_t)old);
    }
    g_graphs.push_back(GraphEntry{key, nullptr, ++g_graph_clock});
    lock.unlock();
    return run_forward(p, t, in_idx, in_w, t_dev, workspace, workspace_bytes, stream_ptr,
                       prelaid, ret);
  }
  // second sighting: capture on the library stream, then launch on the caller's stream
  cudaStream_t cs = capture_stream(key.device);
  if (!cs) {
    lock.unlock();
    return run_forward(p, t, in_idx, in_w, t_dev, workspace, workspace_bytes, stream_ptr,
                       prelaid, ret);
  }
  FMOE_CUDA_TRY(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
  const int v =
      run_forward(p, t, in_idx, in_w, t_dev, workspace, workspace_bytes, cs, prelaid, ret);
  cudaGraph_t graph = nullptr;
  const cudaError_t ec = cudaStreamEndCapture(cs, &graph);
  if (v != FMOE_OK) {
    if (graph) cudaGraphDestroy(graph);
    return v;
  }
  if (ec != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return fail(FMOE_ERR_RUNTIME, std::string("graph capture failed: ") + cudaGetErrorString(ec));
  }
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess)
    return fail(FMOE_ERR_RUNTIME,
                std::string("graph instantiation failed: ") + cudaGetErrorString(ei));
  hit->exec = exec;
  hit->last_use = ++g_graph_clock;
  lock.unlock();
  FMOE_CUDA_TRY(cudaGraphLaunch(exec, stream));
  return FMOE_OK;
}

}  // namespace
}  // namespace fmoe

extern "C" int fmoe_forward(const fmoe_problem* p, const fmoe_tensors* t, void* workspace,
                            size_t workspace_bytes, void* stream_ptr) {
  return forward_cached(p, t, nullptr, nullptr, workspace, workspace_bytes, stream_ptr);
}

extern "C" int fmoe_forward_routed(const fmoe_problem* p, const int32_t* topk_idx,
                                   const float* topk_w, const fmoe_tensors* t, void* workspace,
                                   size_t workspace_bytes, void* stream_ptr) {
  if (!topk_idx || !topk_w) return fail(FMOE_ERR_VALUE, "topk_idx / topk_w must not be NULL");
  return forward_cached(p, t, topk_idx, topk_w, workspace, workspace_bytes, stream_ptr);
}

extern "C" int fmoe_forward_routed_count(const fmoe_problem* p, const int32_t* topk_idx,
                                         const float* topk_w, const int32_t* num_tokens_dev,
                                         const fmoe_tensors* t, void* workspace,
                                         size_t workspace_bytes, void* stream_ptr) {
  if (!topk_idx || !topk_w || !num_tokens_dev)
    return fail(FMOE_ERR_VALUE, "topk_idx / topk_w / num_tokens_dev must not be NULL");
  return forward_cached(p, t, topk_idx, topk_w, workspace, workspace_bytes, stream_ptr, false,
                        num_tokens_dev);
}

extern "C" int fmoe_forward_routed_count_p2p(
    const fmoe_problem* p, const int32_t* topk_idx, const float* topk_w,
    const int32_t* num_tokens_dev, const fmoe_tensors* t, void* workspace,
    size_t workspace_bytes, void* const* peer_out, const int64_t* src_start,
    const int64_t* row_shift, int world, int64_t capacity_rows, int* err, void* stream_ptr) {
  if (!topk_idx || !topk_w || !num_tokens_dev)
    return fail(FMOE_ERR_VALUE, "topk_idx / topk_w / num_tokens_dev must not be NULL");
  if (!peer_out || !src_start || !row_shift || !err || world <= 0 || world > 32 ||
      capacity_rows < 0)
    return fail(FMOE_ERR_VALUE, "fmoe_forward_routed_count_p2p: bad return arguments");
  EpReturn ret;
  std::memset(&ret, 0, sizeof(ret));  // the graph-cache key compares its bytes
  ret.peer_out = peer_out;
  ret.src_start = src_start;
  ret.row_shift = row_shift;
  ret.world = world;
  ret.capacity = capacity_rows;
  ret.err = err;
  return forward_cached(p, t, topk_idx, topk_w, workspace, workspace_bytes, stream_ptr, false,
                        num_tokens_dev, &ret);
}

extern "C" int fmoe_forward_prelaid(const fmoe_problem* p, const fmoe_tensors* t,
                                    void* workspace, size_t workspace_bytes, void* stream_ptr) {
  return forward_cached(p, t, nullptr, nullptr, workspace, workspace_bytes, stream_ptr, true);
}

extern "C" int fmoe_forward_routed_prelaid(const fmoe_problem* p, const int32_t* topk_idx,
                                           const float* topk_w, const fmoe_tensors* t,
                                           void* workspace, size_t workspace_bytes,
                                           void* stream_ptr) {
  if (!topk_idx || !topk_w) return fail(FMOE_ERR_VALUE, "topk_idx / topk_w must not be NULL");
  return forward_cached(p, t, topk_idx, topk_w, workspace, workspace_bytes, stream_ptr, true);
}

extern "C" int fmoe_prelayout_weights(const fmoe_problem* p, const void* gemm1_weights,
                                      const void* gemm2_weights, void* gemm1_out,
                                      void* gemm2_out, void* stream_ptr) {
  int v = validate(p);
  if (v != FMOE_OK) return v;
  if (p->hidden_size % 256 != 0)
    return fail(FMOE_ERR_VALUE, "pre-laid-out weights need hidden_size to be a multiple of 256");
  if (!gemm1_weights || !gemm2_weights || !gemm1_out || !gemm2_out)
    return fail(FMOE_ERR_VALUE, "weight pointers must not be NULL");
  const void* ptrs[] = {gemm1_weights, gemm2_weights, gemm1_out, gemm2_out};
  for (const void* q : ptrs)
    if (!aligned(q, 16)) return fail(FMOE_ERR_VALUE, "weight pointers must be 16-byte aligned");
  const size_t b1 = (size_t)p->num_local_experts * 2 * p->intermediate_size * p->hidden_size;
  const size_t b2 = (size_t)p->num_local_experts * p->hidden_size * p->intermediate_size;
  auto overlaps = [](const void* a, size_t na, const void* b, size_t nb) {
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + nb && y < x + na;
  };
  if (overlaps(gemm1_out, b1, gemm1_weights, b1) || overlaps(gemm1_out, b1, gemm2_weights, b2) ||
      overlaps(gemm2_out, b2, gemm1_weights, b1) || overlaps(gemm2_out, b2, gemm2_weights, b2) ||
      overlaps(gemm1_out, b1, gemm2_out, b2))
    return fail(FMOE_ERR_VALUE, "pre-layout outputs must not overlap the weights or each other");
  FMOE_CUDA_TRY(launch_prelayout(static_cast<const uint8_t*>(gemm1_weights),
                                 static_cast<const uint8_t*>(gemm2_weights),
                                 static_cast<uint8_t*>(gemm1_out), static_cast<uint8_t*>(gemm2_out),
                                 p->num_local_experts, p->hidden_size, p->intermediate_size,
                                 static_cast<cudaStream_t>(stream_ptr)));
  return FMOE_OK;
}

extern "C" int fmoe_set_stage_events(void* const* events) {
  if (!events) {
    g_stage_on = false;
    return FMOE_OK;
  }
  for (int i = 0; i < 6; ++i) {
    if (!events[i]) return fail(FMOE_ERR_VALUE, "stage events must not be NULL");
    g_stage_events[i] = static_cast<cudaEvent_t>(events[i]);
  }
  g_stage_on = true;
  return FMOE_OK;
}

extern "C" int fmoe_route(const fmoe_problem* p, const float* routing_logits,
                          const void* routing_bias, const fmoe_route_out* out, void* workspace,
                          size_t workspace_bytes, void* stream_ptr) {
  int v = validate(p);
  if (v != FMOE_OK) return v;
  if (p->num_tokens == 0) return FMOE_OK;
  if (!routing_logits || !routing_bias || !out || !out->topk_idx || !out->topk_w)
    return fail(FMOE_ERR_VALUE, "routing pointers must not be NULL");
  Carved c;
  v = carve(p, workspace, workspace_bytes, &c);
  if (v != FMOE_OK) return v;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const int bn = tile_n_of(p);
  v = launch_route(p, c, routing_logits, routing_bias, bn, stream);
  if (v != FMOE_OK) return v;
  const size_t n = (size_t)p->num_tokens * p->top_k;
  FMOE_CUDA_TRY(cudaMemcpyAsync(out->topk_idx, c.at<int>(c.L.topk_idx), n * 4,
                                cudaMemcpyDeviceToDevice, stream));
  FMOE_CUDA_TRY(cudaMemcpyAsync(out->topk_w, c.at<float>(c.L.topk_w), n * 4,
                                cudaMemcpyDeviceToDevice, stream));
  return FMOE_OK;
}

extern "C" int fmoe_read_device_error(const fmoe_problem* p, void* workspace, void* stream_ptr,
                                      int32_t* device_error) {
  int v = validate(p);
  if (v != FMOE_OK) return v;
  if (!workspace || !device_error) return fail(FMOE_ERR_VALUE, "NULL argument");
  const WorkspaceLayout L = make_layout(to_geometry(*p));
  int* word = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + L.meta) + kMetaError;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  FMOE_CUDA_TRY(cudaStreamSynchronize(stream));
  int host = 0;
  FMOE_CUDA_TRY(cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost));
  FMOE_CUDA_TRY(cudaMemset(word, 0, sizeof(int)));
  *device_error = host;
  if (host != 0) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "device error word 0x%x", host);
    g_last_error = buf;
  }
  return FMOE_OK;
}

extern "C" int fmoe_poll_device_error(int32_t* device_error) {
  if (!device_error) return fail(FMOE_ERR_VALUE, "device_error must not be NULL");
  *device_error = 0;
  int dev = 0;
  FMOE_CUDA_TRY(cudaGetDevice(&dev));
  if (!error_sink_for(dev, nullptr))
    return fail(FMOE_ERR_RUNTIME, "could not allocate the host-mapped device error word");
  std::lock_guard<std::mutex> lock(g_sink_mu);
  ErrorSink& s = g_sinks[dev];
  volatile unsigned* h = s.host;
  const unsigned count = h[1];
  if (count == s.seen) return FMOE_OK;
  s.seen = count;
  unsigned bits = h[0];
  h[0] = 0;
  // a report whose bits were cleared by a racing poll still counts
  *device_error = (int32_t)(bits != 0 ? bits : 0x40000000u);
  char buf[128];
  std::snprintf(buf, sizeof(buf), "device error word 0x%x reported by a call on device %d",
                (unsigned)*device_error, dev);
  g_last_error = buf;
  return FMOE_OK;
}

extern "C" int fmoe_selftest_inject_device_error(int32_t bits) {
  g_inject_err = bits;
  return FMOE_OK;
}

extern "C" int fmoe_plan_view_get(const fmoe_problem* p, void* workspace, fmoe_plan_view* view) {
  int v = validate(p);
  if (v != FMOE_OK) return v;
  if (!workspace || !view) return fail(FMOE_ERR_VALUE, "NULL argument");
  const WorkspaceLayout L = make_layout(to_geometry(*p));
  uint8_t* b = static_cast<uint8_t*>(workspace);
  view->expert_cnt = reinterpret_cast<const int32_t*>(b + L.expert_cnt);
  view->expert_off = reinterpret_cast<const int32_t*>(b + L.expert_off);
  view->row_token = reinterpret_cast<const int32_t*>(b + L.row_token);
  view->token_row = reinterpret_cast<const int32_t*>(b + L.token_row);
  view->meta = reinterpret_cast<const int32_t*>(b + L.meta);
  view->row_cap = L.row_cap;
  return FMOE_OK;
}
