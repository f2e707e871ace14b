// route.cu -- DeepSeek-V3 grouped top-k routing, local-expert histogram and row plan.
//
// One warp routes one token (the reference runs one thread per token,
// solution/cuda/kernel.cu:408-516). Selection follows kernel.cu:388-516:
//   s = sigmoid(logit), s_wb = s + bias                      (kernel.cu:398-400)
//   group score = sum of the two largest s_wb in the group    (kernel.cu:423-442)
//   keep topk_group groups, ties to the lower group index     (kernel.cu:444-458)
//   pick top_k experts of kept groups by s_wb, ties to the
//   lower expert id                                            (kernel.cu:460-495)
//   w_k = s[idx_k] / (sum_k s[idx_k] + 1e-20) * rsf           (kernel.cu:497-515)
// The sigmoid is the exactly reproducible one from fmoe_common.cuh, so indices and
// weights match the host restatement bit for bit. Output is compact [T, top_k]
// (the reference writes a dense [T, 256] weight matrix).
//
// The same kernel counts each CTA's local routes (kernel.cu:530-545) and the last CTA
// to finish turns the counts into expert offsets (16-row aligned), per-CTA bases for
// the stable scatter, and the chunk list consumed by the grouped GEMMs
// (kernel.cu:594-604 and :665-689 restated on the device, no host round trip).
#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"

namespace fmoe {

namespace {

constexpr int kWarps = kRouteTokensPerCta;
constexpr int kMaxE = 256;       // experts per token supported by the warp layout
constexpr int kMaxGroups = 32;

// True when (va, ia) ranks above (vb, ib): larger value, then smaller index; NaN lowest.
__device__ __forceinline__ bool ranks_above(float va, int ia, float vb, int ib) {
  const bool na = va != va, nb = vb != vb;
  if (na || nb) return (na && nb) ? ia < ib : nb;
  if (va > vb) return true;
  if (va < vb) return false;
  return ia < ib;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

}  // namespace

// Order-preserving map of a float to uint32 (larger float -> larger key). Only used
// for candidates, which are never NaN or -inf; key 0 therefore means "no candidate".
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ bool is_candidate(float v) { return v > -INFINITY; }  // not NaN/-inf

// Routing of one token when every group holds 32 experts (DeepSeek-V3: 8 groups of 32):
// lane l owns expert g * 32 + l of every group g, so scores live in registers and every
// selection step is a warp reduction. Same arithmetic, comparisons and summation order as
// the general path below, hence the same bits.
__device__ __forceinline__ void route_token_g32(const RouteArgs& a, int64_t t, int lane,
                                                int* s_cnt) {
  constexpr int kG = 8;  // groups per token supported here (E <= 256)
  const int ng = a.n_group, K = a.top_k;
  const float* lrow = a.logits + t * a.E;
  float x[kG], b[kG], sg[kG], wb[kG];
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    x[g] = g < ng ? __ldg(lrow + g * 32 + lane) : 0.0f;
    b[g] = g < ng ? bf16_bits_to_float(__ldg(a.bias + g * 32 + lane)) : 0.0f;
  }
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    sg[g] = exact_sigmoid(x[g]);
    wb[g] = g < ng ? __fadd_rn(sg[g], b[g]) : -INFINITY;
  }
  // group score = sum of the two largest candidates (duplicates count twice)
  float gs[kG];
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    const uint32_t k = is_candidate(wb[g]) ? order_key(wb[g]) : 0u;
    const uint32_t k1 = __reduce_max_sync(0xffffffffu, k);
    const unsigned dup = __popc(__ballot_sync(0xffffffffu, k == k1 && k1 != 0u));
    const uint32_t k2 = dup >= 2 ? k1 : __reduce_max_sync(0xffffffffu, k == k1 ? 0u : k);
    gs[g] = __fadd_rn(k1 ? key_value(k1) : -INFINITY, k2 ? key_value(k2) : -INFINITY);
  }
  // kept groups: lane g (< n_group) counts the groups ranking above its own
  const int mg = lane & (kG - 1);
  float own = gs[0];
#pragma unroll
  for (int g = 1; g < kG; ++g)
    if (g == mg) own = gs[g];
  int rank = 0;
#pragma unroll
  for (int g = 0; g < kG; ++g)
    if (g < ng && g != mg) rank += ranks_above(gs[g], g, own, mg);
  const uint32_t keep =
      __ballot_sync(0xffffffffu, lane < ng && rank < a.topk_group) & ((1u << ng) - 1u);
  // top_k rounds: lane-local best (ties to the lower group = lower expert id), then the
  // warp maximum, ties to the lowest expert id
  uint32_t key[kG];
#pragma unroll
  for (int g = 0; g < kG; ++g)
    key[g] = ((keep >> g) & 1u) && is_candidate(wb[g]) ? order_key(wb[g]) : 0u;
  int my_e = -1;
  float my_s = 0.0f, sum = 0.0f;
  for (int k = 0; k < K; ++k) {
    uint32_t bk = 0u;
    int bg = 0;
#pragma unroll
    for (int g = 0; g < kG; ++g)
      if (key[g] > bk) {
        bk = key[g];
        bg = g;
      }
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
    if (kmax == 0u) break;  // fewer than top_k candidates: the rest stay -1 / 0
    const uint32_t win = __reduce_min_sync(
        0xffffffffu, bk == kmax ? (uint32_t)(bg * 32 + lane) : 0xffffffffu);
    const int wl = (int)(win & 31u), wg = (int)(win >> 5);
    float v = sg[0];
#pragma unroll
    for (int g = 1; g < kG; ++g)
      if (g == wg) v = sg[g];
    v = __shfl_sync(0xffffffffu, v, wl);
    sum = __fadd_rn(sum, v);  // selection order, as the reference sums
    if (lane == wl) {
#pragma unroll
      for (int g = 0; g < kG; ++g)
        if (g == wg) key[g] = 0u;
    }
    if (lane == k) {
      my_e = (int)win;
      my_s = v;
    }
  }
  sum = __fadd_rn(sum, 1e-20f);
  if (lane < K) {
    a.topk_idx[t * K + lane] = my_e;
    a.topk_w[t * K + lane] = my_e >= 0 ? __fmul_rn(__fdiv_rn(my_s, sum), a.rsf) : 0.0f;
    const int le = my_e - a.local_offset;
    if (my_e >= 0 && le >= 0 && le < a.E_local) atomicAdd(&s_cnt[le], 1);
  }
}

__global__ void __launch_bounds__(kWarps * 32) route_plan_kernel(RouteArgs a) {
  __shared__ float s_sc[kWarps][kMaxE];
  __shared__ float s_wb[kWarps][kMaxE];
  __shared__ float s_gscore[kWarps][kMaxGroups];
  __shared__ int s_cnt[kMaxLocalExperts];
  __shared__ int s_is_last;
  __shared__ int s_tot[kMaxLocalExperts];
  __shared__ int s_off[kMaxLocalExperts + 1];
  __shared__ int s_choff[kMaxLocalExperts + 1];
  __shared__ int s_sel[kWarps][32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, G = a.E / a.n_group, K = a.top_k;
  const int EPL = (E + 31) / 32;  // experts per lane (lane owns lane + 32 j)
  for (int i = threadIdx.x; i < a.E_local; i += blockDim.x) s_cnt[i] = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();

  const int64_t t = (int64_t)blockIdx.x * kWarps + warp;
  if (t < a.T && a.in_idx) {
    // routed mode: (expert, weight) pairs computed elsewhere (expert-parallel dispatch)
    if (lane < K) {
      const int e = a.in_idx[t * K + lane];
      a.topk_idx[t * K + lane] = e;
      a.topk_w[t * K + lane] = a.in_w[t * K + lane];
      const int le = e - a.local_offset;
      if (e >= 0 && le >= 0 && le < a.E_local) atomicAdd(&s_cnt[le], 1);
    }
  } else if (t < a.T && G == 32) {
    route_token_g32(a, t, lane, s_cnt);
  } else if (t < a.T) {
    // 1) sigmoid + bias (strided, coalesced loads)
    const float* lrow = a.logits + t * E;
    for (int e = lane; e < E; e += 32) {
      const float sg = exact_sigmoid(__ldg(lrow + e));
      s_sc[warp][e] = sg;
      s_wb[warp][e] = __fadd_rn(sg, bf16_bits_to_float(__ldg(a.bias + e)));
    }
    __syncwarp();
    // 2) group scores = sum of the two largest biased scores (NaN and -inf never count,
    //    exactly as the reference's strict '>' scan from -inf)
    if (G == 32) {
      // one expert of every group per lane: warp-wide top-2 per group via redux
      for (int g = 0; g < a.n_group; ++g) {
        const float v = s_wb[warp][g * 32 + lane];
        const uint32_t k = is_candidate(v) ? order_key(v) : 0u;
        const uint32_t k1 = __reduce_max_sync(0xffffffffu, k);
        const unsigned dup = __popc(__ballot_sync(0xffffffffu, k == k1 && k1 != 0u));
        const uint32_t k2 = dup >= 2 ? k1 : __reduce_max_sync(0xffffffffu, k == k1 ? 0u : k);
        if (lane == 0) {
          const float b0 = k1 ? key_value(k1) : -INFINITY;
          const float b1 = k2 ? key_value(k2) : -INFINITY;
          s_gscore[warp][g] = __fadd_rn(b0, b1);
        }
      }
    } else if (lane < a.n_group) {
      float b0 = -INFINITY, b1 = -INFINITY;
      for (int j = 0; j < G; ++j) {
        const float v = s_wb[warp][lane * G + j];
        if (v > b0) {
          b1 = b0;
          b0 = v;
        } else if (v > b1) {
          b1 = v;
        }
      }
      s_gscore[warp][lane] = __fadd_rn(b0, b1);
    }
    __syncwarp();
    // 3) keep topk_group groups (lane 0, tiny serial loop), broadcast as a bit mask
    uint32_t keep = 0;
    if (lane == 0) {
      for (int pick = 0; pick < a.topk_group; ++pick) {
        int best = -1;
        for (int g = 0; g < a.n_group; ++g) {
          if (keep & (1u << g)) continue;
          if (best < 0 || ranks_above(s_gscore[warp][g], g, s_gscore[warp][best], best)) best = g;
        }
        keep |= 1u << best;
      }
    }
    keep = __shfl_sync(0xffffffffu, keep, 0);
    // 4) top_k experts: per round a warp max of the order key, ties to the lowest id
    uint32_t cand = 0;  // bit j: expert lane + 32 j is still a candidate
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < E && ((keep >> (e / G)) & 1u) && is_candidate(s_wb[warp][e])) cand |= 1u << j;
    }
    int* sel = s_sel[warp];
    for (int k = 0; k < K; ++k) {
      uint32_t best_k = 0u;
      int best_e = 0x7fffffff;
      for (uint32_t c = cand; c; c &= c - 1) {
        const int j = __ffs(c) - 1;
        const int e = lane + 32 * j;
        const uint32_t key = order_key(s_wb[warp][e]);
        if (key > best_k) {  // ascending j: ties keep the lower id
          best_k = key;
          best_e = e;
        }
      }
      const uint32_t kmax = __reduce_max_sync(0xffffffffu, best_k);
      const uint32_t win = __reduce_min_sync(0xffffffffu,
                                             (best_k == kmax && kmax != 0u) ? (uint32_t)best_e
                                                                            : 0xffffffffu);
      const int bi = kmax != 0u ? (int)win : -1;
      if (lane == 0) sel[k] = bi;
      if (bi >= 0 && (bi & 31) == lane) cand &= ~(1u << (bi >> 5));
    }
    __syncwarp();
    // 5) weights in selection order, local histogram
    if (lane < K) {
      // each lane needs the same left-to-right sum: compute it redundantly in order
      float sum = 0.0f;
      for (int k = 0; k < K; ++k)
        if (sel[k] >= 0) sum = __fadd_rn(sum, s_sc[warp][sel[k]]);
      sum = __fadd_rn(sum, 1e-20f);
      const int e = sel[lane];
      a.topk_idx[t * K + lane] = e;
      a.topk_w[t * K + lane] = e >= 0 ? __fmul_rn(__fdiv_rn(s_sc[warp][e], sum), a.rsf) : 0.0f;
      const int le = e - a.local_offset;
      if (e >= 0 && le >= 0 && le < a.E_local) atomicAdd(&s_cnt[le], 1);
    }
  }
  __syncthreads();
  const int nctas = gridDim.x;
  if (nctas > 1) {
    for (int i = threadIdx.x; i < a.E_local; i += blockDim.x)
      a.cta_counts[(int64_t)blockIdx.x * a.E_local + i] = s_cnt[i];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int ticket = atomicAdd(a.meta + kMetaTicket, 1);
      s_is_last = ticket == nctas - 1;
    }
    __syncthreads();
    if (!s_is_last) return;
    __threadfence();
  }

  // ---- last CTA: expert totals, per-CTA bases, 16-row aligned offsets, chunks ----
  // cta_base[c][e] = rows of expert e routed by CTAs before c (relative to the expert's
  // first row; the scatter adds expert_off[e])
  for (int e = warp; e < a.E_local; e += kWarps) {
    int run = 0;
    if (nctas == 1) {
      run = s_cnt[e];
      if (lane == 0) a.cta_base[e] = 0;
    } else {
      for (int c0 = 0; c0 < nctas; c0 += 32) {
        const int c = c0 + lane;
        const int v = c < nctas ? __ldcg(a.cta_counts + (int64_t)c * a.E_local + e) : 0;
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        if (c < nctas) a.cta_base[(int64_t)c * a.E_local + e] = run + incl - v;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    if (lane == 0) s_tot[e] = run;
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scans over experts, 32 at a time
    int run_off = 0, run_ch = 0;
    for (int base = 0; base < a.E_local; base += 32) {
      const int e = base + lane;
      const int tot = e < a.E_local ? s_tot[e] : 0;
      const int pad = (tot + kRowAlign - 1) / kRowAlign * kRowAlign;
      const int nch = (tot + a.bn - 1) >> a.bn_log2;
      int io = pad, ic = nch;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int yo = __shfl_up_sync(0xffffffffu, io, o);
        const int yc = __shfl_up_sync(0xffffffffu, ic, o);
        if (lane >= o) {
          io += yo;
          ic += yc;
        }
      }
      if (e < a.E_local) {
        s_off[e] = run_off + io - pad;
        s_choff[e] = run_ch + ic - nch;
      }
      run_off += __shfl_sync(0xffffffffu, io, 31);
      run_ch += __shfl_sync(0xffffffffu, ic, 31);
    }
    if (lane == 0) {
      s_off[a.E_local] = run_off;
      s_choff[a.E_local] = run_ch;
      a.expert_off[a.E_local] = run_off;
      a.meta[kMetaTotalRows] = run_off;
      a.meta[kMetaNumChunks] = run_ch < a.max_chunks ? run_ch : (int)a.max_chunks;
      if (run_off > a.row_cap || run_ch > a.max_chunks)
        atomicOr(a.meta + kMetaError, kErrRowOverflow);
      a.meta[kMetaTicket] = 0;  // ready for the next launch on this workspace
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E_local; e += blockDim.x) {
    a.expert_cnt[e] = s_tot[e];
    a.expert_off[e] = s_off[e];
    const int n = s_tot[e];
    for (int c = 0, r = 0; r < n; ++c, r += a.bn) {
      if (s_choff[e] + c >= a.max_chunks) break;
      Chunk ch;
      ch.expert = e;
      ch.row0 = s_off[e] + r;
      ch.rows = n - r < a.bn ? n - r : a.bn;
      ch.ncols = (ch.rows + kRowAlign - 1) / kRowAlign * kRowAlign;
      a.chunks[s_choff[e] + c] = ch;
    }
  }
}

}  // namespace fmoe
