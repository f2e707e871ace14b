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
  const bool by_nan = (na && nb) ? ia < ib : nb;
  const bool by_value = va > vb || (va == vb && ia < ib);
  return (na || nb) ? by_nan : by_value;
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

// (key, index) a ranks before (key, index) b: larger key, then smaller index.
__device__ __forceinline__ bool before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

__device__ __forceinline__ void cswap(uint32_t (&k)[8], int (&ix)[8], int i, int j) {
  if (!before(k[i], ix[i], k[j], ix[j])) {
    const uint32_t tk = k[i];
    k[i] = k[j];
    k[j] = tk;
    const int ti = ix[i];
    ix[i] = ix[j];
    ix[j] = ti;
  }
}

// Batcher's odd-even merge sort of 8 (19 comparators), descending by (key, -index).
__device__ __forceinline__ void sort8(uint32_t (&k)[8], int (&ix)[8]) {
  cswap(k, ix, 0, 1); cswap(k, ix, 2, 3); cswap(k, ix, 4, 5); cswap(k, ix, 6, 7);
  cswap(k, ix, 0, 2); cswap(k, ix, 1, 3); cswap(k, ix, 4, 6); cswap(k, ix, 5, 7);
  cswap(k, ix, 1, 2); cswap(k, ix, 5, 6);
  cswap(k, ix, 0, 4); cswap(k, ix, 1, 5); cswap(k, ix, 2, 6); cswap(k, ix, 3, 7);
  cswap(k, ix, 2, 4); cswap(k, ix, 3, 5);
  cswap(k, ix, 1, 2); cswap(k, ix, 3, 4); cswap(k, ix, 5, 6);
}

// Routing of one token when every group holds 32 experts (DeepSeek-V3: 8 groups of 32).
// Lane l owns the 8 consecutive experts g * 32 + (l & 3) * 8 + i of group g = l >> 2, so
// the group's top-2 is an in-lane top-2 merged over its 4 lanes by two shuffles, the kept
// groups are ranked from 8 shuffled scores, and each top_k round takes the best head of
// the lanes' sorted candidate lists (one redux; a second one only on an exact tie). Same
// arithmetic, comparisons and summation order as the general path below, hence the same
// bits; a single warp's dependency chain is the cost, so it is kept short.
__device__ __forceinline__ void route_token_g32(const RouteArgs& a, int64_t t, int lane,
                                                int* s_cnt) {
  const int ng = a.n_group, K = a.top_k;
  const int g = lane >> 2;
  const bool live = g < ng;
  const int e0 = g * 32 + (lane & 3) * 8;
  float sg[8];
  uint32_t key[8];
  if (live) {
    const float4* lp = reinterpret_cast<const float4*>(a.logits + t * a.E + e0);
    const float4 x0 = __ldg(lp), x1 = __ldg(lp + 1);
    const uint4 bv = __ldg(reinterpret_cast<const uint4*>(a.bias + e0));
    const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sg[i] = exact_sigmoid(x[i]);
      const uint16_t bbits = (uint16_t)(bw[i >> 1] >> ((i & 1) * 16));
      const float wb = __fadd_rn(sg[i], bf16_bits_to_float(bbits));
      key[i] = is_candidate(wb) ? order_key(wb) : 0u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sg[i] = 0.0f;
      key[i] = 0u;
    }
  }
  // group score = sum of the two largest candidates (duplicates count twice): in-lane
  // top-2, then merged across the group's 4 lanes
  uint32_t m1 = 0u, m2 = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m2 = max(m2, min(m1, key[i]));
    m1 = max(m1, key[i]);
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    const uint32_t p1 = __shfl_xor_sync(0xffffffffu, m1, o);
    const uint32_t p2 = __shfl_xor_sync(0xffffffffu, m2, o);
    m2 = max(min(m1, p1), max(m2, p2));
    m1 = max(m1, p1);
  }
  const float gs =
      __fadd_rn(m1 ? key_value(m1) : -INFINITY, m2 ? key_value(m2) : -INFINITY);
  // kept groups: each lane counts the groups ranking above its own group
  int rank = 0;
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    const float gh = __shfl_sync(0xffffffffu, gs, 4 * h);
    if (h < ng && h != g) rank += ranks_above(gh, h, gs, g);
  }
  const bool keep = live && rank < a.topk_group;
  // this lane's candidates, sorted (ties: lower expert id first)
  int ix[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ix[i] = i;
    if (!keep) key[i] = 0u;
  }
  sort8(key, ix);
  int my_e = -1;
  float my_s = 0.0f, sum = 0.0f;
  int head = 0;  // next unselected entry of the sorted list
  for (int k = 0; k < K; ++k) {
    uint32_t hk = 0u;
    int hi = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j == head) {
        hk = key[j];
        hi = ix[j];
      }
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, hk);
    if (kmax == 0u) break;  // fewer than top_k candidates: the rest stay -1 / 0
    const unsigned tie = __ballot_sync(0xffffffffu, hk == kmax);
    int win;
    if ((tie & (tie - 1u)) == 0u) {
      win = __shfl_sync(0xffffffffu, e0 + hi, __ffs(tie) - 1);
    } else {
      win = (int)__reduce_min_sync(0xffffffffu,
                                   hk == kmax ? (uint32_t)(e0 + hi) : 0xffffffffu);
    }
    const int wl = win >> 3;  // the lane holding expert `win`
    float v = sg[0];
#pragma unroll
    for (int j = 1; j < 8; ++j)
      if (j == hi) v = sg[j];
    v = __shfl_sync(0xffffffffu, v, wl);
    sum = __fadd_rn(sum, v);  // selection order, as the reference sums
    if (lane == wl) ++head;
    if (lane == k) {
      my_e = win;
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
  if (a.inject_err != 0 && blockIdx.x == 0 && threadIdx.x == 0)
    atomicOr(a.meta + kMetaError, a.inject_err);
  __syncthreads();

  const int64_t t = (int64_t)blockIdx.x * kWarps + warp;
  if (t < a.T && a.in_idx) {
    // routed mode: (expert, weight) pairs computed elsewhere (expert-parallel dispatch);
    // with a device-side token count, the slots past it are marked unselected
    const int64_t tn = a.t_dev ? (int64_t)*a.t_dev : a.T;
    if (lane < K) {
      const int e = t < tn ? a.in_idx[t * K + lane] : -1;
      a.topk_idx[t * K + lane] = e;
      a.topk_w[t * K + lane] = t < tn ? a.in_w[t * K + lane] : 0.0f;
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
  if (nctas == 1) {
    for (int e = threadIdx.x; e < a.E_local; e += blockDim.x) {
      a.cta_base[e] = 0;
      s_tot[e] = s_cnt[e];
    }
  } else {
    // Warp w owns CTAs [c0, c1) and lane l experts l, l + 32, ...: each count is read with
    // coalesced loads issued kBatch at a time, so the pass costs a few L2 round trips
    // rather than one per 32 CTAs. Pass 1 sums each warp's range, a scan over the warps
    // gives each range its start, pass 2 writes the bases.
    constexpr int kBatch = 16;
    int* s_part = reinterpret_cast<int*>(&s_sc[0][0]);  // [kWarps][E_local], scores are done
    const int c0 = (int)((int64_t)nctas * warp / kWarps);
    const int c1 = (int)((int64_t)nctas * (warp + 1) / kWarps);
    for (int e = lane; e < a.E_local; e += 32) {
      int sum = 0;
      for (int cb = c0; cb < c1; cb += kBatch) {
        int v[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
          v[q] = cb + q < c1 ? __ldcg(a.cta_counts + (int64_t)(cb + q) * a.E_local + e) : 0;
#pragma unroll
        for (int q = 0; q < kBatch; ++q) sum += v[q];
      }
      s_part[warp * a.E_local + e] = sum;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < a.E_local; e += blockDim.x) {
      int run = 0;
      for (int w = 0; w < kWarps; ++w) {
        const int v = s_part[w * a.E_local + e];
        s_part[w * a.E_local + e] = run;
        run += v;
      }
      s_tot[e] = run;
    }
    __syncthreads();
    for (int e = lane; e < a.E_local; e += 32) {
      int run = s_part[warp * a.E_local + e];
      for (int cb = c0; cb < c1; cb += kBatch) {
        int v[kBatch];
#pragma unroll
        for (int q = 0; q < kBatch; ++q)
          v[q] = cb + q < c1 ? __ldcg(a.cta_counts + (int64_t)(cb + q) * a.E_local + e) : 0;
#pragma unroll
        for (int q = 0; q < kBatch; ++q) {
          if (cb + q < c1) a.cta_base[(int64_t)(cb + q) * a.E_local + e] = run;
          run += v[q];
        }
      }
    }
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
