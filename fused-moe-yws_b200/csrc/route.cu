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

__global__ void __launch_bounds__(kWarps * 32) route_plan_kernel(RouteArgs a) {
  __shared__ float s_sc[kWarps][kMaxE];
  __shared__ float s_wb[kWarps][kMaxE];
  __shared__ float s_gscore[kWarps][kMaxGroups];
  __shared__ int s_cnt[64];
  __shared__ int s_is_last;
  __shared__ int s_tot[64];
  __shared__ int s_off[65];
  __shared__ int s_choff[65];
  __shared__ int s_sel[kWarps][32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, G = a.E / a.n_group, K = a.top_k;
  for (int i = threadIdx.x; i < a.E_local; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();

  const int64_t t = (int64_t)blockIdx.x * kWarps + warp;
  if (t < a.T) {
    // 1) sigmoid + bias into shared memory (strided, coalesced loads)
    const float* lrow = a.logits + t * E;
    for (int e = lane; e < E; e += 32) {
      const float sg = exact_sigmoid(__ldg(lrow + e));
      s_sc[warp][e] = sg;
      s_wb[warp][e] = __fadd_rn(sg, bf16_bits_to_float(__ldg(a.bias + e)));
    }
    __syncwarp();
    // 2) group scores: lane g scans its group exactly like the reference loop
    if (lane < a.n_group) {
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
    // 4) top_k experts by warp-wide arg-max rounds; lane owns experts lane, lane+32, ...
    uint32_t taken = 0;  // bit j: expert lane + 32 j already selected
    int* sel = s_sel[warp];
    for (int k = 0; k < K; ++k) {
      float bv = -INFINITY;
      int bi = -1;
      for (int j = 0; lane + 32 * j < E; ++j) {
        const int e = lane + 32 * j;
        if ((taken >> j) & 1u) continue;
        if (!((keep >> (e / G)) & 1u)) continue;
        const float v = s_wb[warp][e];
        if (!(v > -INFINITY)) continue;  // NaN and -inf are never selected
        if (bi < 0 || ranks_above(v, e, bv, bi)) {
          bv = v;
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ranks_above(ov, oi, bv, bi))) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) sel[k] = bi;
      if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    }
    __syncwarp();
    // 5) weights in selection order, local histogram
    if (lane == 0) {
      float sum = 0.0f;
      for (int k = 0; k < K; ++k)
        if (sel[k] >= 0) sum = __fadd_rn(sum, s_sc[warp][sel[k]]);
      sum = __fadd_rn(sum, 1e-20f);
      for (int k = 0; k < K; ++k) {
        const int e = sel[k];
        a.topk_idx[t * K + k] = e;
        a.topk_w[t * K + k] =
            e >= 0 ? __fmul_rn(__fdiv_rn(s_sc[warp][e], sum), a.rsf) : 0.0f;
        const int le = e - a.local_offset;
        if (e >= 0 && le >= 0 && le < a.E_local) atomicAdd(&s_cnt[le], 1);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.E_local; i += blockDim.x)
    a.cta_counts[(int64_t)blockIdx.x * a.E_local + i] = s_cnt[i];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(a.meta + kMetaTicket, 1);
    s_is_last = ticket == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_is_last) return;
  __threadfence();

  // ---- last CTA: expert totals, 16-row aligned offsets, per-CTA bases, chunks ----
  const int nctas = gridDim.x;
  const volatile int* cc = a.cta_counts;
  for (int e = warp; e < a.E_local; e += kWarps) {
    int sum = 0;
    for (int c = lane; c < nctas; c += 32) sum += cc[(int64_t)c * a.E_local + e];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_tot[e] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0, choff = 0;
    for (int e = 0; e < a.E_local; ++e) {
      s_off[e] = off;
      s_choff[e] = choff;
      off += (s_tot[e] + kRowAlign - 1) / kRowAlign * kRowAlign;
      choff += (s_tot[e] + a.bn - 1) / a.bn;
    }
    s_off[a.E_local] = off;
    s_choff[a.E_local] = choff;
    a.expert_off[a.E_local] = off;
    a.meta[kMetaTotalRows] = off;
    a.meta[kMetaNumChunks] = choff < a.max_chunks ? choff : (int)a.max_chunks;
    if (off > a.row_cap || choff > a.max_chunks) atomicOr(a.meta + kMetaError, kErrRowOverflow);
    a.meta[kMetaTicket] = 0;  // ready for the next launch on this workspace
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
      ch.rows = min(a.bn, n - r);
      ch.ncols = (ch.rows + kRowAlign - 1) / kRowAlign * kRowAlign;
      a.chunks[s_choff[e] + c] = ch;
    }
  }
  // per-CTA base row of each expert: expert offset + rows of the earlier CTAs
  for (int e = warp; e < a.E_local; e += kWarps) {
    int run = s_off[e];
    for (int c0 = 0; c0 < nctas; c0 += 32) {
      const int c = c0 + lane;
      const int v = c < nctas ? cc[(int64_t)c * a.E_local + e] : 0;
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
}

}  // namespace fmoe
