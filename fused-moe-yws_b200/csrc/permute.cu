// permute.cu -- stable expert-major scatter with fused FP8 row gather, and the final
// per-token combine.
//
// scatter_gather_kernel restates the reference's reorder + gather
// (solution/cuda/kernel.cu:553-592 and :761-816) with three changes:
//   * rows are ordered by (local expert, token, k) -- a stable counting sort using the
//     per-CTA bases from route_plan_kernel -- so the permutation is deterministic;
//   * the FP8 rows are copied as 16-byte vectors and stay FP8 (the reference
//     dequantises them to fp32/fp16 in HBM); their per-128-column scales are gathered
//     into a [H/128, row_cap] array beside them;
//   * each expert's segment is padded to 16 rows; padding rows are zeroed.
//
// combine_kernel restates final_reduce_cast_grouped_kernel (kernel.cu:864-891): each
// token sums its local routes in top-k order (the routing weight was already applied
// by the GEMM2 epilogue) and casts to bf16. Tokens with no local route get zeros.
#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"

namespace fmoe {

namespace {
constexpr int kTok = kRouteTokensPerCta;
constexpr int kMaxEntries = kTok * 32;
constexpr int kPreVec = 512;          // 16-byte row vectors prefetched per CTA (8 KB)
constexpr int kPreScales = kTok * 64;  // block scales prefetched per CTA (4 KB)

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
}  // namespace

__global__ void __launch_bounds__(256) scatter_gather_kernel(ScatterArgs a) {
  constexpr int kW = 8;  // warps
  __shared__ int s_row[kMaxEntries];                 // destination row of each entry, or -1
  __shared__ int s_list[kMaxEntries];                // entries with a local route, in order
  __shared__ int s_base[kMaxLocalExperts];           // first row of each expert for this CTA
  __shared__ int s_ecnt[kMaxLocalExperts];
  __shared__ int s_eoff[kMaxLocalExperts];
  __shared__ int s_wcnt[kW][kMaxLocalExperts];       // routes per (warp, expert) in a pass
  __shared__ int s_wn[kW];
  __shared__ int s_nlocal;

  __shared__ uint4 s_pre[kPreVec];     // [token][vector] of this CTA's column slice
  __shared__ float s_pscale[kPreScales];  // [token][block]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t lt = (1u << lane) - 1u;
  const int K = a.top_k, nent = kTok * K;
  const int64_t t0 = (int64_t)blockIdx.x * kTok;
  // this CTA copies 16-byte column vectors [v0, v1) of every local row
  const int vpr = a.H / 16;
  const int v0 = (int)((int64_t)vpr * blockIdx.y / gridDim.y);
  const int v1 = (int)((int64_t)vpr * (blockIdx.y + 1) / gridDim.y);
  const int vw = v1 - v0;
  // this CTA also owns the 128-column scale blocks that start inside its columns, so the
  // scattered 4-byte scale stores are spread over every column part
  const int kb0 = (v0 * 16 + kBlock - 1) / kBlock, kb1 = (v1 * 16 + kBlock - 1) / kBlock;
  const int kbw = kb1 - kb0;
  // The source rows and their scales were complete before the routing kernel passed its
  // own dependency wait (this grid starts only after that), so they are fetched before
  // this kernel's wait: the HBM latency of the copy overlaps the routing kernel instead
  // of following it. Only small slices are prefetched (decode-sized batches).
  const bool pre_rows = kTok * vw <= kPreVec;
  const bool pre_scales = kTok * kbw <= kPreScales;
  if (pre_rows) {
    for (int v = tid; v < kTok * vw; v += blockDim.x) {
      const int64_t t = t0 + v / vw;
      if (t < a.T) s_pre[v] = ld_nc_v4(a.hidden + t * a.H + (v0 + v % vw) * 16);
    }
  }
  if (pre_scales && kbw > 0) {
    for (int v = tid; v < kTok * kbw; v += blockDim.x) {
      const int64_t t = t0 + v / kbw;
      if (t < a.T) s_pscale[v] = __ldg(a.hidden_scale + (int64_t)(kb0 + v % kbw) * a.T + t);
    }
  }
  pdl_wait();
  pdl_trigger();
  // every global index load of the CTA is issued in this one phase
  for (int e = tid; e < a.E_local; e += blockDim.x) {
    const int off = a.expert_off[e];
    s_eoff[e] = off;
    s_ecnt[e] = a.expert_cnt[e];
    s_base[e] = off + a.cta_base[(int64_t)blockIdx.x * a.E_local + e];
  }
  if (tid == 0) s_nlocal = 0;
  // stable rank of each entry (token-major, then k) among the CTA's entries of its expert:
  // rank inside the warp from __match_any_sync, plus the earlier warps' counts
  for (int p0 = 0; p0 < nent; p0 += blockDim.x) {
    for (int i = tid; i < kW * a.E_local; i += blockDim.x) s_wcnt[i / a.E_local][i % a.E_local] = 0;
    const int i = p0 + tid;
    int le = -1;
    if (i < nent) {
      const int64_t t = t0 + i / K;
      if (t < a.T) {
        const int ge = a.topk_idx[t * K + i % K];
        const int l = ge - a.local_offset;
        if (ge >= 0 && l >= 0 && l < a.E_local) le = l;
      }
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, le);
    __syncthreads();  // s_wcnt zeroed, s_base loaded
    if (le >= 0 && (peers & lt) == 0u) s_wcnt[warp][le] = __popc(peers);
    __syncthreads();
    int row = -1;
    if (le >= 0) {
      int rank = __popc(peers & lt);
      for (int w = 0; w < warp; ++w) rank += s_wcnt[w][le];
      row = s_base[le] + rank;
      if (row >= a.row_cap) {
        atomicOr(a.meta + kMetaError, kErrRowOverflow);
        row = -1;
      }
    }
    // compact the local entries in entry order
    const uint32_t has = __ballot_sync(0xffffffffu, row >= 0);
    if (lane == 0) s_wn[warp] = __popc(has);
    __syncthreads();
    int pos = s_nlocal + __popc(has & lt);
    for (int w = 0; w < warp; ++w) pos += s_wn[w];
    if (i < nent) s_row[i] = row;
    if (row >= 0) s_list[pos] = i;
    if (blockIdx.y == 0 && i < nent) {
      const int64_t t = t0 + i / K;
      if (t < a.T) a.token_row[t * K + i % K] = row;
      if (row >= 0) {
        a.row_token[row] = (int)t;
        a.row_w[row] = a.topk_w[t * K + i % K];
      }
    }
    __syncthreads();  // all reads of s_nlocal / s_wn / s_wcnt of this pass are done
    if (le >= 0) {
      // later passes continue after this pass's rows of the same expert
      if ((peers & lt) == 0u) atomicAdd(&s_base[le], __popc(peers));
    }
    if (tid == 0) {
      int n = 0;
      for (int w = 0; w < kW; ++w) n += s_wn[w];
      s_nlocal += n;
    }
    __syncthreads();
  }
  const int n = s_nlocal;
  if (pre_rows) {
    for (int v = tid; v < n * vw; v += blockDim.x) {
      const int li = v / vw, pv = v - li * vw;
      const int i = s_list[li];
      *reinterpret_cast<uint4*>(a.a_perm + (int64_t)s_row[i] * a.H + (v0 + pv) * 16) =
          s_pre[(i / K) * vw + pv];
    }
  } else {
    // kUnroll loads in flight per thread before their stores (a store may alias the next
    // load, so the compiler would otherwise wait for each load in turn)
    constexpr int kUnroll = 4;
    for (int vb = tid; vb < n * vw; vb += kUnroll * blockDim.x) {
      uint4 x[kUnroll];
      int64_t dst[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int v = vb + u * blockDim.x;
        dst[u] = -1;
        if (v < n * vw) {
          const int li = v / vw, pv = v - li * vw;
          const int i = s_list[li];
          x[u] = ld_nc_v4(a.hidden + (t0 + i / K) * a.H + (v0 + pv) * 16);
          dst[u] = (int64_t)s_row[i] * a.H + (v0 + pv) * 16;
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (dst[u] >= 0) *reinterpret_cast<uint4*>(a.a_perm + dst[u]) = x[u];
    }
  }
  if (kbw > 0) {
    if (pre_scales) {
      for (int v = tid; v < n * kbw; v += blockDim.x) {
        const int li = v / kbw, bb = v - li * kbw;
        const int i = s_list[li];
        a.a_scale[(int64_t)(kb0 + bb) * a.row_cap + s_row[i]] = s_pscale[(i / K) * kbw + bb];
      }
    } else {
      constexpr int kUnroll = 4;
      for (int vb = tid; vb < n * kbw; vb += kUnroll * blockDim.x) {
        float x[kUnroll];
        int64_t dst[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int v = vb + u * blockDim.x;
          dst[u] = -1;
          if (v < n * kbw) {
            const int li = v / kbw, bb = v - li * kbw;
            const int i = s_list[li];
            x[u] = __ldg(a.hidden_scale + (int64_t)(kb0 + bb) * a.T + t0 + i / K);
            dst[u] = (int64_t)(kb0 + bb) * a.row_cap + s_row[i];
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (dst[u] >= 0) a.a_scale[dst[u]] = x[u];
      }
    }
  }
  // padding rows of the experts this CTA column owns (expert e goes to x = e % gridDim.x)
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int e = blockIdx.x; e < a.E_local; e += gridDim.x) {
    const int cnt = s_ecnt[e];
    const int r0 = s_eoff[e] + cnt;
    const int npad = (cnt + kRowAlign - 1) / kRowAlign * kRowAlign - cnt;
    if (npad == 0) continue;
    for (int v = tid; v < npad * vw; v += blockDim.x) {
      const int r = r0 + v / vw;
      if (r < a.row_cap)
        *reinterpret_cast<uint4*>(a.a_perm + (int64_t)r * a.H + (v0 + v % vw) * 16) = z;
    }
    for (int v = tid; v < npad * kbw; v += blockDim.x) {
      const int r = r0 + v / kbw;
      if (r < a.row_cap) a.a_scale[(int64_t)(kb0 + v % kbw) * a.row_cap + r] = 0.0f;
    }
    if (blockIdx.y == 0) {
      for (int v = tid; v < npad; v += blockDim.x) {
        if (r0 + v < a.row_cap) {
          a.row_token[r0 + v] = -1;
          a.row_w[r0 + v] = 0.0f;
        }
      }
    }
  }
}

template <int kCombineVec>
__global__ void __launch_bounds__(128) combine_kernel(CombineArgs a) {
  __shared__ int s_rows[32];
  const int64_t t = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  // every earlier kernel of the call has finished: pass its error word on to the host
  if (a.err_sink && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    const int e = *reinterpret_cast<const volatile int*>(a.err_word);
    if (e != 0) report_device_error(a.err_sink, e);
  }
  if (a.t_dev && t >= (int64_t)*a.t_dev) return;  // past the tokens actually present
  __nv_bfloat16* dst = a.out + t * a.H;
  if (a.peer_out) {
    // expert-parallel return: straight into the source rank's buffer (peer memory)
    if (t >= a.src_start[a.world]) return;
    int s = 0;
    while (s + 1 < a.world && t >= a.src_start[s + 1]) ++s;
    const int64_t q = t + a.row_shift[s];
    if (q < 0 || q >= a.capacity) {
      if (threadIdx.x == 0 && blockIdx.y == 0) atomicOr(a.xerr, 2);
      return;
    }
    dst = a.peer_out[s] + q * a.H;
  }
  if (threadIdx.x < a.top_k) s_rows[threadIdx.x] = a.token_row[t * a.top_k + threadIdx.x];
  __syncthreads();
  // this CTA covers 8-element vectors [blockIdx.y * 128 * kCombineVec, + 128 * kCombineVec)
  // of the token's row; thread i takes vectors i, i + 128, ..., so each route's row is read
  // with kCombineVec independent loads in flight
  const int nv = a.H / 8;
  const int vb = (int)blockIdx.y * 128 * kCombineVec + (int)threadIdx.x;
  float acc[kCombineVec][8];
#pragma unroll
  for (int u = 0; u < kCombineVec; ++u)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[u][j] = 0.0f;
  for (int k = 0; k < a.top_k; ++k) {
    const int row = s_rows[k];
    if (row < 0) continue;
    uint4 x[kCombineVec];
#pragma unroll
    for (int u = 0; u < kCombineVec; ++u) {
      const int v = vb + u * 128;
      x[u] = v < nv ? ld_nc_v4(a.ow + (int64_t)row * a.H + v * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kCombineVec; ++u) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&x[u]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[u][2 * j] += f.x;
        acc[u][2 * j + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int u = 0; u < kCombineVec; ++u) {
    const int v = vb + u * 128;
    if (v >= nv) continue;
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[u][2 * j], acc[u][2 * j + 1]);
    *reinterpret_cast<uint4*>(dst + v * 8) = o;
  }
  if (a.peer_out) {
    // the rows are read by the peer after a barrier: one system-scope fence per CTA, after
    // the CTA barrier (cumulative over every thread's stores)
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
  }
}

template __global__ void combine_kernel<1>(CombineArgs a);
template __global__ void combine_kernel<2>(CombineArgs a);

}  // namespace fmoe
