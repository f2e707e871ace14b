// gemm_sm100.cu -- persistent grouped FP8 GEMMs of the fused MoE layer on tcgen05.
//
// Replaces the reference's expert GEMMs (solution/cuda/kernel.cu:1006-1199 SIMT, and
// the CUTLASS Sm80 grouped GEMMs at :73-115 / :1221-1417 fed by weight dequantisation
// passes :924-1003). Both GEMMs here read the FP8 weights straight from HBM through
// TMA, multiply on the 5th-generation tensor cores (kind::f8f6f4, E4M3 x E4M3 -> F32
// in TMEM) and apply the 128-block scales in fp32 per K block ("promotion").
//
// Orientation ("swap AB"): the MMA M side is 128 weight rows, the N side is a chunk of
// up to BN routed token rows of one expert (N = rows rounded up to 16). Every weight
// byte is thus read once per chunk, which is what the bandwidth-bound regime needs, and
// a ragged expert wastes at most 15 MMA columns instead of a 128-row M tile.
//
// GEMM1 (+SwiGLU): tile = 64 gate rows [i0, i0+64) and the matching 64 up rows
//   [I+i0, I+i0+64) of W13 (kernel.cu:829-831 pairs G1[:, c] with G1[:, I + c]).
//   Per K block kb (128): D = W13_tile . A_chunk^T in TMEM; epilogue warps add
//   D * w_scale[row block, kb] * a_scale[token, kb] into fp32 registers. The tile
//   epilogue forms C = x1 * silu(x2) and writes it as an FP8 hi/lo pair on one
//   per-(token, 64-column) scale: C ~ scale * (hi + lo), relative error ~2^-8.
// GEMM2: tile = 128 rows h of W2. Per 64-column C block j: D = W2[:, 64j:64j+64] .
//   hi_j^T + W2[...] . lo_j^T (both into the same accumulator: same scale), promoted
//   with w2_scale[h block, j/2] * c_scale[token, j]. Epilogue writes
//   bf16(D * routing_weight) per routed row for the deterministic combine.
//
// Warp roles (320 threads, one CTA per SM, persistent over the tile list):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2..9  epilogue: warp w reads TMEM lane quadrant (w % 4), column half
//               (w - 2) / 4 of the token tile.
// TMEM: 512 columns = two accumulator buffers of up to 256 columns, so the MMA of
// K block kb+1 overlaps the promotion of block kb.
#include <cuda_fp8.h>

#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"
#include "sm100.cuh"

namespace fmoe {

using namespace sm100;

namespace {

constexpr int kThreads = 320;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory per CTA

template <int BN, bool kG1>
struct Cfg {
  static constexpr int kAK = kG1 ? 128 : 64;                 // weight K bytes per step
  static constexpr int kASwz = kG1 ? 128 : 64;
  static constexpr int kABytes = 128 * kAK;
  static constexpr int kBBytes = BN * 128;                   // token K bytes per step = 128
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int HB = BN / 2;                          // columns per epilogue half
  static constexpr int CW = HB < 32 ? HB : 32;               // TMEM load width
  static constexpr int kExBytes = kG1 ? 2 * 64 * 33 * 4 : 0; // SwiGLU exchange (padded)
  static constexpr int kCbufBytes = 2 * 2 * 2 * HB * 4;      // [parity][half][gate/up][col]
  static constexpr int kBarBytes = 512;
  static constexpr int kFixed = 1024 + kExBytes + kCbufBytes + kBarBytes;
  static constexpr int kStagesRaw = (kSmemLimit - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 16 ? 16 : kStagesRaw;
  static constexpr int kSmemBytes = kFixed + kStages * kStageBytes;
  static constexpr uint32_t kTx = kStageBytes;
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void set_error(int* err, volatile int* abort_flag, int code) {
  atomicOr(err, code);
  *abort_flag = 1;
}

template <int BN, bool kG1>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = Cfg<BN, kG1>;
  constexpr int S = C::kStages, HB = C::HB, CW = C::CW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* ex = reinterpret_cast<float*>(smem + S * C::kStageBytes);
  float* cbuf = reinterpret_cast<float*>(smem + S * C::kStageBytes + C::kExBytes);
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes + C::kExBytes + C::kCbufBytes);
  uint64_t* full = bars;            // [S]
  uint64_t* empty = bars + 16;      // [S]
  uint64_t* tfull = bars + 32;      // [2]
  uint64_t* tempty = bars + 34;     // [2]
  uint64_t* mma_done = bars + 36;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 38);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 39);
  static_assert(40 * 8 <= C::kBarBytes, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int num_tiles = args.meta[kMetaNumChunks] * args.m_tiles;
  const int KS = args.k_steps;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();  // weights: streamed once
      const uint64_t pol_a = policy_evict_last();   // token tiles: re-read by every m tile
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const Chunk ch = args.chunks[tile / args.m_tiles];
        const int m = tile % args.m_tiles;
        for (int ks = 0; ks < KS; ++ks, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = stages + s * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          mbar_arrive_expect_tx(&full[s], C::kTx);
          if constexpr (kG1) {
            const int wrow = ch.expert * 2 * args.I + m * 64;
            tma_load_2d(sa, &tmA, &full[s], ks * 128, wrow, pol_w);
            tma_load_2d(sa + 64 * 128, &tmA, &full[s], ks * 128, wrow + args.I, pol_w);
          } else {
            const int wrow = ch.expert * args.H + m * 128;
            tma_load_2d(sa, &tmA, &full[s], ks * 64, wrow, pol_w);
          }
          tma_load_2d(sb, &tmB, &full[s], ks * 128, ch.row0, pol_a);
        }
      }
      if (!ok) set_error(args.err, abort_flag, kErrTimeoutProducer);
      // drain: every issued load must land before the CTA's shared memory is released
      static const int zero = 0;
      for (int j = it > S ? it - S : 0; j < it; ++j)
        mbar_wait(&full[j % S], (j / S) & 1, &zero);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, acc_it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const Chunk ch = args.chunks[tile / args.m_tiles];
        const uint32_t idesc = idesc_e4m3_f32(128, ch.ncols);
        for (int ks = 0; ks < KS; ++ks, ++it, ++acc_it) {
          const int b = acc_it & 1, use = acc_it >> 1;
          if (!mbar_wait(&tempty[b], (use & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(stages + s * C::kStageBytes);
          const uint64_t adesc = smem_desc_kmajor(sa, C::kASwz);
          const uint64_t bdesc = smem_desc_kmajor(sa + C::kABytes, 128);
          const uint32_t d = tmem + b * 256;
          if constexpr (kG1) {
#pragma unroll
            for (int sub = 0; sub < 4; ++sub)
              mma_f8f6f4(d, adesc + 2 * sub, bdesc + 2 * sub, idesc, sub > 0);
          } else {
            // hi half of the C block, then the lo half, same W2 block, same accumulator
            mma_f8f6f4(d, adesc + 0, bdesc + 0, idesc, 0);
            mma_f8f6f4(d, adesc + 2, bdesc + 2, idesc, 1);
            mma_f8f6f4(d, adesc + 0, bdesc + 4, idesc, 1);
            mma_f8f6f4(d, adesc + 2, bdesc + 6, idesc, 1);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[b]);
        }
      }
      if (!ok) set_error(args.err, abort_flag, kErrTimeoutMma);
      // all issued MMAs must retire before TMEM is released
      static const int zero = 0;
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, &zero);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - 2;          // 0..7
    const int q = warp & 3;           // TMEM lane quadrant this warp may access
    const int half = ew >> 2;         // token column half
    const int tid_h = (ew & 3) * 32 + lane;
    const int r = q * 32 + lane;      // accumulator row = weight row inside the tile
    const int bar_id = 1 + half;      // named barrier of the 4 warps of this half
    float acc[HB];
    int acc_it = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      const Chunk ch = args.chunks[tile / args.m_tiles];
      const int m = tile % args.m_tiles;
      const int ncols = ch.ncols;
#pragma unroll
      for (int j = 0; j < HB; ++j) acc[j] = 0.0f;
      // scale rows of the weight tile
      const float* ws_gate;
      const float* ws_up;
      int ws_step;
      if constexpr (kG1) {
        const int nb2 = 2 * args.I / kBlock, kbh = args.H / kBlock;
        ws_gate = args.w_scale + ((int64_t)ch.expert * nb2 + (m * 64) / kBlock) * kbh;
        ws_up = args.w_scale + ((int64_t)ch.expert * nb2 + (args.I + m * 64) / kBlock) * kbh;
        ws_step = 1;
      } else {
        const int nbh = args.H / kBlock, kbi = args.I / kBlock;
        ws_gate = args.w_scale + ((int64_t)ch.expert * nbh + m) * kbi;
        ws_up = ws_gate;
        ws_step = 2;  // one W2 scale column per two 64-column C blocks
      }
      for (int ks = 0; ks < KS; ++ks, ++acc_it) {
        const int par = acc_it & 1;
        float* cb_half = cbuf + (par * 2 + half) * 2 * HB;
        // combined per-column scale for this K block: w_scale(row block) * act_scale(token)
        {
          const float wg = __ldg(ws_gate + ks / ws_step);
          const float wu = __ldg(ws_up + ks / ws_step);
          const float* as = args.act_scale + (int64_t)ks * args.row_cap + ch.row0 + half * HB;
          for (int idx = tid_h; idx < 2 * HB; idx += 128) {
            const int g = idx / HB, col = idx - g * HB;
            const float sa = (half * HB + col < ncols) ? __ldg(as + col) : 0.0f;
            cb_half[idx] = (g == 0 ? wg : wu) * sa;
          }
        }
        const int b = acc_it & 1, use = acc_it >> 1;
        const bool good = mbar_wait(&tfull[b], use & 1, abort_flag);
        if (named_bar_or(bar_id, 128, !good)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* cb = cb_half + ((kG1 && q >= 2) ? HB : 0);
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + b * 256 + half * HB;
#pragma unroll
        for (int c = 0; c < HB / CW; ++c) {
          if (half * HB + c * CW < ncols) {
            uint32_t v[CW];
            tmem_ld_32x32b<CW>(tbase + c * CW, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < CW; ++i)
              acc[c * CW + i] = fmaf(__uint_as_float(v[i]), cb[c * CW + i], acc[c * CW + i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
      if (!ok) break;

      if constexpr (kG1) {
        // ---- SwiGLU + FP8 hi/lo quantisation of C, per 64-column block m ----
        float* exh = ex + half * 64 * 33;  // [64 rows][33] (32 token columns + pad)
#pragma unroll
        for (int sc = 0; sc < HB / CW; ++sc) {
          const int cbase = half * HB + sc * CW;
          if (cbase < ncols) {
            if (q >= 2) {
#pragma unroll
              for (int i = 0; i < CW; ++i) exh[(r - 64) * 33 + i] = silu(acc[sc * CW + i]);
            }
            named_bar(bar_id, 128);
            if (q < 2) {
#pragma unroll
              for (int i = 0; i < CW; ++i) exh[r * 33 + i] *= acc[sc * CW + i];
            }
            named_bar(bar_id, 128);
            if (q < 2) {
              const int i = r >> 1, p = r & 1;  // token column i, C columns [32p, 32p+32)
              float vals[32];
              float amax = 0.0f;
#pragma unroll
              for (int k = 0; k < 32; ++k) {
                vals[k] = exh[(p * 32 + k) * 33 + (i < CW ? i : 0)];
                amax = fmaxf(amax, fabsf(vals[k]));
              }
              amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
              if (i < CW && cbase + i < ncols) {
                const float inv = amax > 0.0f ? 448.0f / amax : 0.0f;
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int k = 0; k < 32; k += 4) {
                  float x[4], h[4], l[4];
#pragma unroll
                  for (int u = 0; u < 4; ++u) x[u] = vals[k + u] * inv;
                  const __nv_fp8x2_storage_t h01 =
                      __nv_cvt_float2_to_fp8x2(make_float2(x[0], x[1]), __NV_SATFINITE, __NV_E4M3);
                  const __nv_fp8x2_storage_t h23 =
                      __nv_cvt_float2_to_fp8x2(make_float2(x[2], x[3]), __NV_SATFINITE, __NV_E4M3);
                  const __half2_raw hr01 = __nv_cvt_fp8x2_to_halfraw2(h01, __NV_E4M3);
                  const __half2_raw hr23 = __nv_cvt_fp8x2_to_halfraw2(h23, __NV_E4M3);
                  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&hr01));
                  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&hr23));
                  h[0] = f01.x; h[1] = f01.y; h[2] = f23.x; h[3] = f23.y;
#pragma unroll
                  for (int u = 0; u < 4; ++u) l[u] = x[u] - h[u];
                  const __nv_fp8x2_storage_t l01 =
                      __nv_cvt_float2_to_fp8x2(make_float2(l[0], l[1]), __NV_SATFINITE, __NV_E4M3);
                  const __nv_fp8x2_storage_t l23 =
                      __nv_cvt_float2_to_fp8x2(make_float2(l[2], l[3]), __NV_SATFINITE, __NV_E4M3);
                  hi[k / 4] = (uint32_t)h01 | ((uint32_t)h23 << 16);
                  lo[k / 4] = (uint32_t)l01 | ((uint32_t)l23 << 16);
                }
                const int64_t row = ch.row0 + cbase + i;
                uint8_t* dst = args.cq + row * (2 * (int64_t)args.I) + m * 128 + p * 32;
                reinterpret_cast<uint4*>(dst)[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                reinterpret_cast<uint4*>(dst)[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                reinterpret_cast<uint4*>(dst + 64)[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                reinterpret_cast<uint4*>(dst + 64)[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                if (p == 0) args.c_scale[(int64_t)m * args.row_cap + row] = amax / 448.0f;
              }
            }
            named_bar(bar_id, 128);
          }
        }
      } else {
        // ---- weighted expert output rows, bf16, for the deterministic combine ----
        const int h = m * 128 + r;
#pragma unroll
        for (int j = 0; j < HB; ++j) {
          const int col = half * HB + j;
          if (col < ch.rows) {
            const int64_t row = ch.row0 + col;
            const float w = __ldg(args.row_w + row);
            args.ow[row * args.H + h] = __float2bfloat16_rn(acc[j] * w);
          }
        }
      }
    }
    if (!ok) set_error(args.err, abort_flag, kErrTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int BN, bool kG1>
cudaError_t launch_one(const CUtensorMap& a, const CUtensorMap& b, const GemmArgs& args,
                       int grid, cudaStream_t stream) {
  using C = Cfg<BN, kG1>;
  auto* fn = grouped_gemm_kernel<BN, kG1>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (configured_device != dev) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  fn<<<grid, kThreads, C::kSmemBytes, stream>>>(a, b, args);
  return cudaGetLastError();
}

}  // namespace

bool gemm_bn_supported(int bn) {
  return bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256;
}

cudaError_t launch_gemm1(int bn, const CUtensorMap& w13_map, const CUtensorMap& a_map,
                         const GemmArgs& args, int grid, cudaStream_t stream) {
  switch (bn) {
    case 16: return launch_one<16, true>(w13_map, a_map, args, grid, stream);
    case 32: return launch_one<32, true>(w13_map, a_map, args, grid, stream);
    case 64: return launch_one<64, true>(w13_map, a_map, args, grid, stream);
    case 128: return launch_one<128, true>(w13_map, a_map, args, grid, stream);
    case 256: return launch_one<256, true>(w13_map, a_map, args, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm2(int bn, const CUtensorMap& w2_map, const CUtensorMap& cq_map,
                         const GemmArgs& args, int grid, cudaStream_t stream) {
  switch (bn) {
    case 16: return launch_one<16, false>(w2_map, cq_map, args, grid, stream);
    case 32: return launch_one<32, false>(w2_map, cq_map, args, grid, stream);
    case 64: return launch_one<64, false>(w2_map, cq_map, args, grid, stream);
    case 128: return launch_one<128, false>(w2_map, cq_map, args, grid, stream);
    case 256: return launch_one<256, false>(w2_map, cq_map, args, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fmoe
