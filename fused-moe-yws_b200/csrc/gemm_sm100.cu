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
// GEMM1 (+SwiGLU): tile = 128 gate rows [i0, i0+128) and the matching 128 up rows
//   [I+i0, I+i0+128) of W13 (kernel.cu:829-831 pairs G1[:, c] with G1[:, I + c]).
//   Per K block kb (128): D = W13_tile . A_chunk^T in TMEM; epilogue warps add
//   D * w_scale[row block, kb] * a_scale[token, kb] into fp32 registers. The tile
//   epilogue forms C = x1 * silu(x2) and writes it as an FP8 hi/lo pair on one
//   per-(token, 128-column) scale: C ~ scale * (hi + lo), relative error ~2^-8.
// GEMM2: tile = 256 rows h of W2 (two 128-row accumulators). Per 128-column C block j, one
//   MMA of N = 2 BN per accumulator over the stacked [hi_j; lo_j] token tiles gives
//   W2[rows, 128j:128j+128] . hi_j^T and . lo_j^T side by side; their sum is promoted with
//   w2_scale[h block, j] * c_scale[token, j]. The epilogue writes bf16(D * routing_weight)
//   per routed row for the deterministic combine.
// Each K step is three copies: one 32 KB weight box (GEMM1: gate and up tiles through a 3D
// tensor map; GEMM2: a 256-row box), one token box (GEMM2: hi and lo through a 3D map) and
// one bulk copy of the token scales -- the producer thread's issue cost is per copy.
//
// Warp roles (320 threads, one CTA per SM, persistent over the tile list):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2..9  epilogue: warp w reads TMEM lane quadrant (w % 4), column half
//               (w - 2) / 4 of the token tile; thread row r holds both accumulators'
//               row r (GEMM1: gate and up of C column r; GEMM2: output rows r, 128 + r).
// TMEM: 512 columns = two accumulator buffers of up to 256 columns, so the MMA of
// K block kb+1 overlaps the promotion of block kb.
#include <cuda_fp8.h>

#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"
#include "gemm_sched.cuh"
#include "sm100.cuh"

namespace fmoe {

using namespace sm100;

namespace {

constexpr int kThreads = 320;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory per CTA
constexpr int kEpiThreads = 256;    // warps 2..9
constexpr int kBarAll = 3;          // named barrier id over all epilogue warps

template <int BN, bool kG1>
struct Cfg {
  static constexpr int kAcc = 2;                              // accumulators per K step
  static constexpr int kABytes = 2 * 128 * 128;               // gate + up, or 256 W2 rows
  static constexpr int kBBytes = (kG1 ? 1 : 2) * BN * 128;   // tokens (G2: hi and lo)
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int HB = BN / 2;                           // token columns per half
  // TMEM load width: two accumulators are live, so loads go in narrow chunks
  static constexpr int kCWMax = 16;
  static constexpr int CW = HB < kCWMax ? HB : kCWMax;
  // TMEM columns per accumulator. GEMM2 runs one MMA of N = 2 BN over the stacked hi and
  // lo token rows, so an accumulator holds W.hi in columns [0, BN) and W.lo in [BN, 2 BN)
  static constexpr int kAccCols = kG1 ? (BN < 32 ? 32 : BN) : 2 * BN;
  static constexpr int kBufCols = 2 * kAccCols;
  static constexpr int kNBufRaw = 512 / kBufCols;
  static constexpr int kNBuf = kNBufRaw > 8 ? 8 : kNBufRaw;   // accumulator ring depth
  static constexpr int kExBytes = kG1 ? 2 * 128 * (HB + 1) * 4 : 0;  // SwiGLU staging
  static_assert(!kG1 || HB * 4 <= 128, "SwiGLU quantisation maps 4 threads per token column");
  static constexpr int kWscBytes = 2 * 2 * kMaxKSteps * 4;    // [slot][gate/up][k step]
  static constexpr int kSlotBytes = BN * 4;                   // act scales of one K step
  static constexpr int kMaxSlots = 16 + 8 + 2;
  static constexpr int kBarBytes = 1024;
  static constexpr int kFixedMax =
      1024 + kExBytes + kWscBytes + kMaxSlots * kSlotBytes + kBarBytes + 64;
  static constexpr int kStagesRaw = (kSmemLimit - kFixedMax) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 16 ? 16 : kStagesRaw;
  static constexpr int kSlots = kStages + kNBuf + 2;          // scale ring depth
  static constexpr int kFixed =
      1024 + kExBytes + kWscBytes + kSlots * kSlotBytes + kBarBytes + 64;
  static constexpr int kSmemBytes = kFixed + kStages * kStageBytes;
  static constexpr uint32_t kTx = kStageBytes;
  static constexpr int kPartialFloats = kAcc * 128 * BN;      // one split-K partial tile
  static_assert(kStages >= 2, "not enough shared memory for a 2-stage pipeline");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert((16 + 16 + 8 + 8 + 4 + 2 * kMaxSlots + 3) * 8 <= kBarBytes, "barrier area");
  static_assert(kNBuf >= 2, "need at least two accumulator buffers");
};

// fast division: the reference is built with --use_fast_math, which approximates it too
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ void set_error(int* err, volatile int* abort_flag, int code) {
  atomicOr(err, code);
  *abort_flag = 1;
}

// Promote one accumulator: acc[j] += D[row, col_j] * scale_j * sw for this thread's
// half of the token columns (only column chunks below ncols are read).
template <int HB, int CW>
__device__ __forceinline__ void promote(float (&acc)[HB], uint32_t taddr, const float* sa,
                                        float sw, int col0, int ncols) {
#pragma unroll
  for (int c = 0; c < HB / CW; ++c) {
    if (col0 + c * CW < ncols) {
      uint32_t v[CW];
      tmem_ld_32x32b<CW>(taddr + c * CW, v);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < CW; ++i)
        acc[c * CW + i] = fmaf(__uint_as_float(v[i]), sa[c * CW + i] * sw, acc[c * CW + i]);
    }
  }
}

// GEMM2: acc[j] += (D_hi[row, col_j] + D_lo[row, col_j]) * scale_j * sw, the lo columns
// `lo_off` TMEM columns after the hi columns.
template <int HB, int CW>
__device__ __forceinline__ void promote_hilo(float (&acc)[HB], uint32_t taddr, int lo_off,
                                             const float* sa, float sw, int col0, int ncols) {
#pragma unroll
  for (int c = 0; c < HB / CW; ++c) {
    if (col0 + c * CW < ncols) {
      uint32_t h[CW], l[CW];
      tmem_ld_32x32b<CW>(taddr + c * CW, h);
      tmem_ld_32x32b<CW>(taddr + lo_off + c * CW, l);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < CW; ++i)
        acc[c * CW + i] = fmaf(__uint_as_float(h[i]) + __uint_as_float(l[i]),
                               sa[c * CW + i] * sw, acc[c * CW + i]);
    }
  }
}

// Store HB floats (16-byte aligned) as float4 vectors.
template <int HB>
__device__ __forceinline__ void store_row(float* dst, const float (&v)[HB]) {
  if constexpr (HB % 4 == 0) {
#pragma unroll
    for (int j = 0; j < HB; j += 4)
      *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < HB; ++j) dst[j] = v[j];
  }
}

// Load HB floats (16-byte aligned) written by another CTA: L2-coherent loads.
template <int HB>
__device__ __forceinline__ void load_row(float (&v)[HB], const float* src) {
  if constexpr (HB % 4 == 0) {
#pragma unroll
    for (int j = 0; j < HB; j += 4) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(src + j));
      v[j] = x.x;
      v[j + 1] = x.y;
      v[j + 2] = x.z;
      v[j + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < HB; ++j) v[j] = __ldcg(src + j);
  }
}

// acc = sum of the tile's contributions in K order (contributor CTAs cf..cl, each of
// which -- this one included -- has stored its partial before the arrival counter).
// A contributor's partial lives in slot 0 (its range starts inside the tile) or slot 1
// (the tile ends its range); CTAs with an empty range contribute nothing. A batch of
// contributors is loaded before the adds. The order is fixed, so the result does not
// depend on which CTA finishes the tile. Partials come from other CTAs: L2-coherent loads.
template <int HB, int kRegs>
__device__ __forceinline__ void sum_contributions(float (&acc)[HB], const float* partials,
                                                  int64_t elem_off, int stride,
                                                  const StreamK& sk, int64_t tile_begin, int cf,
                                                  int cl) {
  float out[HB];
#pragma unroll
  for (int j = 0; j < HB; ++j) out[j] = 0.0f;
  constexpr int kBatch = kRegs / HB > 0 ? kRegs / HB : 1;  // contributors in flight
  for (int c0 = cf; c0 <= cl; c0 += kBatch) {
    float buf[kBatch][HB];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int c = c0 + u;
      if (c <= cl && sk.start(c) != sk.start(c + 1)) {
        const int slot = sk.start(c) >= tile_begin ? 0 : 1;
        const float* p = partials + (int64_t)(2 * c + slot) * stride + elem_off;
#pragma unroll
        for (int j = 0; j < HB; j += 4) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(p + j));
          buf[u][j] = x.x;
          buf[u][j + 1] = x.y;
          buf[u][j + 2] = x.z;
          buf[u][j + 3] = x.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int c = c0 + u;
      if (c <= cl && sk.start(c) != sk.start(c + 1)) {
#pragma unroll
        for (int j = 0; j < HB; ++j) out[j] += buf[u][j];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < HB; ++j) acc[j] = out[j];
}

template <int BN, bool kG1>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = Cfg<BN, kG1>;
  constexpr int S = C::kStages, HB = C::HB, CW = C::CW, NB = C::kNBuf, SR = C::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* fixed = smem + S * C::kStageBytes;
  float* ex = reinterpret_cast<float*>(fixed);
  float* wsc = reinterpret_cast<float*>(fixed + C::kExBytes);
  float* sring = reinterpret_cast<float*>(fixed + C::kExBytes + C::kWscBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(fixed + C::kExBytes + C::kWscBytes +
                                               SR * C::kSlotBytes);
  uint64_t* full = bars;                 // [S]   TMA -> MMA
  uint64_t* empty = bars + 16;           // [S]   MMA -> TMA
  uint64_t* tfull = bars + 32;           // [NB]  MMA -> epilogue
  uint64_t* tempty = bars + 40;          // [NB]  epilogue -> MMA
  uint64_t* wfull = bars + 48;           // [2]   weight-scale rows, producer -> epilogue
  uint64_t* wempty = bars + 50;          // [2]   epilogue -> producer
  uint64_t* sfull = bars + 52;           // [SR]  scale ring, TMA -> epilogue
  uint64_t* sempty = sfull + C::kMaxSlots;  // [SR] epilogue -> TMA
  uint64_t* mma_done = sempty + C::kMaxSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mma_done + 2);
  volatile int* last_flag = reinterpret_cast<volatile int*>(mma_done + 2) + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    for (int r = 0; r < SR; ++r) {
      mbar_init(&sfull[r], 1);
      mbar_init(&sempty[r], 8);
    }
    for (int r = 0; r < 2; ++r) {
      mbar_init(&wfull[r], 32);
      mbar_init(&wempty[r], 8);
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
  // The producer warp waits for the previous kernel only once its first weight boxes are
  // in flight (below); every other warp waits here, before touching its outputs.
  if (warp != 0) pdl_wait();  // the permute / GEMM1 outputs of the previous kernel are visible
  pdl_trigger();  // let the next kernel's CTAs start their prologue as SMs free up

  const int num_tiles = args.meta[kMetaNumChunks] * args.m_tiles;
  const int KS = args.k_steps;
  const int cta = (int)blockIdx.x;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // The whole warp stages each tile's weight block scales (one W2 row, or the gate and
    // up rows of W13) into a 2-slot shared ring; lane 0 alone issues the copies.
    const uint64_t pol_w = policy_evict_first();  // weights: streamed once
    const uint64_t pol_a = policy_evict_last();   // token tiles: re-read by every m tile
    // The chunk list and the weights do not depend on the previous kernel: the routing plan
    // was complete before it could start this grid (it triggers only after its own
    // dependency wait). So the weight boxes of the first min(S, steps) stages are issued
    // before griddepcontrol.wait, overlapping the pipeline's first HBM latency with the
    // previous kernel's tail; the token tiles and their scales follow after the wait.
    int it = 0, wseg = 0, pre = 0;
    bool ok = true, waited = false;
    Schedule sched(num_tiles, KS, (int)gridDim.x, cta);
    int tile, k0, k1;
    while (ok && sched.next(tile, k0, k1)) {
      const Chunk ch = args.chunks[tile / args.m_tiles];
      const int m = tile % args.m_tiles;
      {
        const int ws = wseg & 1;
        bool w_ok = true;
        if (lane == 0) w_ok = mbar_wait(&wempty[ws], ((wseg >> 1) & 1) ^ 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
          ok = false;
          break;
        }
        const int kbh = (kG1 ? args.H : args.I) / kBlock;
        const float* g;
        const float* u;
        if constexpr (kG1) {
          const int nb2 = 2 * args.I / kBlock;
          g = args.w_scale + ((int64_t)ch.expert * nb2 + m) * kbh;
          u = args.w_scale + ((int64_t)ch.expert * nb2 + args.I / kBlock + m) * kbh;
        } else {
          // h blocks 2 m and 2 m + 1; the second is past the expert when H / 128 is odd
          g = args.w_scale + ((int64_t)ch.expert * (args.H / kBlock) + 2 * m) * kbh;
          u = 2 * m + 1 < args.H / kBlock ? g + kbh : nullptr;
        }
        float* dst = wsc + ws * 2 * kMaxKSteps;
        for (int i = lane; i < kbh; i += 32) {
          dst[i] = __ldg(g + i);
          dst[kMaxKSteps + i] = u ? __ldg(u + i) : 0.0f;
        }
        mbar_arrive(&wfull[ws]);  // every lane: its stores are released by its own arrive
        ++wseg;
      }
      // weight box of K step ks into stage s (the stage's full barrier expects the token
      // tile too)
      auto load_weights = [&](int s, int ks) {
        uint8_t* sa = stages + s * C::kStageBytes;
        mbar_arrive_expect_tx(&full[s], C::kTx);
        if (args.w_pre) {
          // the same 32 KB image, stored contiguously ahead of time: one bulk copy
          const int64_t t = ((int64_t)ch.expert * args.m_tiles + m) * KS + ks;
          bulk_load_1d_hint(sa, args.w_pre + t * kPrelaidTileBytes, kPrelaidTileBytes, &full[s],
                            pol_w);
        } else if constexpr (kG1) {
          // {K, row in half, (expert, gate|up)} box {128, 128, 2}: gate tile, then up tile
          tma_load_3d(sa, &tmA, &full[s], ks * 128, m * 128, 2 * ch.expert, pol_w);
        } else {
          // 256 W2 rows
          tma_load_2d(sa, &tmA, &full[s], ks * 128, ch.expert * args.H + m * 256, pol_w);
        }
      };
      if (!waited) {
        if (lane == 0) {
          pre = k1 - k0 < S ? k1 - k0 : S;  // stages are fresh: no empty wait needed
          for (int i = 0; i < pre; ++i) load_weights(i, k0 + i);
        }
        pdl_wait();
        waited = true;
      }
      if (lane == 0) {
        const float* asrc = args.act_scale + ch.row0;
        for (int ks = k0; ks < k1; ++ks, ++it) {
          const int s = it % S, slot = it % SR;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, abort_flag) ||
              !mbar_wait(&sempty[slot], ((it / SR) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sb = stages + s * C::kStageBytes + C::kABytes;
          if (it >= pre) load_weights(s, ks);
          if constexpr (kG1) {
            tma_load_2d(sb, &tmB, &full[s], ks * 128, ch.row0, pol_a);
          } else {
            // {byte in block, row, 128-byte block} box {128, BN, 2}: hi, then lo
            tma_load_3d(sb, &tmB, &full[s], 0, ch.row0, 2 * ks, pol_a);
          }
          // activation / intermediate scales of this K step for the chunk's columns
          mbar_arrive_expect_tx(&sfull[slot], ch.ncols * 4);
          bulk_load_1d(sring + slot * BN, asrc + (int64_t)ks * args.row_cap, ch.ncols * 4,
                       &sfull[slot]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (!waited) pdl_wait();  // no work: still ordered after the previous kernel
    if (lane == 0) {
      if (!ok) set_error(args.err, abort_flag, kErrTimeoutProducer);
      // drain: every issued copy must land before the CTA's shared memory is released
      static const int zero = 0;
      for (int j = it > S ? it - S : 0; j < it; ++j)
        mbar_wait(&full[j % S], (j / S) & 1, &zero);
      for (int j = it > SR ? it - SR : 0; j < it; ++j)
        mbar_wait(&sfull[j % SR], (j / SR) & 1, &zero);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      Schedule sched(num_tiles, KS, (int)gridDim.x, cta);
      int tile, k0, k1;
      while (ok && sched.next(tile, k0, k1)) {
        const Chunk ch = args.chunks[tile / args.m_tiles];
        const uint32_t idesc = idesc_e4m3_f32(128, kG1 ? ch.ncols : 2 * BN);
        for (int ks = k0; ks < k1; ++ks, ++it) {
          const int b = it % NB, use = it / NB;
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
          const uint32_t d = tmem + b * C::kBufCols;
          // accumulator 0: weight rows 0..127 of the stage, 1: rows 128..255. For GEMM2 the
          // hi and lo token tiles are adjacent in shared memory, so one MMA of N = 2 BN
          // multiplies a weight tile with both (an MMA costs about the same up to N = 64)
          const uint64_t a0 = smem_desc_kmajor(sa, 128);
          const uint64_t a1 = smem_desc_kmajor(sa + 128 * 128, 128);
          const uint64_t bd = smem_desc_kmajor(sa + C::kABytes, 128);
#pragma unroll
          for (int sub = 0; sub < 4; ++sub) {
            mma_f8f6f4(d, a0 + 2 * sub, bd + 2 * sub, idesc, sub > 0);
            mma_f8f6f4(d + C::kAccCols, a1 + 2 * sub, bd + 2 * sub, idesc, sub > 0);
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
    const int tid_e = ew * 32 + lane;  // 0..255
    const int r = q * 32 + lane;      // accumulator row = weight row inside the tile
    const int bar_half = 1 + half;    // named barrier of the 4 warps of this half
    float acc_g[HB];  // accumulator 0 (GEMM1 gate, GEMM2 rows 0..127 of the tile)
    float acc_u[HB];  // accumulator 1 (GEMM1 up, GEMM2 rows 128..255)
    int it = 0, wseg = 0;
    bool ok = true;
    Schedule sched(num_tiles, KS, (int)gridDim.x, cta);
    int tile, k0, k1;
    while (sched.next(tile, k0, k1)) {
      const Chunk ch = args.chunks[tile / args.m_tiles];
      const int m = tile % args.m_tiles;
      const int ncols = ch.ncols;
      // weight block scales of this tile, staged by the producer warp
      const int ws = wseg & 1;
      if (ok && !mbar_wait(&wfull[ws], (wseg >> 1) & 1, abort_flag)) ok = false;
      const float* wrow = wsc + ws * 2 * kMaxKSteps;
#pragma unroll
      for (int j = 0; j < HB; ++j) {
        acc_g[j] = 0.0f;
        acc_u[j] = 0.0f;
      }
      const SplitRole role = split_role(sched, tile, k0, k1);
      if (role.split && role.pair && role.head) {
        // the tile's tail was this CTA's successor's first split segment: wait for its
        // partial and start the accumulators from it (overlaps the first K steps' MMAs)
        bool ready = true;
        if (tid_e == 0 && ok) ready = wait_nonzero(args.tile_counters + role.cf, abort_flag);
        if (named_bar_or(kBarAll, kEpiThreads, !ready || !ok)) {
          if (ok) set_error(args.err, abort_flag, kErrTimeoutEpilogue);
          ok = false;
        } else {
          const float* pp = args.partials + (int64_t)(2 * role.cl) * C::kPartialFloats;
          load_row<HB>(acc_g, pp + (0 * 128 + r) * BN + half * HB);
          load_row<HB>(acc_u, pp + (1 * 128 + r) * BN + half * HB);
        }
      }
      for (int ks = k0; ks < k1; ++ks, ++it) {
        const int b = it % NB, use = it / NB;
        const int slot = it % SR, suse = it / SR;
        if (!ok) continue;
        if (!mbar_wait(&sfull[slot], suse & 1, abort_flag) ||
            !mbar_wait(&tfull[b], use & 1, abort_flag)) {
          ok = false;
          continue;
        }
        tc_fence_after();
        const float* sa = sring + slot * BN + half * HB;
        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + b * C::kBufCols + half * HB;
        if constexpr (kG1) {
          promote<HB, CW>(acc_g, tb, sa, wrow[ks], half * HB, ncols);
          promote<HB, CW>(acc_u, tb + C::kAccCols, sa, wrow[kMaxKSteps + ks], half * HB, ncols);
        } else {
          promote_hilo<HB, CW>(acc_g, tb, BN, sa, wrow[ks], half * HB, ncols);
          promote_hilo<HB, CW>(acc_u, tb + C::kAccCols, BN, sa, wrow[kMaxKSteps + ks], half * HB,
                               ncols);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[b]);
          mbar_arrive(&sempty[slot]);
        }
      }
      // the weight-scale slot is free again once this warp's promotions are done
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&wempty[ws]);
      ++wseg;
      // one abort decision for all epilogue warps (nobody waits at a barrier alone)
      if (named_bar_or(kBarAll, kEpiThreads, !ok)) {
        ok = false;
        break;
      }

      // ---- stream-K: a partial segment publishes its fp32 partial; the contributor that
      //      completes the tile's K range sums all contributions in K order and finishes ----
      if (role.split && role.pair) {
        float* part = args.partials + (int64_t)(2 * cta + role.slot) * C::kPartialFloats;
        if (!role.head) {
          // tail owner: publish the partial and move on (the head owner finishes the tile)
          store_row<HB>(part + (0 * 128 + r) * BN + half * HB, acc_g);
          store_row<HB>(part + (1 * 128 + r) * BN + half * HB, acc_u);
          named_bar(kBarAll, kEpiThreads);
          if (tid_e == 0) red_release_add(args.tile_counters + role.cf, k1 - k0);
          continue;
        }
        if (tid_e == 0) args.tile_counters[role.cf] = 0;  // ready for the next launch
      } else if (role.split) {
        // position of the tile in the stream-K step space
        const StreamK& sk = sched.sk;
        const int64_t tile_begin = role.tb;
        const int slot = role.slot;
        float* part = args.partials + (int64_t)(2 * cta + slot) * C::kPartialFloats;
        store_row<HB>(part + (0 * 128 + r) * BN + half * HB, acc_g);
        store_row<HB>(part + (1 * 128 + r) * BN + half * HB, acc_u);
        __threadfence();
        named_bar(kBarAll, kEpiThreads);
        const int cf = sk.cta_of(tile_begin), cl = sk.cta_of(tile_begin + KS - 1);
        if (tid_e == 0) {
          const int done = atomicAdd(args.tile_counters + cf, k1 - k0) + (k1 - k0);
          const bool last = done == KS;
          if (last) args.tile_counters[cf] = 0;  // ready for the next launch
          *last_flag = last;
        }
        named_bar(kBarAll, kEpiThreads);
        if (!*last_flag) continue;
        __threadfence();
        constexpr int kRegs = 32;
        sum_contributions<HB, kRegs>(acc_g, args.partials, (0 * 128 + r) * BN + half * HB,
                                     C::kPartialFloats, sk, tile_begin, cf, cl);
        sum_contributions<HB, kRegs>(acc_u, args.partials, (1 * 128 + r) * BN + half * HB,
                                     C::kPartialFloats, sk, tile_begin, cf, cl);
      }

      if constexpr (kG1) {
        // ---- SwiGLU + FP8 hi/lo quantisation of C, per 128-column block m ----
        // thread row r holds gate (x1) and up (x2) of C column 128 m + r for this half's
        // token columns; C goes to shared memory first so the accumulators die here
        float* exh = ex + half * 128 * (HB + 1);  // [128 rows][HB + 1]
#pragma unroll
        for (int i = 0; i < HB; ++i) exh[r * (HB + 1) + i] = acc_g[i] * silu(acc_u[i]);
        named_bar(bar_half, 128);
        // 4 threads per token column, 32 C columns each
        const int i = tid_h >> 2, p = tid_h & 3;
        const bool active = i < HB;
        float vals[32];
        float amax = 0.0f;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          vals[k] = exh[(p * 32 + k) * (HB + 1) + (active ? i : 0)];
          amax = fmaxf(amax, fabsf(vals[k]));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        if (active && half * HB + i < ncols) {
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
          const int64_t row = ch.row0 + half * HB + i;
          uint8_t* dst = args.cq + row * (2 * (int64_t)args.I) + m * 256 + p * 32;
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
          reinterpret_cast<uint4*>(dst + 128)[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          reinterpret_cast<uint4*>(dst + 128)[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
          if (p == 0) args.c_scale[(int64_t)m * args.row_cap + row] = amax / 448.0f;
        }
        named_bar(bar_half, 128);  // exh is reused by the next tile
      } else {
        // ---- weighted expert output rows, bf16, for the deterministic combine ----
        const int h = m * 256 + r;
        const bool second = h + 128 < args.H;  // rows 128..255 exist unless H / 128 is odd
#pragma unroll
        for (int j = 0; j < HB; ++j) {
          const int col = half * HB + j;
          if (col < ch.rows) {
            const int64_t row = ch.row0 + col;
            const float w = __ldg(args.row_w + row);
            args.ow[row * args.H + h] = __float2bfloat16_rn(acc_g[j] * w);
            if (second) args.ow[row * args.H + h + 128] = __float2bfloat16_rn(acc_u[j] * w);
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
  return launch_pdl(fn, dim3(grid), dim3(kThreads), C::kSmemBytes, stream, a, b, args);
}

// Weight pre-layout: every (expert, m tile, K step) weight tile the GEMMs load -- GEMM1:
// gate rows [128 m, 128 m + 128) then up rows [I + 128 m, ...) of W13; GEMM2: rows
// [256 m, 256 m + 256) of W2; 128 K bytes each -- written as the 32 KB shared-memory image a
// SWIZZLE_128B tensor-map load produces (16-byte chunk c of row r at chunk c ^ (r % 8)),
// tiles ordered [expert][m tile][K step]. One CTA per tile, one 16-byte chunk per thread
// step; reads and writes are coalesced per 128-byte row.
__global__ void __launch_bounds__(256) prelayout_kernel(const uint8_t* __restrict__ w,
                                                        uint8_t* __restrict__ out, int rows,
                                                        int cols, int m_tiles, int k_steps,
                                                        int gemm1, int I) {
  const int64_t tile = blockIdx.x;
  const int ks = (int)(tile % k_steps);
  const int m = (int)((tile / k_steps) % m_tiles);
  const int64_t e = tile / ((int64_t)k_steps * m_tiles);
  const uint8_t* src = w + e * (int64_t)rows * cols;
  uint8_t* dst = out + tile * kPrelaidTileBytes;
  for (int i = threadIdx.x; i < 256 * 8; i += blockDim.x) {
    const int r = i >> 3, c = i & 7;
    const int srow = gemm1 ? (r < 128 ? 128 * m + r : I + 128 * m + (r - 128)) : 256 * m + r;
    const uint4 v =
        *reinterpret_cast<const uint4*>(src + (int64_t)srow * cols + ks * 128 + c * 16);
    *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) * 16)) = v;
  }
}

}  // namespace

cudaError_t launch_prelayout(const uint8_t* w13, const uint8_t* w2, uint8_t* w13_out,
                             uint8_t* w2_out, int E_local, int H, int I, cudaStream_t stream) {
  const int64_t t1 = (int64_t)E_local * (I / 128) * (H / 128);
  const int64_t t2 = (int64_t)E_local * (H / 256) * (I / 128);
  prelayout_kernel<<<(unsigned)t1, 256, 0, stream>>>(w13, w13_out, 2 * I, H, I / 128, H / 128,
                                                     1, I);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  prelayout_kernel<<<(unsigned)t2, 256, 0, stream>>>(w2, w2_out, H, I, H / 256, I / 128, 0, I);
  return cudaGetLastError();
}

bool gemm_bn_supported(int bn) { return bn == 16 || bn == 32 || bn == 64 || bn == 128; }

size_t gemm_partial_bytes() {
  static_assert(Cfg<64, false>::kPartialFloats <= 128 * 256, "partial slot size");
  // stream-K: two partial slots per CTA; one partial tile is at most 2 accumulators x 128
  // rows x 64 columns of fp32 (decode GEMM1) or 128 token rows x 256 columns (throughput)
  return (size_t)2 * kMaxSms * 128 * 256 * sizeof(float);
}

cudaError_t launch_gemm1(int bn, const CUtensorMap& w13_map, const CUtensorMap& a_map,
                         const GemmArgs& args, int grid, cudaStream_t stream) {
  switch (bn) {
    case 16: return launch_one<16, true>(w13_map, a_map, args, grid, stream);
    case 32: return launch_one<32, true>(w13_map, a_map, args, grid, stream);
    case 64: return launch_one<64, true>(w13_map, a_map, args, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm2(int bn, const CUtensorMap& w2_map, const CUtensorMap& cq_map,
                         const GemmArgs& args, int grid, cudaStream_t stream) {
  switch (bn) {
    case 16: return launch_one<16, false>(w2_map, cq_map, args, grid, stream);
    case 32: return launch_one<32, false>(w2_map, cq_map, args, grid, stream);
    case 64: return launch_one<64, false>(w2_map, cq_map, args, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fmoe
