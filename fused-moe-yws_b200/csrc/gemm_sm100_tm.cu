// gemm_sm100_tm.cu -- throughput ("token-major") family of the grouped FP8 GEMMs, used
// when experts receive many rows (large T, skewed routing, the expert-parallel layer).
//
// Same operator as gemm_sm100.cu (reference solution/cuda/kernel.cu:1006-1199 and the
// CUTLASS grouped GEMMs at :73-115 / :1221-1417), other orientation: the MMA M side is
// 128 routed token rows of one expert, the N side is 256 weight rows. Per 128-K block one
// tcgen05.mma M128 x N256 x K128 (four K = 32 instructions) fills a 256-column TMEM
// accumulator; an epilogue thread owns one token row, so the block-scale promotion is a
// single FMA per element with a per-thread scalar (token scale x weight-block scale).
//   GEMM1: N = 128 gate rows [128 m, 128 m + 128) + the matching 128 up rows of W13; the
//          thread holding token row r and C columns [64 j, 64 j + 64) reads gate columns
//          64 j.. and up columns 128 + 64 j..: SwiGLU is thread-local; the per-(token,
//          128-column) amax is combined across the 2 column slices through shared memory.
//   GEMM2: N = 256 rows of W2 (two 128-row scale blocks); the thread owns 128 consecutive
//          output columns of its token row (one scale block) and stores them as 256
//          contiguous bytes.
// Warps: 0 TMA producer (also stages each tile's weight-scale rows into a 2-slot ring),
// 1 TMEM allocator + MMA issuer, 2..9 epilogue (TMEM lane quadrant = warp % 4, column
// slice = (warp - 2) / 4). Ten warps put at most three on an SM sub-partition, so a thread
// can hold 168 registers: its 128 accumulators stay in registers, and the per-step waits,
// fences and barrier arrivals are paid by 8 warps instead of 16 (18 warps capped a thread
// at 96 registers, which put spills on the K loop; measured 3-12 % slower).
// Two 256-column TMEM accumulators let the MMA of K block kb+1 overlap the promotion of kb. The schedule (data-parallel waves, stream-K tail), bounded
// waits, abort protocol and error reporting are those of gemm_sm100.cu.
#include <cuda_fp8.h>

#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"
#include "gemm_sched.cuh"
#include "sm100.cuh"

namespace fmoe {

using namespace sm100;

namespace {

constexpr int kTmThreads = 320;     // 10 warps
constexpr int kTmEpiThreads = 256;  // warps 2..9
constexpr int kTmBarAll = 1;        // named barrier over the epilogue warps
constexpr int kTmSmemLimit = 232448;

template <bool kG1>
struct TmCfg {
  static constexpr int kABytes = kG1 ? 128 * 128 : 2 * 128 * 128;  // tokens (G2: hi + lo)
  static constexpr int kBBytes = 256 * 128;                        // 256 weight rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kNBuf = 2;                                  // 2 x 256 TMEM columns
  static constexpr int kSlotBytes = 128 * 4;                       // token scales, one K step
  static constexpr int kAxBytes = kG1 ? 4 * 128 * 4 : 0;           // amax exchange
  static constexpr int kWscBytes = 2 * 2 * kMaxKSteps * 4;         // [slot][row 0/1][k step]
  static constexpr int kMaxSlots = 16 + 2 + 2;
  static constexpr int kBarBytes = 1024;
  static constexpr int kFixedMax =
      1024 + kAxBytes + kWscBytes + kMaxSlots * kSlotBytes + kBarBytes + 64;
  static constexpr int kStagesRaw = (kTmSmemLimit - kFixedMax) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 16 ? 16 : kStagesRaw;
  static constexpr int kSlots = kStages + kNBuf + 2;
  static constexpr int kFixed = 1024 + kAxBytes + kWscBytes + kSlots * kSlotBytes + kBarBytes + 64;
  static constexpr int kSmemBytes = kFixed + kStages * kStageBytes;
  static constexpr int kPartialFloats = 128 * 256;
  static_assert(kStages >= 2, "pipeline depth");
  static_assert(kSmemBytes <= kTmSmemLimit, "shared memory budget");
  static_assert((16 + 16 + 2 + 2 + 4 + 2 * kMaxSlots + 4 + 4) * 8 <= kBarBytes, "barrier area");
};

// fast division: the reference is built with --use_fast_math, which approximates it too
__device__ __forceinline__ float silu_tm(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// acc[i] += D[i] * s, W TMEM columns per load, as packed FMAs (each lane of fma.rn.f32x2
// rounds like fmaf). GEMM1 loads 8 columns at a time: beside its 64 gate and 64 up
// accumulators that leaves fewer values to spill and reload in every K step (measured
// 5-12 % faster for GEMM1 than 16-column loads).
template <int N, int W = 16>
__device__ __forceinline__ void promote_tm(float (&acc)[N], uint32_t taddr, float s) {
  const float2 s2 = make_float2(s, s);
#pragma unroll
  for (int c = 0; c < N / W; ++c) {
    uint32_t v[W];
    tmem_ld_32x32b<W>(taddr + c * W, v);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < W; i += 2) {
      const float2 r = __ffma2_rn(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])),
                                  s2, make_float2(acc[c * W + i], acc[c * W + i + 1]));
      acc[c * W + i] = r.x;
      acc[c * W + i + 1] = r.y;
    }
  }
}

template <int N>
__device__ __forceinline__ void store_vec(float* dst, const float (&v)[N]) {
#pragma unroll
  for (int j = 0; j < N; j += 4)
    *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

// Load N floats written by another CTA (16-byte aligned): L2-coherent loads.
template <int N>
__device__ __forceinline__ void load_vec(float (&v)[N], const float* src) {
#pragma unroll
  for (int j = 0; j < N; j += 4) {
    const float4 x = __ldcg(reinterpret_cast<const float4*>(src + j));
    v[j] = x.x;
    v[j + 1] = x.y;
    v[j + 2] = x.z;
    v[j + 3] = x.w;
  }
}

// Sum of a tile's stream-K contributions (partials in [row][256] layout), in K order; CTAs
// with an empty range contribute nothing. Partials come from other CTAs: L2-coherent loads.
template <int N>
__device__ __forceinline__ void sum_tm(float (&acc)[N], const float* partials, int64_t off,
                                       const StreamK& sk, int64_t tile_begin, int cf, int cl) {
#pragma unroll
  for (int j = 0; j < N; ++j) acc[j] = 0.0f;
  for (int c = cf; c <= cl; ++c) {
    if (sk.start(c) == sk.start(c + 1)) continue;
    const int slot = sk.start(c) >= tile_begin ? 0 : 1;
    const float* p = partials + (int64_t)(2 * c + slot) * (128 * 256) + off;
#pragma unroll
    for (int j = 0; j < N; j += 4) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(p + j));
      acc[j] += x.x;
      acc[j + 1] += x.y;
      acc[j + 2] += x.z;
      acc[j + 3] += x.w;
    }
  }
}

template <bool kG1>
__global__ void __launch_bounds__(kTmThreads, 1)
    grouped_gemm_tm_kernel(const __grid_constant__ CUtensorMap tmA,
                           const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using C = TmCfg<kG1>;
  constexpr int S = C::kStages, NB = C::kNBuf, SR = C::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* fixed = smem + S * C::kStageBytes;
  float* ax = reinterpret_cast<float*>(fixed);
  float* wsc = reinterpret_cast<float*>(fixed + C::kAxBytes);
  float* sring = reinterpret_cast<float*>(fixed + C::kAxBytes + C::kWscBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(fixed + C::kAxBytes + C::kWscBytes +
                                               SR * C::kSlotBytes);
  uint64_t* full = bars;          // [S]  TMA -> MMA
  uint64_t* empty = bars + 16;    // [S]  MMA -> TMA
  uint64_t* tfull = bars + 32;    // [2]  MMA -> epilogue
  uint64_t* tempty = bars + 34;   // [2]  epilogue -> MMA
  uint64_t* wfull = bars + 36;    // [2]  weight-scale rows, producer -> epilogue
  uint64_t* wempty = bars + 38;   // [2]  epilogue -> producer
  uint64_t* sfull = bars + 40;    // [SR] token-scale ring, TMA -> epilogue
  uint64_t* sempty = sfull + C::kMaxSlots;
  uint64_t* mma_done = sempty + C::kMaxSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mma_done + 2);
  volatile int* last_flag = abort_flag + 1;
  // segment descriptors {tile, k0 | k1 << 8, chunk row0, chunk rows} beside the 2-slot
  // weight-scale ring: the producer walks the schedule and publishes each segment with its
  // scales (tile < 0: no more work), so the epilogue warps hold no schedule state in
  // registers and read no chunk record from global memory at the end of a tile
  int4* segd = reinterpret_cast<int4*>(mma_done + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kTmEpiThreads / 32);
    }
    for (int r = 0; r < SR; ++r) {
      mbar_init(&sfull[r], 1);
      mbar_init(&sempty[r], kTmEpiThreads / 32);
    }
    for (int r = 0; r < 2; ++r) {
      mbar_init(&wfull[r], 32);
      mbar_init(&wempty[r], kTmEpiThreads / 32);
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
  pdl_wait();
  pdl_trigger();

  const int num_tiles = args.meta[kMetaNumChunks] * args.m_tiles;
  const int KS = args.k_steps;
  const int cta = (int)blockIdx.x;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // The whole warp stages each tile's weight block scales into a 2-slot shared ring;
    // lane 0 alone issues the copies.
    // Weight tiles: every token tile of an expert reads the same weight rows. The data-parallel
    // prefix deals tiles round-robin, so one wave of CTAs covers gridDim.x consecutive tiles;
    // when an expert's tiles fit in one wave its weight rows are read close together in time
    // and are not worth keeping, when they span several waves the later waves re-read them
    // from L2 only if they were kept.
    const uint64_t pol_once = policy_evict_first();
    const uint64_t pol_keep = policy_evict_last();
    const uint64_t pol_a = policy_evict_last();
    int it = 0, wseg = 0;
    bool ok = true;
    Schedule sched(num_tiles, KS, (int)gridDim.x, cta);
    int tile, k0, k1;
    while (ok && sched.next(tile, k0, k1)) {
      const Chunk ch = args.chunks[tile / args.m_tiles];
      const int m = tile % args.m_tiles;
      const int e_tiles = (__ldg(args.expert_cnt + ch.expert) + 127) / 128 * args.m_tiles;
      const uint64_t pol_w = e_tiles > (int)gridDim.x ? pol_keep : pol_once;
      {
        // GEMM1: gate block m and up block I/128 + m (H/128 values each);
        // GEMM2: h blocks 2 m and 2 m + 1 (I/128 values each)
        const int ws = wseg & 1;
        bool w_ok = true;
        if (lane == 0) w_ok = mbar_wait(&wempty[ws], ((wseg >> 1) & 1) ^ 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
          ok = false;
          break;
        }
        const float* g;
        const float* u;
        int n;
        if constexpr (kG1) {
          const int nb2 = 2 * args.I / kBlock;
          n = args.H / kBlock;
          g = args.w_scale + ((int64_t)ch.expert * nb2 + m) * n;
          u = args.w_scale + ((int64_t)ch.expert * nb2 + args.I / kBlock + m) * n;
        } else {
          n = args.I / kBlock;
          g = args.w_scale + ((int64_t)ch.expert * (args.H / kBlock) + 2 * m) * n;
          u = g + n;
        }
        float* dst = wsc + ws * 2 * kMaxKSteps;
        for (int i = lane; i < n; i += 32) {
          dst[i] = __ldg(g + i);
          dst[kMaxKSteps + i] = __ldg(u + i);
        }
        if (lane == 0) segd[ws] = make_int4(tile, k0 | (k1 << 8), ch.row0, ch.rows);
        mbar_arrive(&wfull[ws]);  // every lane: its stores are released by its own arrive
        ++wseg;
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
          uint8_t* sa = stages + s * C::kStageBytes;
          uint8_t* sb = sa + C::kABytes;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          if constexpr (kG1) {
            tma_load_2d(sa, &tmA, &full[s], ks * 128, ch.row0, pol_a);
          } else {
            tma_load_2d(sa, &tmA, &full[s], ks * 256, ch.row0, pol_a);                    // hi
            tma_load_2d(sa + 128 * 128, &tmA, &full[s], ks * 256 + 128, ch.row0, pol_a);  // lo
          }
          if (args.w_pre) {
            // the weight tile's 32 KB image stored ahead of time: one contiguous bulk copy
            const int64_t t = ((int64_t)ch.expert * args.m_tiles + m) * KS + ks;
            bulk_load_1d_hint(sb, args.w_pre + t * kPrelaidTileBytes, kPrelaidTileBytes,
                              &full[s], pol_w);
          } else if constexpr (kG1) {
            const int wrow = ch.expert * 2 * args.I + m * 128;
            tma_load_2d(sb, &tmB, &full[s], ks * 128, wrow, pol_w);
            tma_load_2d(sb + 128 * 128, &tmB, &full[s], ks * 128, wrow + args.I, pol_w);
          } else {
            const int wrow = ch.expert * args.H + m * 256;
            tma_load_2d(sb, &tmB, &full[s], ks * 128, wrow, pol_w);
            tma_load_2d(sb + 128 * 128, &tmB, &full[s], ks * 128, wrow + 128, pol_w);
          }
          mbar_arrive_expect_tx(&sfull[slot], ch.ncols * 4);
          bulk_load_1d(sring + slot * 128, asrc + (int64_t)ks * args.row_cap, ch.ncols * 4,
                       &sfull[slot]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (ok) {
      // end of work for the epilogue
      const int ws = wseg & 1;
      bool w_ok = true;
      if (lane == 0) w_ok = mbar_wait(&wempty[ws], ((wseg >> 1) & 1) ^ 1, abort_flag);
      ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (ok) {
        if (lane == 0) segd[ws] = make_int4(-1, 0, 0, 0);
        mbar_arrive(&wfull[ws]);
      }
    }
    if (lane == 0) {
      if (!ok) {
        atomicOr(args.err, kErrTimeoutProducer);
        *abort_flag = 1;
      }
      // drain: every issued copy must land before the CTA's shared memory is released
      static const int zero = 0;
      for (int j = it > S ? it - S : 0; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1, &zero);
      for (int j = it > SR ? it - SR : 0; j < it; ++j)
        mbar_wait(&sfull[j % SR], (j / SR) & 1, &zero);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      const uint32_t idesc = idesc_e4m3_f32(128, 256);
      Schedule sched(num_tiles, KS, (int)gridDim.x, cta);
      int tile, k0, k1;
      while (ok && sched.next(tile, k0, k1)) {
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
          const uint32_t d = tmem + b * 256;
          const uint64_t bd = smem_desc_kmajor(sa + C::kABytes, 128);
          if constexpr (kG1) {
            const uint64_t ad = smem_desc_kmajor(sa, 128);
#pragma unroll
            for (int sub = 0; sub < 4; ++sub) mma_f8f6f4(d, ad + 2 * sub, bd + 2 * sub, idesc, sub > 0);
          } else {
            // hi and lo parts of the C block share one scale -> one accumulator
            const uint64_t ah = smem_desc_kmajor(sa, 128);
            const uint64_t al = smem_desc_kmajor(sa + 128 * 128, 128);
#pragma unroll
            for (int sub = 0; sub < 4; ++sub) mma_f8f6f4(d, ah + 2 * sub, bd + 2 * sub, idesc, sub > 0);
#pragma unroll
            for (int sub = 0; sub < 4; ++sub) mma_f8f6f4(d, al + 2 * sub, bd + 2 * sub, idesc, 1);
          }
          tc_commit(&empty[s]);
          tc_commit(&tfull[b]);
        }
      }
      if (!ok) {
        atomicOr(args.err, kErrTimeoutMma);
        *abort_flag = 1;
      }
      // all issued MMAs must retire before TMEM is released
      static const int zero = 0;
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, &zero);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - 2;        // 0..7
    const int q = warp & 3;         // TMEM lane quadrant = token rows 32 q .. 32 q + 31
    const int j = ew >> 2;          // column slice 0..1
    const int tid_e = ew * 32 + lane;
    const int row = q * 32 + lane;  // token row inside the tile
    constexpr int NA = kG1 ? 64 : 128;
    float acc[NA];
    float acc_u[kG1 ? 64 : 1];
    int it = 0, wseg = 0;
    bool ok = true;
    for (;;) {
      // next segment and its weight-scale rows, staged by the producer into the 2-slot ring;
      // one decision for all epilogue warps (nobody waits at a barrier alone)
      const int ws = wseg & 1;
      const bool have = mbar_wait(&wfull[ws], (wseg >> 1) & 1, abort_flag);
      if (named_bar_or(kTmBarAll, kTmEpiThreads, !have)) {
        ok = have;
        break;
      }
      int k0, k1, row0, rows;
      {
        const int4 d = segd[ws];
        if (d.x < 0) break;  // no more work
        k0 = d.y & 0xff;
        k1 = d.y >> 8;
        row0 = d.z;
        rows = d.w;
      }
      // GEMM2's routing weight of this thread's row, loaded now: its latency is hidden by the
      // K loop instead of stalling the tile's finalize
      const float w_row = !kG1 && row < rows ? __ldg(args.row_w + row0 + row) : 0.0f;
      const float* wrow = wsc + ws * 2 * kMaxKSteps;
#pragma unroll
      for (int i = 0; i < NA; ++i) acc[i] = 0.0f;
      if constexpr (kG1) {
#pragma unroll
        for (int i = 0; i < 64; ++i) acc_u[i] = 0.0f;
      }
      {
        // the descriptor fields are re-read from shared memory where needed, so no
        // schedule state stays live across the K loop
        const Schedule sc(num_tiles, KS, (int)gridDim.x, cta);
        const SplitRole role = split_role(sc, segd[ws].x, k0, k1);
        if (role.split && role.pair && role.head) {
        // start from the tail owner's partial (see SplitRole)
        bool ready = true;
        if (tid_e == 0 && ok) ready = wait_nonzero(args.tile_counters + role.cf, abort_flag);
        if (named_bar_or(kTmBarAll, kTmEpiThreads, !ready || !ok)) {
          if (ok) {
            atomicOr(args.err, kErrTimeoutEpilogue);
            *abort_flag = 1;
          }
          ok = false;
        } else {
          const float* pp = args.partials + (int64_t)(2 * role.cl) * C::kPartialFloats + row * 256;
          if constexpr (kG1) {
            load_vec<64>(acc, pp + 64 * j);
            load_vec<64>(acc_u, pp + 128 + 64 * j);
          } else {
            load_vec<128>(acc, pp + 128 * j);
          }
        }
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
        const float st = sring[slot * 128 + row];  // token scale (rows >= ncols: unused)
        const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + b * 256;
        if constexpr (kG1) {
          promote_tm<64, 8>(acc, tb + 64 * j, st * wrow[ks]);
          promote_tm<64, 8>(acc_u, tb + 128 + 64 * j, st * wrow[kMaxKSteps + ks]);
        } else {
          promote_tm<128>(acc, tb + 128 * j, st * wrow[j * kMaxKSteps + ks]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[b]);
          mbar_arrive(&sempty[slot]);
        }
      }
      // the weight-scale slot (and its descriptor) is free again once this warp's
      // promotions are done
      const int tile = segd[ws].x;
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&wempty[ws]);
      ++wseg;
      // one abort decision for all epilogue warps (nobody waits at a barrier alone)
      if (named_bar_or(kTmBarAll, kTmEpiThreads, !ok)) {
        ok = false;
        break;
      }
      const Schedule sched(num_tiles, KS, (int)gridDim.x, cta);
      const SplitRole role = split_role(sched, tile, k0, k1);
      const int m = tile % args.m_tiles;
      // ---- stream-K partial tiles ([row][256] fp32), finished by the last contributor ----
      if (role.split && role.pair) {
        if (!role.head) {
          // tail owner: publish the partial and move on (the head owner finishes the tile)
          float* part =
              args.partials + (int64_t)(2 * cta + role.slot) * C::kPartialFloats + row * 256;
          if constexpr (kG1) {
            store_vec<64>(part + 64 * j, acc);
            store_vec<64>(part + 128 + 64 * j, acc_u);
          } else {
            store_vec<128>(part + 128 * j, acc);
          }
          named_bar(kTmBarAll, kTmEpiThreads);
          if (tid_e == 0) red_release_add(args.tile_counters + role.cf, k1 - k0);
          continue;
        }
        if (tid_e == 0) args.tile_counters[role.cf] = 0;  // ready for the next launch
      } else if (role.split) {
        const StreamK& sk = sched.sk;
        const int64_t tile_begin = role.tb;
        const int slot = role.slot;
        float* part = args.partials + (int64_t)(2 * cta + slot) * C::kPartialFloats + row * 256;
        if constexpr (kG1) {
          store_vec<64>(part + 64 * j, acc);
          store_vec<64>(part + 128 + 64 * j, acc_u);
        } else {
          store_vec<128>(part + 128 * j, acc);
        }
        __threadfence();
        named_bar(kTmBarAll, kTmEpiThreads);
        const int cf = sk.cta_of(tile_begin), cl = sk.cta_of(tile_begin + KS - 1);
        if (tid_e == 0) {
          const int done = atomicAdd(args.tile_counters + cf, k1 - k0) + (k1 - k0);
          const bool last = done == KS;
          if (last) args.tile_counters[cf] = 0;  // ready for the next launch
          *last_flag = last;
        }
        named_bar(kTmBarAll, kTmEpiThreads);
        if (!*last_flag) continue;
        __threadfence();
        if constexpr (kG1) {
          sum_tm<64>(acc, args.partials, row * 256 + 64 * j, sk, tile_begin, cf, cl);
          sum_tm<64>(acc_u, args.partials, row * 256 + 128 + 64 * j, sk, tile_begin, cf, cl);
        } else {
          sum_tm<128>(acc, args.partials, row * 256 + 128 * j, sk, tile_begin, cf, cl);
        }
      }

      const bool real = row < rows;  // rows past the chunk belong to the next expert
      const int64_t grow = (int64_t)row0 + row;
      if constexpr (kG1) {
        // ---- SwiGLU, then FP8 hi/lo on one per-(token, 128-column) scale ----
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          acc[i] = acc[i] * silu_tm(acc_u[i]);
          amax = fmaxf(amax, fabsf(acc[i]));
        }
        ax[j * 128 + row] = amax;
        named_bar(kTmBarAll, kTmEpiThreads);
        amax = fmaxf(ax[row], ax[128 + row]);
        if (real) {
          const float inv = amax > 0.0f ? 448.0f / amax : 0.0f;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
          uint32_t hi[8], lo[8];
#pragma unroll
          for (int k = 0; k < 32; k += 4) {
            float x[4], h[4], l[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) x[u] = acc[32 * hh + k + u] * inv;
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
          // full 32-byte sectors (the workspace is 256-byte aligned, 2I a multiple of 256):
          // 16-byte stores scattered over 32 rows per instruction stalled the epilogue for
          // microseconds per tile while the TMA loads saturated the memory system
          uint8_t* dst = args.cq + grow * (2 * (int64_t)args.I) + m * 256 + j * 64 + 32 * hh;
          st_global_v8(dst, hi);
          st_global_v8(dst + 128, lo);
          }
          if (j == 0) args.c_scale[(int64_t)m * args.row_cap + grow] = amax / 448.0f;
        }
        named_bar(kTmBarAll, kTmEpiThreads);  // ax is reused by the next tile
      } else {
        // ---- weighted expert output: 128 consecutive bf16 of this token row ----
        if (real) {
          const float w = w_row;
          // 32-byte stores: full sectors (H is a multiple of 256 on this path)
          __nv_bfloat16* dst = args.ow + grow * args.H + m * 256 + 128 * j;
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            uint32_t o[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const __nv_bfloat162 h =
                  __floats2bfloat162_rn(acc[16 * v + 2 * u] * w, acc[16 * v + 2 * u + 1] * w);
              o[u] = *reinterpret_cast<const uint32_t*>(&h);
            }
            st_global_v8(dst + 16 * v, o);
          }
        }
      }
    }
    if (!ok) {
      atomicOr(args.err, kErrTimeoutEpilogue);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kG1>
cudaError_t launch_tm(const CUtensorMap& a, const CUtensorMap& b, const GemmArgs& args, int grid,
                      cudaStream_t stream) {
  using C = TmCfg<kG1>;
  auto* fn = grouped_gemm_tm_kernel<kG1>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (configured_device != dev) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  return launch_pdl(fn, dim3(grid), dim3(kTmThreads), C::kSmemBytes, stream, a, b, args);
}

}  // namespace

cudaError_t launch_gemm1_tm(const CUtensorMap& a_map, const CUtensorMap& w13_map,
                            const GemmArgs& args, int grid, cudaStream_t stream) {
  return launch_tm<true>(a_map, w13_map, args, grid, stream);
}

cudaError_t launch_gemm2_tm(const CUtensorMap& cq_map, const CUtensorMap& w2_map,
                            const GemmArgs& args, int grid, cudaStream_t stream) {
  return launch_tm<false>(cq_map, w2_map, args, grid, stream);
}

}  // namespace fmoe
