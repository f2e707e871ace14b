/*
 * fmoe_oracle.c -- CPU restatement of the routing and row-permutation steps of the
 * DeepSeek-V3 FP8 block-scaled fused-MoE operator.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA path: only the
 * test suite, __graft_entry__.smoke() and the CPU-baseline leg of bench.py load it.
 * The product library never links or calls it.
 *
 * What it restates (reference = YuWei-CH/Fused-MoE-YWS, solution/cuda/kernel.cu):
 *   - sigmoid + bias                        kernel.cu:388-401 (sigmoid_bias_kernel)
 *   - group top-2 sums, top-k_group groups,
 *     top-k experts, renormalised weights   kernel.cu:408-516 (routing_select_kernel)
 *   - local-expert histogram / row order    kernel.cu:530-592 (count/reorder kernels)
 *
 * Deliberate, documented differences from the reference:
 *   1. The reference computes 1/(1+expf(-x)) with --use_fast_math expf, which no CPU
 *      can reproduce bit for bit. Both this oracle and the CUDA routing kernel use the
 *      same hand-written exp (Cody-Waite range reduction ln2 = hi + lo, degree-7 Taylor
 *      polynomial on |r| <= ln2/2 evaluated by Horner with explicit fused multiply-adds,
 *      then an exact two-step 2^n scaling). Every operation is an IEEE-754
 *      single-precision add/mul/fma/div with round-to-nearest, so CPU and GPU agree
 *      bit for bit. Compile with -ffp-contract=off and without -ffast-math.
 *   2. The reference reorders rows with atomics, so the row order inside an expert is
 *      non-deterministic (kernel.cu:572-576). Here rows are ordered by
 *      (local expert, token, k): a stable counting sort. The CUDA permute kernel
 *      produces exactly this order, so the permutation is checked bit-exactly.
 *   3. Expert segments are padded to a multiple of 16 rows (the MMA N granularity);
 *      padding rows carry token -1.
 *   4. Non-finite scores: an expert whose biased score is NaN or -inf is never
 *      selected (the reference's strict '>' against -inf has the same effect), and a
 *      group whose score is NaN ranks below every finite group. The reference reads
 *      keep_group[-1] when fewer than topk_group groups have a finite score
 *      (kernel.cu:446-457); here the lowest-index remaining groups are kept instead.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__FAST_MATH__)
#error "fmoe_oracle.c must be compiled without -ffast-math"
#endif

/* ------------------------------------------------------------------------- */
/* Exact-by-construction exp / sigmoid (shared algorithm with csrc/route.cu)  */
/* ------------------------------------------------------------------------- */

static float pow2i(int n) { /* 2^n for n in [-126, 127], exact */
  uint32_t bits = (uint32_t)(n + 127) << 23;
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

float fmoe_oracle_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97208404541015625f) return 0.0f;
  const float n = rintf(x * 1.44269502162933349609375f); /* round(x / ln2) */
  float r = fmaf(n, -0.693145751953125f, x);              /* ln2 high part (exact n*hi) */
  r = fmaf(n, -1.428606765330187045e-06f, r);              /* ln2 low part */
  float p = 1.98412701138295233249664306640625e-04f;       /* 1/7! */
  p = fmaf(p, r, 1.388888922519981861114501953125e-03f);   /* 1/6! */
  p = fmaf(p, r, 8.333333767950534820556640625e-03f);      /* 1/5! */
  p = fmaf(p, r, 4.1666667908430099487304687500e-02f);     /* 1/4! */
  p = fmaf(p, r, 1.6666667163372039794921875e-01f);        /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni / 2;
  const int n2 = ni - n1;
  return (p * pow2i(n1)) * pow2i(n2);
}

float fmoe_oracle_sigmoid(float x) {
  const float e = fmoe_oracle_expf(-x);
  return 1.0f / (1.0f + e);
}

static float bf16_to_f32(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

/* a ranks above b: larger value first, then smaller index. NaN ranks lowest. */
static int ranks_above(float va, int ia, float vb, int ib) {
  const int na = va != va, nb = vb != vb;
  if (na || nb) {
    if (na && nb) return ia < ib;
    return nb;
  }
  if (va > vb) return 1;
  if (va < vb) return 0;
  return ia < ib;
}

/*
 * Route T tokens. Follows kernel.cu:388-516.
 *   logits   fp32 [T, E]
 *   bias     bf16 bits [E]
 *   out_idx  int32 [T, K]  (global expert ids in selection order, -1 if unfilled)
 *   out_w    fp32  [T, K]  (s / (sum s + 1e-20) * rsf, 0 for unfilled slots)
 *   out_s    optional fp32 [T, E] sigmoid scores (may be NULL)
 * Returns 0 on success, -1 on bad geometry.
 */
int fmoe_oracle_route(int64_t T, int E, int n_group, int topk_group, int top_k,
                      const float* logits, const uint16_t* bias, float rsf,
                      int32_t* out_idx, float* out_w, float* out_s) {
  if (E <= 0 || E > 1024 || n_group <= 0 || E % n_group != 0 || topk_group <= 0 ||
      topk_group > n_group || top_k <= 0 || top_k > 32 || n_group > 64)
    return -1;
  const int G = E / n_group;
  float s[1024], swb[1024], gscore[64];
  int keep[64], taken[1024];
  for (int64_t t = 0; t < T; ++t) {
    const float* lrow = logits + t * E;
    for (int e = 0; e < E; ++e) {
      s[e] = fmoe_oracle_sigmoid(lrow[e]);              /* kernel.cu:398 */
      swb[e] = s[e] + bf16_to_f32(bias[e]);             /* kernel.cu:400 */
      if (out_s) out_s[t * E + e] = s[e];
      taken[e] = 0;
    }
    /* group score = sum of the two largest biased scores (kernel.cu:423-442) */
    for (int g = 0; g < n_group; ++g) {
      float b0 = -INFINITY, b1 = -INFINITY;
      for (int j = 0; j < G; ++j) {
        const float v = swb[g * G + j];
        if (v > b0) {
          b1 = b0;
          b0 = v;
        } else if (v > b1) {
          b1 = v;
        }
      }
      gscore[g] = b0 + b1;
      keep[g] = 0;
    }
    /* keep topk_group groups, ties to the lower group index (kernel.cu:444-458) */
    for (int pick = 0; pick < topk_group; ++pick) {
      int best = -1;
      for (int g = 0; g < n_group; ++g) {
        if (keep[g]) continue;
        if (best < 0 || ranks_above(gscore[g], g, gscore[best], best)) best = g;
      }
      keep[best] = 1;
    }
    /* top_k experts among kept groups, ties to the lower expert id (kernel.cu:460-495) */
    int32_t* irow = out_idx + t * top_k;
    float* wrow = out_w + t * top_k;
    for (int k = 0; k < top_k; ++k) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        if (taken[e] || !keep[e / G]) continue;
        const float v = swb[e];
        if (!(v > -INFINITY)) continue; /* NaN and -inf never selected */
        if (best < 0 || ranks_above(v, e, swb[best], best)) best = e;
      }
      irow[k] = best;
      if (best >= 0) taken[best] = 1;
    }
    /* weights from the unbiased scores, summed in selection order (kernel.cu:497-515) */
    float sum = 0.0f;
    for (int k = 0; k < top_k; ++k)
      if (irow[k] >= 0) sum = sum + s[irow[k]];
    sum = sum + 1e-20f;
    for (int k = 0; k < top_k; ++k)
      wrow[k] = irow[k] >= 0 ? (s[irow[k]] / sum) * rsf : 0.0f;
  }
  return 0;
}

/*
 * Deterministic expert-major row plan (kernel.cu:530-592 restated, stable order).
 *   topk_idx   int32 [T, K]
 *   expert_cnt int32 [E_local]        rows per local expert
 *   expert_off int32 [E_local + 1]    first row of each expert, 16-row aligned segments
 *   row_token  int32 [row_cap]        token of each row, -1 for padding / unused rows
 *   row_k      int32 [row_cap]        top-k slot of each row, -1 for padding
 *   token_row  int32 [T, K]           row of each (token, k), -1 if not local
 * Returns the padded row total, or -1 if row_cap is too small.
 */
int64_t fmoe_oracle_plan(int64_t T, int top_k, int E_local, int local_offset,
                         const int32_t* topk_idx, int32_t* expert_cnt, int32_t* expert_off,
                         int32_t* row_token, int32_t* row_k, int32_t* token_row,
                         int64_t row_cap) {
  for (int e = 0; e < E_local; ++e) expert_cnt[e] = 0;
  for (int64_t i = 0; i < T * top_k; ++i) {
    const int le = topk_idx[i] - local_offset;
    if (topk_idx[i] >= 0 && le >= 0 && le < E_local) expert_cnt[le]++;
  }
  int64_t off = 0;
  for (int e = 0; e < E_local; ++e) {
    expert_off[e] = (int32_t)off;
    off += ((int64_t)expert_cnt[e] + 15) / 16 * 16;
  }
  expert_off[E_local] = (int32_t)off;
  if (off > row_cap) return -1;
  for (int64_t r = 0; r < row_cap; ++r) {
    row_token[r] = -1;
    row_k[r] = -1;
  }
  int32_t fill[1024];
  for (int e = 0; e < E_local; ++e) fill[e] = 0;
  for (int64_t t = 0; t < T; ++t) {
    for (int k = 0; k < top_k; ++k) {
      const int g = topk_idx[t * top_k + k];
      const int le = g - local_offset;
      if (g >= 0 && le >= 0 && le < E_local) {
        const int64_t r = expert_off[le] + fill[le]++;
        row_token[r] = (int32_t)t;
        row_k[r] = k;
        token_row[t * top_k + k] = (int32_t)r;
      } else {
        token_row[t * top_k + k] = -1;
      }
    }
  }
  return off;
}
