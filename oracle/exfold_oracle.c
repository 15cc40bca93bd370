/*
 * CPU oracle for the ExFold routing-transform hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain scalar C, what the
 * reference computes on this path so that the CUDA kernels can be checked
 * against it.  It is never linked into the product library and nothing in the
 * product calls it; tests, the smoke check and the benchmark's CPU-baseline leg
 * load it through oracle/oracle.py.
 *
 * Build with -ffp-contract=off: every float operation below is one IEEE
 * binary32 operation, in the order written, so the results are reproducible
 * bit for bit.  Each function cites the reference lines it restates
 * (paths relative to the reference project root).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------- */
/* Exact elementwise math shared (by definition, not by code) with the kernels.
 *
 * exp: Cody-Waite range reduction x = n*ln2 + r with ln2 split into a 15-bit
 * head (so n*ln2_hi is exact) and a tail, then the degree-7 Taylor polynomial
 * of e^r on |r| <= ln2/2 evaluated by Horner with fused multiply-adds
 * (truncation error < 6e-9 relative), then scaling by 2^n through the
 * exponent field.  Inputs are clamped to [-87, 88] so 2^n stays normal.
 * The router's selection key sigmoid(x)+bias is built from this function, so
 * the kernels evaluate the very same operation sequence. */
static const float kLog2e = 0x1.715476p+0f;
static const float kLn2Hi = 0x1.62e4p-1f;
static const float kLn2Lo = 0x1.7f7d1cp-20f;
static const float kInvFact[8] = {1.0f, 1.0f, 0x1p-1f, 0x1.555556p-3f, 0x1.555556p-5f,
                                  0x1.111112p-7f, 0x1.6c16c2p-10f, 0x1.a01a02p-13f};

ORC_API float orc_exp(float x) {
  if (!(x > -87.0f)) x = -87.0f; /* NaN maps to the lower clamp */
  if (x > 88.0f) x = 88.0f;
  const float n = rintf(x * kLog2e);
  float r = fmaf(n, -kLn2Hi, x);
  r = fmaf(n, -kLn2Lo, r);
  float p = kInvFact[7];
  for (int i = 6; i >= 0; --i) p = fmaf(p, r, kInvFact[i]);
  const int ni = (int)n;
  return p * u2f((uint32_t)(ni + 127) << 23);
}

ORC_API float orc_sigmoid(float x) {
  const float e = orc_exp(-x);
  return 1.0f / (1.0f + e);
}

/* sqrt(softplus(x)), the "sqrtsoftplus" router score of vLLM's fused_topk_bias
 * (vllm fused_topk_bias_router.py: F.softplus(gating_output).sqrt()), used by
 * exfold/deepseek_v4/vllm_patch.py:175-209 through module.scoring_func.
 * softplus(x) = max(x, 0) + log1p(exp(-|x|)) with the exp above (NaN maps to
 * its lower clamp, so softplus(NaN) = log1p(e^-87)); log1p(y), 0 < y <= 1, as
 * 2 atanh(u) with u = y / (2 + y) <= 1/3: 2u (1 + u^2/3 + u^4/5 + ... + u^14/15)
 * by Horner in u^2 with fused multiply-adds (truncation below 2e-9 relative);
 * then the IEEE square root. */
static const float kInvOdd[8] = {1.0f,           0x1.555556p-2f, 0x1.99999ap-3f, 0x1.24924ap-3f,
                                 0x1.c71c72p-4f, 0x1.745d18p-4f, 0x1.3b13b2p-4f, 0x1.111112p-4f};
ORC_API float orc_log1p_unit(float y) {
  const float u = y / (2.0f + y);
  const float s = u * u;
  float p = kInvOdd[7];
  for (int i = 6; i >= 0; --i) p = fmaf(p, s, kInvOdd[i]);
  return (2.0f * u) * p;
}
ORC_API float orc_sqrtsoftplus(float x) {
  const float e = orc_exp(-fabsf(x));
  return sqrtf(fmaxf(x, 0.0f) + orc_log1p_unit(e));
}
static inline float orc_score(int scoring, float x) {
  return scoring == 1 ? orc_sigmoid(x) : orc_sqrtsoftplus(x);
}

/* Total order on float keys: IEEE 754 totalOrder (a NaN ranks by its sign bit: above +inf
 * when clear, below -inf when set), except that -0 ranks equal to +0. */
ORC_API uint32_t orc_key(float x) {
  const uint32_t b = f2u(x);
  const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return k == 0x7FFFFFFFu ? 0x80000000u : k;
}

/* (key desc, index asc): is (ka, ia) ranked before (kb, ib)? */
static inline int before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

/* ------------------------------------------------------------------------- */
/* Router top-k.
 * scoring 0 = softmax: select on the logits (softmax is monotone), weights
 *   e_i = exp(x_i - x_max) over the selected slots divided by their sum when
 *   renormalize, else by the sum over all experts in index order.  Semantics
 *   of tests/test_qwen3_kernels.py:35-37 (softmax, topk, divide by sum) and
 *   of vLLM fused_topk called at exfold/qwen3/vllm_patch.py:98-109.
 * scoring 1 = sigmoid with bias: select on sigmoid(x)+bias, weights are the
 *   unbiased sigmoid of the selected experts, divided by their sum when
 *   renormalize, then times routed_scaling_factor.  Semantics of vLLM
 *   fused_topk_bias called at exfold/deepseek_v4/vllm_patch.py:175-209.
 * Slots are ordered by (key desc, expert asc). */
ORC_API void orc_router_topk(const float* logits, int64_t tokens, int experts, int top_k,
                             int scoring, const float* bias, int renormalize, float scaling,
                             float* out_w, int32_t* out_ids) {
  uint32_t* keys = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)experts);
  char* taken = (char*)malloc((size_t)experts);
  for (int64_t t = 0; t < tokens; ++t) {
    const float* x = logits + t * experts;
    for (int e = 0; e < experts; ++e) {
      float k = x[e];
      if (scoring != 0) k = orc_score(scoring, x[e]) + (bias ? bias[e] : 0.0f);
      keys[e] = orc_key(k);
      taken[e] = 0;
    }
    int32_t* ids = out_ids + t * top_k;
    for (int s = 0; s < top_k; ++s) {
      int best = -1;
      for (int e = 0; e < experts; ++e) {
        if (taken[e]) continue;
        if (best < 0 || before(keys[e], e, keys[best], best)) best = e;
      }
      taken[best] = 1;
      ids[s] = best;
    }
    float* w = out_w + t * top_k;
    if (scoring == 0) {
      const float m = x[ids[0]];
      float sum = 0.0f;
      for (int s = 0; s < top_k; ++s) {
        w[s] = orc_exp(x[ids[s]] - m);
        sum = sum + w[s];
      }
      if (!renormalize) {
        sum = 0.0f;
        for (int e = 0; e < experts; ++e) sum = sum + orc_exp(x[e] - m);
      }
      for (int s = 0; s < top_k; ++s) w[s] = w[s] / sum;
    } else {
      float sum = 0.0f;
      for (int s = 0; s < top_k; ++s) {
        w[s] = orc_score(scoring, x[ids[s]]);
        sum = sum + w[s];
      }
      /* sqrtsoftplus clamps the divisor at 1e-20 (vllm fused_topk_bias_router.py
       * _topk_softplus_sqrt_torch: sum.clamp(min=1e-20)) */
      if (scoring == 2 && sum < 1e-20f) sum = 1e-20f;
      if (renormalize)
        for (int s = 0; s < top_k; ++s) w[s] = w[s] / sum;
    }
    if (scaling != 1.0f)
      for (int s = 0; s < top_k; ++s) w[s] = w[s] * scaling;
  }
  free(keys);
  free(taken);
}

/* ------------------------------------------------------------------------- */
/* Hash routing (DeepSeek-V4 hash-MoE layers): vllm fused_topk_bias_router.py
 * (hash_indices_table[input_tokens], weights = the unbiased scores gathered at
 * those ids, renormalised, times the scaling factor), called by
 * exfold/deepseek_v4/vllm_patch.py:175-209 with module.gate.tid2eid.  Routes
 * keep the table's order.  scoring 1 = sigmoid, 2 = sqrtsoftplus.  A token id
 * outside the table gives ids -1 and weights 0; a table entry outside
 * [0, experts) keeps its id and gets weight 0 (both would index out of range
 * in the reference). */
ORC_API void orc_router_hash(const float* logits, int64_t tokens, int experts, int top_k,
                             int scoring, const int64_t* token_ids, const int32_t* table,
                             int64_t table_rows, int renormalize, float scaling,
                             float* out_w, int32_t* out_ids) {
  for (int64_t t = 0; t < tokens; ++t) {
    float* w = out_w + t * top_k;
    int32_t* ids = out_ids + t * top_k;
    const int64_t tid = token_ids[t];
    if (tid < 0 || tid >= table_rows) {
      for (int s = 0; s < top_k; ++s) {
        ids[s] = -1;
        w[s] = 0.0f;
      }
      continue;
    }
    float sum = 0.0f;
    for (int s = 0; s < top_k; ++s) {
      const int32_t e = table[tid * top_k + s];
      ids[s] = e;
      w[s] = (e >= 0 && e < experts) ? orc_score(scoring, logits[t * experts + e]) : 0.0f;
      sum = sum + w[s];
    }
    if (scoring == 2 && sum < 1e-20f) sum = 1e-20f;
    if (renormalize)
      for (int s = 0; s < top_k; ++s) w[s] = w[s] / sum;
    if (scaling != 1.0f)
      for (int s = 0; s < top_k; ++s) w[s] = w[s] * scaling;
  }
}

/* ------------------------------------------------------------------------- */
/* Qwen3 prefill fold, exfold/qwen3/kernels.py:31-94 (_project_prefill_kernel).
 * The first target_k slots are retained as given (the input is assumed sorted
 * by weight).  Each omitted slot j = target_k..top_k-1, in order, goes to the
 * retained position with the smallest loss[src][retained] (first position on
 * ties), adding w_j * coeff[src][target]; a minimum loss >= 1e30 drops the
 * transfer (kernels.py:74).  All other retained weights get + 0.0 (kernels.py:
 * 75-79 adds a masked 0.0 to every slot). */
ORC_API void orc_fold_qwen3(const float* w, const int32_t* ids, int64_t tokens, int top_k,
                            int target_k, const float* coeff, const float* loss, int experts,
                            float* out_w, int32_t* out_ids) {
  for (int64_t t = 0; t < tokens; ++t) {
    const float* tw = w + t * top_k;
    const int32_t* ti = ids + t * top_k;
    float acc[64];
    for (int p = 0; p < target_k; ++p) acc[p] = tw[p];
    for (int j = target_k; j < top_k; ++j) {
      const int src = ti[j];
      int pos = 0;
      float best = loss[(int64_t)src * experts + ti[0]];
      for (int p = 1; p < target_k; ++p) {
        const float c = loss[(int64_t)src * experts + ti[p]];
        if (c < best) { best = c; pos = p; }
      }
      const int tgt = ti[pos];
      const float scale = (best < 1.0e30f) ? coeff[(int64_t)src * experts + tgt] : 0.0f;
      const float add = tw[j] * scale;
      for (int p = 0; p < target_k; ++p) acc[p] = acc[p] + (p == pos ? add : 0.0f);
    }
    for (int p = 0; p < target_k; ++p) {
      out_w[t * target_k + p] = acc[p];
      out_ids[t * target_k + p] = ti[p];
    }
  }
}

/* ------------------------------------------------------------------------- */
/* DeepSeek-V4 prefill fold, exfold/deepseek_v4/csrc/exfold_kernels.cu:17-118.
 * Stable insertion sort by weight descending (48-59); omitted slot j goes to
 * the first retained position with loss strictly below FLT_MAX and minimal
 * (67-79, no 1e30 guard).  renorm_mode 1 rescales to the original L2 norm
 * (101-110); mode 2 scales each transfer by clamp(1 - confidence_loss, 0, 1)
 * and spreads the lost mass over the retained weights in proportion
 * (80-99). */
ORC_API void orc_fold_dsv4(const float* w, const int32_t* ids, int64_t tokens, int top_k,
                           int target_k, const float* coeff, const float* sel_loss,
                           const float* conf_loss, int experts, int renorm_mode, float* out_w,
                           int32_t* out_ids) {
  for (int64_t t = 0; t < tokens; ++t) {
    float lw[64], rw[64];
    int li[64];
    float l2 = 0.0f;
    for (int p = 0; p < top_k; ++p) {
      lw[p] = w[t * top_k + p];
      li[p] = ids[t * top_k + p];
      l2 = l2 + lw[p] * lw[p];
    }
    for (int p = 1; p < top_k; ++p) {
      const float cw = lw[p];
      const int ci = li[p];
      int ins = p;
      while (ins > 0 && cw > lw[ins - 1]) {
        lw[ins] = lw[ins - 1];
        li[ins] = li[ins - 1];
        --ins;
      }
      lw[ins] = cw;
      li[ins] = ci;
    }
    float rsum = 0.0f;
    for (int p = 0; p < target_k; ++p) {
      rw[p] = lw[p];
      rsum = rsum + rw[p];
    }
    float fallback = 0.0f;
    for (int j = target_k; j < top_k; ++j) {
      const int src = li[j];
      float best = FLT_MAX;
      int bp = 0;
      for (int p = 0; p < target_k; ++p) {
        const float c = sel_loss[(int64_t)src * experts + li[p]];
        if (c < best) { best = c; bp = p; }
      }
      const int tgt = li[bp];
      float conf = 1.0f;
      if (renorm_mode == 2) {
        const float cl = conf_loss[(int64_t)src * experts + tgt];
        conf = fminf(fmaxf(1.0f - cl, 0.0f), 1.0f);
        fallback = fallback + lw[j] * (1.0f - conf);
      }
      lw[bp] = lw[bp] + lw[j] * coeff[(int64_t)src * experts + tgt] * conf;
    }
    if (renorm_mode == 2 && rsum > 1.0e-20f) {
      const float fs = fallback / rsum;
      for (int p = 0; p < target_k; ++p) lw[p] = lw[p] + rw[p] * fs;
    }
    float scale = 1.0f;
    if (renorm_mode == 1) {
      float f2 = 0.0f;
      for (int p = 0; p < target_k; ++p) f2 = f2 + lw[p] * lw[p];
      if (f2 > 1.0e-20f) scale = sqrtf(l2 / f2);
    }
    for (int p = 0; p < target_k; ++p) {
      out_w[t * target_k + p] = lw[p] * scale;
      out_ids[t * target_k + p] = li[p];
    }
  }
}

/* ------------------------------------------------------------------------- */
/* Decode importance.  The reference sums w * norm[e] with float atomics
 * (exfold/qwen3/kernels.py:369-398; exfold_kernels.cu:146-151), whose order
 * is not fixed.  Here each product is formed in fp32 (one rounding), clamped
 * as below, converted to a 2^-32 fixed point with round-to-nearest-even
 * and summed in int64: exact and independent of order and of how the batch is
 * split across GPUs.  A NaN product counts 0 (the reference's fp32 sum would
 * turn NaN and rank that expert first); products are clamped to |p| <= 2^24,
 * so one route adds at most 2^56 and the int64 sum, which wraps modulo 2^64,
 * is exact while an expert's true total stays below 2^31 in magnitude. */
ORC_API int64_t orc_fixed_point(float p) {
  if (p != p) return 0;
  p = fminf(fmaxf(p, -16777216.0f), 16777216.0f);
  return (int64_t)llrintf(p * 4294967296.0f);
}

ORC_API void orc_importance(const float* w, const int32_t* ids, int64_t routes,
                            const float* norms, int experts, int64_t* importance) {
  for (int e = 0; e < experts; ++e) importance[e] = 0;
  for (int64_t r = 0; r < routes; ++r) {
    const int e = ids[r];
    if (e < 0 || e >= experts) continue;
    /* modulo 2^64, as the kernels' int64 atomics (signed overflow is undefined in C) */
    importance[e] = (int64_t)((uint64_t)importance[e] +
                              (uint64_t)orc_fixed_point(w[r] * norms[e]));
  }
}

/* Experts ordered by (importance desc, expert asc); the Triton selector packs
 * (float bits << 32 | ~expert) for the same order (kernels.py:413-420) and
 * the CUDA kernel's descending radix sort is stable (exfold_kernels.cu:154-159). */
ORC_API void orc_order(const int64_t* importance, int experts, int32_t* order) {
  for (int e = 0; e < experts; ++e) {
    int rank = 0;
    for (int o = 0; o < experts; ++o)
      if (importance[o] > importance[e] || (importance[o] == importance[e] && o < e)) ++rank;
    order[rank] = e;
  }
}

/* Qwen3 reroute with a given subset, exfold/qwen3/kernels.py:154-232
 * (_reroute_decode_kernel).  A route whose expert is in the subset is
 * unchanged; otherwise it goes to the subset member with the smallest loss
 * (first in subset order on ties) and its weight is multiplied by
 * coeff[src][tgt], or by 0 when that loss is >= 1e30 (kernels.py:222). */
ORC_API void orc_reroute_qwen3(const float* w, const int32_t* ids, int64_t routes,
                               const int32_t* subset, int subset_size, const float* coeff,
                               const float* loss, int experts, float* out_w, int32_t* out_ids) {
  char* in_subset = (char*)calloc((size_t)experts, 1);
  int32_t* tgt = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  float* scale = (float*)malloc(sizeof(float) * (size_t)experts);
  for (int p = 0; p < subset_size; ++p) in_subset[subset[p]] = 1;
  for (int e = 0; e < experts; ++e) {
    int pos = 0;
    float best = loss[(int64_t)e * experts + subset[0]];
    for (int p = 1; p < subset_size; ++p) {
      const float c = loss[(int64_t)e * experts + subset[p]];
      if (c < best) { best = c; pos = p; }
    }
    tgt[e] = subset[pos];
    scale[e] = best < 1.0e30f ? coeff[(int64_t)e * experts + subset[pos]] : 0.0f;
  }
  for (int64_t r = 0; r < routes; ++r) {
    const int e = ids[r];
    if (e < 0 || e >= experts || in_subset[e]) { /* out-of-range ids pass through */
      out_w[r] = w[r];
      out_ids[r] = e;
    } else {
      out_w[r] = w[r] * scale[e];
      out_ids[r] = tgt[e];
    }
  }
  free(in_subset); free(tgt); free(scale);
}

/* Qwen3 decode: select_and_reroute_decode (kernels.py:423-491).  The subset
 * is the first `budget` experts of the order, zero-importance experts
 * included, then the reroute above.  budget >= experts or an empty batch
 * returns the input unchanged (kernels.py:449-450). */
ORC_API void orc_decode_qwen3(const float* w, const int32_t* ids, int64_t batch, int top_k,
                              const float* norms, const float* coeff, const float* loss,
                              int experts, int budget, float* out_w, int32_t* out_ids,
                              int32_t* out_subset) {
  const int64_t routes = batch * top_k;
  if (budget >= experts || batch == 0) {
    memcpy(out_w, w, sizeof(float) * (size_t)routes);
    memcpy(out_ids, ids, sizeof(int32_t) * (size_t)routes);
    return;
  }
  int64_t* imp = (int64_t*)malloc(sizeof(int64_t) * (size_t)experts);
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  orc_importance(w, ids, routes, norms, experts, imp);
  orc_order(imp, experts, order);
  if (out_subset)
    for (int p = 0; p < budget; ++p) out_subset[p] = order[p];
  orc_reroute_qwen3(w, ids, routes, order, budget, coeff, loss, experts, out_w, out_ids);
  free(imp); free(order);
}

/* DeepSeek-V4 decode, exfold_kernels.cu:120-201.  An expert is retained when
 * it is among the first `budget` of the order and its importance is positive
 * (161-164).  A retained or zero-importance expert maps to itself with scale
 * 1 (166-173); any other expert maps to the retained expert of smallest loss
 * strictly below FLT_MAX, first in importance order on ties, with scale
 * coeff[src][tgt] (174-192); if no loss qualifies it maps to itself. */
static void dsv4_apply(const int64_t* imp, const float* w, const int32_t* ids, int64_t routes,
                       const float* coeff, const float* loss, int experts, int budget,
                       float* out_w, int32_t* out_ids);

ORC_API void orc_decode_dsv4(const float* w, const int32_t* ids, int64_t batch, int top_k,
                             const float* norms, const float* coeff, const float* loss,
                             int experts, int budget, float* out_w, int32_t* out_ids) {
  const int64_t routes = batch * top_k;
  int64_t* imp = (int64_t*)malloc(sizeof(int64_t) * (size_t)experts);
  orc_importance(w, ids, routes, norms, experts, imp);
  dsv4_apply(imp, w, ids, routes, coeff, loss, experts, budget, out_w, out_ids);
  free(imp);
}

/* Decode from an importance vector summed elsewhere (a batch sharded over ranks): the select,
 * table and apply steps of orc_decode_qwen3 (variant 0, without its passthrough) or
 * orc_decode_dsv4 (variant 1) on this rank's routes. */
ORC_API void orc_decode_apply(const int64_t* imp, const float* w, const int32_t* ids,
                              int64_t routes, const float* coeff, const float* loss, int experts,
                              int budget, int variant, float* out_w, int32_t* out_ids) {
  if (variant == 1) {
    dsv4_apply(imp, w, ids, routes, coeff, loss, experts, budget, out_w, out_ids);
    return;
  }
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  orc_order(imp, experts, order);
  orc_reroute_qwen3(w, ids, routes, order, budget, coeff, loss, experts, out_w, out_ids);
  free(order);
}

static void dsv4_apply(const int64_t* imp, const float* w, const int32_t* ids, int64_t routes,
                       const float* coeff, const float* loss, int experts, int budget,
                       float* out_w, int32_t* out_ids) {
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  char* kept = (char*)calloc((size_t)experts, 1);
  int32_t* tgt = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  float* scale = (float*)malloc(sizeof(float) * (size_t)experts);
  orc_order(imp, experts, order);
  for (int p = 0; p < budget && p < experts; ++p)
    if (imp[order[p]] > 0) kept[order[p]] = 1;
  for (int e = 0; e < experts; ++e) {
    tgt[e] = e;
    scale[e] = 1.0f;
    if (kept[e] || imp[e] <= 0) continue;
    float best = FLT_MAX;
    int bt = e;
    for (int p = 0; p < budget && p < experts; ++p) {
      if (imp[order[p]] <= 0) continue;
      const float c = loss[(int64_t)e * experts + order[p]];
      if (c < best) { best = c; bt = order[p]; }
    }
    tgt[e] = bt;
    scale[e] = bt == e ? 1.0f : coeff[(int64_t)e * experts + bt];
  }
  for (int64_t r = 0; r < routes; ++r) {
    const int e = ids[r];
    if (e < 0 || e >= experts) { /* out-of-range ids pass through */
      out_ids[r] = e;
      out_w[r] = w[r];
      continue;
    }
    out_ids[r] = tgt[e];
    out_w[r] = w[r] * scale[e];
  }
  free(order); free(kept); free(tgt); free(scale);
}

/* ------------------------------------------------------------------------- */
/* Static decode table, exfold/qwen3/vllm_patch.py:130-143: the `budget`
 * experts of largest calibrated norm are kept (ordered by norm desc, expert
 * asc); every other expert maps to the kept expert of smallest loss (first in
 * that order on ties) with scale coeff[src][tgt]; kept experts map to
 * themselves with scale 1. */
ORC_API void orc_static_table(const float* norms, const float* coeff, const float* loss,
                              int experts, int budget, int32_t* target, float* scale) {
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  char* kept = (char*)calloc((size_t)experts, 1);
  for (int e = 0; e < experts; ++e) {
    int rank = 0;
    const uint32_t ke = orc_key(norms[e]);
    for (int o = 0; o < experts; ++o)
      if (before(orc_key(norms[o]), o, ke, e)) ++rank;
    order[rank] = e;
  }
  for (int p = 0; p < budget; ++p) kept[order[p]] = 1;
  for (int e = 0; e < experts; ++e) {
    if (kept[e]) { target[e] = e; scale[e] = 1.0f; continue; }
    int pos = 0;
    float best = loss[(int64_t)e * experts + order[0]];
    for (int p = 1; p < budget; ++p) {
      const float c = loss[(int64_t)e * experts + order[p]];
      if (c < best) { best = c; pos = p; }
    }
    target[e] = order[pos];
    scale[e] = coeff[(int64_t)e * experts + order[pos]];
  }
  free(order); free(kept);
}

/* In-place static remap, exfold/qwen3/kernels.py:295-319: ids = target[ids],
 * w = w * scale[ids]. */
ORC_API void orc_static_remap(float* w, int32_t* ids, int64_t routes, int experts,
                              const int32_t* target, const float* scale) {
  for (int64_t r = 0; r < routes; ++r) {
    const int e = ids[r];
    if (e < 0 || e >= experts) continue; /* out-of-range ids are left alone */
    w[r] = w[r] * scale[e];
    ids[r] = target[e];
  }
}

/* ------------------------------------------------------------------------- */
/* moe_align / permute.  Semantics of vLLM moe_align_block_size as documented
 * in its Python wrapper (vllm/model_executor/layers/fused_moe/
 * moe_align_block_size.py:11-93, including its worked example): routes
 * grouped by expert, each expert padded to a multiple of block_size with the
 * sentinel numel, experts in ascending order, routes of one expert in
 * ascending flat index.  expert_ids names the expert of every block; blocks
 * past num_tokens_post_pad hold -1.  Routes with an id outside [0, experts)
 * are not placed. */
ORC_API int64_t orc_moe_align_capacity(int64_t numel, int experts, int block_size,
                                       int pad_sorted) {
  int64_t cap = numel + (int64_t)experts * (block_size - 1);
  if (pad_sorted) cap = (cap + block_size - 1) / block_size * block_size;
  if (numel < experts && numel * block_size < cap) cap = numel * block_size;
  return cap;
}

ORC_API void orc_moe_align(const int32_t* ids, int64_t numel, int experts, int block_size,
                           int64_t capacity, int32_t* sorted_ids, int32_t* expert_ids,
                           int32_t* num_post_pad) {
  int64_t* count = (int64_t*)calloc((size_t)experts, sizeof(int64_t));
  int64_t* offset = (int64_t*)calloc((size_t)experts + 1, sizeof(int64_t));
  for (int64_t r = 0; r < numel; ++r)
    if (ids[r] >= 0 && ids[r] < experts) count[ids[r]]++;
  for (int e = 0; e < experts; ++e) {
    const int64_t padded = (count[e] + block_size - 1) / block_size * block_size;
    offset[e + 1] = offset[e] + padded;
  }
  const int64_t blocks = (capacity + block_size - 1) / block_size;
  for (int64_t i = 0; i < capacity; ++i) sorted_ids[i] = (int32_t)numel;
  for (int64_t b = 0; b < blocks; ++b) expert_ids[b] = -1;
  for (int e = 0; e < experts; ++e)
    for (int64_t b = offset[e] / block_size; b < offset[e + 1] / block_size; ++b)
      expert_ids[b] = e;
  int64_t* fill = (int64_t*)calloc((size_t)experts, sizeof(int64_t));
  for (int64_t r = 0; r < numel; ++r) {
    const int e = ids[r];
    if (e < 0 || e >= experts) continue;
    sorted_ids[offset[e] + fill[e]++] = (int32_t)r;
  }
  *num_post_pad = (int32_t)offset[experts];
  free(count); free(offset); free(fill);
}
