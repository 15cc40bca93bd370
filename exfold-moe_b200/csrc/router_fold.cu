// Router top-k and prefill fold kernels (sm_100a).
//
// router_kernel: one pass over the router logits per token, optionally fused with the ExFold
// prefill fold, so the [tokens][top_k] routing tensors never reach HBM.
//   * A token is owned by a group of L = E/32 lanes; each lane holds 32 logits in registers
//     (8 coalesced streaming loads of 4 logits: 16 bytes fp32, 8 bytes bf16 / fp16, converted to
//     fp32 exactly) and stages them in shared memory as fp32.
//   * Selection: the exact top-k set is contained in the candidates whose key is >= theta, where
//     theta is the k-th largest maximum over groups of 4 consecutive keys (k distinct elements
//     reach it, so the k-th largest key is >= theta).  theta comes from a register bitonic
//     network over the group maxima (19-comparator sort per lane, then log2(L) shuffle merges).
//     For the sigmoid router the network runs on fast approximate keys and theta is lowered by
//     twice their error bound, which keeps the containment.  Candidates (typically 9-12 of the
//     E experts) are ranked exactly by (key desc, expert asc); a token with more than
//     kMaxCand candidates (ties, constant rows) takes an exact k-round selection instead.
//   * Fold: omitted slots are spread over the group's lanes, their loss/scale gathers hit the
//     L2-resident E x E tables, and the transfers are accumulated in slot order.
// fold_kernel: the fold alone from precomputed top-k routes (one thread per token), for the
//   reference-compatible API that receives (weights, ids).
#include <float.h>

#include <atomic>

#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"

namespace exf {

constexpr int kMaxK = 8;
constexpr int kMaxCand = 32;


template <int E>
struct RouterShape {
  static constexpr int L = E / 32;        // lanes per token
  static constexpr int TPW = 32 / L;      // tokens per warp
  static constexpr int WARPS = (E >= 128) ? 4 : 2;
  static constexpr int ROW = E + 16;      // padded staging row (floats)
};

__device__ __forceinline__ void cx_desc(uint32_t& a, uint32_t& b) {
  const uint32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}

// Optimal 19-comparator network for 8 inputs, descending.
__device__ __forceinline__ void sort8_desc(uint32_t (&v)[8]) {
  cx_desc(v[0], v[2]); cx_desc(v[1], v[3]); cx_desc(v[4], v[6]); cx_desc(v[5], v[7]);
  cx_desc(v[0], v[4]); cx_desc(v[1], v[5]); cx_desc(v[2], v[6]); cx_desc(v[3], v[7]);
  cx_desc(v[0], v[1]); cx_desc(v[2], v[3]); cx_desc(v[4], v[5]); cx_desc(v[6], v[7]);
  cx_desc(v[2], v[4]); cx_desc(v[3], v[5]);
  cx_desc(v[1], v[4]); cx_desc(v[3], v[6]);
  cx_desc(v[1], v[2]); cx_desc(v[3], v[4]); cx_desc(v[5], v[6]);
}

// a, b sorted descending -> a = the 8 largest of both, sorted descending.
__device__ __forceinline__ void merge8_desc(uint32_t (&a)[8], const uint32_t (&b)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = max(a[i], b[7 - i]);
  cx_desc(a[0], a[4]); cx_desc(a[1], a[5]); cx_desc(a[2], a[6]); cx_desc(a[3], a[7]);
  cx_desc(a[0], a[2]); cx_desc(a[1], a[3]); cx_desc(a[4], a[6]); cx_desc(a[5], a[7]);
  cx_desc(a[0], a[1]); cx_desc(a[2], a[3]); cx_desc(a[4], a[5]); cx_desc(a[6], a[7]);
}


template <int E>
struct __align__(16) RouterSmem {
  using S = RouterShape<E>;
  static constexpr int CSTR = kMaxCand + 1;  // candidate rows: groups land on distinct banks
  static constexpr int SSTR = 12;            // slot rows: 16-byte aligned, distinct bank quads
  __align__(16) float vals[S::WARPS][S::TPW][S::ROW];
  __align__(16) unsigned long long cand[S::WARPS][S::TPW][CSTR];  // key << 32 | ~expert
  __align__(16) float cval[S::WARPS][S::TPW][CSTR];
  __align__(16) int sidx[S::WARPS][S::TPW][SSTR];   // selected experts, router order
  __align__(16) float sval[S::WARPS][S::TPW][SSTR]; // logit (softmax) / exact sigmoid
  __align__(16) float sw[S::WARPS][S::TPW][SSTR];   // unnormalised weight
  __align__(16) float wf[S::WARPS][S::TPW][SSTR];   // final weight, router order
  __align__(16) int fidx[S::WARPS][S::TPW][SSTR];   // fold order (DeepSeek-V4: weight-sorted)
  __align__(16) float fw[S::WARPS][S::TPW][SSTR];
  __align__(16) int fpos[S::WARPS][S::TPW][SSTR];   // omitted slot -> retained position
  __align__(16) float ft[S::WARPS][S::TPW][SSTR];   // omitted slot -> transfer
  __align__(16) float ff[S::WARPS][S::TPW][SSTR];   // omitted slot -> lost mass (blend)
  __align__(16) float acc[S::WARPS][S::TPW][SSTR];  // folded retained weights
};

template <int E, int SCORING, int FOLD, typename LT>
__global__ void __launch_bounds__(RouterShape<E>::WARPS * 32)
    router_kernel(const RouterParams p) {
  const LT* logits = static_cast<const LT*>(p.logits);
  using S = RouterShape<E>;
  constexpr int L = S::L;
  constexpr int TPW = S::TPW;
  __shared__ RouterSmem<E> sm;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane / L;
  const int r = lane % L;
  const unsigned gmask = (L == 32 ? 0xffffffffu : ((1u << L) - 1u)) << (g * L);
  const int K = p.top_k;
  const int P = p.target_k;
  const int64_t total = (int64_t)p.layers * p.tokens;
  const int64_t stride = (int64_t)gridDim.x * S::WARPS * TPW;

  float* sv = sm.vals[warp][g];
  unsigned long long* cand = sm.cand[warp][g];
  float* cval = sm.cval[warp][g];
  int* sidx = sm.sidx[warp][g];
  float* sval = sm.sval[warp][g];
  float* swt = sm.sw[warp][g];
  float* wf = sm.wf[warp][g];

  // (layer, token) of this group's token, advanced incrementally (no 64-bit division per step)
  int64_t gt = ((int64_t)blockIdx.x * S::WARPS + warp) * TPW + g;
  int64_t layer = gt < total ? gt / p.tokens : 0;
  int64_t tok = gt - layer * p.tokens;
  // logits of the current token are prefetched one iteration ahead
  float4 nv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    nv[i] = gt < total ? ld_stream_logits4(logits + gt * E + 4 * (r + L * i))
                       : make_float4(0.f, 0.f, 0.f, 0.f);

  for (int64_t base = gt - g; base < total; base += stride, gt += stride) {
    const bool valid = gt < total;
    const float* brow = (SCORING != EXF_SOFTMAX && p.bias) ? p.bias + layer * E : nullptr;

    // ---- stage, selection keys (IEEE total order; exact logits or fast sigmoid) -------------
    uint32_t keys[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int col = 4 * (r + L * i);
      const float4 v = nv[i];
      *reinterpret_cast<float4*>(sv + col) = v;
      float x[4] = {v.x, v.y, v.z, v.w};
      if (SCORING != EXF_SOFTMAX) {
        const float4 b = brow ? __ldg(reinterpret_cast<const float4*>(brow + col))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        x[0] = approx_score<SCORING>(x[0]) + b.x;
        x[1] = approx_score<SCORING>(x[1]) + b.y;
        x[2] = approx_score<SCORING>(x[2]) + b.z;
        x[3] = approx_score<SCORING>(x[3]) + b.w;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) keys[4 * i + c] = order_key(x[c]);
    }

    // ---- threshold: k-th largest group-of-4 maximum over the token --------------------------
    uint32_t top[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      top[i] = max(max(keys[4 * i], keys[4 * i + 1]), max(keys[4 * i + 2], keys[4 * i + 3]));
    sort8_desc(top);
#pragma unroll
    for (int off = 1; off < L; off <<= 1) {
      uint32_t other[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) other[i] = __shfl_xor_sync(0xffffffffu, top[i], off);
      merge8_desc(top, other);
    }
    uint32_t theta = top[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
      if (i == K - 1) theta = top[i];
    if (SCORING != EXF_SOFTMAX)
      theta = order_key(float_of_key(theta) - 2.0f * kSigmoidMargin);
    else if (theta == kKeyPosZero)
      theta = kKeyNegZero;  // -0 ranks equal to +0

    // ---- candidates ------------------------------------------------------------------------
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) mask |= (keys[j] >= theta ? 1u : 0u) << j;
    const int cnt = __popc(mask);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < L; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off, L);
      if (r >= off) incl += o;
    }
    const int ncand = __shfl_sync(0xffffffffu, incl, L - 1, L);
    const bool overflow = ncand > kMaxCand;

    // prefetch the next token's logits; they land while this token is ranked and folded
    const int64_t layer_now = layer;
    {
      const int64_t ngt = gt + stride;
      tok += stride;
      while (tok >= p.tokens && layer < p.layers) {
        tok -= p.tokens;
        ++layer;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        nv[i] = ngt < total ? ld_stream_logits4(logits + ngt * E + 4 * (r + L * i))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();

    if (valid && !overflow) {
      int off = incl - cnt;
      uint32_t m = mask;
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        const int col = 4 * (r + L * (j >> 2)) + (j & 3);
        const float x = sv[col];
        float val;
        uint32_t k;
        if (SCORING != EXF_SOFTMAX) {
          val = exact_score<SCORING>(x);
          k = key_of(__fadd_rn(val, brow ? __ldg(brow + col) : 0.0f));
        } else {
          val = x;
          k = key_of(x);
        }
        cand[off] = ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)col);
        cval[off] = val;
        ++off;
      }
    }
    __syncwarp();
    if (valid && !overflow) {
      for (int c = r; c < ncand; c += L) {
        const unsigned long long pc = cand[c];
        int rank = 0;
        for (int o = 0; o < ncand; ++o) rank += (cand[o] > pc) ? 1 : 0;
        if (rank < K) {
          sidx[rank] = (int)(0xFFFFFFFFu - (uint32_t)pc);
          sval[rank] = cval[c];
        }
      }
    } else if (valid) {
      // Exact k rounds over all E keys, recomputed from the staged logits each round (rare
      // path: ties or constant rows).  Group-uniform branch; shuffles use the group mask.
      uint32_t taken = 0;
      for (int s = 0; s < K; ++s) {
        unsigned long long best = 0;  // every packed key is nonzero and unique
        int bj = -1;
        for (int j = 0; j < 32; ++j) {
          if ((taken >> j) & 1u) continue;
          const int col = 4 * (r + L * (j >> 2)) + (j & 3);
          const float x = sv[col];
          const uint32_t k =
              (SCORING != EXF_SOFTMAX)
                  ? key_of(__fadd_rn(exact_score<SCORING>(x), brow ? __ldg(brow + col) : 0.0f))
                  : key_of(x);
          const unsigned long long pk =
              ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)col);
          if (pk > best) {
            best = pk;
            bj = j;
          }
        }
        const unsigned long long mine = best;
#pragma unroll
        for (int off = 1; off < L; off <<= 1) {
          const unsigned long long o = __shfl_xor_sync(gmask, best, off, L);
          best = o > best ? o : best;
        }
        if (bj >= 0 && mine == best) taken |= 1u << bj;
        if (r == 0) {
          const int col = (int)(0xFFFFFFFFu - (uint32_t)best);
          sidx[s] = col;
          sval[s] = (SCORING != EXF_SOFTMAX) ? exact_score<SCORING>(sv[col]) : sv[col];
        }
      }
    }
    __syncwarp();

    // ---- weights: each slot computed once, by lane (slot % L) ---------------------------------
    if (valid) {
      for (int s = r; s < K; s += L)
        swt[s] = (SCORING == EXF_SOFTMAX) ? exact_exp(__fsub_rn(sval[s], sval[0])) : sval[s];
    }
    __syncwarp();
    float norm = 0.0f;
    bool divide = true;
    if (SCORING == EXF_SOFTMAX && !p.renormalize) {
      // normaliser over all experts: per-lane partial sums, combined in lane order
      const float m = sval[0];
      float part = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = 4 * (r + L * (j >> 2)) + (j & 3);
        part = __fadd_rn(part, exact_exp(__fsub_rn(sv[col], m)));
      }
#pragma unroll
      for (int q = 0; q < L; ++q) norm = __fadd_rn(norm, __shfl_sync(0xffffffffu, part, q, L));
    } else if (SCORING != EXF_SOFTMAX && !p.renormalize) {
      divide = false;
    } else {
      for (int s = 0; s < K; ++s) norm = __fadd_rn(norm, swt[s]);
      // sqrtsoftplus clamps the divisor (vLLM fused_topk_bias: sum.clamp(min=1e-20))
      if (SCORING == EXF_SQRTSOFTPLUS && norm < 1.0e-20f) norm = 1.0e-20f;
    }
    if (valid) {
      for (int s = r; s < K; s += L) {
        float x = divide ? __fdiv_rn(swt[s], norm) : swt[s];
        if (p.scaling != 1.0f) x = __fmul_rn(x, p.scaling);
        wf[s] = x;
      }
    }
    __syncwarp();

    if (FOLD == kFoldNone) {
      if (valid) {
        for (int s = r; s < K; s += L) {
          p.out_w[gt * K + s] = wf[s];
          p.out_ids[gt * K + s] = sidx[s];
        }
      }
      __syncwarp();
      continue;
    }

    // ---- prefill fold ----------------------------------------------------------------------
    const float* coeff = p.coeff + layer_now * E * E;
    const float* sel = p.sel_loss + layer_now * E * E;
    const int* fidx = sidx;
    const float* fw = wf;
    if (FOLD == kFoldDsv4) {
      // stable sort by weight descending: each slot's rank under (weight desc, slot asc)
      int* oidx = sm.fidx[warp][g];
      float* ow = sm.fw[warp][g];
      if (valid) {
        for (int s = r; s < K; s += L) {
          const float ws = wf[s];
          const uint32_t ks = key_of(ws);
          int pos = 0;
          for (int q = 0; q < K; ++q) {
            const uint32_t kq = key_of(wf[q]);
            pos += (kq > ks || (kq == ks && q < s)) ? 1 : 0;
          }
          oidx[pos] = sidx[s];
          ow[pos] = ws;
        }
      }
      __syncwarp();
      fidx = oidx;
      fw = ow;
    }
    int* fpos = sm.fpos[warp][g];
    float* ft = sm.ft[warp][g];
    float* ff = sm.ff[warp][g];
    float* acc = sm.acc[warp][g];
    if (valid) {
      const bool blend = FOLD == kFoldDsv4 && p.renorm_mode == EXF_RENORM_SIMILARITY_BLEND;
      const float* conf_tab = blend ? p.conf_loss + layer_now * E * E : nullptr;
      for (int j = P + r; j < K; j += L) {
        const int src = fidx[j];
        const float wj = fw[j];
        const float* lrow = sel + (int64_t)src * E;
        const float* crow = coeff + (int64_t)src * E;
        // every retained candidate's loss, scale (and confidence) in flight at once
        float lv[kMaxK], cv[kMaxK], qv[kMaxK];
        int tv[kMaxK];
#pragma unroll
        for (int q = 0; q < kMaxK; ++q) {
          if (q < P) {
            tv[q] = fidx[q];
            lv[q] = __ldg(lrow + tv[q]);
            cv[q] = __ldg(crow + tv[q]);
            qv[q] = blend ? __ldg(conf_tab + (int64_t)src * E + tv[q]) : 0.0f;
          }
        }
        int pos = 0;
        float best = (FOLD == kFoldQwen3) ? lv[0] : FLT_MAX;
#pragma unroll
        for (int q = (FOLD == kFoldQwen3) ? 1 : 0; q < kMaxK; ++q) {
          if (q < P && lv[q] < best) {
            best = lv[q];
            pos = q;
          }
        }
        float s_val = cv[0], cl = qv[0];
#pragma unroll
        for (int q = 1; q < kMaxK; ++q) {
          if (q == pos) {
            s_val = cv[q];
            cl = qv[q];
          }
        }
        if (FOLD == kFoldQwen3) {
          ft[j] = __fmul_rn(wj, best < 1.0e30f ? s_val : 0.0f);
        } else {
          float conf = 1.0f;
          float lost = 0.0f;
          if (blend) {
            conf = fminf(fmaxf(__fsub_rn(1.0f, cl), 0.0f), 1.0f);
            lost = __fmul_rn(wj, __fsub_rn(1.0f, conf));
          }
          ft[j] = __fmul_rn(__fmul_rn(wj, s_val), conf);
          ff[j] = lost;
        }
        fpos[j] = pos;
      }
    }
    __syncwarp();
    if (valid) {
      const bool blend = FOLD == kFoldDsv4 && p.renorm_mode == EXF_RENORM_SIMILARITY_BLEND;
      float fs = 0.0f;
      bool spread = false;
      if (blend) {
        float fallback = 0.0f, rsum = 0.0f;
        for (int j = P; j < K; ++j) fallback = __fadd_rn(fallback, ff[j]);
        for (int q = 0; q < P; ++q) rsum = __fadd_rn(rsum, fw[q]);
        spread = rsum > 1.0e-20f;
        if (spread) fs = __fdiv_rn(fallback, rsum);
      }
      for (int q = r; q < P; q += L) {
        const float wq = fw[q];
        float a = wq;
        for (int j = P; j < K; ++j) {
          const int pj = fpos[j];
          if (FOLD == kFoldQwen3)
            a = __fadd_rn(a, q == pj ? ft[j] : 0.0f);
          else if (q == pj)
            a = __fadd_rn(a, ft[j]);
        }
        if (spread) a = __fadd_rn(a, __fmul_rn(wq, fs));
        acc[q] = a;
      }
    }
    __syncwarp();
    if (valid) {
      float scale = 1.0f;
      if (FOLD == kFoldDsv4 && p.renorm_mode == EXF_RENORM_ROUTER_L2) {
        float l2 = 0.0f, f2 = 0.0f;
        for (int s = 0; s < K; ++s) l2 = __fadd_rn(l2, __fmul_rn(wf[s], wf[s]));
        for (int q = 0; q < P; ++q) f2 = __fadd_rn(f2, __fmul_rn(acc[q], acc[q]));
        if (f2 > 1.0e-20f) scale = __fsqrt_rn(__fdiv_rn(l2, f2));
      }
      for (int q = r; q < P; q += L) {
        p.out_w[gt * P + q] = (FOLD == kFoldDsv4) ? __fmul_rn(acc[q], scale) : acc[q];
        p.out_ids[gt * P + q] = fidx[q];
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------------------------

// One token's fold, thread-local: w / id are the top_k routes in router order (K <= 8).  Writes
// the target_k folded weights (renorm applied) and ids.  Every retained candidate's loss, scale and
// confidence are gathered together so each omitted route costs one round trip to L2.
template <int VARIANT>
__device__ __forceinline__ void fold_token(const float (&w)[kMaxK], const int (&id)[kMaxK], int K,
                                           int P, int E, const float* coeff, const float* sel,
                                           const float* conf_tab, int renorm_mode,
                                           float (&out)[kMaxK], int (&fid)[kMaxK]) {
  auto cl = [E](int e) { return e < 0 ? 0 : (e >= E ? E - 1 : e); };
  float fw[kMaxK];
  if (VARIANT == EXF_DSV4) {
    // stable sort descending by weight: rank under (weight desc, slot asc)
#pragma unroll
    for (int s = 0; s < kMaxK; ++s) {
      fw[s] = 0.0f;
      fid[s] = 0;
    }
#pragma unroll
    for (int s = 0; s < kMaxK; ++s) {
      if (s < K) {
        const uint32_t ks = key_of(w[s]);
        int pos = 0;
#pragma unroll
        for (int q = 0; q < kMaxK; ++q)
          if (q < K && ranks_before(key_of(w[q]), q, ks, s)) ++pos;
#pragma unroll
        for (int q = 0; q < kMaxK; ++q)
          if (q == pos) {
            fw[q] = w[s];
            fid[q] = id[s];
          }
      }
    }
  } else {
#pragma unroll
    for (int s = 0; s < kMaxK; ++s) {
      fw[s] = w[s];
      fid[s] = id[s];
    }
  }
  const bool blend = VARIANT == EXF_DSV4 && renorm_mode == EXF_RENORM_SIMILARITY_BLEND;
  float acc[kMaxK];
#pragma unroll
  for (int q = 0; q < kMaxK; ++q) acc[q] = fw[q];
  float fallback = 0.0f;
#pragma unroll
  for (int j = 1; j < kMaxK; ++j) {
    if (j < P || j >= K) continue;
    const int src = cl(fid[j]);
    const float* lrow = sel + (int64_t)src * E;
    const float* crow = coeff + (int64_t)src * E;
    const float* qrow = blend ? conf_tab + (int64_t)src * E : nullptr;
    float lv[kMaxK], cv[kMaxK], qv[kMaxK];
#pragma unroll
    for (int q = 0; q < kMaxK; ++q) {
      if (q < P) {
        const int t = cl(fid[q]);
        lv[q] = __ldg(lrow + t);
        cv[q] = __ldg(crow + t);
        qv[q] = blend ? __ldg(qrow + t) : 0.0f;
      }
    }
    int pos = 0;
    float best = (VARIANT == EXF_QWEN3) ? lv[0] : FLT_MAX;
#pragma unroll
    for (int q = (VARIANT == EXF_QWEN3) ? 1 : 0; q < kMaxK; ++q)
      if (q < P && lv[q] < best) {
        best = lv[q];
        pos = q;
      }
    float s_val = cv[0], cl_val = qv[0];
#pragma unroll
    for (int q = 1; q < kMaxK; ++q)
      if (q == pos) {
        s_val = cv[q];
        cl_val = qv[q];
      }
    if (VARIANT == EXF_QWEN3) {
      const float add = __fmul_rn(fw[j], best < 1.0e30f ? s_val : 0.0f);
#pragma unroll
      for (int q = 0; q < kMaxK; ++q)
        if (q < P) acc[q] = __fadd_rn(acc[q], q == pos ? add : 0.0f);
    } else {
      float conf = 1.0f;
      if (blend) {
        conf = fminf(fmaxf(__fsub_rn(1.0f, cl_val), 0.0f), 1.0f);
        fallback = __fadd_rn(fallback, __fmul_rn(fw[j], __fsub_rn(1.0f, conf)));
      }
      const float add = __fmul_rn(__fmul_rn(fw[j], s_val), conf);
#pragma unroll
      for (int q = 0; q < kMaxK; ++q)
        if (q == pos) acc[q] = __fadd_rn(acc[q], add);
    }
  }
  float scale = 1.0f;
  if (VARIANT == EXF_DSV4) {
    if (blend) {
      float rsum = 0.0f;
#pragma unroll
      for (int q = 0; q < kMaxK; ++q)
        if (q < P) rsum = __fadd_rn(rsum, fw[q]);
      if (rsum > 1.0e-20f) {
        const float fs = __fdiv_rn(fallback, rsum);
#pragma unroll
        for (int q = 0; q < kMaxK; ++q)
          if (q < P) acc[q] = __fadd_rn(acc[q], __fmul_rn(fw[q], fs));
      }
    } else if (renorm_mode == EXF_RENORM_ROUTER_L2) {
      float l2 = 0.0f, f2 = 0.0f;
#pragma unroll
      for (int q = 0; q < kMaxK; ++q) {
        if (q < K) l2 = __fadd_rn(l2, __fmul_rn(w[q], w[q]));
        if (q < P) f2 = __fadd_rn(f2, __fmul_rn(acc[q], acc[q]));
      }
      if (f2 > 1.0e-20f) scale = __fsqrt_rn(__fdiv_rn(l2, f2));
    }
  }
#pragma unroll
  for (int q = 0; q < kMaxK; ++q) out[q] = (VARIANT == EXF_DSV4) ? __fmul_rn(acc[q], scale) : acc[q];
}

// Fold of precomputed routes, one thread per token, semantics as the fold stage above.
template <typename WT, typename IT, int VARIANT>
__global__ void __launch_bounds__(256) fold_kernel(const FoldParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.tokens) return;
  const int K = p.top_k;
  const int P = p.target_k;
  const WT* wrow = static_cast<const WT*>(p.w) + t * K;
  const IT* irow = static_cast<const IT*>(p.ids) + t * K;
  float w[kMaxK];
  int id[kMaxK];
#pragma unroll
  for (int s = 0; s < kMaxK; ++s) {
    w[s] = (s < K) ? to_f32(wrow[s]) : 0.0f;
    id[s] = (s < K) ? (int)irow[s] : 0;
  }
  float out[kMaxK];
  int fid[kMaxK];
  fold_token<VARIANT>(w, id, K, P, p.experts, p.coeff, p.sel_loss, p.conf_loss, p.renorm_mode, out,
                      fid);
  WT* ow = static_cast<WT*>(p.out_w) + t * P;
  IT* oi = static_cast<IT*>(p.out_ids) + t * P;
#pragma unroll
  for (int q = 0; q < kMaxK; ++q)
    if (q < P) {
      ow[q] = from_f32<WT>(out[q]);
      oi[q] = (IT)fid[q];
    }
}

// ---------------------------------------------------------------------------------------------
// Hash routing (DeepSeek-V4 hash-MoE layers; vLLM fused_topk_bias with hash_indices_table, called
// from exfold/deepseek_v4/vllm_patch.py:175-209): the routes of token t are table[token_ids[t]],
// in table order; their weights are the unbiased scores of those experts, renormalised (the
// sqrtsoftplus divisor clamped at 1e-20) and scaled.  One thread per token.  A token id outside
// the table gives ids -1 and weights 0; a table entry outside [0, experts) keeps its id and
// gets weight 0, so nothing is read out of range.
template <int SCORING, typename TID, typename LT>
__global__ void __launch_bounds__(256) router_hash_kernel(
    const LT* logits, int64_t tokens, int E, int K, const TID* token_ids, const int32_t* table,
    int64_t rows, int renormalize, float scaling, float* out_w, int32_t* out_ids) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= tokens) return;
  const int64_t tid = (int64_t)token_ids[t];
  float* ow = out_w + t * K;
  int32_t* oi = out_ids + t * K;
  if (tid < 0 || tid >= rows) {
    for (int s = 0; s < K; ++s) {
      ow[s] = 0.0f;
      oi[s] = -1;
    }
    return;
  }
  const int32_t* trow = table + tid * K;
  const LT* xrow = logits + t * E;
  float w[kMaxK];
  int id[kMaxK];
  float sum = 0.0f;
#pragma unroll
  for (int s = 0; s < kMaxK; ++s) {
    if (s < K) {
      const int e = __ldg(trow + s);
      id[s] = e;
      w[s] = (e >= 0 && e < E) ? exact_score<SCORING>(logit_f32<LT>(xrow[e])) : 0.0f;
      sum = __fadd_rn(sum, w[s]);
    }
  }
  if (SCORING == EXF_SQRTSOFTPLUS && sum < 1.0e-20f) sum = 1.0e-20f;
#pragma unroll
  for (int s = 0; s < kMaxK; ++s) {
    if (s < K) {
      float x = renormalize ? __fdiv_rn(w[s], sum) : w[s];
      if (scaling != 1.0f) x = __fmul_rn(x, scaling);
      ow[s] = x;
      oi[s] = id[s];
    }
  }
}

template <int SCORING, typename TID, typename LT>
static cudaError_t launch_hash_t(const void* logits, int64_t tokens, int E, int K,
                                 const void* token_ids, const int32_t* table, int64_t rows,
                                 int renormalize, float scaling, float* out_w, int32_t* out_ids,
                                 cudaStream_t stream) {
  const unsigned blocks = (unsigned)((tokens + 255) / 256);
  router_hash_kernel<SCORING, TID, LT><<<blocks, 256, 0, stream>>>(
      static_cast<const LT*>(logits), tokens, E, K, static_cast<const TID*>(token_ids), table,
      rows, renormalize, scaling, out_w, out_ids);
  return cudaGetLastError();
}

template <int SCORING, typename LT>
static cudaError_t launch_hash_l(const void* logits, int64_t tokens, int E, int K,
                                 const void* token_ids, int id_dtype, const int32_t* table,
                                 int64_t rows, int renormalize, float scaling, float* out_w,
                                 int32_t* out_ids, cudaStream_t s) {
  return id_dtype == EXF_I32
             ? launch_hash_t<SCORING, int32_t, LT>(logits, tokens, E, K, token_ids, table, rows,
                                                   renormalize, scaling, out_w, out_ids, s)
             : launch_hash_t<SCORING, int64_t, LT>(logits, tokens, E, K, token_ids, table, rows,
                                                   renormalize, scaling, out_w, out_ids, s);
}

template <int SCORING>
static cudaError_t launch_hash_s(const void* logits, int logit_dtype, int64_t tokens, int E,
                                 int K, const void* token_ids, int id_dtype, const int32_t* table,
                                 int64_t rows, int renormalize, float scaling, float* out_w,
                                 int32_t* out_ids, cudaStream_t s) {
  switch (logit_dtype) {
    case EXF_F32:
      return launch_hash_l<SCORING, float>(logits, tokens, E, K, token_ids, id_dtype, table, rows,
                                           renormalize, scaling, out_w, out_ids, s);
    case EXF_BF16:
      return launch_hash_l<SCORING, __nv_bfloat16>(logits, tokens, E, K, token_ids, id_dtype,
                                                   table, rows, renormalize, scaling, out_w,
                                                   out_ids, s);
    default:
      return launch_hash_l<SCORING, __half>(logits, tokens, E, K, token_ids, id_dtype, table,
                                            rows, renormalize, scaling, out_w, out_ids, s);
  }
}

cudaError_t launch_router_hash(const void* logits, int logit_dtype, int64_t tokens, int experts,
                               int top_k, int scoring, const void* token_ids, int id_dtype,
                               const int32_t* table, int64_t table_rows, int renormalize,
                               float scaling, float* out_w, int32_t* out_ids, cudaStream_t s) {
  if (scoring == EXF_SQRTSOFTPLUS)
    return launch_hash_s<EXF_SQRTSOFTPLUS>(logits, logit_dtype, tokens, experts, top_k, token_ids,
                                           id_dtype, table, table_rows, renormalize, scaling,
                                           out_w, out_ids, s);
  return launch_hash_s<EXF_SIGMOID>(logits, logit_dtype, tokens, experts, top_k, token_ids,
                                    id_dtype, table, table_rows, renormalize, scaling, out_w,
                                    out_ids, s);
}

// ---------------------------------------------------------------------------------------------
// Host launchers
template <int E, int SCORING, int FOLD, typename LT>
static cudaError_t launch_router_l(const RouterParams& p, cudaStream_t stream) {
  using S = RouterShape<E>;
  auto kern = router_kernel<E, SCORING, FOLD, LT>;
  const int64_t total = (int64_t)p.layers * p.tokens;
  const int64_t per_block = (int64_t)S::WARPS * S::TPW;
  int64_t blocks = (total + per_block - 1) / per_block;
  const int cap = persistent_grid(reinterpret_cast<const void*>(kern), S::WARPS * 32, 0);
  if (cap > 0 && blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  kern<<<(unsigned)blocks, S::WARPS * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int E, int SCORING, int FOLD>
static cudaError_t launch_router_e(const RouterParams& p, cudaStream_t stream) {
  switch (p.logit_dtype) {
    case EXF_F32: return launch_router_l<E, SCORING, FOLD, float>(p, stream);
    case EXF_BF16: return launch_router_l<E, SCORING, FOLD, __nv_bfloat16>(p, stream);
    default: return launch_router_l<E, SCORING, FOLD, __half>(p, stream);
  }
}

template <int SCORING, int FOLD>
static cudaError_t launch_router_s(int experts, const RouterParams& p, cudaStream_t stream) {
  switch (experts) {
    case 64: return launch_router_e<64, SCORING, FOLD>(p, stream);
    case 128: return launch_router_e<128, SCORING, FOLD>(p, stream);
    case 256: return launch_router_e<256, SCORING, FOLD>(p, stream);
    case 512: return launch_router_e<512, SCORING, FOLD>(p, stream);
    default: return cudaErrorNotSupported;
  }
}

// The tile kernels keep a CTA per SM streaming 32- or 16-token tiles; a launch below about
// 32768 rows gives each warp at most one tile, and the generic kernel's shorter per-token chain
// then finishes first (L2 flushed, us per launch, tile / generic: E = 128 softmax + fold at 4096
// rows 12.3 / 10.2, 16384 rows 14.3 / 14.3, 65536 rows 22.5 / 26.6; E = 256 biased sigmoid +
// DeepSeek fold 22.5 / 12.3, 24.6 / 20.6, 49.2 / 55.3; without a fold 16.4 / 12.3 at 4096 and
// 40.9 / 38.9 at 65536 rows).
static std::atomic<int64_t> g_tile_min_rows{32768};

int64_t router_tile_min_rows(int64_t rows) {
  return rows >= 0 ? g_tile_min_rows.exchange(rows) : g_tile_min_rows.load();
}

cudaError_t launch_router(int experts, int scoring, int fold, const RouterParams& p,
                          cudaStream_t stream) {
  const int64_t rows = p.tokens * p.layers;
  const int64_t min_rows = g_tile_min_rows.load(std::memory_order_relaxed);
  if (rows >= min_rows && router_tpt_eligible(experts, scoring, fold, p))
    return launch_router_tpt(fold, p, stream);
  if (rows >= (fold == kFoldNone ? 4 * min_rows : min_rows) &&
      router_biased_eligible(experts, scoring, fold, p))
    return launch_router_biased(fold, p, stream);
  if (scoring == EXF_SOFTMAX) {
    if (fold == kFoldNone) return launch_router_s<EXF_SOFTMAX, kFoldNone>(experts, p, stream);
    if (fold == kFoldQwen3) return launch_router_s<EXF_SOFTMAX, kFoldQwen3>(experts, p, stream);
    return launch_router_s<EXF_SOFTMAX, kFoldDsv4>(experts, p, stream);
  }
  if (scoring == EXF_SQRTSOFTPLUS) {
    if (fold == kFoldNone) return launch_router_s<EXF_SQRTSOFTPLUS, kFoldNone>(experts, p, stream);
    if (fold == kFoldQwen3) return launch_router_s<EXF_SQRTSOFTPLUS, kFoldQwen3>(experts, p, stream);
    return launch_router_s<EXF_SQRTSOFTPLUS, kFoldDsv4>(experts, p, stream);
  }
  if (fold == kFoldNone) return launch_router_s<EXF_SIGMOID, kFoldNone>(experts, p, stream);
  if (fold == kFoldQwen3) return launch_router_s<EXF_SIGMOID, kFoldQwen3>(experts, p, stream);
  return launch_router_s<EXF_SIGMOID, kFoldDsv4>(experts, p, stream);
}

template <typename WT, typename IT>
static cudaError_t launch_fold_t(int variant, const FoldParams& p, cudaStream_t stream) {
  const unsigned blocks = (unsigned)((p.tokens + 255) / 256);
  if (variant == EXF_QWEN3)
    fold_kernel<WT, IT, EXF_QWEN3><<<blocks, 256, 0, stream>>>(p);
  else
    fold_kernel<WT, IT, EXF_DSV4><<<blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

template <typename WT>
static cudaError_t launch_fold_w(int id_dtype, int variant, const FoldParams& p,
                                 cudaStream_t stream) {
  return id_dtype == EXF_I32 ? launch_fold_t<WT, int32_t>(variant, p, stream)
                             : launch_fold_t<WT, int64_t>(variant, p, stream);
}

cudaError_t launch_fold(int w_dtype, int id_dtype, int variant, const FoldParams& p,
                        cudaStream_t stream) {
  switch (w_dtype) {
    case EXF_F32: return launch_fold_w<float>(id_dtype, variant, p, stream);
    case EXF_BF16: return launch_fold_w<__nv_bfloat16>(id_dtype, variant, p, stream);
    default: return launch_fold_w<__half>(id_dtype, variant, p, stream);
  }
}

}  // namespace exf
