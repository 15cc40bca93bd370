// Biased-sigmoid router top-8 (+ DeepSeek-V4 prefill fold) for 256 experts (sm_100a).
//
// router_biased_kernel serves the prefill router of DeepSeek-style models: experts ranked by
// sigmoid(x) + bias (IEEE totalOrder keys, -0 = +0, lowest expert first on ties), weights = the
// unbiased sigmoid of the 8 selected experts (renormalised or not, times a scaling factor),
// optionally fused with the ExFold prefill fold (exfold/deepseek_v4/csrc/exfold_kernels.cu:17-118:
// stable sort by weight, each omitted route folded onto the retained expert of smallest selection
// loss, renorm modes 0/1/2).
//   * Tiles of 16 tokens x 1 KB (fp32 logits; 512 B rows of bf16 / fp16 logits, twice the
//     slots) stream through a ring of shared-memory slots filled by bulk copies (cp.async.bulk,
//     mbarrier completion) and shared by the CTA's 8 warps, as in router_tpt.cu.  A warp takes
//     two tiles (A, B) at a time.  For the group maxima, lanes 2r and 2r+1 split token r of a
//     tile: lane half h reads the 32 groups of columns 128h..128h+127 in the chunk order
//     u ^ (lane & 7) (16-byte fp32 chunks) or u ^ (lane & 15) (8-byte 16-bit chunks), so the
//     lanes of each quarter-warp / half-warp hit different banks.  16-bit logits are converted
//     to fp32 exactly on load.
//     Everything after that is per token with one lane each: lane 2r ranks token r of A, lane
//     2r+1 token r of B.
//   * Approximate scores a~ = 0.5 tanh.approx(x / 2) + (0.5 + bias): one MUFU operation per
//     expert.  Over every finite fp32 x, 0.5 tanh.approx(x / 2) + 0.5 is within 4.0e-6 of the
//     sigmoid on B200 (exhaustive sweep) and exact_sigmoid within 9e-8, so |a~ - exact score|
//     <= kErrAbs + kErrRel |score| with a factor-2 margin (the roundings of the bias terms are
//     the relative part).
//   * Each lane keys its 32 group maxima (groups of 4 columns, maxima by three-input max; the
//     key is the maximum's raw bits as a signed integer with the low 6 bits naming the group)
//     and sorts them (4 x 19-comparator networks, 3 merges); one merge with the partner
//     lane gives the token's 8 groups with the largest approximate maxima and the 9th largest.
//     The token's lane reads those 8 groups' logits (fp32: from the tile slot, which the warp
//     holds until then; 16-bit: from L2, the slot refilled before the sort), re-scores them and
//     keys each group's maximum exactly (exact_sigmoid + bias).  With A8 the
//     smallest exact head score, every expert of the exact top 8 has a~ >= A8 - err(A8) =: bound.
//     If the 9th group maximum is below bound, the exact top 8 is the 8 heads plus the other
//     elements of the 8 groups that reach bound (typically 0-2), inserted exactly; otherwise
//     every element of the row that reaches bound is inserted (every element, for a row whose
//     scores are not all finite): exact, slower.
//   * Fold: the argmin over the retained experts of the selection loss (the first minimal loss
//     below FLT_MAX).  fp32 logits: the fp32 losses are gathered from L2.  16-bit logits: the
//     layer's loss table sits in shared memory as the high 16 bits of each float (128 KB), a
//     monotone truncation; the argmin is exact when the smallest truncated loss is unique and
//     below truncated FLT_MAX, otherwise (ties, values near FLT_MAX) the fp32 losses are read
//     from global memory.  Scales and confidence losses are gathered from L2.
#include <float.h>

#include <mutex>

#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"
#include "exf_tile.cuh"

namespace exf {
namespace {
using namespace tile;

constexpr int kE = 256;
constexpr int kK = 8;
constexpr int kWarps = 8;                // warps per CTA, each ranking two tiles at a time
constexpr int kRows = 16;                // tokens per tile

// |approximate - exact score| <= kErrAbs + kErrRel |score| (see the header comment).
constexpr float kErrAbs = 1.0e-5f;
constexpr float kErrRel = 4.0e-7f;

template <int FOLD, typename LT>
struct BiasedSmem {
  // 16 KB tiles of fp32 logits (8 KB of bf16 / fp16): the fold's 128 KB table leaves room for 6
  // (12), without it 13 (26)
  // fp32 logits: the fold's argmins read the fp32 loss table from L2, which leaves 13 tile slots,
  // and each slot is held until the lane pair has read its token's 8 head groups (65536 tokens,
  // P = 3, L2 flushed: 49.1 -> 41.0 us; either change alone gains nothing).  16-bit logits: the
  // table's high halves in shared memory and the heads reloaded from L2 (38.9 us; 43.0 the other
  // way).
  static constexpr bool kSmemTable = FOLD != kFoldNone && sizeof(LT) == 2;
  static constexpr bool kHeadsSmem = sizeof(LT) == 4;
  static constexpr int kSlots = (kSmemTable ? 6 : 13) * (4 / sizeof(LT));
  // group chunk order of lane t: u ^ (t & kSwz) (16-byte fp32 chunks: quarter-warps, 8-byte
  // 16-bit chunks: half-warps hit distinct banks)
  static constexpr uint32_t kSwz = sizeof(LT) == 4 ? 7u : 15u;
  LT tile[kSlots][kRows * kE];
  uint16_t loss_hi[kSmemTable ? kE * kE : 8];  // high 16 bits of each loss
  float cterm[kE];         // 0.5 + bias (rounded), the constant of the approximate score
  float bias[kE];          // the current layer's bias (zeros without one)
  uint64_t bar[kSlots];    // tile copies
  long long seq[kSlots];   // CTA-local index of the tile whose copy the slot's barrier tracks
  long long done[kSlots];  // CTA-local index of the last tile whose copy was waited for
  int next;                // next tile of the current layer to hand out
  int failed;              // a wait timed out: the remaining tiles are marked, not ranked
};
template <int FOLD, typename LT>
constexpr size_t biased_smem_bytes() { return sizeof(BiasedSmem<FOLD, LT>); }
static_assert(biased_smem_bytes<kFoldDsv4, float>() <= 232448, "router_biased: shared memory");
static_assert(biased_smem_bytes<kFoldNone, float>() <= 232448, "router_biased: shared memory");
static_assert(biased_smem_bytes<kFoldDsv4, __half>() <= 232448, "router_biased: shared memory");
static_assert(biased_smem_bytes<kFoldNone, __half>() <= 232448, "router_biased: shared memory");

// 4 logits from global memory through the read-only path, as floats
template <typename LT>
__device__ __forceinline__ float4 ldg_logits4(const LT* p) {
  if constexpr (sizeof(LT) == 4) {
    return __ldg(reinterpret_cast<const float4*>(p));
  } else {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const float2 a = logit2_f32<LT>(u.x), b = logit2_f32<LT>(u.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
}

__device__ __forceinline__ float tanh_approx(float x) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// approximate biased score; c = 0.5 + bias
__device__ __forceinline__ float approx_biased(float x, float c) {
  return __fmaf_rn(0.5f, tanh_approx(__fmul_rn(0.5f, x)), c);
}
__device__ __forceinline__ float lane4(const float4& v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}
// FLT_MAX with its low 16 bits cleared: a truncated loss below it is below FLT_MAX
constexpr uint32_t kFltMaxHi = 0x7F7F0000u;

// merge8 (exf_tile.cuh) that keeps the two largest values dropped so far: d1 >= d2 (over a whole
// merge tree: the 9th and 10th largest inputs)
__device__ __forceinline__ void merge8_2(int32_t* a, const int32_t* b, int32_t& d1,
                                         int32_t& d2) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int32_t lo = min(a[i], b[7 - i]);
    a[i] = max(a[i], b[7 - i]);
    d2 = max(d2, min(d1, lo));
    d1 = max(d1, lo);
  }
  cxs32(a[0], a[4]); cxs32(a[1], a[5]); cxs32(a[2], a[6]); cxs32(a[3], a[7]);
  cxs32(a[0], a[2]); cxs32(a[1], a[3]); cxs32(a[4], a[6]); cxs32(a[5], a[7]);
  cxs32(a[0], a[1]); cxs32(a[2], a[3]); cxs32(a[4], a[5]); cxs32(a[6], a[7]);
}

// A truncated signed key (low 6 bits replaced) rounded up in value: low bits set for a positive
// float, cleared for a negative one.
__device__ __forceinline__ float key_ceil(int32_t k) {
  return __int_as_float(k >= 0 ? (k | 63) : (k & ~63));
}

// Sorted insertion of (packed key, sigmoid) into the descending list T / S, dropping the last.
__device__ __forceinline__ void insert8p(uint64_t (&T)[kK], float (&S)[kK], uint64_t v, float s) {
#pragma unroll
  for (int q = 0; q < kK; ++q) {
    const bool sw = T[q] < v;
    const uint64_t tv = T[q];
    const float ts = S[q];
    T[q] = sw ? v : tv;
    S[q] = sw ? s : ts;
    v = sw ? tv : v;
    s = sw ? ts : s;
  }
}
__device__ __forceinline__ void cx64p(uint64_t& a, uint64_t& b, float& sa, float& sb) {
  const bool sw = a < b;
  const uint64_t ta = a;
  const float tsa = sa;
  a = sw ? b : a;
  b = sw ? ta : b;
  sa = sw ? sb : sa;
  sb = sw ? tsa : sb;
}
__device__ __forceinline__ void sort8p(uint64_t (&v)[kK], float (&s)[kK]) {
  cx64p(v[0], v[2], s[0], s[2]); cx64p(v[1], v[3], s[1], s[3]);
  cx64p(v[4], v[6], s[4], s[6]); cx64p(v[5], v[7], s[5], s[7]);
  cx64p(v[0], v[4], s[0], s[4]); cx64p(v[1], v[5], s[1], s[5]);
  cx64p(v[2], v[6], s[2], s[6]); cx64p(v[3], v[7], s[3], s[7]);
  cx64p(v[0], v[1], s[0], s[1]); cx64p(v[2], v[3], s[2], s[3]);
  cx64p(v[4], v[5], s[4], s[5]); cx64p(v[6], v[7], s[6], s[7]);
  cx64p(v[2], v[4], s[2], s[4]); cx64p(v[3], v[5], s[3], s[5]);
  cx64p(v[1], v[4], s[1], s[4]); cx64p(v[3], v[6], s[3], s[6]);
  cx64p(v[1], v[2], s[1], s[2]); cx64p(v[3], v[4], s[3], s[4]); cx64p(v[5], v[6], s[5], s[6]);
}

// Exact top 8 of one row by insertion of every element whose approximate score reaches bound
// (or is NaN); every element when all is set.  Out of line: rarely taken.
template <typename LT>
__device__ __noinline__ void exact_top8_biased(const LT* grow, const float* cterm,
                                               const float* bias, float bound, bool all,
                                               uint64_t* out, float* out_s) {
  uint64_t T[kK];
  float S[kK];
#pragma unroll
  for (int q = 0; q < kK; ++q) {
    T[q] = 0;
    S[q] = 0.0f;
  }
#pragma unroll 1
  for (int c0 = 0; c0 < kE / 4; c0 += 8) {
    float4 xs[8];  // 8 chunks in flight
#pragma unroll
    for (int u = 0; u < 8; ++u) xs[u] = ldg_logits4(grow + 4 * (c0 + u));
#pragma unroll 1
    for (int u = 0; u < 8; ++u) {
      const int c = c0 + u;
      const float4 cc = *reinterpret_cast<const float4*>(cterm + 4 * c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xj = lane4(xs[u], j);
        const float a = approx_biased(xj, lane4(cc, j));
        if (all || !(a < bound)) {
          const float sg = exact_sigmoid(xj);
          insert8p(T, S, pack(key_of(__fadd_rn(sg, bias[4 * c + j])), 4 * c + j), sg);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kK; ++q) {
    out[q] = T[q];
    out_s[q] = S[q];
  }
}

template <int FOLD, int P, typename LT>
__global__ void __launch_bounds__(kWarps * 32, 1) router_biased_kernel(const RouterParams p) {
  using Smem = BiasedSmem<FOLD, LT>;
  constexpr int kSlots = Smem::kSlots;
  extern __shared__ __align__(128) uint8_t biased_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(biased_raw);
  const LT* logits = static_cast<const LT*>(p.logits);
  const int t = threadIdx.x & 31;
  const int h = t & 1;         // column half of this lane in the group maxima; tile B after it
  const int r = t >> 1;        // token of the tile
  const uint32_t swz = static_cast<uint32_t>(t) & Smem::kSwz;  // chunk order of this lane
  const int64_t tokens = p.tokens;
  // Tiles never straddle a layer (the last one of a layer may be short): global tile g is tile
  // g % tpl of layer g / tpl.  This CTA ranks the contiguous range [g0, g0 + nk).
  const int64_t tpl = (tokens + kRows - 1) / kRows;
  const int64_t ntiles = tpl * p.layers;
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * ntiles / gridDim.x;
  const int64_t nk = (static_cast<int64_t>(blockIdx.x) + 1) * ntiles / gridDim.x - g0;
  volatile long long* seq = sm.seq;
  volatile int* failed = &sm.failed;

  auto issue = [&](int64_t k) {  // local tile k into slot k % kSlots
    const int slot = static_cast<int>(k % kSlots);
    const int64_t l = (g0 + k) / tpl, tl = (g0 + k) - l * tpl;
    const int64_t rows = tokens - tl * kRows < kRows ? tokens - tl * kRows : kRows;
    const uint32_t bytes = static_cast<uint32_t>(rows * kE * sizeof(LT));
    bar_expect(&sm.bar[slot], bytes);
    bulk_load(sm.tile[slot], logits + (l * tokens + tl * kRows) * kE, bytes, &sm.bar[slot]);
  };
  // Launched as a programmatic dependent of the previous kernel in the stream.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      bar_init(&sm.bar[s]);
      sm.seq[s] = -1;
      sm.done[s] = -1;
    }
    sm.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int s = 0; s < kSlots && s < nk; ++s) {
      sm.seq[s] = s;
      issue(s);
    }
  }

  // Group maxima of tile k for this lane's half of token r (lanes past the end of a short tile
  // use the tile's first token): pk = the token's 8 largest packed maxima, p9 the 9th.  Waits for
  // the tile's copy and refills the slot afterwards; false if a wait timed out.  Warp-uniform.
  auto group_maxima = [&](int64_t k, int rowi, int32_t (&pk)[kK], int32_t& p9,
                          int32_t& p10, bool own, float4 (&xo)[kK]) -> bool {
    const int slot = static_cast<int>(k % kSlots);
    bool ok = !*failed;
    if (ok && t == 0) {
      uint32_t i = 0;
      while (seq[slot] != k && !*failed && i < kSpinLimit)
        if (++i > 16) __nanosleep(32);
      ok = seq[slot] == k;
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) ok = bar_wait(&sm.bar[slot], static_cast<uint32_t>(k / kSlots) & 1u);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      if (t == 0) sm.done[slot] = k;
    } else {
      *failed = 1;
    }
    // approximate group maxima, keyed: the only reads of the tile
    int32_t g[32];
    if (ok) {
      const LT* rowp = sm.tile[slot] + rowi * kE;
#pragma unroll
      for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = 32 * h + static_cast<int>(static_cast<uint32_t>(8 * s + i) ^ swz);
          const float4 v = load_logits4(rowp + 4 * c);
          const float4 cc = *reinterpret_cast<const float4*>(sm.cterm + 4 * c);
          const float m = fmax_nan(fmax3_nan(approx_biased(v.x, cc.x), approx_biased(v.y, cc.y),
                                             approx_biased(v.z, cc.z)),
                                   approx_biased(v.w, cc.w));
          const uint32_t id = (static_cast<uint32_t>(h) << 5) | (8 * s + i);
          g[8 * s + i] = static_cast<int32_t>((__float_as_uint(m) & ~63u) | (63u - id));
        }
    }
    auto refill = [&]() {
      // the tile is consumed: refill its slot with local tile k + kSlots (generic-proxy reads of
      // the slot are ordered before the bulk copy that overwrites it)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (t == 0 && ok && k + kSlots < nk) {
        issue(k + kSlots);
        __threadfence_block();
        seq[slot] = k + kSlots;
      }
    };
    if constexpr (!Smem::kHeadsSmem) refill();  // before the sorting network
    p9 = INT32_MIN;
    p10 = INT32_MIN;
#pragma unroll
    for (int q = 0; q < kK; ++q) pk[q] = INT32_MIN;
    if (ok) {
      sort8<int32_t, cxs32>(g);
      sort8<int32_t, cxs32>(g + 8);
      sort8<int32_t, cxs32>(g + 16);
      sort8<int32_t, cxs32>(g + 24);
      merge8_2(g, g + 8, p9, p10);
      merge8_2(g + 16, g + 24, p9, p10);
      merge8_2(g, g + 16, p9, p10);
      // the partner lane's 8 groups: both lanes end with the same sorted top 8 of the token
      int32_t o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __shfl_xor_sync(0xffffffffu, g[i], 1);
      const int32_t o9 = __shfl_xor_sync(0xffffffffu, p9, 1);
      const int32_t o10 = __shfl_xor_sync(0xffffffffu, p10, 1);
      merge8_2(g, o, p9, p10);
      // the partner's two largest dropped values
      p10 = max(p10, min(p9, o9));
      p9 = max(p9, o9);
      p10 = max(p10, o10);
#pragma unroll
      for (int q = 0; q < kK; ++q) pk[q] = g[q];
      if (Smem::kHeadsSmem && own) {  // this lane's token: the 8 head groups' logits from the slot
        const LT* rowp = sm.tile[slot] + rowi * kE;
#pragma unroll
        for (int q = 0; q < kK; ++q) {
          const uint32_t id = 63u - (static_cast<uint32_t>(pk[q]) & 63u);
          const uint32_t hh = id >> 5, i = id & 31u;
          const uint32_t osw = (static_cast<uint32_t>(t) & (Smem::kSwz & ~1u)) | hh;
          xo[q] = load_logits4(rowp + 4 * static_cast<int>(32 * hh + (i ^ osw)));
        }
      }
    }
    if constexpr (Smem::kHeadsSmem) refill();
    return ok;
  };

  for (int64_t ks = 0; ks < nk;) {
    const int64_t l = (g0 + ks) / tpl;
    const int64_t ke = ((l + 1) * tpl - g0) < nk ? (l + 1) * tpl - g0 : nk;
    const int n = static_cast<int>(ke - ks);
    // ---- this layer's bias terms and truncated losses into shared memory (the previous
    // layer's readers have passed the barrier at the end of the segment loop) ----------------
    if (threadIdx.x == 0) sm.next = 0;
    {
      const float* brow = p.bias ? p.bias + l * kE : nullptr;
      for (int e = threadIdx.x; e < kE; e += kWarps * 32) {
        const float b = brow ? brow[e] : 0.0f;
        sm.bias[e] = b;
        sm.cterm[e] = __fadd_rn(0.5f, b);
      }
      if (Smem::kSmemTable) {
        // 16 loads in flight per thread before their stores: the 256 KB table costs 4 L2 (or,
        // after L2 was flushed, DRAM) round trips instead of one per few 16-byte vectors
        constexpr int kBatch = 16;
        constexpr int kStride = kWarps * 32;
        static_assert((kE * kE / 4) % (kBatch * kStride) == 0, "loss table copy batches");
        const uint4* src = reinterpret_cast<const uint4*>(p.sel_loss + l * kE * kE);
        uint2* dst = reinterpret_cast<uint2*>(sm.loss_hi);
        for (int i0 = threadIdx.x; i0 < kE * kE / 4; i0 += kBatch * kStride) {
          uint4 v[kBatch];
#pragma unroll
          for (int b = 0; b < kBatch; ++b) v[b] = __ldg(src + i0 + b * kStride);
#pragma unroll
          for (int b = 0; b < kBatch; ++b)
            dst[i0 + b * kStride] = make_uint2(__byte_perm(v[b].x, v[b].y, 0x7632),
                                               __byte_perm(v[b].z, v[b].w, 0x7632));
        }
      }
    }
    __syncthreads();
    const float* coeff = FOLD != kFoldNone ? p.coeff + l * kE * kE : nullptr;
    const float* selg = FOLD != kFoldNone ? p.sel_loss + l * kE * kE : nullptr;
    const bool blend = FOLD == kFoldDsv4 && p.renorm_mode == EXF_RENORM_SIMILARITY_BLEND;
    const float* conf = blend ? p.conf_loss + l * kE * kE : nullptr;
    const int64_t tile0 = (g0 + ks) - l * tpl;  // the segment's first tile within the layer

    while (true) {
      int j = 0;
      if (t == 0) j = atomicAdd(&sm.next, 2);
      j = __shfl_sync(0xffffffffu, j, 0);
      if (j >= n) break;
      const bool has_b = j + 1 < n;
      // ======== phase 1: group maxima of tiles A and B (the only reads of the tiles) =========
      const int64_t tok_a = (tile0 + j) * kRows, tok_b = tok_a + kRows;
      const int ra = tok_a + r < tokens ? r : 0;
      const int rb = has_b && tok_b + r < tokens ? r : 0;
      // this lane's token from phase 2 on: r of A (h = 0) or r of B (h = 1); a lane without a
      // token ranks A's (in bounds, discarded)
      const bool use_b = h && has_b;
      // Tiles A and B in a loop that is not unrolled (one copy of the group-maxima code: the
      // kernel's instruction fetch was a top stall); each lane keeps its own tile's result.
      int32_t pk[kK] = {}, p9 = INT32_MIN, p10 = INT32_MIN;
      float4 xq[kK];  // the 8 head groups' logits
      bool ok = true;
#pragma unroll 1
      for (int which = 0; which < (has_b ? 2 : 1); ++which) {
        int32_t tk[kK], t9 = INT32_MIN, t10 = INT32_MIN;
        ok = group_maxima(ks + j + which, which ? rb : ra, tk, t9, t10,
                          which == (use_b ? 1 : 0), xq) && ok;
        if (which == (use_b ? 1 : 0)) {
#pragma unroll
          for (int q = 0; q < kK; ++q) pk[q] = tk[q];
          p9 = t9;
          p10 = t10;
        }
      }
      const bool valid = use_b ? tok_b + r < tokens : (h == 0 && tok_a + r < tokens);
      const int64_t orow = l * tokens + (use_b ? tok_b : tok_a) + r;
      const LT* grow = logits + (l * tokens + (use_b ? tok_b + rb : tok_a + ra)) * kE;

      if (!ok) {
        if (valid) {
          const int width = FOLD == kFoldNone ? kK : P;
          for (int q = 0; q < width; ++q) {
            p.out_w[orow * width + q] = 0.0f;
            p.out_ids[orow * width + q] = -1;
          }
        }
        continue;
      }

      // ======== phase 2: exact keys of the 8 groups' maxima (heads), then the extras ==========
      uint64_t T[kK];
      float S[kK];
      float av[kK][4];
      int em[kK];
      int cq[kK];
#pragma unroll
      for (int q = 0; q < kK; ++q) {
        const uint32_t id = 63u - (pk[q] & 63u);
        const uint32_t hh = id >> 5, i = id & 31u;
        // chunk order of the lane (of this lane's pair) that took the maximum
        const uint32_t osw = (static_cast<uint32_t>(t) & (Smem::kSwz & ~1u)) | hh;
        cq[q] = static_cast<int>(32 * hh + (i ^ osw));
        if constexpr (!Smem::kHeadsSmem)
          xq[q] = ldg_logits4(grow + 4 * cq[q]);  // all loads in flight before any use
      }
#pragma unroll
      for (int q = 0; q < kK; ++q) {
        const int c = cq[q];
        const float4 x = xq[q];
        const float4 cc = *reinterpret_cast<const float4*>(sm.cterm + 4 * c);
        av[q][0] = approx_biased(x.x, cc.x);
        av[q][1] = approx_biased(x.y, cc.y);
        av[q][2] = approx_biased(x.z, cc.z);
        av[q][3] = approx_biased(x.w, cc.w);
        const float mx = fmaxf(fmaxf(av[q][0], av[q][1]), fmaxf(av[q][2], av[q][3]));
        const int e = av[q][0] == mx ? 0 : (av[q][1] == mx ? 1 : (av[q][2] == mx ? 2 : 3));
        em[q] = e;
        const float sg = exact_sigmoid(lane4(x, e));
        T[q] = pack(key_of(__fadd_rn(sg, sm.bias[4 * c + e])), 4 * c + e);
        S[q] = sg;
      }
      bool sorted = true;
#pragma unroll
      for (int q = 0; q + 1 < kK; ++q) sorted = sorted && T[q] > T[q + 1];
      if (!sorted) sort8p(T, S);
      const float a8 = float_of_key(static_cast<uint32_t>(T[kK - 1] >> 32));
      const float bound = __fsub_rn(a8, __fmaf_rn(kErrRel, fabsf(a8), kErrAbs));
      // The 9th and 10th largest approximate maxima rounded up.  Keys are the raw bits of the
      // maxima compared as signed integers, so negative maxima rank in reverse among themselves:
      // when a negative maximum is named, every other negative one is larger and the test below
      // fails (the exact path ranks the row); when the 9th or 10th is negative, every negative
      // maximum is below the positive bound.
      const float g9 = key_ceil(p9);
      const float g10 = key_ceil(p10);
      const bool nonfinite = (pk[0] & ~63) >= 0x7F800000;  // +inf or NaN approximate maximum
      if (!nonfinite && g10 < bound) {
        // every element outside the 8 groups and the 9th is below bound: insert the other
        // elements of the 8 groups that reach bound (their logits are in registers) ...
        uint32_t xm = 0;
#pragma unroll
        for (int q = 0; q < kK; ++q)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            xm |= (e != em[q] && !(av[q][e] < bound) ? 1u : 0u) << (4 * q + e);
        while (xm) {
          const int site = __ffs(xm) - 1;
          xm &= xm - 1;
          const int q = site >> 2, e = site & 3;
          float4 xs = xq[0];
          int cs = cq[0];
#pragma unroll
          for (int qq = 1; qq < kK; ++qq)
            if (qq == q) {
              xs = xq[qq];
              cs = cq[qq];
            }
          const int col = 4 * cs + e;
          const float sg = exact_sigmoid(lane4(xs, e));
          insert8p(T, S, pack(key_of(__fadd_rn(sg, sm.bias[col])), col), sg);
        }
        // ... and, when the 9th group's maximum reaches bound, the elements of that group that do
        if (!(g9 < bound)) {
          const uint32_t id = 63u - (p9 & 63u);
          const uint32_t hh = id >> 5, i = id & 31u;
          const uint32_t osw = (static_cast<uint32_t>(t) & (Smem::kSwz & ~1u)) | hh;
          const int c = static_cast<int>(32 * hh + (i ^ osw));
          const float4 x = ldg_logits4(grow + 4 * c);
          const float4 cc = *reinterpret_cast<const float4*>(sm.cterm + 4 * c);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float xe = lane4(x, e);
            if (!(approx_biased(xe, lane4(cc, e)) < bound)) {
              const float sg = exact_sigmoid(xe);
              insert8p(T, S, pack(key_of(__fadd_rn(sg, sm.bias[4 * c + e])), 4 * c + e), sg);
            }
          }
        }
      } else {
        uint64_t Te[kK];
        float Se[kK];
        exact_top8_biased<LT>(grow, sm.cterm, sm.bias, bound, nonfinite, Te, Se);
#pragma unroll
        for (int q = 0; q < kK; ++q) {
          T[q] = Te[q];
          S[q] = Se[q];
        }
      }

      // ======== phase 3: weights, fold, store ===================================================
      int id[kK];
      float w[kK];
      {
        float norm = 0.0f;
#pragma unroll
        for (int s = 0; s < kK; ++s) {
          id[s] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(T[s]));
          norm = __fadd_rn(norm, S[s]);
        }
#pragma unroll
        for (int s = 0; s < kK; ++s) {
          float x = p.renormalize ? __fdiv_rn(S[s], norm) : S[s];
          if (p.scaling != 1.0f) x = __fmul_rn(x, p.scaling);
          w[s] = x;
        }
      }
      if constexpr (FOLD == kFoldNone) {
        if (valid) {
          float4* ow = reinterpret_cast<float4*>(p.out_w + orow * kK);
          int4* oi = reinterpret_cast<int4*>(p.out_ids + orow * kK);
          ow[0] = make_float4(w[0], w[1], w[2], w[3]);
          ow[1] = make_float4(w[4], w[5], w[6], w[7]);
          oi[0] = make_int4(id[0], id[1], id[2], id[3]);
          oi[1] = make_int4(id[4], id[5], id[6], id[7]);
        }
      } else {
        // ---- DeepSeek-V4 fold: stable sort by weight (desc, slot asc); the key carries the
        // expert id below the slot, the weight rides along ------------------------------------
        uint64_t wk[kK];
        float fw[kK];
#pragma unroll
        for (int s = 0; s < kK; ++s) {
          wk[s] = (static_cast<uint64_t>(key_of(w[s])) << 32) |
                  (static_cast<uint64_t>(kK - 1 - s) << 8) | (static_cast<uint32_t>(id[s]) & 0xFFu);
          fw[s] = w[s];
        }
        sort8p(wk, fw);
        int fidx[kK];
#pragma unroll
        for (int s = 0; s < kK; ++s) fidx[s] = static_cast<int>(wk[s] & 0xFFu);

        // argmins from the truncated losses in shared memory, then every scale (and confidence
        // loss) gathered from L2 at once
        int fpos[kK], ftgt[kK];
#pragma unroll
        for (int j2 = P; j2 < kK; ++j2) {
          const int src = fidx[j2];
          int pos = 0;
          if constexpr (!Smem::kSmemTable) {
            // the fp32 argmin from L2: the first minimal loss below FLT_MAX
            float lv[P];
#pragma unroll
            for (int q = 0; q < P; ++q) lv[q] = __ldg(selg + src * kE + fidx[q]);
            float bf = FLT_MAX;
#pragma unroll
            for (int q = 0; q < P; ++q) {
              pos = lv[q] < bf ? q : pos;
              bf = lv[q] < bf ? lv[q] : bf;
            }
          } else {
          const uint16_t* lrow = sm.loss_hi + src * kE;
          float hb = __int_as_float(0x7F800000);  // +inf
          bool tie = false;
#pragma unroll
          for (int q = 0; q < P; ++q) {
            const float v = __uint_as_float(static_cast<uint32_t>(lrow[fidx[q]]) << 16);
            tie = v == hb || (v < hb ? false : tie);
            pos = v < hb ? q : pos;
            hb = v < hb ? v : hb;
          }
          if (!(hb <= __uint_as_float(kFltMaxHi))) {
            pos = 0;  // no loss below FLT_MAX (+inf, NaN): the first retained expert
          } else if (tie || hb == __uint_as_float(kFltMaxHi)) {
            // not decided by the truncated losses: the fp32 argmin (first minimal loss below
            // FLT_MAX)
            float bf = FLT_MAX;
            pos = 0;
#pragma unroll
            for (int q = 0; q < P; ++q) {
              const float c = __ldg(selg + src * kE + fidx[q]);
              if (c < bf) {
                bf = c;
                pos = q;
              }
            }
          }
          }
          int tgt = fidx[0];
#pragma unroll
          for (int q = 1; q < P; ++q)
            if (q == pos) tgt = fidx[q];
          fpos[j2] = pos;
          ftgt[j2] = tgt;
        }
        float scv[kK], clv[kK];
#pragma unroll
        for (int j2 = P; j2 < kK; ++j2) {
          scv[j2] = __ldg(coeff + fidx[j2] * kE + ftgt[j2]);
          clv[j2] = blend ? __ldg(conf + fidx[j2] * kE + ftgt[j2]) : 0.0f;
        }
        float ft[kK], ff[kK];
#pragma unroll
        for (int j2 = P; j2 < kK; ++j2) {
          float cf = 1.0f, lost = 0.0f;
          if (blend) {
            cf = fminf(fmaxf(__fsub_rn(1.0f, clv[j2]), 0.0f), 1.0f);
            lost = __fmul_rn(fw[j2], __fsub_rn(1.0f, cf));
          }
          ft[j2] = __fmul_rn(__fmul_rn(fw[j2], scv[j2]), cf);
          ff[j2] = lost;
        }
        float acc[P];
#pragma unroll
        for (int q = 0; q < P; ++q) {
          float a = fw[q];
#pragma unroll
          for (int j2 = P; j2 < kK; ++j2)
            if (fpos[j2] == q) a = __fadd_rn(a, ft[j2]);
          acc[q] = a;
        }
        if (blend) {
          float fallback = 0.0f, rsum = 0.0f;
#pragma unroll
          for (int j2 = P; j2 < kK; ++j2) fallback = __fadd_rn(fallback, ff[j2]);
#pragma unroll
          for (int q = 0; q < P; ++q) rsum = __fadd_rn(rsum, fw[q]);
          if (rsum > 1.0e-20f) {
            const float fs = __fdiv_rn(fallback, rsum);
#pragma unroll
            for (int q = 0; q < P; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(fw[q], fs));
          }
        }
        float scale = 1.0f;
        const bool l2mode = p.renorm_mode == EXF_RENORM_ROUTER_L2;
        if (l2mode) {
          float l2 = 0.0f, f2 = 0.0f;
#pragma unroll
          for (int s = 0; s < kK; ++s) l2 = __fadd_rn(l2, __fmul_rn(w[s], w[s]));
#pragma unroll
          for (int q = 0; q < P; ++q) f2 = __fadd_rn(f2, __fmul_rn(acc[q], acc[q]));
          if (f2 > 1.0e-20f) scale = __fsqrt_rn(__fdiv_rn(l2, f2));
        }
        if (valid) {
#pragma unroll
          for (int q = 0; q < P; ++q) {
            p.out_w[orow * P + q] = l2mode ? __fmul_rn(acc[q], scale) : acc[q];
            p.out_ids[orow * P + q] = fidx[q];
          }
        }
      }
    }
    // this layer's table reads are done before the next layer's tables are written
    __syncthreads();
    ks = ke;
  }

  // copies still in flight after a time-out land before the CTA's shared memory is released
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s)
      if (sm.seq[s] > sm.done[s])
        bar_wait(&sm.bar[s], static_cast<uint32_t>(sm.seq[s] / kSlots) & 1u);
  }
}

template <int FOLD, int P, typename LT>
cudaError_t launch_biased_l(const RouterParams& p, cudaStream_t stream) {
  auto kern = router_biased_kernel<FOLD, P, LT>;
  constexpr size_t smem = biased_smem_bytes<FOLD, LT>();
  static std::mutex mu;
  static bool allowed[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!allowed[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      allowed[dev] = true;
    }
  }
  int64_t blocks = (p.tokens + kRows - 1) / kRows * p.layers;
  const int sms = sm_count();
  if (sms > 0 && blocks > sms) blocks = sms;
  if (blocks < 1) blocks = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int FOLD, int P>
cudaError_t launch_biased(const RouterParams& p, cudaStream_t stream) {
  switch (p.logit_dtype) {
    case EXF_F32: return launch_biased_l<FOLD, P, float>(p, stream);
    case EXF_BF16: return launch_biased_l<FOLD, P, __nv_bfloat16>(p, stream);
    default: return launch_biased_l<FOLD, P, __half>(p, stream);
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

bool router_biased_eligible(int experts, int scoring, int fold, const RouterParams& p) {
  return experts == kE && scoring == EXF_SIGMOID && fold != kFoldQwen3 && p.top_k == kK &&
         p.target_k >= 1 && p.target_k <= kK && aligned16(p.logits) &&
         (fold != kFoldNone || (aligned16(p.out_w) && aligned16(p.out_ids))) &&
         (fold == kFoldNone || aligned16(p.sel_loss));
}

cudaError_t launch_router_biased(int fold, const RouterParams& p, cudaStream_t stream) {
  if (fold == kFoldNone) return launch_biased<kFoldNone, kK>(p, stream);
  switch (p.target_k) {
    case 1: return launch_biased<kFoldDsv4, 1>(p, stream);
    case 2: return launch_biased<kFoldDsv4, 2>(p, stream);
    case 3: return launch_biased<kFoldDsv4, 3>(p, stream);
    case 4: return launch_biased<kFoldDsv4, 4>(p, stream);
    case 5: return launch_biased<kFoldDsv4, 5>(p, stream);
    case 6: return launch_biased<kFoldDsv4, 6>(p, stream);
    case 7: return launch_biased<kFoldDsv4, 7>(p, stream);
    default: return launch_biased<kFoldDsv4, 8>(p, stream);
  }
}

}  // namespace exf
