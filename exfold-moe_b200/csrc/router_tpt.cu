// Router top-8 (+ Qwen3 prefill fold) for 128 experts, one token per thread (sm_100a).
//
// router_tpt_kernel serves the prefill router of 128-expert softmax models (top-8, renormalised),
// optionally fused with the ExFold prefill fold (exfold/qwen3/kernels.py:9-94 semantics):
//   * The logits stream through a ring of 10 tile slots (32 tokens x 512 B each) per CTA, filled
//     by bulk copies (cp.async.bulk, mbarrier completion) and shared by 10 warps (168
//     registers each; 10 rather than 8 warps: 2.8 instead of 3.5 tiles per warp and launch at
//     131072 tokens, 23.1 instead of 24.6 us per launch; 16-bit logits: 20 slots of 8 KB shared
//     by 14 warps): a warp takes
//     the next tile of the layer, ranks it, and refills the slot with the tile 10 places ahead
//     as soon as its selection has read it, publishing the tile index so that the slot's next
//     reader knows which barrier phase to wait for.  Lane t owns token t of the tile and reads
//     its row in the chunk order i ^ (t & 7): rows are 512 B apart, so the 8 lanes of each
//     quarter-warp hit 8 different 16-byte bank quads and the reads are conflict-free.  bf16 /
//     fp16 logits: 8 KB tiles in twice the slots, 8-byte chunks in the order i ^ (t & 15), and
//     exact group-maximum keys (below), so ties need no fallback.
//   * The 32 groups of 4 consecutive columns give 32 group maxima (three-input max.f32; for bf16
//     logits a packed max.bf16x2 first); each is keyed as its raw bits compared as a signed
//     integer (positive floats rank by value above every negative one), with the low 5 bits
//     replaced by the group's slot, and the keys go through a sorting network (4 x 19-comparator sorts, 3 merges) whose top 8 name the 8
//     groups with the largest maxima.  Those groups are reloaded (their exact maxima are then
//     in descending order unless two truncated keys tie; then they are sorted as (key desc,
//     column asc)), and every other element of those groups that reaches the 8th maximum is
//     inserted.  When the 9th largest maximum (the largest value the merges drop) is below the
//     8th in its truncated key and the 8th maximum is positive, this is the exact top 8 (every
//     element that reaches it lies in those groups; no zeros, so -0 and +0 cannot tie; the named
//     maxima are then positive floats, compared as floats).  For
//     16-bit logits the truncation loses nothing and equal keys sort by group, so only the sign
//     of the 8th maximum and NaN rows decide.  Other
//     tokens (a group outside the 8 close to the 8th maximum, zeros among the candidates, NaN)
//     insert every element of every group that reaches the truncated bound instead (every
//     element, for a row with a NaN): exact, slower.
//   * The fold's loss lookups (4 per omitted route) go to a shared-memory copy of the layer's
//     128 x 128 loss table, loaded once per CTA and layer: scattered 4-byte reads from L1/L2 cost
//     one pass per distinct line (32 per warp instruction), shared memory only its bank
//     conflicts.  The one scale per omitted route is read from L2 while the weights are
//     computed.  Each CTA ranks a contiguous range of the (layer, tile) sequence, so it loads
//     one table per layer boundary it crosses.
#include <float.h>

#include <mutex>
#include <type_traits>

#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"
#include "exf_tile.cuh"

namespace exf {
namespace {
using namespace tile;

constexpr int kE = 128;
constexpr int kK = 8;
#ifndef EXF_TPT_SLOTS
#define EXF_TPT_SLOTS 10
#endif
constexpr int kRows = 32;                // tokens per tile: one per lane
// Warps per CTA, each ranking one tile at a time.  A warp's tile latency bounds the kernel, so
// more warps help until the register file runs out (registers are allocated per SM sub-partition,
// so 9-12 warps cap a thread at 168 registers and 13-16 at 128): 10 for fp32 logits (12-16
// measured slower per launch: they share 10 slots), 14 for 16-bit logits with their 20 slots
// (21.7 us per 131072-token launch against 23.6 us with 10 warps).
template <typename LT>
constexpr int tpt_warps() {
  return sizeof(LT) == 4 ? 10 : 14;
}

// Tile slots per CTA (a ring shared by its warps): 16 KB tiles of fp32 logits, 8 KB of bf16 /
// fp16 logits, so the 16-bit ring has twice the slots in the same shared memory.
template <typename LT>
struct TptSmem {
  static constexpr int kSlots = sizeof(LT) == 4 ? EXF_TPT_SLOTS : 2 * EXF_TPT_SLOTS;
  // Lane t reads the 16-byte (fp32) / 8-byte (16-bit) group chunks of its row in the order
  // u ^ (t & kSwz): rows are 512 / 256 bytes apart, so each quarter-warp (16-byte loads) or
  // half-warp (8-byte loads) hits distinct banks.
  static constexpr int kSwz = sizeof(LT) == 4 ? 7 : 15;
  LT tile[kSlots][kRows * kE];
  float loss[kE * kE];     // the current layer's selection-loss table (fold only)
  uint64_t bar[kSlots];    // tile copies
  uint64_t tbar;           // table copies
  long long seq[kSlots];   // CTA-local index of the tile whose copy the slot's barrier tracks
  long long done[kSlots];  // CTA-local index of the last tile whose copy was waited for
  int next;                // next tile of the current layer to hand out
  int failed;              // a wait timed out: the remaining tiles are marked, not ranked
};
template <typename LT>
constexpr size_t tpt_smem_bytes() {
  return sizeof(TptSmem<LT>) + 128;  // + alignment slack
}
static_assert(tpt_smem_bytes<float>() <= 232448, "router_tpt: shared memory over the limit");
static_assert(tpt_smem_bytes<__nv_bfloat16>() <= 232448, "router_tpt: shared memory over the limit");

// Exact top 8 of one row by insertion of every element (key at least lb) of every group whose
// maximum reaches lb; -0 ranks equal to +0.  Out of line: rarely taken, and kept out of the
// instruction cache of the hot loop.
template <typename LT>
__device__ __noinline__ void exact_top8(const LT* rowp, int swz, uint32_t lb, uint64_t* out) {
  uint64_t T[kK];
#pragma unroll
  for (int q = 0; q < kK; ++q) T[q] = 0;
#pragma unroll 1
  for (int u = 0; u < 32; ++u) {
    const int cbase = 4 * (u ^ swz);
    const float4 v = load_logits4(rowp + cbase);
    const uint32_t k[4] = {key_of(v.x), key_of(v.y), key_of(v.z), key_of(v.w)};
    if (max(max(k[0], k[1]), max(k[2], k[3])) < lb) continue;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (k[e] >= lb) insert8(T, pack(k[e], cbase + e));
  }
#pragma unroll
  for (int q = 0; q < kK; ++q) out[q] = T[q];
}

// Copies local tiles [from, kSlots) (of the first segment of a one-layer launch) into their
// slots and publishes each tile index after its copy is issued.
template <typename LT>
__device__ __noinline__ void issue_held_back(TptSmem<LT>& sm, const LT* logits, int64_t g0,
                                             int64_t tpl, int64_t tokens, int from, int64_t nk) {
  constexpr int kSlots = TptSmem<LT>::kSlots;
  for (int s = from; s < kSlots && s < nk; ++s) {
    const int64_t l = (g0 + s) / tpl, tl = (g0 + s) - l * tpl;
    const int64_t rows = tokens - tl * kRows < kRows ? tokens - tl * kRows : kRows;
    const uint32_t bytes = static_cast<uint32_t>(rows * kE * sizeof(LT));
    bar_expect(&sm.bar[s], bytes);
    bulk_load(sm.tile[s], logits + (l * tokens + tl * kRows) * kE, bytes, &sm.bar[s]);
    __threadfence_block();
    *reinterpret_cast<volatile long long*>(&sm.seq[s]) = s;
  }
}

template <int FOLD, int P, typename LT>
__global__ void __launch_bounds__(tpt_warps<LT>() * 32, 1) router_tpt_kernel(const RouterParams p) {
  extern __shared__ uint8_t tpt_raw[];
  using Smem = TptSmem<LT>;
  constexpr int kSlots = Smem::kSlots;
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(tpt_raw) + 127) &
                                      ~static_cast<uintptr_t>(127));
  const LT* logits = static_cast<const LT*>(p.logits);
  const int t = threadIdx.x & 31;
  const int swz = t & Smem::kSwz;
  const int64_t tokens = p.tokens;
  // Tiles never straddle a layer (the last one of a layer may be short): global tile g is tile
  // g % tpl of layer g / tpl.  This CTA ranks the contiguous range [g0, g0 + nk), so it crosses
  // few layer boundaries; its local tile k is global tile g0 + k.
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
  // Launched as a programmatic dependent of the previous kernel in the stream: let the next
  // launch's CTAs take SMs as this grid's CTAs exit, and wait here until the previous grid has
  // completed and its writes are visible (a no-op for an ordinary launch).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // A one-layer launch starts with kFirstSlots tile copies and issues the other slots once its
  // first tile is in: with every slot of every CTA issued at once (24 MB over the GPU) each copy
  // completes only when the whole burst has drained, about 3 us after the start.  131072-token
  // layer: 23.28 -> 22.16 us fp32, 21.69 -> 20.61 us bf16 (2 to 6 first slots measured, 4 best).
  // A launch over several layers has its start amortised and issues every slot at once.
  constexpr int kFirstSlots = 4;
  const int first_slots = p.layers == 1 && kFirstSlots < kSlots ? kFirstSlots : kSlots;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      bar_init(&sm.bar[s]);
      sm.seq[s] = -1;
      sm.done[s] = -1;
    }
    bar_init(&sm.tbar);
    sm.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (FOLD != kFoldNone && nk > 0) {  // the first layer's table ahead of the first tiles
      bar_expect(&sm.tbar, kE * kE * sizeof(float));
      bulk_load(sm.loss, p.sel_loss + (g0 / tpl) * kE * kE, kE * kE * sizeof(float), &sm.tbar);
    }
    for (int s = 0; s < first_slots && s < nk; ++s) {
      sm.seq[s] = s;
      issue(s);
    }
  }
  __syncthreads();

  // thread 0: phase (0, 1, ...) of the table copy issued and not yet waited for (-1: none)
  int64_t table_pending = FOLD != kFoldNone && nk > 0 ? 0 : -1;
  // layer segments of the range: [ks, ke) of local tiles in layer l, the phase-th segment
  int phase = 0;
  for (int64_t ks = 0; ks < nk; ++phase) {
    const int64_t l = (g0 + ks) / tpl;
    const int64_t ke = ((l + 1) * tpl - g0) < nk ? (l + 1) * tpl - g0 : nk;
    const int n = static_cast<int>(ke - ks);
    // ---- this layer's loss table into shared memory (all reads of the previous one are done)
    if (threadIdx.x == 0) {
      sm.next = 0;
      if (FOLD != kFoldNone && phase > 0 && !*failed) {
        bar_expect(&sm.tbar, kE * kE * sizeof(float));
        bulk_load(sm.loss, p.sel_loss + l * kE * kE, kE * kE * sizeof(float), &sm.tbar);
        table_pending = phase;
      }
    }
    __syncthreads();
    if (FOLD != kFoldNone) {
      bool ok = !*failed && bar_wait(&sm.tbar, static_cast<uint32_t>(phase) & 1u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) *failed = 1;
      if (threadIdx.x == 0 && ok) table_pending = -1;
    }
    const float* coeff = p.coeff + l * kE * kE;

    while (true) {
      int j = 0;
      if (t == 0) j = atomicAdd(&sm.next, 1);
      j = __shfl_sync(0xffffffffu, j, 0);
      if (j >= n) break;
      const int64_t k = ks + j;
      const int slot = static_cast<int>(k % kSlots);
      // the slot must hold tile k's copy before its barrier parity means anything: the lane that
      // refills a slot publishes the tile index after issuing the copy
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
      // the slots held back at the start of a one-layer launch, once its first tile is in (out
      // of line: the tile loop's code stays as small as without it)
      if (k == 0 && ok && t == 0 && first_slots < kSlots)
        issue_held_back<LT>(sm, logits, g0, tpl, tokens, first_slots, nk);
      const int64_t tok = (g0 + k - l * tpl) * kRows + t;
      const bool valid = tok < tokens;
      const int64_t row = l * tokens + tok;
      const LT* rowp = sm.tile[slot] + t * kE;
      uint64_t T[kK];

      // ======== phase 1: the selection, the only part that reads the tile =====================
      if (ok) {
        // ---- group maxima (step u reads group u ^ swz: columns 4 (u ^ swz) .. + 3) ------------
        // A float maximum keyed once equals the key maximum except that -0 may stand for +0
        // (harmless: zeros never reach the fast path's theta, and the exact path merges them);
        // a NaN makes the group's key all ones, which the exact path below takes over.  The key
        // keeps its high 27 bits; the low 5 hold 31 - u (fp32: a constant per step) or, for
        // 16-bit logits, 31 - group, so that equal keys sort by ascending group, i.e. ascending
        // column.
        // Keys are the raw bits of the float maxima compared as signed integers: positive floats
        // (and +inf, and the canonical NaN that max.NaN returns, above +inf) rank by value above
        // every negative one; negative floats rank in reverse among themselves, which only the
        // exact path sees (the fast path needs a positive 8th maximum).
        constexpr bool kExactKeys = sizeof(LT) == 2;
        int32_t pk[32];
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t grp = static_cast<uint32_t>((8 * s + i) ^ swz);
            float m;
            if constexpr (std::is_same<LT, __nv_bfloat16>::value) {
              // bf16: the packed maximum of the two pairs, then of its halves (bf16 -> fp32 is
              // exact and monotone, so this is the maximum of the converted values; NaN
              // propagates as the canonical NaN)
              const uint2 u = *reinterpret_cast<const uint2*>(rowp + 4 * grp);
              uint32_t r2;
              asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r2) : "r"(u.x), "r"(u.y));
              m = fmax_nan(__uint_as_float(r2 << 16), __uint_as_float(r2 & 0xFFFF0000u));
            } else {
              const float4 v = load_logits4(rowp + 4 * grp);
              m = fmax_nan(fmax3_nan(v.x, v.y, v.z), v.w);
            }
            pk[8 * s + i] = static_cast<int32_t>((__float_as_uint(m) & ~31u) |
                                                 (31u - (kExactKeys ? grp : 8 * s + i)));
          }
        sort8<int32_t, cxs32>(pk);
        sort8<int32_t, cxs32>(pk + 8);
        sort8<int32_t, cxs32>(pk + 16);
        sort8<int32_t, cxs32>(pk + 24);
        int32_t p9 = INT32_MIN;  // the 9th largest packed maximum
        merge8s(pk, pk + 8, p9);
        merge8s(pk + 16, pk + 24, p9);
        merge8s(pk, pk + 16, p9);

        // ---- the 8 named groups: exact maxima, sorted by (key desc, column asc) -------------
        // A 16-bit logit converted to fp32 has its low 16 bits all zeros, so for 16-bit logits
        // the truncated keys are exact: the named groups' maxima are in (value desc, column asc)
        // order, and an element of any other group either is below the 8th maximum or equals it
        // at a higher column, so it is not in the top 8.  fp32 keys lose their low 5 bits: the
        // order holds when the truncated keys differ, and the other groups are excluded when the
        // 9th truncated maximum is below the 8th.  The fast path needs the 8th truncated maximum
        // positive (no zeros or negative values among the candidates) and no NaN in the row;
        // the named maxima are then positive, their order keys are their bits with the sign bit
        // set, and every comparison below is a float comparison of positive values.
        const bool apart = kExactKeys || (p9 >> 5) < (pk[kK - 1] >> 5);
        const bool nan_row = pk[0] > 0x7F80001F;  // above +inf: max.NaN found a NaN
        const bool fast = apart && pk[kK - 1] >= 32 && !nan_row;
        float4 xv[kK];
        int cb[kK], emax[kK];
#pragma unroll
        for (int i = 0; i < kK; ++i) {
          const uint32_t slot = 31u - (static_cast<uint32_t>(pk[i]) & 31u);
          cb[i] = 4 * static_cast<int>(kExactKeys ? slot : slot ^ static_cast<uint32_t>(swz));
          const float4 v = load_logits4(rowp + cb[i]);
          xv[i] = v;
          const float m = fmaxf(fmax3(v.x, v.y, v.z), v.w);
          emax[i] = v.x == m ? 0 : (v.y == m ? 1 : (v.z == m ? 2 : 3));
          T[i] = pack(__float_as_uint(m) | 0x80000000u, cb[i] + emax[i]);
        }
        if (!kExactKeys) {
          uint32_t dmin = 0xFFFFFFFFu;  // truncated keys differ where the xor reaches bit 5
#pragma unroll
          for (int i = 0; i + 1 < kK; ++i)
            dmin = min(dmin, static_cast<uint32_t>(pk[i] ^ pk[i + 1]));
          if (dmin < 32u) sort8<uint64_t, cx64>(T);
        }

        if (fast) {
          // other elements of the named groups that reach theta: a mask over the 32 (group,
          // element) sites, each inserted after a reload from the tile (typically 0-2 of them)
          const float theta = __uint_as_float(static_cast<uint32_t>(T[kK - 1] >> 32) & 0x7FFFFFFFu);
          uint32_t xm = 0, mm = 0, slo = 0, shi = 0;
#pragma unroll
          for (int i = 0; i < kK; ++i) {
            const uint32_t grp = static_cast<uint32_t>(cb[i]) >> 2;
            if (i < 6)
              slo |= grp << (5 * i);
            else
              shi |= grp << (5 * (i - 6));
            xm |= (xv[i].x >= theta ? 1u : 0u) << (4 * i);
            xm |= (xv[i].y >= theta ? 2u : 0u) << (4 * i);
            xm |= (xv[i].z >= theta ? 4u : 0u) << (4 * i);
            xm |= (xv[i].w >= theta ? 8u : 0u) << (4 * i);
            mm |= 1u << (4 * i + emax[i]);
          }
          xm &= ~mm;
          while (xm) {
            const int site = __ffs(xm) - 1;
            xm &= xm - 1;
            const int i = site >> 2;
            const uint32_t grp = (i < 6 ? slo >> (5 * i) : shi >> (5 * (i - 6))) & 31u;
            const int col = 4 * static_cast<int>(grp) + (site & 3);
            insert8(T, pack(__float_as_uint(logit_f32<LT>(rowp[col])) | 0x80000000u, col));
          }
        } else if (valid) {
          // exact insertion over every element of every group whose maximum reaches the bound:
          // the 8th truncated maximum rounded down in value (a row with a NaN: every element)
          const uint32_t b8 = static_cast<uint32_t>(pk[kK - 1]);
          const uint32_t lb = pk[kK - 1] >= 0 ? (b8 & ~31u) | 0x80000000u : ~(b8 | 31u);
          uint64_t Te[kK];
          exact_top8<LT>(rowp, swz, nan_row ? 0u : lb, Te);
#pragma unroll
          for (int q = 0; q < kK; ++q) T[q] = Te[q];
        }
      }

      // ---- the tile is consumed: refill its slot with local tile k + kSlots ------------------
      // (generic-proxy accesses to the slot are ordered before the bulk copy that overwrites it)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (t == 0 && ok && k + kSlots < nk) {
        issue(k + kSlots);
        __threadfence_block();
        seq[slot] = k + kSlots;
      }

      // ======== phase 2: weights, fold and store from registers and the tables ===============
      if (ok) {
        int id[kK];
        float val[kK];
#pragma unroll
        for (int s = 0; s < kK; ++s) {
          id[s] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(T[s]));
          val[s] = float_of_key(static_cast<uint32_t>(T[s] >> 32));
        }
        // fold targets: slot j >= P folds onto the first retained q of minimal loss; the scales
        // of the targets are gathered from L2 while the weights are computed
        float best[kK], scale[kK];
        int fp[kK];
        if (FOLD != kFoldNone) {
#pragma unroll
          for (int j = P; j < kK; ++j) {
            const float* lrow = sm.loss + id[j] * kE;
            float b = lrow[id[0]];
            int pos = 0, tgt = id[0];
#pragma unroll
            for (int q = 1; q < P; ++q) {
              const float lq = lrow[id[q]];
              if (lq < b) {
                b = lq;
                pos = q;
                tgt = id[q];
              }
            }
            best[j] = b;
            fp[j] = pos;
            scale[j] = __ldg(coeff + id[j] * kE + tgt);
          }
        }

        float w[kK];
        {
          float norm = 0.0f;
#pragma unroll
          for (int s = 0; s < kK; ++s) {
            w[s] = exact_exp_le88(__fsub_rn(val[s], val[0]));  // val[s] <= val[0], or NaN
            norm = __fadd_rn(norm, w[s]);
          }
#pragma unroll
          for (int s = 0; s < kK; ++s) {
            float x = __fdiv_rn(w[s], norm);
            if (p.scaling != 1.0f) x = __fmul_rn(x, p.scaling);
            w[s] = x;
          }
        }

        if (FOLD == kFoldNone) {
          if (valid) {
            float4* ow = reinterpret_cast<float4*>(p.out_w + row * kK);
            int4* oi = reinterpret_cast<int4*>(p.out_ids + row * kK);
            ow[0] = make_float4(w[0], w[1], w[2], w[3]);
            ow[1] = make_float4(w[4], w[5], w[6], w[7]);
            oi[0] = make_int4(id[0], id[1], id[2], id[3]);
            oi[1] = make_int4(id[4], id[5], id[6], id[7]);
          }
        } else {
          // ---- Qwen3 prefill fold: transfers added to their targets in slot order -------------
          float ft[kK];
#pragma unroll
          for (int j = P; j < kK; ++j) ft[j] = __fmul_rn(w[j], best[j] < 1.0e30f ? scale[j] : 0.0f);
          float acc[P];
#pragma unroll
          for (int q = 0; q < P; ++q) {
            float a = w[q];
#pragma unroll
            for (int j = P; j < kK; ++j) a = __fadd_rn(a, q == fp[j] ? ft[j] : 0.0f);
            acc[q] = a;
          }
          if (valid) {
            if constexpr (P == 4) {
              *reinterpret_cast<float4*>(p.out_w + row * P) =
                  make_float4(acc[0], acc[1], acc[2], acc[3]);
              *reinterpret_cast<int4*>(p.out_ids + row * P) =
                  make_int4(id[0], id[1], id[2], id[3]);
            } else {
#pragma unroll
              for (int q = 0; q < P; ++q) {
                p.out_w[row * P + q] = acc[q];
                p.out_ids[row * P + q] = id[q];
              }
            }
          }
        }
      } else if (valid) {
        // the tile never arrived: mark the routes invalid rather than leave stale values
        const int width = FOLD == kFoldNone ? kK : P;
        for (int q = 0; q < width; ++q) {
          p.out_w[row * width + q] = 0.0f;
          p.out_ids[row * width + q] = -1;
        }
      }
    }
    // this layer's table reads are ordered before the copy of the next layer's table
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    ks = ke;
  }

  // copies still in flight after a time-out land before the CTA's shared memory is released
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s)
      if (sm.seq[s] > sm.done[s])
        bar_wait(&sm.bar[s], static_cast<uint32_t>(sm.seq[s] / kSlots) & 1u);
    if (table_pending >= 0) bar_wait(&sm.tbar, static_cast<uint32_t>(table_pending) & 1u);
  }
}

template <int FOLD, int P, typename LT>
cudaError_t launch_tpt_l(const RouterParams& p, cudaStream_t stream) {
  auto kern = router_tpt_kernel<FOLD, P, LT>;
  constexpr size_t smem = tpt_smem_bytes<LT>();
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
  cfg.blockDim = dim3(tpt_warps<LT>() * 32);
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
cudaError_t launch_tpt(const RouterParams& p, cudaStream_t stream) {
  switch (p.logit_dtype) {
    case EXF_F32: return launch_tpt_l<FOLD, P, float>(p, stream);
    case EXF_BF16: return launch_tpt_l<FOLD, P, __nv_bfloat16>(p, stream);
    default: return launch_tpt_l<FOLD, P, __half>(p, stream);
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

bool router_tpt_eligible(int experts, int scoring, int fold, const RouterParams& p) {
  return experts == kE && scoring == EXF_SOFTMAX && fold != kFoldDsv4 && p.top_k == kK &&
         p.renormalize && p.target_k >= 1 && p.target_k <= kK && aligned16(p.logits) &&
         aligned16(p.out_w) && aligned16(p.out_ids) &&
         (fold == kFoldNone || aligned16(p.sel_loss));
}

cudaError_t launch_router_tpt(int fold, const RouterParams& p, cudaStream_t stream) {
  if (fold == kFoldNone) return launch_tpt<kFoldNone, kK>(p, stream);
  switch (p.target_k) {
    case 1: return launch_tpt<kFoldQwen3, 1>(p, stream);
    case 2: return launch_tpt<kFoldQwen3, 2>(p, stream);
    case 3: return launch_tpt<kFoldQwen3, 3>(p, stream);
    case 4: return launch_tpt<kFoldQwen3, 4>(p, stream);
    case 5: return launch_tpt<kFoldQwen3, 5>(p, stream);
    case 6: return launch_tpt<kFoldQwen3, 6>(p, stream);
    case 7: return launch_tpt<kFoldQwen3, 7>(p, stream);
    default: return launch_tpt<kFoldQwen3, 8>(p, stream);
  }
}

}  // namespace exf
