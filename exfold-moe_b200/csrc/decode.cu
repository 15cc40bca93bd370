// Decode expert budget kernels (sm_100a).
//
// decode_kernel is one CTA of 1024 threads doing the whole transform for a decode batch:
//   1. importance[e] = sum over routes of w * norm[e] as 2^-32 fixed point in int64 (shared-
//      memory 64-bit atomics into per-warp-group copies, then summed: exact, so independent of
//      the order the atomics land in), or
//      read from a caller-reduced vector (batch sharded over GPUs), or skipped when the caller
//      gives the subset explicitly;
//   2. order = experts by (importance desc, expert asc), E/ (1024/E) comparisons per thread;
//   3. per-expert target table: one warp per source expert, the subset's losses read from the
//      L2-resident loss row by all 32 lanes, argmin by a (loss, position) shuffle reduction that
//      reproduces the sequential strict-< scan of the reference;
//   4. apply the table to every route.
// A decode batch is at most a few thousand routes (B x k), so the single CTA keeps every phase
// on chip and the transform costs one launch.  For E <= 128 the loss and scale tables (2 x 64 KB
// at E = 128) are bulk-copied into shared memory at the start (plain and sharded decode), so that
// the copy overlaps phases 1 and 2 and phase 3 reads them on chip instead of making two dependent
// L2 round trips.
// For a batch sharded over GPUs (kImportanceExchanged) phase 1 is followed by an exchange with the
// peer ranks inside the launch: each rank's vector goes to every rank's exchange buffer by NVLink
// peer stores, and every rank sums the R vectors in rank order (exact integers), so one launch per
// layer replaces importance launch + all-reduce + apply launch.
// decode_importance_kernel is the multi-CTA first phase for a sharded or very large batch.
#include <float.h>

#include <mutex>

#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"
#include "exf_tile.cuh"

namespace exf {

constexpr int kDecodeThreads = 1024;
constexpr int kMaxExperts = 1024;
constexpr int kSmemTableExperts = 128;  // tables of at most this many experts go to shared memory



constexpr int kRouteUnroll = 8;   // routes per thread with their loads in flight together
constexpr int kTableBatch = 4;    // source experts per warp with their loss reads in flight together

// Private importance histograms during phase 1: kHistInts 64-bit counters shared out as
// 2048 / E copies, one per group of warps, so that the (compare-and-swap) 64-bit shared atomics
// only collide within a warp; they alias the arrays that phase 1 does not use.
constexpr int kHistLongs = 2048;

struct DecodeSmem {
  long long imp[kMaxExperts];
  float norm[kMaxExperts];
  union {
    long long hist[kHistLongs];
    struct {
      int order[kMaxExperts];
      int rank[kMaxExperts];
      int tgt[kMaxExperts];
      float scale[kMaxExperts];
    };
  };
  unsigned char keep[kMaxExperts];
};
static_assert(sizeof(long long) * kHistLongs <= 4 * 4 * kMaxExperts, "hist alias");

// Sequential strict-< argmin semantics as a (value, position) reduction.
//   Qwen3 (exfold/qwen3/kernels.py:186-212): start from position 0; later NaNs never win, so
//   NaN -> +inf, ties -> first position; a NaN at position 0 wins outright.
//   DeepSeek-V4 (exfold_kernels.cu:175-187): start from FLT_MAX; only values strictly below
//   FLT_MAX qualify; positions of non-positive importance are skipped.
__device__ __forceinline__ void argmin_merge(float& v, int& pos, float ov, int opos) {
  if (ov < v || (ov == v && opos < pos)) {
    v = ov;
    pos = opos;
  }
}

template <typename WT, typename IT>
__device__ void merge_routes(const DecodeParams& p);

// ---- peer exchange: self-validating 8-byte words (see kXchSlots) ------------------------------
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* ptr, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(ptr), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* ptr) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;  // 2 s

// sm.imp holds this rank's vector; afterwards the sum over the ranks.  A word that has not
// arrived within p.wait_ns (2 s by default) leaves the local vector in place and sets
// *p.status = 1: the ranks' subsets then differ, and the exchange buffers must be rebuilt.
__device__ void exchange_importance(const DecodeParams& p, DecodeSmem& sm) {
  __shared__ unsigned long long s_call;
  __shared__ int s_late;
  const int E = p.experts, R = p.world, me = p.rank, tid = threadIdx.x;
  unsigned long long* own = reinterpret_cast<unsigned long long*>(p.peers[me]);
  if (tid == 0) {
    s_call = own[kXchEpoch] + 1;  // written by this rank's previous call (stream order)
    s_late = 0;
  }
  __syncthreads();
  const unsigned long long call = s_call;
  const unsigned long long tag = (call & 0xFFFFFFFFull) << 32;
  const int64_t par = static_cast<int64_t>(call & 1);
  // this rank's words into slot (par, me) of every rank's buffer
  for (int i = tid; i < R * E * 2; i += kDecodeThreads) {
    const int r = i / (2 * E), k = i - r * 2 * E;  // k = 2 e + h
    const unsigned long long v = static_cast<unsigned long long>(sm.imp[k >> 1]);
    const unsigned long long half = (k & 1) ? (v >> 32) : (v & 0xFFFFFFFFull);
    st_relaxed_sys(reinterpret_cast<unsigned long long*>(p.peers[r]) + kXchSlots +
                       ((par * R + me) * E) * 2 + k,
                   tag | half);
  }
  // the sum is staged in hist (free between phases 1 and 2) so that sm.imp changes only if every
  // rank's vector arrived
  for (int e = tid; e < E; e += kDecodeThreads) sm.hist[e] = 0;
  __syncthreads();  // every local read of sm.imp is done before it is overwritten below
  // poll this rank's slots of parity par: one (rank, expert) word pair per thread, so that the
  // first load of every pair is in flight at once; the ranks' values are added into hist[e] with
  // 64-bit shared atomics (modulo 2^64, as the single-GPU sums: any order gives the same sum)
  const unsigned long long limit = p.wait_ns ? p.wait_ns : kDefaultWaitNs;
  const unsigned long long t0 = global_ns();
  bool late = false;
  for (int i = tid; i < R * E && !late; i += kDecodeThreads) {
    const int r = i / E, e = i - r * E;
    const unsigned long long* wp = own + kXchSlots + ((par * R + r) * E + e) * 2;
    unsigned long long lo = ld_relaxed_sys(wp), hi = ld_relaxed_sys(wp + 1);
    // time-bounded, and iteration-bounded too (at least ~4 s of 64 ns sleeps)
    for (uint32_t it = 0; (lo ^ tag) >> 32 || (hi ^ tag) >> 32; ++it) {
      if (global_ns() - t0 > limit || it >= (1u << 26)) {
        late = true;
        break;
      }
      __nanosleep(64);
      lo = ld_relaxed_sys(wp);
      hi = ld_relaxed_sys(wp + 1);
    }
    if (!late)
      atomicAdd(reinterpret_cast<unsigned long long*>(&sm.hist[e]), (hi << 32) | (lo & 0xFFFFFFFFull));
  }
  if (late) atomicExch(&s_late, 1);
  __syncthreads();
  if (s_late == 0)
    for (int e = tid; e < E; e += kDecodeThreads) sm.imp[e] = sm.hist[e];
  if (tid == 0) {
    own[kXchEpoch] = call;
    if (s_late != 0 && p.status) *p.status = 1;
  }
  __syncthreads();
}

// Phase 3 for the source experts of warp `warp`: loss row argmins over the subset and the chosen
// targets' scales, read from `loss` / `coeff` (the shared-memory copies or the global tables).
template <bool kOnChip>
__device__ __forceinline__ float table_load(const float* t, int64_t i) {
  if constexpr (kOnChip) return t[i];
  else return __ldg(t + i);
}
template <bool kOnChip>
__device__ __forceinline__ void target_table(const DecodeParams& p, DecodeSmem& sm,
                                             const float* loss, const float* coeff);

template <typename WT, typename IT, bool MERGE = false>
__global__ void __launch_bounds__(kDecodeThreads, 1) decode_kernel(const DecodeParams p) {
  __shared__ DecodeSmem sm;
  // [2][E][E] loss, then coeff, then the copies' mbarrier, from the first 128-byte boundary of the
  // dynamic shared memory (tables_smem; never for MERGE, whose launch has none).  The declared
  // alignment stays 16 so that the static layout is that of a kernel without the tables (a
  // 128-byte aligned declaration padded it and measured 4 us slower in the fused layer launch).
  extern __shared__ __align__(16) float dsm[];
  float* dtab = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(dsm) + 127) &
                                         ~static_cast<uintptr_t>(127));
  uint64_t* tab_bar = reinterpret_cast<uint64_t*>(dtab + 2 * p.experts * p.experts);
  const int E = p.experts;
  const int D = p.budget;
  const int tid = threadIdx.x;
  const WT* w = static_cast<const WT*>(p.w);
  const IT* ids = static_cast<const IT*>(p.ids);
  // launched as a programmatic dependent: nothing the previous kernel wrote is read before this
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const bool tsm = !MERGE && p.tables_smem != 0;
  if (tsm && tid == 0) {
    const uint32_t bytes = static_cast<uint32_t>(E) * E * sizeof(float);
    tile::bar_init(tab_bar);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tile::bar_expect(tab_bar, 2 * bytes);
    tile::bulk_load(dtab, p.loss, bytes, tab_bar);
    tile::bulk_load(dtab + E * E, p.coeff, bytes, tab_bar);
  }

  // ---- 1. importance ------------------------------------------------------------------------
  const int copies = kHistLongs / E < 32 ? kHistLongs / E : 32;  // >= 2 for E <= 1024
  long long* hist = sm.hist + ((tid >> 5) % copies) * E;
  const bool from_routes = p.source == kImportanceFromRoutes || p.source == kImportanceExchanged;
  // the first batch of routes is loaded before the barrier, beside the norms, and kept in
  // registers for phase 4 (not in the decode fused with the expert layer, whose launch measured
  // 4 us slower per Qwen3 layer with it)
  constexpr bool kEarly = !MERGE;
  WT wr0[kRouteUnroll];
  IT raw0[kRouteUnroll];
  if (kEarly && from_routes) {
#pragma unroll
    for (int j = 0; j < kRouteUnroll; ++j) {
      const int64_t r = j * kDecodeThreads + tid;
      raw0[j] = r < p.routes ? ids[r] : (IT)-1;
      wr0[j] = r < p.routes ? w[r] : from_f32<WT>(0.0f);
    }
  }
  for (int e = tid; e < E; e += kDecodeThreads) {
    sm.imp[e] = (p.source == kImportanceGiven) ? p.importance[e] : 0;
    if (from_routes) sm.norm[e] = __ldg(p.norms + e);
    sm.keep[e] = 0;
  }
  if (from_routes)
    for (int i = tid; i < copies * E; i += kDecodeThreads) sm.hist[i] = 0;
  __syncthreads();
  if (from_routes) {
    for (int64_t base = 0; base < p.routes; base += kRouteUnroll * kDecodeThreads) {
      WT wr[kRouteUnroll];
      int er[kRouteUnroll];
#pragma unroll
      for (int j = 0; j < kRouteUnroll; ++j) {
        const int64_t r = base + j * kDecodeThreads + tid;
        const bool kept = kEarly && base == 0;
        er[j] = kept ? (int)raw0[j] : (r < p.routes ? (int)ids[r] : -1);
        wr[j] = kept ? wr0[j] : (r < p.routes ? w[r] : from_f32<WT>(0.0f));
      }
#pragma unroll
      for (int j = 0; j < kRouteUnroll; ++j) {
        const int e = er[j];
        if (e < 0 || e >= E) continue;
        const long long q = fixed_point(__fmul_rn(to_f32(wr[j]), sm.norm[e]));
        atomicAdd(reinterpret_cast<unsigned long long*>(&hist[e]), (unsigned long long)q);
      }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kDecodeThreads) {
      long long acc = 0;
      for (int c = 0; c < copies; ++c) acc += sm.hist[c * E + e];
      sm.imp[e] = acc;
    }
    __syncthreads();
  }
  if (p.source == kImportanceExchanged) exchange_importance(p, sm);

  // ---- 2. order -------------------------------------------------------------------------------
  if (p.source == kSubsetGiven) {
    for (int e = tid; e < E; e += kDecodeThreads) sm.rank[e] = E;  // not in subset
    __syncthreads();
    for (int q = tid; q < D; q += kDecodeThreads) {
      const int e = p.subset[q];
      const bool ok = e >= 0 && e < E;
      sm.order[q] = ok ? e : 0;  // an out-of-range subset entry never reads outside the tables
      if (ok) sm.keep[e] = 1;
    }
  } else {
    // threads per expert: TP consecutive lanes split the comparison loop
    int tp = 1;
    while (tp < 32 && tp * 2 * E <= kDecodeThreads) tp *= 2;
    const int e = tid / tp;
    const int sub = tid % tp;
    int cnt = 0;
    if (e < E) {
      const long long ie = sm.imp[e];
      for (int o = sub; o < E; o += tp) {
        const long long io = sm.imp[o];
        cnt += (io > ie || (io == ie && o < e)) ? 1 : 0;
      }
    }
    for (int off = tp >> 1; off > 0; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off, tp);
    if (e < E && sub == 0) {
      sm.order[cnt] = e;
      sm.rank[e] = cnt;
    }
    __syncthreads();
    for (int e2 = tid; e2 < E; e2 += kDecodeThreads) {
      const bool in_budget = sm.rank[e2] < D;
      sm.keep[e2] = (p.variant == EXF_QWEN3) ? in_budget : (in_budget && sm.imp[e2] > 0);
    }
  }
  __syncthreads();
  if (p.out_subset) {
    for (int q = tid; q < D; q += kDecodeThreads) p.out_subset[q] = sm.order[q];
  }

  // ---- 3. target table ----------------------------------------------------------------------
  // (from the shared-memory copies of the tables when their copy has landed; a copy that has
  // not landed within the bounded wait leaves the global tables in use)
  bool on_chip = false;
  if (tsm) on_chip = __syncthreads_and(tile::bar_wait(tab_bar, 0) ? 1 : 0) != 0;
  if (on_chip)
    target_table<true>(p, sm, dtab, dtab + E * E);
  else
    target_table<false>(p, sm, p.loss, p.coeff);
  __syncthreads();

  // ---- 4. apply -----------------------------------------------------------------------------
  const bool qwen3 = p.variant == EXF_QWEN3;
  WT* ow = static_cast<WT*>(p.out_w);
  IT* oi = static_cast<IT*>(p.out_ids);
  for (int64_t base = 0; base < p.routes; base += kRouteUnroll * kDecodeThreads) {
    IT raw[kRouteUnroll];
    WT wr[kRouteUnroll];
#pragma unroll
    for (int j = 0; j < kRouteUnroll; ++j) {
      const int64_t r = base + j * kDecodeThreads + tid;
      const bool kept = kEarly && from_routes && base == 0;  // loaded in phase 1
      raw[j] = kept ? raw0[j] : (r < p.routes ? ids[r] : (IT)-1);
      wr[j] = kept ? wr0[j] : (r < p.routes ? w[r] : from_f32<WT>(0.0f));
    }
#pragma unroll
    for (int j = 0; j < kRouteUnroll; ++j) {
      const int64_t r = base + j * kDecodeThreads + tid;
      if (r >= p.routes) continue;
      const int e = (int)raw[j];
      if (e < 0 || e >= E) {
        ow[r] = wr[j];
        oi[r] = raw[j];
      } else if (qwen3) {
        if (sm.keep[e]) {
          ow[r] = wr[j];
          oi[r] = raw[j];
        } else {
          // exfold/qwen3/kernels.py:214-225: the scale is cast to the weight dtype first
          const float s = to_f32(from_f32<WT>(sm.scale[e]));
          ow[r] = from_f32<WT>(__fmul_rn(to_f32(wr[j]), s));
          oi[r] = (IT)sm.tgt[e];
        }
      } else {
        ow[r] = from_f32<WT>(__fmul_rn(to_f32(wr[j]), sm.scale[e]));
        oi[r] = (IT)sm.tgt[e];
      }
    }
  }
  if constexpr (MERGE) merge_routes<WT, IT>(p);
  // a table copy still in flight after a timed-out wait lands before the shared memory is freed
  if (tsm && !on_chip && tid == 0) tile::bar_wait(tab_bar, 0);
}

template <bool kOnChip>
__device__ __forceinline__ void target_table(const DecodeParams& p, DecodeSmem& sm,
                                             const float* loss, const float* coeff) {
  const int E = p.experts;
  const int D = p.budget;
  const int tid = threadIdx.x;
  // A warp builds the rows of kTableBatch source experts at once: their loss reads are issued
  // together, the first and the chosen loss come out of the reduction, and only the scale of
  // each chosen target is a second round trip.
  const int warp = tid >> 5;
  const int lane = tid & 31;
  constexpr int kWarps = kDecodeThreads / 32;
  const bool qwen3 = p.variant == EXF_QWEN3;
  for (int e0 = warp; e0 < E; e0 += kTableBatch * kWarps) {
    int ex[kTableBatch];
    bool act[kTableBatch];
    float v[kTableBatch], first[kTableBatch];
    int pos[kTableBatch];
#pragma unroll
    for (int i = 0; i < kTableBatch; ++i) {
      ex[i] = e0 + i * kWarps;
      act[i] = ex[i] < E && (qwen3 || (!sm.keep[ex[i]] && sm.imp[ex[i]] > 0));
      v[i] = INFINITY;
      pos[i] = 0x7fffffff;
      first[i] = 0.0f;
    }
    for (int q = lane; q < D; q += 32) {
      const int o = sm.order[q];
      const bool use = qwen3 || sm.imp[o] > 0;
      float c[kTableBatch];
#pragma unroll
      for (int i = 0; i < kTableBatch; ++i)
        c[i] = (act[i] && use) ? table_load<kOnChip>(loss, (int64_t)ex[i] * E + o) : 0.0f;
#pragma unroll
      for (int i = 0; i < kTableBatch; ++i) {
        if (!act[i] || !use) continue;
        if (qwen3) {
          // exfold/qwen3/kernels.py:186-212: NaN never wins after position 0
          if (q == 0) first[i] = c[i];
          const float cv = (c[i] != c[i]) ? INFINITY : c[i];
          if (cv < v[i]) {
            v[i] = cv;
            pos[i] = q;
          }
        } else if (c[i] < FLT_MAX && c[i] < v[i]) {  // exfold_kernels.cu:175-187
          v[i] = c[i];
          pos[i] = q;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kTableBatch; ++i) {
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v[i], off);
        const int op = __shfl_xor_sync(0xffffffffu, pos[i], off);
        argmin_merge(v[i], pos[i], ov, op);
      }
      first[i] = __shfl_sync(0xffffffffu, first[i], 0);  // position 0 is lane 0's
    }
    float sc[kTableBatch];
    int tg[kTableBatch];
#pragma unroll
    for (int i = 0; i < kTableBatch; ++i) {
      tg[i] = ex[i];
      sc[i] = 1.0f;
      if (!act[i]) continue;
      if (qwen3) {
        float best = v[i];  // finite whenever a position won on its own
        if (first[i] != first[i] || pos[i] == 0x7fffffff) {
          pos[i] = 0;
          best = first[i];
        }
        tg[i] = sm.order[pos[i]];
        sc[i] = (best < 1.0e30f) ? table_load<kOnChip>(coeff, (int64_t)ex[i] * E + tg[i]) : 0.0f;
      } else if (pos[i] != 0x7fffffff) {
        tg[i] = sm.order[pos[i]];
        sc[i] = (tg[i] == ex[i]) ? 1.0f : table_load<kOnChip>(coeff, (int64_t)ex[i] * E + tg[i]);
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < kTableBatch; ++i)
        if (ex[i] < E) {
          sm.tgt[ex[i]] = tg[i];
          sm.scale[ex[i]] = sc[i];
        }
    }
  }
}

// ---- 5. (decode for the expert layer) the layer's routes, from the routes phase 4 wrote ------
// Routes of one token that the table sent to the same expert become one route: the first keeps
// the sum of their weights (fp32, slot order), the others get id -1 (so the expert layer computes
// that expert once for the token).  Out-of-range ids also get -1.  moe_align and the gather of
// token rows then run over these routes in one multi-CTA launch (align_gather_kernel).
// Phase 4's writes are read back through L1 after the barrier (same CTA), never through the
// read-only path.
template <typename WT, typename IT>
__device__ void merge_routes(const DecodeParams& p) {
  const int E = p.experts;
  const int K = p.top_k;
  const int R = static_cast<int>(p.routes);
  const WT* ow = static_cast<const WT*>(p.out_w);
  const IT* oi = static_cast<const IT*>(p.out_ids);
  __syncthreads();
  for (int t = threadIdx.x; t < R / K; t += kDecodeThreads) {
    int e[8];
    float g[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      e[j] = -1;
      g[j] = 0.0f;
      if (j < K) {
        const int x = static_cast<int>(oi[t * K + j]);
        e[j] = (x >= 0 && x < E) ? x : -1;
        g[j] = e[j] >= 0 ? to_f32(ow[t * K + j]) : 0.0f;
      }
    }
#pragma unroll
    for (int j = 1; j < 8; ++j) {
      bool merged = false;
#pragma unroll
      for (int f = 0; f < j; ++f) {
        if (!merged && e[j] >= 0 && e[f] == e[j]) {
          g[f] = __fadd_rn(g[f], g[j]);
          merged = true;
        }
      }
      if (merged) {
        e[j] = -1;
        g[j] = 0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < K) {
        p.gemm_ids[t * K + j] = e[j];
        p.gemm_w[t * K + j] = g[j];
      }
  }
}

// Multi-CTA importance: per-CTA shared-memory histogram, then one 64-bit global atomic per
// expert per CTA into the caller's (zeroed) vector.
template <typename WT, typename IT>
__global__ void __launch_bounds__(256) decode_importance_kernel(const void* wv, const void* idv,
                                                                int64_t routes, int experts,
                                                                const float* norms,
                                                                int64_t* importance) {
  __shared__ long long hist[kMaxExperts];
  const WT* w = static_cast<const WT*>(wv);
  const IT* ids = static_cast<const IT*>(idv);
  for (int e = threadIdx.x; e < experts; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < routes;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)ids[r];
    if (e < 0 || e >= experts) continue;
    const long long q = fixed_point(__fmul_rn(to_f32(w[r]), __ldg(norms + e)));
    atomicAdd(reinterpret_cast<unsigned long long*>(&hist[e]), (unsigned long long)q);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < experts; e += blockDim.x)
    if (hist[e] != 0)
      atomicAdd(reinterpret_cast<unsigned long long*>(importance + e), (unsigned long long)hist[e]);
}

// Static decode table (exfold/qwen3/vllm_patch.py:130-143): keep the `budget` experts of largest
// calibrated norm, map every other expert to the kept expert of smallest loss.
__global__ void __launch_bounds__(kDecodeThreads, 1) static_table_kernel(
    const float* norms, const float* coeff, const float* loss, int E, int D, int32_t* target,
    float* scale_out) {
  __shared__ int order[kMaxExperts];
  __shared__ int rank[kMaxExperts];
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += kDecodeThreads) {
    const uint32_t ke = key_of(__ldg(norms + e));
    int cnt = 0;
    for (int o = 0; o < E; ++o) cnt += ranks_before(key_of(__ldg(norms + o)), o, ke, e) ? 1 : 0;
    order[cnt] = e;
    rank[e] = cnt;
  }
  __syncthreads();
  const int warp = tid >> 5;
  const int lane = tid & 31;
  for (int e = warp; e < E; e += kDecodeThreads / 32) {
    if (rank[e] < D) {
      if (lane == 0) {
        target[e] = e;
        scale_out[e] = 1.0f;
      }
      continue;
    }
    const float* lrow = loss + (int64_t)e * E;
    float v = INFINITY;
    int pos = 0x7fffffff;
    for (int q = lane; q < D; q += 32) {
      const float c = __ldg(lrow + order[q]);
      const float cv = (c != c) ? INFINITY : c;
      if (cv < v) {
        v = cv;
        pos = q;
      }
    }
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int op = __shfl_xor_sync(0xffffffffu, pos, off);
      argmin_merge(v, pos, ov, op);
    }
    const float first = __ldg(lrow + order[0]);
    if (first != first || pos == 0x7fffffff) pos = 0;
    if (lane == 0) {
      target[e] = order[pos];
      scale_out[e] = __ldg(coeff + (int64_t)e * E + order[pos]);
    }
  }
}

// In-place remap (exfold/qwen3/kernels.py:295-319): ids = target[ids], w = w * scale[ids].
template <typename WT, typename IT>
__global__ void __launch_bounds__(256) static_remap_kernel(void* wv, void* idv, int64_t routes,
                                                           int experts, const int32_t* target,
                                                           const float* scale) {
  WT* w = static_cast<WT*>(wv);
  IT* ids = static_cast<IT*>(idv);
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < routes;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)ids[r];
    if (e < 0 || e >= experts) continue;
    w[r] = from_f32<WT>(__fmul_rn(to_f32(w[r]), __ldg(scale + e)));
    ids[r] = (IT)__ldg(target + e);
  }
}

// ---------------------------------------------------------------------------------------------
// Whether the loss and scale tables of a launch go to shared memory: E <= 128 and both tables
// 16-byte aligned (the bulk copies' rule; E * E * 4 is then a multiple of 16 for even E).
static bool tables_fit(const DecodeParams& p) {
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  return p.experts >= 2 && p.experts <= kSmemTableExperts && p.experts % 2 == 0 && p.loss &&
         p.coeff && a16(p.loss) && a16(p.coeff);
}

template <typename WT, typename IT, bool MERGE = false>
static cudaError_t launch_decode_t(const DecodeParams& pin, cudaStream_t s) {
  auto kern = decode_kernel<WT, IT, MERGE>;
  constexpr size_t kMaxTables = 2 * kSmemTableExperts * kSmemTableExperts * sizeof(float) + 144;
  static std::mutex mu;
  static bool allowed[64] = {};
  DecodeParams p = pin;
  // (not for the decode fused with the expert layer, whose launch measured slower with it; the
  // plain 48-layer decode, with the first routes kept in registers, 13.40 -> 12.88 us per layer)
  p.tables_smem = !MERGE && tables_fit(p) ? 1 : 0;
  if (p.tables_smem) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!allowed[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kMaxTables));
      if (e != cudaSuccess) return e;
      allowed[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes =
      p.tables_smem ? 2 * static_cast<size_t>(p.experts) * p.experts * sizeof(float) + 144 : 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_decode_merge(const DecodeParams& p, cudaStream_t s) {
  return launch_decode_t<float, int32_t, true>(p, s);
}

cudaError_t launch_decode(int w_dtype, int id_dtype, const DecodeParams& p, cudaStream_t s) {
  const bool i32 = id_dtype == EXF_I32;
  switch (w_dtype) {
    case EXF_F32: return i32 ? launch_decode_t<float, int32_t>(p, s) : launch_decode_t<float, int64_t>(p, s);
    case EXF_BF16:
      return i32 ? launch_decode_t<__nv_bfloat16, int32_t>(p, s)
                 : launch_decode_t<__nv_bfloat16, int64_t>(p, s);
    default: return i32 ? launch_decode_t<__half, int32_t>(p, s) : launch_decode_t<__half, int64_t>(p, s);
  }
}

template <typename WT, typename IT>
static cudaError_t launch_importance_t(const void* w, const void* ids, int64_t routes, int experts,
                                       const float* norms, int64_t* imp, cudaStream_t s) {
  int64_t blocks = (routes + 255) / 256;
  const int cap = 2 * sm_count();
  if (cap > 0 && blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  decode_importance_kernel<WT, IT><<<(unsigned)blocks, 256, 0, s>>>(w, ids, routes, experts, norms, imp);
  return cudaGetLastError();
}

cudaError_t launch_importance(int w_dtype, int id_dtype, const void* w, const void* ids,
                              int64_t routes, int experts, const float* norms, int64_t* imp,
                              cudaStream_t s) {
  const bool i32 = id_dtype == EXF_I32;
  switch (w_dtype) {
    case EXF_F32:
      return i32 ? launch_importance_t<float, int32_t>(w, ids, routes, experts, norms, imp, s)
                 : launch_importance_t<float, int64_t>(w, ids, routes, experts, norms, imp, s);
    case EXF_BF16:
      return i32 ? launch_importance_t<__nv_bfloat16, int32_t>(w, ids, routes, experts, norms, imp, s)
                 : launch_importance_t<__nv_bfloat16, int64_t>(w, ids, routes, experts, norms, imp, s);
    default:
      return i32 ? launch_importance_t<__half, int32_t>(w, ids, routes, experts, norms, imp, s)
                 : launch_importance_t<__half, int64_t>(w, ids, routes, experts, norms, imp, s);
  }
}

cudaError_t launch_static_table(const float* norms, const float* coeff, const float* loss, int E,
                                int D, int32_t* target, float* scale, cudaStream_t s) {
  static_table_kernel<<<1, kDecodeThreads, 0, s>>>(norms, coeff, loss, E, D, target, scale);
  return cudaGetLastError();
}

template <typename WT, typename IT>
static cudaError_t launch_remap_t(void* w, void* ids, int64_t routes, int experts,
                                  const int32_t* target, const float* scale, cudaStream_t s) {
  int64_t blocks = (routes + 255) / 256;
  const int cap = 4 * sm_count();
  if (cap > 0 && blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  static_remap_kernel<WT, IT><<<(unsigned)blocks, 256, 0, s>>>(w, ids, routes, experts, target, scale);
  return cudaGetLastError();
}

cudaError_t launch_static_remap(int w_dtype, int id_dtype, void* w, void* ids, int64_t routes,
                                int experts, const int32_t* target, const float* scale,
                                cudaStream_t s) {
  const bool i32 = id_dtype == EXF_I32;
  switch (w_dtype) {
    case EXF_F32:
      return i32 ? launch_remap_t<float, int32_t>(w, ids, routes, experts, target, scale, s)
                 : launch_remap_t<float, int64_t>(w, ids, routes, experts, target, scale, s);
    case EXF_BF16:
      return i32 ? launch_remap_t<__nv_bfloat16, int32_t>(w, ids, routes, experts, target, scale, s)
                 : launch_remap_t<__nv_bfloat16, int64_t>(w, ids, routes, experts, target, scale, s);
    default:
      return i32 ? launch_remap_t<__half, int32_t>(w, ids, routes, experts, target, scale, s)
                 : launch_remap_t<__half, int64_t>(w, ids, routes, experts, target, scale, s);
  }
}

}  // namespace exf
