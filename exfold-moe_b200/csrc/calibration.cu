// Calibration statistics of the pairwise scalar projectors on the GPU (sm_100a): the
// accumulator PairwiseScalarStats of exfold/qwen3/calibration.py:9-140.
//
// calib_update_kernel (calibration.py:49-95): one warp per token at a time.  The token's k <= 8
// unweighted expert outputs stream through shared memory in 256-column chunks (bf16; 128 for
// fp32) by cp.async, three chunks in flight per warp; lane l copies and reads only its own
// 16-byte unit of each row, so the pipeline needs no barrier.  Each lane accumulates the 36
// pairwise dot products (squared norms on the diagonal) of its columns in fp32; a butterfly
// reduction in a fixed order gives the token's totals.  The 56 ordered pairs of routes with
// different experts and the 8 norms are then split over the lanes: each adds, in fp64, the fp32
// products w_s <u_s, u_d>, w_s ||u_d||^2, w_s ||u_s||^2 (w_s = ||u_s||) into the [E, E]
// statistics, and ||u_s|| and 1 into the per-expert norm sum and count, with 64-bit atomics in
// L2 (the reference's index_add_).  The FMA chains make this pass issue-bound; it serves fp32
// outputs and the shapes the tensor-core pass does not take.
// calib_gram_kernel, the same update for bf16 / fp16 outputs with k in {1, 2, 4, 8} and a hidden
// size that is a multiple of 128, on the tensor cores: 128 / k tokens' routes are 128 consecutive
// rows of the [tokens * k, hidden] outputs, and one tcgen05.mma chain (M = N = 128, K = 16 per
// instruction, fp32 in TMEM) computes their Gram matrix X X^T, with the same TMA-loaded tile as
// both operands.  Only the 128 / k diagonal k x k blocks are used (1/16 of the products at k = 8),
// which the tensor cores still do in less time than the tile takes to arrive from HBM.  The
// products are exact in fp32; each 128-column slice is summed by the tensor core into one of 4
// TMEM accumulators in turn, and the slices' sums are added in fp32 with round-to-nearest (the
// tensor core's own fp32 chains drop low bits, 1.8e-5 of a dot product over 2048 columns).  Warp
// roles as in moe_gemm.cu: warp 0 streams 16 KB tiles through an 8-stage ring, warp 1 issues
// the MMAs, warps 2-5 read their 32 rows' k columns from TMEM and add the same fp64 updates as
// calib_update_kernel.
// calib_finalize_kernel (calibration.py:97-126): the closed form element by element in fp64,
// a device flag for non-finite statistics.  calib_norms_kernel (calibration.py:128-140): mean
// norm per expert, the lower median of the observed experts for the others.
#include <float.h>

#include <mutex>

#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"
#include "exf_tc.cuh"

namespace exf {

namespace {

constexpr int kCalibK = 8;
constexpr int kPairs = kCalibK * (kCalibK + 1) / 2;  // s <= d

__device__ __forceinline__ int pair_index(int s, int d) {  // s <= d
  return s * kCalibK - s * (s - 1) / 2 + (d - s);
}

// 16 bytes of one output row -> fp32 (8 bf16 / fp16 values or 4 fp32 values)
template <typename T>
struct Unit {
  static constexpr int kElems = 16 / sizeof(T);
};
__device__ __forceinline__ void to_f32(const uint4& q, float (&v)[8], __nv_bfloat16*) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void to_f32(const uint4& q, float (&v)[8], __half*) {
  const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void to_f32(const uint4& q, float (&v)[8], float*) {
  v[0] = __uint_as_float(q.x);
  v[1] = __uint_as_float(q.y);
  v[2] = __uint_as_float(q.z);
  v[3] = __uint_as_float(q.w);
  v[4] = v[5] = v[6] = v[7] = 0.0f;
}

constexpr int kStages = 3;          // chunks in flight per warp
constexpr int kUpdWarps = 8;
// [warp][stage][route][lane] 16-byte units: a lane copies and reads only its own units
struct CalibSmem {
  uint4 buf[kUpdWarps][kStages][kCalibK][32];
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_prior() {  // all but the newest kStages-1 groups
  asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 1) : "memory");
}

template <typename T, typename IT>
__global__ void __launch_bounds__(kUpdWarps * 32) calib_update_kernel(
    const T* out, const IT* ids, int64_t tokens, int K, int H, int E, double* dot, double* tsq,
    double* ssq, double* nsum, double* ncnt) {
  extern __shared__ uint4 calib_raw[];
  CalibSmem& sm = *reinterpret_cast<CalibSmem*>(calib_raw);
  constexpr int EL = Unit<T>::kElems;  // elements per lane per chunk
  constexpr int CW = 32 * EL;          // chunk width
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t wstride = (int64_t)gridDim.x * kUpdWarps;
  const int64_t t0 = (int64_t)blockIdx.x * kUpdWarps + warp;
  const int nch = (H + CW - 1) / CW;
  // this warp's work is the flat sequence (token t0 + i * wstride, chunk c), f = i * nch + c
  const int64_t mine = t0 < tokens ? (tokens - t0 + wstride - 1) / wstride : 0;
  const int64_t nflat = mine * nch;
  auto issue = [&](int64_t f) {
    if (f < nflat) {
      const int64_t t = t0 + (f / nch) * wstride;
      const int c = (int)(f % nch);
      const int h = c * CW + lane * EL;
      const bool in = h < H;
      const T* src = out + t * K * (int64_t)H + (in ? h : 0);
      const int st = (int)(f % kStages);
#pragma unroll
      for (int s = 0; s < kCalibK; ++s)
        if (s < K) cp_async16(&sm.buf[warp][st][s][lane], src + (int64_t)s * H, in);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int j = 0; j < kStages - 1; ++j) issue(j);

  float acc[kPairs];
#pragma unroll
  for (int p = 0; p < kPairs; ++p) acc[p] = 0.0f;
  for (int64_t f = 0; f < nflat; ++f) {
    issue(f + kStages - 1);
    cp_async_wait_prior();
    const int st = (int)(f % kStages);
    float v[kCalibK][8];
#pragma unroll
    for (int s = 0; s < kCalibK; ++s) {
      if (s < K) {
        to_f32(sm.buf[warp][st][s][lane], v[s], static_cast<T*>(nullptr));
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[s][i] = 0.0f;
      }
    }
#pragma unroll
    for (int s = 0; s < kCalibK; ++s)
#pragma unroll
      for (int d = s; d < kCalibK; ++d) {
        float a = acc[pair_index(s, d)];
#pragma unroll
        for (int i = 0; i < EL; ++i) a = __fmaf_rn(v[s][i], v[d][i], a);
        acc[pair_index(s, d)] = a;
      }
    if ((int)(f % nch) != nch - 1) continue;

    // ---- the token is complete: its totals, then the statistics updates
    const int64_t t = t0 + (f / nch) * wstride;
    float mine_p = 0.0f, mine_q = 0.0f;  // lane l keeps pair l, lanes 0..3 also pair 32 + l
#pragma unroll
    for (int p = 0; p < kPairs; ++p) {
      float a = acc[p];
      acc[p] = 0.0f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, off));
      if (p < 32) {
        if (lane == p) mine_p = a;
      } else if (lane == p - 32) {
        mine_q = a;
      }
    }
    auto total = [&](int p) {  // the token's total of pair p, from the lane that keeps it
      const float lo = __shfl_sync(0xffffffffu, mine_p, p & 31);
      const float hi = __shfl_sync(0xffffffffu, mine_q, p & 31);
      return p < 32 ? lo : hi;
    };
    const IT* irow = ids + t * K;
    // tasks: 56 ordered pairs (s != d) and 8 norms, two per lane
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int task = lane + 32 * r;
      int s, d;
      if (task < 56) {
        s = task / 7;
        const int dd = task % 7;
        d = dd + (dd >= s ? 1 : 0);
      } else {
        s = task - 56;
        d = s;
      }
      // every lane takes part in the shuffles; the tasks beyond K are dropped afterwards
      const float sq_s = total(pair_index(s, s));
      const float sq_d = total(pair_index(d, d));
      const float pd = total(s <= d ? pair_index(s, d) : pair_index(d, s));
      if (s >= K || d >= K) continue;
      const int es = (int)irow[s];
      if (es < 0 || es >= E) continue;
      const float w = __fsqrt_rn(sq_s);
      if (task >= 56) {
        atomicAdd(nsum + es, (double)w);
        atomicAdd(ncnt + es, 1.0);
        continue;
      }
      const int ed = (int)irow[d];
      if (ed < 0 || ed >= E || ed == es) continue;
      const int64_t idx = (int64_t)es * E + ed;
      atomicAdd(dot + idx, (double)__fmul_rn(pd, w));
      atomicAdd(tsq + idx, (double)__fmul_rn(sq_d, w));
      atomicAdd(ssq + idx, (double)__fmul_rn(sq_s, w));
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}


// ---- tensor-core Gram pass ----------------------------------------------------------------------
constexpr int kGramRows = 128;                          // MMA M = N: 128 / k tokens x k routes
constexpr int kGramBK = 64;                             // 16-bit columns per 128-byte row
constexpr int kGramStages = 8;
constexpr int kGramTile = kGramRows * kGramBK * 2;      // 16 KB
constexpr int kGramThreads = 192;                       // TMA, MMA, 4 epilogue warps
// The tensor core's fp32 accumulation chains drop low bits (toward zero) as they go: a 2048-long
// chain lost up to 1.8e-5 of a dot product.  Chains of kGramPartKb k-blocks (K = 128) go to one
// of kGramSlots TMEM accumulators in turn, and the epilogue adds the partial products of a block
// in fp32 with round-to-nearest.
constexpr int kGramPartKb = 2;
constexpr int kGramSlots = 4;
constexpr int kGramTmemCols = kGramSlots * kGramRows;   // all 512 columns

struct GramSmem {
  alignas(1024) uint8_t tiles[kGramStages][kGramTile];
  alignas(8) uint64_t full[kGramStages];
  alignas(8) uint64_t empty[kGramStages];
  alignas(8) uint64_t acc_full[kGramSlots];
  alignas(8) uint64_t acc_empty[kGramSlots];
  alignas(8) uint64_t drain;
  uint32_t tmem_base;
  int failed;
};
constexpr size_t kGramSmemBytes = sizeof(GramSmem) + 1024;  // + alignment slack

template <bool BF16, typename IT, int KT>
__global__ void __launch_bounds__(kGramThreads, 1) calib_gram_kernel(
    const __grid_constant__ CUtensorMap map, const IT* ids, int64_t tokens, int H, int E,
    double* dot, double* tsq, double* ssq, double* nsum, double* ncnt) {
  using namespace tc;
  extern __shared__ uint8_t gram_raw[];
  GramSmem& sm = *reinterpret_cast<GramSmem*>(
      (reinterpret_cast<uintptr_t>(gram_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t nblocks = (tokens * KT + kGramRows - 1) / kGramRows;
  const int kblocks = H / kGramBK;
  const int nparts = kblocks / kGramPartKb;
  constexpr uint32_t kIdesc = idesc_f16(kGramRows, kGramRows, BF16);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGramStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < kGramSlots; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&sm.drain, 1);
    sm.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, kGramTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = sm.tmem_base;
  volatile int* failed = &sm.failed;

  if (warp == 0) {
    // ---- TMA producer: rows [128 b, 128 b + 128) x columns [64 kb, 64 kb + 64); rows past the
    // last route read as zeros
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      for (int64_t b = blockIdx.x; b < nblocks && ok; b += gridDim.x)
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kGramStages;
          ok = mbar_wait(&sm.empty[s], ((g / kGramStages) & 1) ^ 1, failed);
          if (!ok) break;
          mbar_expect_tx(&sm.full[s], kGramTile);
          tma_load_2d(sm.tiles[s], &map, &sm.full[s], kb * kGramBK,
                      static_cast<int>(b * kGramRows));
        }
      for (uint32_t j = g > kGramStages ? g - kGramStages : 0; j < g; ++j)
        mbar_wait_drain(&sm.full[j % kGramStages], (j / kGramStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer: partial u (k-blocks [2 u', 2 u' + 2) of a block) accumulates X X^T over
    // its 128 columns into TMEM slot u mod 4, columns [128 (u mod 4), +128)
    if (lane == 0) {
      uint32_t g = 0, u = 0;
      bool ok = true;
      for (int64_t b = blockIdx.x; b < nblocks && ok; b += gridDim.x)
        for (int pt = 0; pt < nparts && ok; ++pt, ++u) {
          const int a = u % kGramSlots;
          ok = mbar_wait(&sm.acc_empty[a], ((u / kGramSlots) & 1) ^ 1, failed);
          if (!ok) break;
          fence_after_sync();
          const uint32_t acc = tmem + static_cast<uint32_t>(a * kGramRows);
          for (int j = 0; j < kGramPartKb; ++j, ++g) {
            const int s = g % kGramStages;
            ok = mbar_wait(&sm.full[s], (g / kGramStages) & 1, failed);
            if (!ok) break;
            fence_after_sync();
            const uint32_t base = smem_addr(sm.tiles[s]);
#pragma unroll
            for (int k = 0; k < kGramBK / 16; ++k) {
              const uint64_t d = smem_desc(base + k * 32);
              mma_kind_f16(acc, d, d, kIdesc, (j > 0 || k > 0) ? 1u : 0u);
            }
            mma_commit(&sm.empty[s]);
          }
          if (!ok) break;
          mma_commit(&sm.acc_full[a]);
        }
      mma_commit(&sm.drain);
      mbar_wait_drain(&sm.drain, 0);
    }
  } else {
    // ---- epilogue: warp q owns TMEM lanes (rows) 32q .. 32q + 31, i.e. 32 / k whole tokens,
    // whose k columns lie in columns 32q .. 32q + 31
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const int s = r % KT;          // route of the token (128 is a multiple of k)
    const int gl = lane - s;       // lane of the token's route 0
    uint32_t u = 0;
    bool live = true;
    for (int64_t b = blockIdx.x; b < nblocks && live; b += gridDim.x) {
      // this row of the token's k x k block: G[s][d] = the sum over the partials of
      // v[k * (lane / k) + d]
      float gr[KT];
#pragma unroll
      for (int d = 0; d < KT; ++d) gr[d] = 0.0f;
      for (int pt = 0; pt < nparts; ++pt, ++u) {
        const int a = u % kGramSlots;
        const bool ok = mbar_wait(&sm.acc_full[a], (u / kGramSlots) & 1, failed);
        fence_after_sync();
        // warp-uniform: the TMEM load below is collective
        if (!__all_sync(0xffffffffu, ok && !*failed)) {
          live = false;
          break;
        }
        float v[32];
        tmem_load32(tmem + static_cast<uint32_t>(a * kGramRows + 32 * q) +
                        (static_cast<uint32_t>(32 * q) << 16),
                    v);
        // the slot has been read: the MMA thread may fill it again
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.acc_empty[a]);
#pragma unroll
        for (int d = 0; d < KT; ++d) {
          float x = v[d];
#pragma unroll
          for (int c = 1; c < 32 / KT; ++c)
            if (lane / KT == c) x = v[c * KT + d];
          gr[d] = __fadd_rn(gr[d], x);
        }
      }
      if (!live) break;
      float sq_s = gr[0];
#pragma unroll
      for (int d = 1; d < KT; ++d)
        if (s == d) sq_s = gr[d];
      const int64_t row = b * kGramRows + r;
      const int64_t t = row / KT;
      const bool valid = t < tokens;
      const int es_raw = valid ? static_cast<int>(ids[row]) : -1;
      const int es = (es_raw >= 0 && es_raw < E) ? es_raw : -1;
      const float w = __fsqrt_rn(sq_s);
      float sq_d[KT];
      int ed[KT];
#pragma unroll
      for (int d = 0; d < KT; ++d) {
        sq_d[d] = __shfl_sync(0xffffffffu, sq_s, gl + d);
        ed[d] = __shfl_sync(0xffffffffu, es, gl + d);
      }
      if (es < 0) continue;
      atomicAdd(nsum + es, (double)w);
      atomicAdd(ncnt + es, 1.0);
#pragma unroll
      for (int d = 0; d < KT; ++d) {
        if (d == s || ed[d] < 0 || ed[d] == es) continue;
        const int64_t idx = (int64_t)es * E + ed[d];
        atomicAdd(dot + idx, (double)__fmul_rn(gr[d], w));
        atomicAdd(tsq + idx, (double)__fmul_rn(sq_d[d], w));
        atomicAdd(ssq + idx, (double)__fmul_rn(sq_s, w));
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after_sync();
    tmem_free(tmem, kGramTmemCols);
  }
  // a wait that timed out left statistics out: make them non-finite, which finalize reports
  if (threadIdx.x == 0 && sm.failed) atomicAdd(dot, __longlong_as_double(0x7FF8000000000000ll));
}

__global__ void __launch_bounds__(256) calib_finalize_kernel(
    const double* dot, const double* tsq, const double* ssq, int E, double ridge, double lo,
    double hi, float* coeff, float* loss, int32_t* nonfinite) {
  const int64_t n = (int64_t)E * E;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const double d = dot[i], t = tsq[i], s = ssq[i];
    if (!(isfinite(d) && isfinite(t) && isfinite(s)) && nonfinite) atomicExch(nonfinite, 1);
    const bool observed = s > 0.0;
    const double denom = __dadd_rn(t, ridge);
    double c = 0.0;
    if (observed && denom > 0.0) c = __ddiv_rn(d, denom);
    c = fmin(fmax(c, lo), hi);
    // source_sq - 2 * coefficient * dot + coefficient.square() * target_sq
    const double residual =
        __dadd_rn(__dsub_rn(s, __dmul_rn(__dmul_rn(2.0, c), d)), __dmul_rn(__dmul_rn(c, c), t));
    double l = 1.0e30;
    if (observed) l = __ddiv_rn(fmax(residual, 0.0), s);
    l = fmin(l, 1.0e30);
    const bool diag = (i / E) == (i % E);
    if (diag) l = 1.0e30;
    if (!observed || l >= 1.0e30) c = 0.0;
    if (diag) c = 1.0;
    coeff[i] = __double2float_rn(c);
    loss[i] = __double2float_rn(l);
  }
}

__global__ void __launch_bounds__(1024) calib_norms_kernel(const double* nsum, const double* ncnt,
                                                           int E, float* norms) {
  __shared__ double mean[1024];
  __shared__ int obs[1024];
  __shared__ double median;
  const int e = threadIdx.x;
  if (e == 0) median = 1.0;
  if (e < E) {
    const double c = ncnt[e];
    mean[e] = __ddiv_rn(nsum[e], c > 1.0 ? c : 1.0);
    obs[e] = c > 0.0;
  }
  __syncthreads();
  int n = 0;
  for (int o = 0; o < E; ++o) n += obs[o];
  if (e < E && obs[e]) {
    // rank among the observed means, ties by index: the lower median has rank (n - 1) / 2
    int rank = 0;
    for (int o = 0; o < E; ++o)
      rank += (obs[o] && (mean[o] < mean[e] || (mean[o] == mean[e] && o < e))) ? 1 : 0;
    if (rank == (n - 1) / 2) median = mean[e];
  }
  __syncthreads();
  if (e < E) norms[e] = __double2float_rn(obs[e] ? mean[e] : median);
}

template <typename T, typename IT>
cudaError_t launch_update_t(const void* out, const void* ids, int64_t tokens, int K, int H, int E,
                            double* dot, double* tsq, double* ssq, double* nsum, double* ncnt,
                            cudaStream_t s) {
  auto kern = calib_update_kernel<T, IT>;
  static bool opted[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !opted[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(CalibSmem));
    if (e != cudaSuccess) return e;
    opted[dev] = true;
  }
  int64_t blocks = (tokens + kUpdWarps - 1) / kUpdWarps;
  const int lim = 2 * sm_count();
  if (lim > 0 && blocks > lim) blocks = lim;
  if (blocks < 1) blocks = 1;
  kern<<<(unsigned)blocks, kUpdWarps * 32, sizeof(CalibSmem), s>>>(
      static_cast<const T*>(out), static_cast<const IT*>(ids), tokens, K, H, E, dot, tsq, ssq,
      nsum, ncnt);
  return cudaGetLastError();
}

template <bool BF16, typename IT, int KT>
cudaError_t launch_gram_k(const CUtensorMap& map, const void* ids, int64_t tokens, int H, int E,
                          double* dot, double* tsq, double* ssq, double* nsum, double* ncnt,
                          cudaStream_t s) {
  auto kern = calib_gram_kernel<BF16, IT, KT>;
  static std::mutex mu;
  static bool opted[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!opted[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kGramSmemBytes);
      if (e != cudaSuccess) return e;
      opted[dev] = true;
    }
  }
  int64_t blocks = (tokens * KT + kGramRows - 1) / kGramRows;
  const int sms = sm_count();
  if (sms > 0 && blocks > sms) blocks = sms;
  if (blocks < 1) blocks = 1;
  kern<<<(unsigned)blocks, kGramThreads, kGramSmemBytes, s>>>(
      map, static_cast<const IT*>(ids), tokens, H, E, dot, tsq, ssq, nsum, ncnt);
  return cudaGetLastError();
}

// The tensor-core pass when the shape allows it (bf16 / fp16 outputs, k in {1, 2, 4, 8}, hidden
// a multiple of 128, rows addressable by 32-bit TMA coordinates); cudaErrorNotSupported otherwise.
template <bool BF16>
cudaError_t launch_gram(int id_dtype, const void* out, const void* ids, int64_t tokens, int K,
                        int H, int E, double* dot, double* tsq, double* ssq, double* nsum,
                        double* ncnt, cudaStream_t s) {
  if ((K != 1 && K != 2 && K != 4 && K != 8) || H % (kGramBK * kGramPartKb) != 0 ||
      tokens * K > (int64_t)0x7FFFFF00)
    return cudaErrorNotSupported;
  CUtensorMap map;
  if (!tc::make_map(&map, out, (uint64_t)tokens * K, (uint64_t)H, kGramRows,
                    BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16))
    return cudaErrorNotSupported;
  const bool i32 = id_dtype == EXF_I32;
#define EXF_GRAM_K(KV)                                                                        \
  case KV:                                                                                    \
    return i32 ? launch_gram_k<BF16, int32_t, KV>(map, ids, tokens, H, E, dot, tsq, ssq,      \
                                                  nsum, ncnt, s)                               \
               : launch_gram_k<BF16, int64_t, KV>(map, ids, tokens, H, E, dot, tsq, ssq,      \
                                                  nsum, ncnt, s);
  switch (K) {
    EXF_GRAM_K(1)
    EXF_GRAM_K(2)
    EXF_GRAM_K(4)
    default:
      EXF_GRAM_K(8)
  }
#undef EXF_GRAM_K
}

template <typename T>
cudaError_t launch_update_w(int id_dtype, const void* out, const void* ids, int64_t tokens, int K,
                            int H, int E, double* dot, double* tsq, double* ssq, double* nsum,
                            double* ncnt, cudaStream_t s) {
  return id_dtype == EXF_I32
             ? launch_update_t<T, int32_t>(out, ids, tokens, K, H, E, dot, tsq, ssq, nsum, ncnt, s)
             : launch_update_t<T, int64_t>(out, ids, tokens, K, H, E, dot, tsq, ssq, nsum, ncnt, s);
}

}  // namespace

cudaError_t launch_calib_update(int out_dtype, int id_dtype, const void* out, const void* ids,
                                int64_t tokens, int K, int H, int E, double* dot, double* tsq,
                                double* ssq, double* nsum, double* ncnt, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (out_dtype == EXF_BF16 || out_dtype == EXF_F16) {
    const cudaError_t e =
        out_dtype == EXF_BF16
            ? launch_gram<true>(id_dtype, out, ids, tokens, K, H, E, dot, tsq, ssq, nsum, ncnt, s)
            : launch_gram<false>(id_dtype, out, ids, tokens, K, H, E, dot, tsq, ssq, nsum, ncnt,
                                 s);
    if (e != cudaErrorNotSupported) return e;
  }
  switch (out_dtype) {
    case EXF_F32:
      return launch_update_w<float>(id_dtype, out, ids, tokens, K, H, E, dot, tsq, ssq, nsum, ncnt, s);
    case EXF_BF16:
      return launch_update_w<__nv_bfloat16>(id_dtype, out, ids, tokens, K, H, E, dot, tsq, ssq,
                                            nsum, ncnt, s);
    default:
      return launch_update_w<__half>(id_dtype, out, ids, tokens, K, H, E, dot, tsq, ssq, nsum, ncnt, s);
  }
}

cudaError_t launch_calib_finalize(const double* dot, const double* tsq, const double* ssq, int E,
                                  double ridge, double lo, double hi, float* coeff, float* loss,
                                  int32_t* nonfinite, cudaStream_t s) {
  const int64_t n = (int64_t)E * E;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  calib_finalize_kernel<<<(unsigned)blocks, 256, 0, s>>>(dot, tsq, ssq, E, ridge, lo, hi, coeff,
                                                         loss, nonfinite);
  return cudaGetLastError();
}

cudaError_t launch_calib_norms(const double* nsum, const double* ncnt, int E, float* norms,
                               cudaStream_t s) {
  calib_norms_kernel<<<1, 1024, 0, s>>>(nsum, ncnt, E, norms);
  return cudaGetLastError();
}

}  // namespace exf
