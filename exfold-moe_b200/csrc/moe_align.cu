// moe_align / permute (sm_100a): group routes by expert, pad each expert to a multiple of the
// GEMM block size, name each block's expert.  Routes of one expert keep ascending flat order
// (a stable counting sort), so the permutation is deterministic.
//
// numel <= kAlignSmall: one CTA does count, scan and stable scatter in shared memory (or, for
// the expert layer, every CTA counts and each places and gathers a slice of the routes).
// Larger: count (one CTA per 2048-route chunk, shared-memory histogram) -> scan (one CTA:
// column prefix over chunks, padded exclusive scan over experts, padding and block->expert
// fill) -> stable scatter (one CTA per chunk).  The [chunks][experts] int32 table lives in the
// caller's workspace.
#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"

namespace exf {

constexpr int kAlignThreads = 512;
constexpr int kAlignWarps = kAlignThreads / 32;
constexpr int kAlignMaxExperts = 512;
constexpr int64_t kAlignChunk = 2048;
constexpr int64_t kAlignSmall = 8192;


struct AlignSmem {
  int count[kAlignMaxExperts];
  int base[kAlignMaxExperts];
  int off[kAlignMaxExperts + 1];
  int wcnt[kAlignWarps][kAlignMaxExperts];
  int scan[kAlignThreads];
};

template <typename IT>
__device__ __forceinline__ int expert_of(const IT* ids, int64_t r, int64_t end, int E) {
  if (r >= end) return -1;
  const int e = (int)ids[r];
  return (e >= 0 && e < E) ? e : -1;
}

// One round of the stable scatter: route r (expert e, -1 for none) of the CTA's 512 consecutive
// routes goes to base[e] + (routes of expert e before it in the round); base advances.
__device__ __forceinline__ int scatter_round(int64_t r, int e, int E, AlignSmem& sm,
                                             int32_t* sorted_ids) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (int x = lane; x < E; x += 32) sm.wcnt[warp][x] = 0;
  __syncwarp();
  const unsigned m = __match_any_sync(0xffffffffu, e);
  const int lane_rank = __popc(m & lt);
  if (e >= 0 && lane_rank == 0) sm.wcnt[warp][e] = __popc(m);
  __syncthreads();
  int slot = -1;
  if (e >= 0) {
    int prefix = 0;
    for (int w = 0; w < warp; ++w) prefix += sm.wcnt[w][e];
    slot = sm.base[e] + prefix + lane_rank;
    sorted_ids[slot] = (int32_t)r;
  }
  __syncthreads();
  for (int x = tid; x < E; x += kAlignThreads) {
    int add = 0;
    for (int w = 0; w < kAlignWarps; ++w) add += sm.wcnt[w][x];
    sm.base[x] += add;
  }
  __syncthreads();
  return slot;
}

// Stable scatter of routes [start, end): base[e] holds the next slot of expert e.
template <typename IT>
__device__ void stable_scatter(const IT* ids, int64_t start, int64_t end, int E, AlignSmem& sm,
                               int32_t* sorted_ids) {
  for (int64_t s0 = start; s0 < end; s0 += kAlignThreads) {
    const int64_t r = s0 + threadIdx.x;
    scatter_round(r, expert_of(ids, r, end, E), E, sm, sorted_ids);
  }
}

// Padded exclusive scan over experts (counts in sm.count) -> sm.off[0..E].
__device__ void padded_scan(const AlignParams& p, AlignSmem& sm) {
  const int tid = threadIdx.x;
  const int E = p.experts;
  const int BM = p.block_size;
  // experts per thread: E <= kAlignMaxExperts == kAlignThreads, so one expert per thread
  const int lane = tid & 31, warp = tid >> 5;
  const int c = tid < E ? sm.count[tid] : 0;
  const int padded = (c + BM - 1) / BM * BM;
  // inclusive scan of the padded counts: within each warp by shuffles, then over warp totals
  int v = padded;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  if (lane == 31) sm.scan[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kAlignWarps ? sm.scan[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, t, d);
      if (lane >= d) t += o;
    }
    if (lane < kAlignWarps) sm.scan[kAlignWarps + lane] = t;  // inclusive over warps
  }
  __syncthreads();
  if (warp > 0) v += sm.scan[kAlignWarps + warp - 1];
  if (tid < E) sm.off[tid + 1] = v;
  if (tid == 0) sm.off[0] = 0;
  __syncthreads();
}

// Padding slots of each expert, the tail past the padded total and the expert of each block,
// from sm.off and sm.count; the work is split over `parts` CTAs, this one doing part `part`.
__device__ void fill_padding(const AlignParams& p, const AlignSmem& sm, int part, int parts) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int E = p.experts;
  const int BM = p.block_size;
  const int total = sm.off[E];
  // padding slots of each expert, one warp per expert
  for (int e = part * kAlignWarps + warp; e < E; e += parts * kAlignWarps) {
    const int q0 = sm.off[e] + sm.count[e], q1 = sm.off[e + 1];
    for (int q = q0 + lane; q < q1; q += 32) p.sorted_ids[q] = (int32_t)p.numel;
  }
  const int64_t stride = (int64_t)parts * kAlignThreads;
  const int64_t first = (int64_t)part * kAlignThreads + tid;
  for (int64_t q = total + first; q < p.capacity; q += stride) p.sorted_ids[q] = (int32_t)p.numel;
  const int64_t nblocks = (p.capacity + BM - 1) / BM;
  const int used = total / BM;
  for (int64_t b = first; b < nblocks; b += stride) {
    int e = -1;
    if (b < used) {
      const int start = (int)b * BM;
      int lo = 0, hi = E - 1;  // last expert with off[e] <= start
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sm.off[mid] <= start) lo = mid; else hi = mid - 1;
      }
      e = lo;
    }
    p.expert_ids[b] = e;
  }
  if (part == 0 && tid == 0) *p.num_post_pad = total;
}

// Padded scan and fill by one CTA.
__device__ void scan_and_fill(const AlignParams& p, AlignSmem& sm) {
  padded_scan(p, sm);
  fill_padding(p, sm, 0, 1);
}

template <typename IT>
__global__ void __launch_bounds__(kAlignThreads, 1) align_small_kernel(const AlignParams p) {
  constexpr int kPer = static_cast<int>(kAlignSmall / kAlignThreads);
  __shared__ AlignSmem sm;
  const IT* ids = static_cast<const IT*>(p.ids);
  const int tid = threadIdx.x;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // every id this thread handles, loaded once (all loads in flight together): route
  // j * 512 + tid for round j
  int ex[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) ex[j] = expert_of(ids, (int64_t)j * kAlignThreads + tid, p.numel, p.experts);
  for (int e = tid; e < p.experts; e += kAlignThreads) sm.count[e] = 0;
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (ex[j] >= 0) atomicAdd(&sm.count[ex[j]], 1);
  __syncthreads();
  scan_and_fill(p, sm);
  for (int e = tid; e < p.experts; e += kAlignThreads) sm.base[e] = sm.off[e];
  __syncthreads();
  const int rounds = static_cast<int>((p.numel + kAlignThreads - 1) / kAlignThreads);
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (j < rounds) scatter_round((int64_t)j * kAlignThreads + tid, ex[j], p.experts, sm, p.sorted_ids);
}

// moe_align fused with the gather of token rows (numel <= kAlignSmall, the expert layer at
// decode): every CTA counts all routes (they are few; an L2-resident read) and places only its
// own slice [s0, s0 + slice) of consecutive routes, at the slots the one-CTA kernel gives them
// (routes of an expert in earlier slices come first, then the slice's own in flat order); then
// it copies the token row of each route it placed: xs[slot] = x[route / top_k] (16-byte
// vectors).  Padding, tail and block names are split over the CTAs.  CTA 0 also zeroes
// zero[0, zero_n) (the expert layer kernel's tile counters).
template <typename IT>
__global__ void __launch_bounds__(kAlignThreads, 1)
    align_gather_kernel(const AlignParams p, const uint4* __restrict__ x, int top_k, int row_vecs,
                        uint4* __restrict__ xs, int slice, int32_t* zero, int zero_n) {
  __shared__ AlignSmem sm;
  __shared__ int slot_of[kAlignThreads];
  const IT* ids = static_cast<const IT*>(p.ids);
  const int tid = threadIdx.x;
  const int E = p.experts;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (blockIdx.x == 0)
    for (int i = tid; i < zero_n; i += kAlignThreads) zero[i] = 0;  // the expert layer's counters
  const int64_t s0 = (int64_t)blockIdx.x * slice;
  const int64_t s1 = s0 + slice < p.numel ? s0 + slice : p.numel;
  for (int e = tid; e < E; e += kAlignThreads) {
    sm.count[e] = 0;
    sm.base[e] = 0;
  }
  __syncthreads();
  for (int64_t r = tid; r < p.numel; r += kAlignThreads) {
    const int e = expert_of(ids, r, p.numel, E);
    if (e >= 0) {
      atomicAdd(&sm.count[e], 1);
      if (r < s0) atomicAdd(&sm.base[e], 1);  // routes of e placed by earlier slices
    }
  }
  __syncthreads();
  padded_scan(p, sm);
  for (int e = tid; e < E; e += kAlignThreads) sm.base[e] += sm.off[e];
  __syncthreads();
  fill_padding(p, sm, blockIdx.x, gridDim.x);
  for (int64_t r0 = s0; r0 < s1; r0 += kAlignThreads) {
    slot_of[tid] = scatter_round(r0 + tid, expert_of(ids, r0 + tid, s1, E), E, sm, p.sorted_ids);
    __syncthreads();
    const int n = s1 - r0 < kAlignThreads ? (int)(s1 - r0) : kAlignThreads;
    for (int i = tid; i < n * row_vecs; i += kAlignThreads) {
      const int k = i / row_vecs;
      const int c = i - k * row_vecs;
      const int slot = slot_of[k];
      if (slot >= 0) xs[(int64_t)slot * row_vecs + c] = x[(r0 + k) / top_k * row_vecs + c];
    }
    __syncthreads();  // slot_of is rewritten by the next round
  }
}

template <typename IT>
__global__ void __launch_bounds__(kAlignThreads) align_count_kernel(const AlignParams p) {
  __shared__ int hist[kAlignMaxExperts];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const IT* ids = static_cast<const IT*>(p.ids);
  const int64_t start = (int64_t)blockIdx.x * kAlignChunk;
  const int64_t end = min(start + kAlignChunk, p.numel);
  for (int e = threadIdx.x; e < p.experts; e += kAlignThreads) hist[e] = 0;
  __syncthreads();
  for (int64_t r = start + threadIdx.x; r < end; r += kAlignThreads) {
    const int e = expert_of(ids, r, end, p.experts);
    if (e >= 0) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.experts; e += kAlignThreads)
    p.table[(int64_t)blockIdx.x * p.experts + e] = hist[e];
}

__global__ void __launch_bounds__(kAlignThreads, 1) align_scan_kernel(const AlignParams p) {
  __shared__ AlignSmem sm;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  const int E = p.experts;
  // Column prefix of expert tid over the chunks.  The loads of kBatch chunks are issued before
  // any of their stores: a load after a store to the same table cannot be hoisted above it, so a
  // one-chunk-at-a-time loop would wait one L2 round trip per chunk.
  constexpr int kBatch = 32;
  if (tid < E) {
    int run = 0;
    for (int64_t b0 = 0; b0 < p.chunks; b0 += kBatch) {
      int c[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) c[j] = b0 + j < p.chunks ? p.table[(b0 + j) * E + tid] : 0;
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (b0 + j < p.chunks) {
          p.table[(b0 + j) * E + tid] = run;  // routes of expert tid in chunks before b0 + j
          run += c[j];
        }
    }
    sm.count[tid] = run;
  }
  __syncthreads();
  scan_and_fill(p, sm);
  if (tid < E) {
    const int o = sm.off[tid];
    for (int64_t b0 = 0; b0 < p.chunks; b0 += kBatch) {
      int c[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) c[j] = b0 + j < p.chunks ? p.table[(b0 + j) * E + tid] : 0;
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (b0 + j < p.chunks) p.table[(b0 + j) * E + tid] = c[j] + o;
    }
  }
}

template <typename IT>
__global__ void __launch_bounds__(kAlignThreads, 1) align_scatter_kernel(const AlignParams p) {
  __shared__ AlignSmem sm;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const IT* ids = static_cast<const IT*>(p.ids);
  for (int e = threadIdx.x; e < p.experts; e += kAlignThreads)
    sm.base[e] = p.table[(int64_t)blockIdx.x * p.experts + e];
  __syncthreads();
  const int64_t start = (int64_t)blockIdx.x * kAlignChunk;
  const int64_t end = min(start + kAlignChunk, p.numel);
  stable_scatter(ids, start, end, p.experts, sm, p.sorted_ids);
}

// ---------------------------------------------------------------------------------------------
int64_t align_workspace_bytes(int64_t numel, int experts) {
  if (numel <= kAlignSmall) return 0;
  const int64_t chunks = (numel + kAlignChunk - 1) / kAlignChunk;
  return chunks * experts * (int64_t)sizeof(int32_t);
}

int align_max_experts() { return kAlignMaxExperts; }

// Every align kernel is launched as a programmatic dependent of the kernel before it in the
// stream (its launch overlaps that kernel's tail; it reads nothing before griddepcontrol.wait).
static cudaError_t launch_dependent(void (*kern)(AlignParams), unsigned grid, const AlignParams& p,
                                    cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kAlignThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename IT>
static cudaError_t launch_align_t(AlignParams p, cudaStream_t s) {
  if (p.numel <= kAlignSmall) return launch_dependent(align_small_kernel<IT>, 1, p, s);
  p.chunks = (p.numel + kAlignChunk - 1) / kAlignChunk;
  cudaError_t e = launch_dependent(align_count_kernel<IT>, (unsigned)p.chunks, p, s);
  if (e == cudaSuccess) e = launch_dependent(align_scan_kernel, 1, p, s);
  if (e == cudaSuccess) e = launch_dependent(align_scatter_kernel<IT>, (unsigned)p.chunks, p, s);
  return e;
}

cudaError_t launch_align(int id_dtype, const AlignParams& p, cudaStream_t s) {
  return id_dtype == EXF_I32 ? launch_align_t<int32_t>(p, s) : launch_align_t<int64_t>(p, s);
}

int64_t align_gather_max_numel() { return kAlignSmall; }

cudaError_t launch_align_gather(const AlignParams& p, const void* x, int top_k, int hidden,
                                void* xs, int32_t* zero, int zero_n, cudaStream_t s) {
  if (p.numel < 1 || p.numel > kAlignSmall || hidden % 8 != 0) return cudaErrorInvalidValue;
  // slices of at least 16 routes, one CTA each, at most one CTA per SM
  const int sms = sm_count() > 0 ? sm_count() : 1;
  int64_t slice = (p.numel + sms - 1) / sms;
  if (slice < 16) slice = 16;
  const unsigned grid = (unsigned)((p.numel + slice - 1) / slice);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kAlignThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, align_gather_kernel<int32_t>, p, static_cast<const uint4*>(x),
                         top_k, hidden / 8, static_cast<uint4*>(xs), (int)slice, zero, zero_n);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace exf

// ---- fixed scratch for exf_moe_align_noalloc ---------------------------------------------------
// Some callers cannot allocate device memory when they call moe_align (see exfold_b200.h); for
// them the [chunks][experts] count table lives in this file-scope array instead of a caller
// workspace.  1 MiB of int32 entries; every GPU that loads the library holds it until exit.
// The count kernel writes every entry the scan reads, so no call needs it zeroed.
#include <mutex>

namespace exf {

constexpr int64_t kAlignStaticTableInts = 262144;
static __device__ __align__(256) int32_t g_align_static_table[kAlignStaticTableInts];

constexpr int kStaticTableDevices = 64;
static std::mutex g_static_table_mu;
static int32_t* g_static_table_addr[kStaticTableDevices] = {};

int64_t align_static_table_ints() { return kAlignStaticTableInts; }

// Device address of the current device's copy of the array.  In host code the symbol names a
// host-side stand-in, so the address is looked up once per device, with that device current.
static cudaError_t align_static_table(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kStaticTableDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_static_table_mu);
  if (g_static_table_addr[dev] == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_align_static_table);
    if (e != cudaSuccess) return e;
    g_static_table_addr[dev] = static_cast<int32_t*>(addr);
  }
  *out = g_static_table_addr[dev];
  return cudaSuccess;
}

cudaError_t launch_align_static(int id_dtype, AlignParams p, cudaStream_t s) {
  if (align_workspace_bytes(p.numel, p.experts) > 0) {
    int32_t* table = nullptr;
    const cudaError_t e = align_static_table(&table);
    if (e != cudaSuccess) return e;
    p.table = table;
  }
  return launch_align(id_dtype, p, s);
}

}  // namespace exf
