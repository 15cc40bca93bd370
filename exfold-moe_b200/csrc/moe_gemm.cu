// Grouped SwiGLU expert GEMMs on the 5th-generation tensor cores (sm_100a: tcgen05 + TMA).
//
// After moe_align, routes are grouped by expert and padded to blocks (128 routes at prefill, 64 at
// decode).  Per MoE layer:
//   gather : xs[m] = x[token(sorted_ids[m])] (bf16 rows of real routes; at <= 8192 routes done
//            inside the moe_align launch, align_gather_kernel in moe_align.cu)
//   GEMM-1 : act[m, n] = silu(xs[m] . W1[e, n]) * (xs[m] . W3[e, n]) for n in a 128-wide tile;
//            gate and up rows of W13[e] are stacked into one N = 256 MMA so both accumulators
//            sit side by side in TMEM and the SwiGLU epilogue needs no second pass
//   GEMM-2 : out[route, h] = w_route * (act[m] . W2[e, h])         (N = 256 tile of H)
//   combine: y[t, h] = sum over the token's routes of out[route, h] (fixed order: deterministic)
//
// Prefill (expert_gemm_kernel): routes on the M side.  Both GEMMs share one mainloop in a
// persistent kernel: one CTA per SM walks 128 x 256 output tiles (one expert each); warp 0
// streams 128 x 64 A and 256 x 64 B bf16 tiles with TMA (128-byte swizzle) through a 4-stage
// mbarrier ring that runs on across tiles; one elected
// thread of warp 1 issues tcgen05.mma (M = 128, N = BN, K = 16, fp32 accumulation in TMEM) and
// releases each stage with tcgen05.commit; warps 2-5 read the accumulator with tcgen05.ld and run
// the epilogue.  Two TMEM accumulators (all 512 columns) let the epilogue of one tile overlap
// the mainloop of the next.  The N tiles of one M block run side by side on neighbouring CTAs,
// so A tiles and the expert's weight tiles are reused from L2.
// Decode (expert_layer_t_kernel, experts holding 64 routes or fewer on average): both GEMMs in
// one persistent launch, weight rows on the M side, blocks of 64 routes on the N side (see the
// comment above that kernel).
// Every mbarrier wait is bounded: on time-out the CTA records an error in *status, skips the
// rest of its work, still frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "exf_common.cuh"
#include "exf_launch.h"
#include "exf_moe.h"
#include "exf_tc.cuh"

namespace exf {
using namespace tc;

constexpr int kBM = 128;              // rows per M block (moe_align block size)
constexpr int kBK = 64;               // bf16 elements per 128-byte swizzled row
constexpr int kATileBytes = kBM * kBK * 2;   // 16 KB
constexpr int kGemmThreads = 192;     // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kTmemCols = 512;       // two accumulators of up to 256 fp32 columns

// The MMA N tile of the prefill kernel: 256 (4 stages of 48 KB); 128 (6 stages of 32 KB) is
// kept as a configuration.
template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kBTileBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kATileBytes + kBTileBytes;
  static constexpr uint32_t kIdesc = idesc_f16(kBM, BN, true);  // bf16, M=128, N=BN
};

template <int BN>
struct GemmSmem {
  alignas(1024) uint8_t tiles[GemmCfg<BN>::kStages][GemmCfg<BN>::kStageBytes];
  alignas(8) uint64_t full[GemmCfg<BN>::kStages];
  alignas(8) uint64_t empty[GemmCfg<BN>::kStages];
  alignas(8) uint64_t acc_full[2];   // accumulator b holds a finished tile
  alignas(8) uint64_t acc_empty[2];  // the epilogue has read accumulator b
  alignas(8) uint64_t drain;         // every MMA issued by the CTA has completed
  uint32_t tmem_base;
  int failed;
};
template <int BN>
constexpr size_t gemm_smem_bytes() { return sizeof(GemmSmem<BN>) + 1024; }  // + alignment slack

// ---- the shared mainloop + per-GEMM epilogue ------------------------------------------------
enum GemmKind { kGemmSwiGLU = 0, kGemmDown = 1 };

template <int KIND, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    expert_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, const ExpertGemmParams p) {
  constexpr int kBN = BN;
  constexpr int kStages = GemmCfg<BN>::kStages;
  constexpr int kBTileBytes = GemmCfg<BN>::kBTileBytes;
  constexpr int kStageBytes = GemmCfg<BN>::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  GemmSmem<BN>& sm = *reinterpret_cast<GemmSmem<BN>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&sm.drain, 1);
    sm.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  // Launched as a programmatic dependent: the set-up above overlaps the previous kernel's tail;
  // nothing it wrote is read before this wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Tiles t = m_block * n_tiles + n_tile, strided over the persistent CTAs: the N tiles of one
  // block run side by side (A and the expert's weights are reused from L2).  Blocks past the
  // padded route count, or of no expert, are skipped by every role alike.
  const int post = *p.num_post_pad;
  const int m_used = (post + kBM - 1) / kBM < p.m_blocks ? (post + kBM - 1) / kBM : p.m_blocks;
  const int ntiles = m_used * p.n_tiles;
  auto tile_expert = [&](int t, int& m_block, int& n_tile) {
    m_block = t / p.n_tiles;
    n_tile = t - m_block * p.n_tiles;
    const int e = p.expert_ids[m_block];
    return (e >= 0 && e < p.experts) ? e : -1;
  };
  const uint32_t tmem = sm.tmem_base;
  volatile int* failed = &sm.failed;
  const int kblocks = p.k / kBK;

  if (warp == 0) {
    // ---- TMA producer: one stage ring across all of this CTA's tiles
    if (lane == 0) {
      uint32_t g = 0;  // k-blocks issued
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int m_block, n_tile;
        const int expert = tile_expert(t, m_block, n_tile);
        if (expert < 0) continue;
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kStages;
          ok = mbar_wait(&sm.empty[s], ((g / kStages) & 1) ^ 1, failed);
          if (!ok) break;
          uint8_t* a_dst = sm.tiles[s];
          uint8_t* b_dst = sm.tiles[s] + kATileBytes;
          mbar_expect_tx(&sm.full[s], kStageBytes);
          tma_load_2d(a_dst, &map_a, &sm.full[s], kb * kBK, m_block * kBM);
          if (KIND == kGemmSwiGLU) {
            // gate rows [n0, n0+128) and up rows [I + n0, I + n0 + 128) of W13[expert]
            const int row0 = expert * 2 * p.n_total + n_tile * (kBN / 2);
            tma_load_2d(b_dst, &map_b, &sm.full[s], kb * kBK, row0);
            tma_load_2d(b_dst + kBTileBytes / 2, &map_b, &sm.full[s], kb * kBK,
                        row0 + p.n_total);
          } else {
            tma_load_2d(b_dst, &map_b, &sm.full[s], kb * kBK, expert * p.n_total + n_tile * kBN);
          }
        }
      }
      // copies still in flight (only after a time-out) land before shared memory is released
      for (uint32_t j = g > kStages ? g - kStages : 0; j < g; ++j)
        mbar_wait_drain(&sm.full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer (one thread): tile i accumulates into TMEM columns [256 (i & 1), +256)
    if (lane == 0) {
      uint32_t g = 0;  // k-blocks consumed
      int i = 0;       // tiles accumulated
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int m_block, n_tile;
        if (tile_expert(t, m_block, n_tile) < 0) continue;
        const int b = i & 1;
        ok = mbar_wait(&sm.acc_empty[b], ((i >> 1) & 1) ^ 1, failed);
        if (!ok) break;
        fence_after_sync();
        const uint32_t acc = tmem + static_cast<uint32_t>(b * kBN);
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kStages;
          ok = mbar_wait(&sm.full[s], (g / kStages) & 1, failed);
          if (!ok) break;
          fence_after_sync();
          const uint32_t a_base = smem_addr(sm.tiles[s]);
          const uint32_t b_base = a_base + kATileBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_kind_f16(acc, smem_desc(a_base + k * 32), smem_desc(b_base + k * 32),
                     GemmCfg<BN>::kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&sm.empty[s]);
        }
        if (!ok) break;
        mma_commit(&sm.acc_full[b]);
        ++i;
      }
      // every MMA this thread issued has completed before TMEM is released
      mma_commit(&sm.drain);
      mbar_wait_drain(&sm.drain, 0);
    }
  } else {
    // ---- epilogue: warps 2-5 own TMEM lanes 32*(warp%4) .. +31, one output row per thread
    const int q = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      int m_block, n_tile;
      if (tile_expert(t, m_block, n_tile) < 0) continue;
      const int b = i & 1;
      const bool ok = mbar_wait(&sm.acc_full[b], (i >> 1) & 1, failed);
      fence_after_sync();
      if (!ok || *failed) break;
      const int row = m_block * kBM + q * 32 + lane;
      const uint32_t taddr = tmem + static_cast<uint32_t>(b * kBN) + ((uint32_t)(q * 32) << 16);
      if (KIND == kGemmSwiGLU) {
        // act[row, n0 + c] = silu(gate) * up; gate in columns [0,128), up in [128,256)
        __nv_bfloat16* dst = p.act + (int64_t)row * p.n_total + n_tile * (kBN / 2);
#pragma unroll 1
        for (int c = 0; c < kBN / 2; c += 32) {
          float gt[32], up[32];
          tmem_load32(taddr + c, gt);
          tmem_load32(taddr + kBN / 2 + c, up);
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float a0 = gt[2 * j] / (1.0f + __expf(-gt[2 * j])) * up[2 * j];
            const float a1 = gt[2 * j + 1] / (1.0f + __expf(-gt[2 * j + 1])) * up[2 * j + 1];
            packed[j] = pack_bf16(a0, a1);
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
        }
      } else {
        // out[route, n0 + c] = w_route * acc for real routes; padding rows are dropped.  The
        // TMEM loads are warp-collective, so every lane runs them and only the stores are
        // predicated.
        const int route = p.sorted_ids[row];
        const bool real = route < p.numel;
        const float wr = real ? p.route_w[route] : 0.0f;
        __nv_bfloat16* dst = p.out + (int64_t)(real ? route : 0) * p.hidden + n_tile * kBN;
#pragma unroll 1
        for (int c = 0; c < kBN; c += 32) {
          float v[32];
          tmem_load32(taddr + c, v);
          if (real) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              d4[j] = make_uint4(pack_bf16(v[8 * j] * wr, v[8 * j + 1] * wr),
                                 pack_bf16(v[8 * j + 2] * wr, v[8 * j + 3] * wr),
                                 pack_bf16(v[8 * j + 4] * wr, v[8 * j + 5] * wr),
                                 pack_bf16(v[8 * j + 6] * wr, v[8 * j + 7] * wr));
          }
        }
      }
      // the accumulator has been read: the MMA thread may start the tile after next in it
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
      ++i;
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after_sync();
    tmem_free(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && sm.failed && p.status) atomicExch(p.status, 1);
}

// ---- decode: one persistent kernel for the whole expert layer, routes on the N side ------------
// At decode an expert holds a few routes, so a 128-row block of routes is mostly padding, and the
// MMA work of that padding, not the weight stream, bounds the layer.  Here a tile is 256 weight
// rows of one expert (two 128-row MMA tiles on the M side, all real) times a block of BT = 64 of
// its routes (the N side; the moe_align block size of this path):
//   GEMM-1 tile (block, f): gate rows [128 f, +128) and up rows [I + 128 f, +128) of W13[e]
//     against the block's gathered token rows xs, K = H; the epilogue writes
//     act[r][128 f + i] = silu(gate) * up for the block's real routes;
//   GEMM-2 tile (block, f): rows [256 f, +256) of W2[e] against act, K = I; the epilogue writes
//     out[route][256 f + i] = w_route * D.
// Every pipeline stage holds two 16 KB weight tiles and one 8 KB route tile (80 % weights), in
// both GEMMs.  One launch runs both GEMMs so that no SM idles at the end of GEMM-1 (its 1 MB
// tiles come in few rounds per SM): warp 0 takes tiles from a counter shared by all CTAs, all
// GEMM-1 tiles first, block by block, then the GEMM-2 tiles; before loading act for a GEMM-2
// tile it waits until every epilogue warp that wrote the block's act rows has counted itself off
// (release / acquire on sync[1 + block], with proxy fences: act is written by plain stores and
// read by TMA).  A GEMM-1 tile never waits for anything but earlier tiles of its own CTA, so the
// GEMM-1 tiles a GEMM-2 tile needs always finish: each was handed out earlier to a running CTA
// whose producer had issued all of its loads before taking another tile.  Warp 0 passes tile
// numbers to the MMA warp and the epilogue warps through a ring in shared memory.  Roles, the
// stage ring, TMEM double buffering and bounded waits otherwise as in expert_gemm_kernel; a
// time-out anywhere marks the CTA failed, and the rest of the CTA drains and returns.
struct ExpertLayerParams {
  const int32_t* num_post_pad;
  const int32_t* expert_ids;   // [m_blocks]
  const int32_t* sorted_ids;   // [m_blocks * BT]
  int experts;
  int numel;
  int hidden;
  int inter;
  int m_blocks;
  int* status;
  __nv_bfloat16* act;          // [m_blocks * BT][inter]
  const float* route_w;        // [numel]
  __nv_bfloat16* out;          // [numel][hidden]
  int32_t* sync;               // [0] next tile; [1 + b] GEMM-1 epilogue warps done with block b
};

template <int BT>
struct LCfg {
  static constexpr int kWTile = 128 * kBK * 2;   // 16 KB: 128 weight rows x 64 K
  static constexpr int kTTile = BT * kBK * 2;    // BT route rows x 64 K
  static constexpr int kStageBytes = 2 * kWTile + kTTile;
  static constexpr int kStages = (200 * 1024) / kStageBytes;
  static constexpr int kAccCols = 2 * BT;        // two M tiles of BT columns
  static constexpr int kTmemCols = 2 * kAccCols; // two tiles in flight
  static constexpr int kRing = 8;                // tile numbers handed to the MMA and epilogue
  static constexpr uint32_t kIdesc = idesc_f16(128, BT, true);  // bf16, M = 128, N = BT
};

template <int BT>
struct LSmem {
  alignas(1024) uint8_t tiles[LCfg<BT>::kStages][LCfg<BT>::kStageBytes];
  alignas(8) uint64_t full[LCfg<BT>::kStages];
  alignas(8) uint64_t empty[LCfg<BT>::kStages];
  alignas(8) uint64_t acc_full[2];
  alignas(8) uint64_t acc_empty[2];
  alignas(8) uint64_t ring_full[LCfg<BT>::kRing];
  alignas(8) uint64_t ring_empty[LCfg<BT>::kRing];
  alignas(8) uint64_t drain;
  int ring[LCfg<BT>::kRing];
  uint32_t tmem_base;
  int failed;
};
template <int BT>
constexpr size_t layer_smem_bytes() { return sizeof(LSmem<BT>) + 1024; }
static_assert(layer_smem_bytes<64>() <= 232448, "decode expert layer shared memory");

// Tile t of the layer over `blocks` route blocks: GEMM-1 tiles [0, blocks * n1) block-major,
// then GEMM-2 tiles block-major.
struct LayerTile {
  int kind;   // kGemmSwiGLU or kGemmDown
  int blk;
  int ft;
};
__device__ __forceinline__ LayerTile layer_tile(int t, int blocks, int n1, int n2) {
  LayerTile r;
  const int s_tiles = blocks * n1;
  if (t < s_tiles) {
    r.kind = kGemmSwiGLU;
    r.blk = t / n1;
    r.ft = t - r.blk * n1;
  } else {
    t -= s_tiles;
    r.kind = kGemmDown;
    r.blk = t / n2;
    r.ft = t - r.blk * n2;
  }
  return r;
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int BT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    expert_layer_t_kernel(const __grid_constant__ CUtensorMap map_w13,
                          const __grid_constant__ CUtensorMap map_xs,
                          const __grid_constant__ CUtensorMap map_w2,
                          const __grid_constant__ CUtensorMap map_act,
                          const ExpertLayerParams p) {
  using C = LCfg<BT>;
  constexpr int kStages = C::kStages;
  constexpr int kRing = C::kRing;
  extern __shared__ uint8_t smem_raw[];
  LSmem<BT>& sm = *reinterpret_cast<LSmem<BT>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    for (int j = 0; j < kRing; ++j) {
      mbar_init(&sm.ring_full[j], 1);
      mbar_init(&sm.ring_empty[j], 5);  // the MMA thread and the four epilogue warps
    }
    mbar_init(&sm.drain, 1);
    sm.failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, C::kTmemCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int post = *p.num_post_pad;
  const int blocks = (post + BT - 1) / BT < p.m_blocks ? (post + BT - 1) / BT : p.m_blocks;
  const int n1 = p.inter / 128;  // GEMM-1 tiles per block
  const int n2 = p.hidden / 256; // GEMM-2 tiles per block
  const int total = blocks * (n1 + n2);
  const uint32_t tmem = sm.tmem_base;
  volatile int* failed = &sm.failed;
  auto expert_of = [&](const LayerTile& lt) {
    const int e = p.expert_ids[lt.blk];
    return (e >= 0 && e < p.experts) ? e : -1;
  };

  if (warp == 0) {
    // ---- scheduler + TMA producer (one thread)
    if (lane == 0) {
      uint32_t g = 0;  // stages issued
      bool ok = true;
      int t = atomicAdd(p.sync, 1);
      for (int j = 0; ok; ++j) {
        const int tile = t < total ? t : -1;
        const int slot = j % kRing;
        ok = mbar_wait(&sm.ring_empty[slot], ((j / kRing) & 1) ^ 1, failed);
        if (!ok) break;
        sm.ring[slot] = tile;
        mbar_arrive(&sm.ring_full[slot]);
        if (tile < 0) break;
        t = atomicAdd(p.sync, 1);  // the next tile: its latency overlaps this tile's loads
        const LayerTile lt = layer_tile(tile, blocks, n1, n2);
        const int expert = expert_of(lt);
        if (expert < 0) continue;
        const bool down = lt.kind == kGemmDown;
        if (down) {
          // act rows of the block: every epilogue warp of its n1 GEMM-1 tiles has counted itself
          // off (bounded wait; the GEMM-1 tiles were handed out earlier to running CTAs)
          const int32_t* flag = p.sync + 1 + lt.blk;
          const int want = 4 * n1;
          uint32_t it = 0;
          while (ld_acquire_gpu(flag) < want) {
            if (*failed || ++it >= kWaitLimit) {
              *failed = 1;
              ok = false;
              break;
            }
            __nanosleep(128);
          }
          if (!ok) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        const int kblocks = (down ? p.inter : p.hidden) / kBK;
        const CUtensorMap* mw = down ? &map_w2 : &map_w13;
        const CUtensorMap* mt = down ? &map_act : &map_xs;
        // the two 128-row weight tiles: gate and up rows of W13[e], or 256 rows of W2[e]
        const int row0 = down ? expert * p.hidden + lt.ft * 256 : expert * 2 * p.inter + lt.ft * 128;
        const int row1 = down ? row0 + 128 : row0 + p.inter;
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kStages;
          ok = mbar_wait(&sm.empty[s], ((g / kStages) & 1) ^ 1, failed);
          if (!ok) break;
          uint8_t* st = sm.tiles[s];
          mbar_expect_tx(&sm.full[s], C::kStageBytes);
          tma_load_2d(st, mw, &sm.full[s], kb * kBK, row0);
          tma_load_2d(st + C::kWTile, mw, &sm.full[s], kb * kBK, row1);
          tma_load_2d(st + 2 * C::kWTile, mt, &sm.full[s], kb * kBK, lt.blk * BT);
        }
      }
      // (after a failure the consumers leave their waits on the failed flag)
      for (uint32_t j = g > kStages ? g - kStages : 0; j < g; ++j)
        mbar_wait_drain(&sm.full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer: tile i accumulates into TMEM columns [kAccCols (i & 1), +kAccCols)
    if (lane == 0) {
      uint32_t g = 0;
      int i = 0;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int slot = j % kRing;
        ok = mbar_wait(&sm.ring_full[slot], (j / kRing) & 1, failed);
        if (!ok) break;
        const int tile = sm.ring[slot];
        mbar_arrive(&sm.ring_empty[slot]);
        if (tile < 0) break;
        const LayerTile lt = layer_tile(tile, blocks, n1, n2);
        if (expert_of(lt) < 0) continue;
        const int kblocks = (lt.kind == kGemmDown ? p.inter : p.hidden) / kBK;
        const int b = i & 1;
        ok = mbar_wait(&sm.acc_empty[b], ((i >> 1) & 1) ^ 1, failed);
        if (!ok) break;
        fence_after_sync();
        const uint32_t acc = tmem + static_cast<uint32_t>(b * C::kAccCols);
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kStages;
          ok = mbar_wait(&sm.full[s], (g / kStages) & 1, failed);
          if (!ok) break;
          fence_after_sync();
          const uint32_t w_base = smem_addr(sm.tiles[s]);
          const uint32_t t_base = w_base + 2 * C::kWTile;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint32_t on = (kb > 0 || k > 0) ? 1u : 0u;
            mma_kind_f16(acc, smem_desc(w_base + k * 32), smem_desc(t_base + k * 32), C::kIdesc,
                         on);
            mma_kind_f16(acc + BT, smem_desc(w_base + C::kWTile + k * 32),
                         smem_desc(t_base + k * 32), C::kIdesc, on);
          }
          mma_commit(&sm.empty[s]);
        }
        if (!ok) break;
        mma_commit(&sm.acc_full[b]);
        ++i;
      }
      mma_commit(&sm.drain);
      mbar_wait_drain(&sm.drain, 0);
    }
  } else {
    // ---- epilogue: warps 2-5 own TMEM lanes 32 (warp % 4) .. +31, i.e. 32 weight rows of each
    // M tile; columns are the block's routes.  Lane j fetches route j of each 32-route chunk and
    // shares it.
    const int q = warp & 3;
    int i = 0;
    for (int j = 0;; ++j) {
      const int slot = j % kRing;
      int tile = -2;  // -2: the wait failed
      if (lane == 0 && mbar_wait(&sm.ring_full[slot], (j / kRing) & 1, failed)) {
        tile = sm.ring[slot];
        mbar_arrive(&sm.ring_empty[slot]);
      }
      tile = __shfl_sync(0xffffffffu, tile, 0);
      if (tile < 0) break;
      const LayerTile lt = layer_tile(tile, blocks, n1, n2);
      if (expert_of(lt) < 0) continue;
      const int b = i & 1;
      const bool ok = mbar_wait(&sm.acc_full[b], (i >> 1) & 1, failed);
      fence_after_sync();
      if (!ok || *failed) break;
      const uint32_t taddr =
          tmem + static_cast<uint32_t>(b * C::kAccCols) + ((uint32_t)(q * 32) << 16);
      if (lt.kind == kGemmSwiGLU) {
        const int feat = lt.ft * 128 + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BT; c += 32) {
          const bool real_l = p.sorted_ids[lt.blk * BT + c + lane] < p.numel;
          float gt[32], up[32];
          tmem_load32(taddr + c, gt);
          tmem_load32(taddr + BT + c, up);
          __nv_bfloat16* dst = p.act + (int64_t)(lt.blk * BT + c) * p.inter + feat;
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const bool real = __shfl_sync(0xffffffffu, real_l, r);
            if (real)
              dst[(int64_t)r * p.inter] =
                  __float2bfloat16_rn(gt[r] / (1.0f + __expf(-gt[r])) * up[r]);
          }
        }
      } else {
        const int feat = lt.ft * 256 + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BT; c += 32) {
          const int route_l = p.sorted_ids[lt.blk * BT + c + lane];
          const float w_l = route_l < p.numel ? p.route_w[route_l] : 0.0f;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {  // the two M tiles: features feat and feat + 128
            float v[32];
            tmem_load32(taddr + h * BT + c, v);
#pragma unroll
            for (int r = 0; r < 32; ++r) {
              const int route = __shfl_sync(0xffffffffu, route_l, r);
              const float wr = __shfl_sync(0xffffffffu, w_l, r);
              if (route < p.numel)
                p.out[(int64_t)route * p.hidden + feat + h * 128] = __float2bfloat16_rn(v[r] * wr);
            }
          }
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
      ++i;
      if (lt.kind == kGemmSwiGLU) {
        // this warp's act rows of the tile are written: make them visible to the TMA loads of
        // the block's GEMM-2 tiles (any CTA), then count the warp off
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_gpu_add(p.sync + 1 + lt.blk, 1);
      }
    }
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after_sync();
    tmem_free(tmem, C::kTmemCols);
  }
  if (threadIdx.x == 0 && sm.failed && p.status) atomicExch(p.status, 1);
}

// ---- gather and combine ---------------------------------------------------------------------
// Both passes give one thread one 16-byte vector per grid-stride step, so a warp's accesses stay
// in one region of memory at a time (unrolling a thread over vectors a grid stride apart measured
// 20 % slower at prefill: its loads spread over distant pages).
// xs[m] = x[sorted_ids[m] / top_k] for the real routes of the used rows (16-byte vectors); also
// zeroes zero[0, zero_n).  Padding rows keep whatever the workspace holds: the GEMM rows are
// independent, GEMM-1's padding rows only feed GEMM-2's padding rows, and those are never stored.
__global__ void __launch_bounds__(256) gather_rows_kernel(const __nv_bfloat16* x,
                                                          const int32_t* sorted_ids,
                                                          const int32_t* num_post_pad,
                                                          int64_t rows, int numel, int top_k,
                                                          int hidden, __nv_bfloat16* xs,
                                                          int32_t* zero, int zero_n) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < zero_n; i += gridDim.x * blockDim.x)
    zero[i] = 0;  // the decode expert layer kernel's counters
  const int vec = hidden / 8;
  const int64_t used = *num_post_pad < rows ? *num_post_pad : rows;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < used * vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / vec;
    const int c = (int)(i - m * vec);
    const int route = sorted_ids[m];
    if (route < numel)
      reinterpret_cast<uint4*>(xs + m * hidden)[c] =
          reinterpret_cast<const uint4*>(x + (int64_t)(route / top_k) * hidden)[c];
  }
}

// y[t] = sum_j out[t * top_k + j] in fp32, route order fixed; routes whose expert id is out of
// range were never placed by moe_align and contribute nothing.  top_k <= 8: the loads of all of
// a vector's routes are issued before the sum (one round trip per vector, not top_k).
__global__ void __launch_bounds__(256, 4) combine_kernel(const __nv_bfloat16* __restrict__ out,
                                                      const int32_t* __restrict__ ids, int experts,
                                                      int64_t tokens, int top_k, int hidden,
                                                      __nv_bfloat16* y) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int vec = hidden / 8;
  const uint4* out4 = reinterpret_cast<const uint4*>(out);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tokens * vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vec;
    const int c = (int)(i - t * vec);
    uint4 v[8];
    bool use[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = j < top_k ? __ldg(ids + t * top_k + j) : -1;
      use[j] = e >= 0 && e < experts;
      if (use[j]) v[j] = __ldg(out4 + (t * top_k + j) * vec + c);
    }
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (!use[j]) continue;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]);
    o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]);
    o.w = pack_bf16(acc[6], acc[7]);
    reinterpret_cast<uint4*>(y)[i] = o;
  }
}

// ---- host side ---------------------------------------------------------------------------------
// The kernels need more than 48 KB of dynamic shared memory: opt in once per device.
static cudaError_t allow_gemm_smem() {
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return cudaSuccess;
  const int s256 = (int)gemm_smem_bytes<256>();
  if ((e = cudaFuncSetAttribute(expert_layer_t_kernel<64>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)layer_smem_bytes<64>())) != cudaSuccess ||
      (e = cudaFuncSetAttribute(expert_gemm_kernel<kGemmSwiGLU, 256>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, s256)) != cudaSuccess ||
      (e = cudaFuncSetAttribute(expert_gemm_kernel<kGemmDown, 256>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, s256)) != cudaSuccess)
    return e;
  done[dev] = true;
  return cudaSuccess;
}

// Launch as a programmatic dependent of the previous kernel in the stream (the kernel calls
// griddepcontrol.wait before reading anything that kernel wrote).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// One CTA per SM (192 KB of pipeline stages and all 512 TMEM columns), never more than tiles.
static unsigned persistent_tiles(const ExpertGemmParams& p) {
  const int64_t tiles = (int64_t)p.m_blocks * p.n_tiles;
  const int sms = sm_count();
  int64_t g = sms > 0 && tiles > sms ? sms : tiles;
  return (unsigned)(g > 0 ? g : 1);
}

int64_t moe_capacity(int64_t numel, int experts) {
  int64_t cap = numel + (int64_t)experts * (kBM - 1);
  cap = (cap + kBM - 1) / kBM * kBM;
  if (numel < experts && numel * kBM < cap) cap = numel * kBM;
  return cap;
}

static int64_t up256(int64_t b) { return (b + 255) / 256 * 256; }

MoeWorkspace moe_workspace(int64_t tokens, int top_k, int experts, int hidden, int inter,
                           void* base) {
  MoeWorkspace w{};
  const int64_t numel = tokens * top_k;
  const int64_t cap = moe_capacity(numel, experts);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off += up256(bytes);
    return base ? static_cast<uint8_t*>(base) + o : nullptr;
  };
  w.capacity = cap;
  w.sorted_ids = reinterpret_cast<int32_t*>(take(cap * 4));
  w.expert_ids = reinterpret_cast<int32_t*>(take((cap / 64) * 4));  // blocks of 64 routes or more
  w.num_post_pad = reinterpret_cast<int32_t*>(take(4));
  w.align_bytes = align_workspace_bytes(numel, experts);
  w.align_ws = take(w.align_bytes > 0 ? w.align_bytes : 4);
  w.xs = reinterpret_cast<__nv_bfloat16*>(take(cap * hidden * 2));
  w.act = reinterpret_cast<__nv_bfloat16*>(take(cap * inter * 2));
  w.out = reinterpret_cast<__nv_bfloat16*>(take(numel * hidden * 2));
  w.layer_sync_ints = (int)(1 + cap / 64);
  w.layer_sync = reinterpret_cast<int32_t*>(take(w.layer_sync_ints * 4));
  w.bytes = off;
  return w;
}

// GEMM-1 (+ SwiGLU) and GEMM-2 of launch_moe_experts with an N tile of BN.
template <int BN>
static cudaError_t launch_gemms(const MoeArgs& a, const MoeWorkspace& w, cudaStream_t s) {
  const int64_t numel = a.tokens * a.top_k;
  const int64_t cap = w.capacity;
  constexpr size_t smem = gemm_smem_bytes<BN>();
  CUtensorMap ma, mb;
  if (!make_map(&ma, w.xs, cap, a.hidden, kBM) ||
      !make_map(&mb, a.w13, (uint64_t)a.experts * 2 * a.inter, a.hidden, BN / 2))
    return cudaErrorInvalidValue;
  ExpertGemmParams p{};
  p.num_post_pad = w.num_post_pad;
  p.expert_ids = w.expert_ids;
  p.sorted_ids = w.sorted_ids;
  p.experts = a.experts;
  p.numel = (int)numel;
  p.hidden = a.hidden;
  p.status = a.status;
  p.k = a.hidden;
  p.n_total = a.inter;
  p.act = w.act;
  p.m_blocks = (int)(cap / kBM);
  p.n_tiles = a.inter / (BN / 2);
  cudaError_t e = launch_pdl(expert_gemm_kernel<kGemmSwiGLU, BN>, persistent_tiles(p),
                             kGemmThreads, smem, s, ma, mb, p);
  if (e != cudaSuccess) return e;
  if (!make_map(&ma, w.act, cap, a.inter, kBM) ||
      !make_map(&mb, a.w2, (uint64_t)a.experts * a.hidden, a.inter, BN))
    return cudaErrorInvalidValue;
  p.k = a.inter;
  p.n_total = a.hidden;
  p.route_w = a.topk_w;
  p.out = w.out;
  p.n_tiles = a.hidden / BN;
  return launch_pdl(expert_gemm_kernel<kGemmDown, BN>, persistent_tiles(p), kGemmThreads, smem,
                    s, ma, mb, p);
}

// The decode expert layer (both GEMMs, routes on the N side; see expert_layer_t_kernel) over
// routes aligned into blocks of BT.
template <int BT>
static cudaError_t launch_layer_t(const MoeArgs& a, const MoeWorkspace& w, cudaStream_t s) {
  const int64_t cap = w.capacity;
  CUtensorMap m13, mxs, m2, mact;
  if (!make_map(&m13, a.w13, (uint64_t)a.experts * 2 * a.inter, a.hidden, 128) ||
      !make_map(&mxs, w.xs, cap, a.hidden, BT) ||
      !make_map(&m2, a.w2, (uint64_t)a.experts * a.hidden, a.inter, 128) ||
      !make_map(&mact, w.act, cap, a.inter, BT))
    return cudaErrorInvalidValue;
  ExpertLayerParams p{};
  p.num_post_pad = w.num_post_pad;
  p.expert_ids = w.expert_ids;
  p.sorted_ids = w.sorted_ids;
  p.experts = a.experts;
  p.numel = (int)(a.tokens * a.top_k);
  p.hidden = a.hidden;
  p.inter = a.inter;
  p.m_blocks = (int)(cap / BT);
  p.status = a.status;
  p.act = w.act;
  p.route_w = a.topk_w;
  p.out = w.out;
  p.sync = w.layer_sync;
  const int sms = sm_count();
  return launch_pdl(expert_layer_t_kernel<BT>, sms > 0 ? (unsigned)sms : 1u, kGemmThreads,
                    layer_smem_bytes<BT>(), s, m13, mxs, m2, mact, p);
}

// The moe_align block size, which also picks the GEMM kernels: 128-row blocks of routes on the M
// side (prefill); when the experts hold 64 routes or fewer on average (decode), blocks of 64
// routes on the N side.  (Blocks of 32 measured at most 2 % faster on a few decode shapes and
// 43 % slower at 512 tokens x top-8 over 64 experts: an expert's two blocks read its weights
// twice.)
constexpr int kDecodeBlock = 64;
static int gemm_block(int64_t numel, int experts) {
  return numel > (int64_t)experts * 64 ? kBM : kDecodeBlock;
}

// Steps 3-5 of launch_moe_experts: GEMM-1 + SwiGLU, GEMM-2, combine, from token rows already
// gathered into w.xs in the order of routes aligned into blocks of gemm_block.
static cudaError_t launch_moe_gemms(const MoeArgs& a, const MoeWorkspace& w, cudaStream_t s) {
  cudaError_t e = allow_gemm_smem();
  if (e != cudaSuccess) return e;
  // 3-4. GEMM-1 + SwiGLU, GEMM-2
  e = gemm_block(a.tokens * a.top_k, a.experts) == kDecodeBlock
          ? launch_layer_t<kDecodeBlock>(a, w, s)
          : launch_gemms<256>(a, w, s);
  if (e != cudaSuccess) return e;
  // 5. combine the routes of each token
  const int64_t work = a.tokens * (a.hidden / 8);
  int64_t blocks = (work + 255) / 256;
  const int lim = 8 * sm_count();
  if (lim > 0 && blocks > lim) blocks = lim;
  return launch_pdl(combine_kernel, (unsigned)(blocks > 0 ? blocks : 1), 256, 0, s,
                    static_cast<const __nv_bfloat16*>(w.out), a.topk_ids, a.experts, a.tokens,
                    a.top_k, a.hidden, static_cast<__nv_bfloat16*>(a.y));
}

// Steps 2-5 of launch_moe_experts, from routes already aligned into w (blocks of gemm_block).
static cudaError_t launch_moe_compute(const MoeArgs& a, const MoeWorkspace& w, cudaStream_t s) {
  const int64_t numel = a.tokens * a.top_k;
  const int64_t cap = w.capacity;
  // 2. gather token rows into route order
  const int64_t work = cap * (a.hidden / 8);
  int64_t blocks = (work + 255) / 256;
  const int lim = 8 * sm_count();
  if (lim > 0 && blocks > lim) blocks = lim;
  const cudaError_t e =
      launch_pdl(gather_rows_kernel, (unsigned)(blocks > 0 ? blocks : 1), 256, 0, s,
                 static_cast<const __nv_bfloat16*>(a.x), static_cast<const int32_t*>(w.sorted_ids),
                 static_cast<const int32_t*>(w.num_post_pad), cap, (int)numel, a.top_k, a.hidden,
                 w.xs, w.layer_sync, w.layer_sync_ints);
  return e != cudaSuccess ? e : launch_moe_gemms(a, w, s);
}

cudaError_t launch_moe_experts(const MoeArgs& a, const MoeWorkspace& w, cudaStream_t s) {
  // 1-2. moe_align with the GEMM's blocks, then the gather of token rows; at decode sizes both
  // in one launch of one CTA per SM
  const int64_t numel = a.tokens * a.top_k;
  AlignParams ap{a.topk_ids, numel, a.experts, gemm_block(numel, a.experts), w.capacity,
                 w.sorted_ids, w.expert_ids, w.num_post_pad, static_cast<int32_t*>(w.align_ws), 0};
  if (numel <= align_gather_max_numel()) {
    const cudaError_t e = launch_align_gather(ap, a.x, a.top_k, a.hidden, w.xs, w.layer_sync,
                                              w.layer_sync_ints, s);
    return e != cudaSuccess ? e : launch_moe_gemms(a, w, s);
  }
  const cudaError_t e = launch_align(0 /*int32*/, ap, s);
  return e != cudaSuccess ? e : launch_moe_compute(a, w, s);
}

int64_t decode_moe_workspace_bytes(int64_t tokens, int top_k, int experts, int hidden,
                                   int inter) {
  return moe_workspace(tokens, top_k, experts, hidden, inter, nullptr).bytes +
         2 * up256(tokens * top_k * 4);
}

cudaError_t launch_decode_moe_experts(DecodeParams d, const MoeArgs& a, void* workspace,
                                      cudaStream_t s) {
  const MoeWorkspace w = moe_workspace(a.tokens, a.top_k, a.experts, a.hidden, a.inter, workspace);
  uint8_t* extra = static_cast<uint8_t*>(workspace) + w.bytes;
  d.top_k = a.top_k;
  d.gemm_w = reinterpret_cast<float*>(extra);
  d.gemm_ids = reinterpret_cast<int32_t*>(extra + up256(a.tokens * a.top_k * 4));
  // 1. decode, with the routes of one token to one expert merged
  cudaError_t e = launch_decode_merge(d, s);
  if (e != cudaSuccess) return e;
  // 2. moe_align over the merged routes and the gather of token rows, one launch
  const int64_t numel = a.tokens * a.top_k;
  AlignParams ap{d.gemm_ids, numel, a.experts, gemm_block(numel, a.experts), w.capacity,
                 w.sorted_ids, w.expert_ids, w.num_post_pad, static_cast<int32_t*>(w.align_ws), 0};
  e = launch_align_gather(ap, a.x, a.top_k, a.hidden, w.xs, w.layer_sync, w.layer_sync_ints, s);
  if (e != cudaSuccess) return e;
  // 3. the expert layer over the merged routes
  MoeArgs m = a;
  m.topk_w = d.gemm_w;
  m.topk_ids = d.gemm_ids;
  return launch_moe_gemms(m, w, s);
}

}  // namespace exf
