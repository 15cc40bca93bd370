// Kernel parameter blocks and host launchers (internal to libexfold_b200.so).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exf {

enum FoldKind { kFoldNone = 0, kFoldQwen3 = 1, kFoldDsv4 = 2 };

struct RouterParams {
  const void* logits;    // [layers][tokens][E] of logit_dtype
  int64_t tokens;        // per layer
  int layers;
  int top_k;
  const float* bias;     // [layers][E] or null
  int renormalize;
  float scaling;
  int target_k;
  int renorm_mode;
  const float* coeff;    // [layers][E][E]
  const float* sel_loss;
  const float* conf_loss;
  float* out_w;          // [layers][tokens][top_k or target_k]
  int32_t* out_ids;
  int logit_dtype;       // EXF_F32, EXF_BF16 or EXF_F16
};

struct FoldParams {
  const void* w;
  const void* ids;
  int64_t tokens;
  int top_k;
  int target_k;
  int experts;
  int renorm_mode;
  const float* coeff;
  const float* sel_loss;
  const float* conf_loss;
  void* out_w;
  void* out_ids;
};

enum DecodeSource {
  kImportanceFromRoutes = 0,
  kImportanceGiven = 1,
  kSubsetGiven = 2,
  kImportanceExchanged = 3  // from routes, then summed with the peer ranks' vectors in-launch
};

// Peer exchange of the sharded decode importance.  Every rank owns one buffer of
// exchange_longs(E, R) 64-bit words (zeroed before first use) laid out as
//   [kXchEpoch]                      calls made so far on this buffer (written by its rank only)
//   [kXchSlots + ((p R + r) E + e) 2 + h]   half h of rank r's importance of expert e, written
//                                            by rank r during a call of parity p
// Each word is (call number << 32) | 32-bit half, stored with one 8-byte store (single-copy
// atomic), so a receiver that reads the current call number in a word also reads its half: no
// fence or separate flag is needed.  A call numbered c writes this rank's vector into slot
// (c & 1, rank) of every rank's buffer by NVLink peer stores, then polls (bounded) its own slots
// of parity c & 1 until every word carries c, and sums the R vectors in rank order.  Two
// parities suffice: a rank writes call c + 2 only after reading every rank's call c + 1, which
// each rank writes only after finishing call c.
constexpr int kMaxPeers = 8;
constexpr int64_t kXchEpoch = 0;
constexpr int64_t kXchSlots = 16;
constexpr int64_t exchange_longs(int experts, int world) {
  return kXchSlots + 4 * static_cast<int64_t>(world) * experts;
}

struct DecodeParams {
  const void* w;
  const void* ids;
  int64_t routes;
  int experts;
  int budget;
  int variant;
  int source;
  const float* norms;
  const int64_t* importance;
  const int32_t* subset;
  const float* coeff;
  const float* loss;
  void* out_w;
  void* out_ids;
  int32_t* out_subset;
  // decode for the expert layer (launch_decode_merge only): the routes that the table sent to
  // one expert twice in a token become one route
  int top_k;
  float* gemm_w;            // [routes] weights for the expert layer (merged in slot order)
  int32_t* gemm_ids;        // [routes] expert of each route; -1 for a merged or invalid route
  // kImportanceExchanged only: this process's mapping of every rank's exchange buffer
  int world;
  int rank;
  int64_t* peers[kMaxPeers];
  int32_t* status;          // set to 1 when a peer's vector did not arrive in time (may be null)
  unsigned long long wait_ns;
  // set by the launcher: the loss and scale tables are copied into shared memory at the start
  // (E <= 128, 16-byte aligned tables)
  int tables_smem;
};

struct AlignParams {
  const void* ids;
  int64_t numel;
  int experts;
  int block_size;
  int64_t capacity;
  int32_t* sorted_ids;
  int32_t* expert_ids;
  int32_t* num_post_pad;
  int32_t* table;  // [chunks][experts]
  int64_t chunks;
};

cudaError_t launch_router(int experts, int scoring, int fold, const RouterParams& p, cudaStream_t s);
// Rows (tokens x layers) from which launch_router takes the tile kernels; sets it when rows >= 0
// and returns the previous value.
int64_t router_tile_min_rows(int64_t rows);
cudaError_t launch_router_hash(const void* logits, int logit_dtype, int64_t tokens, int experts,
                               int top_k, int scoring, const void* token_ids, int id_dtype,
                               const int32_t* table, int64_t table_rows, int renormalize,
                               float scaling, float* out_w, int32_t* out_ids, cudaStream_t s);
// One token per thread, bulk-copied tiles: 128 experts, softmax, top-8, renormalised, Qwen3 fold
// or none, 16-byte aligned logits and outputs.
bool router_tpt_eligible(int experts, int scoring, int fold, const RouterParams& p);
cudaError_t launch_router_tpt(int fold, const RouterParams& p, cudaStream_t s);
// Two lanes per token, bulk-copied tiles: 256 experts, biased sigmoid, top-8, DeepSeek-V4 fold or
// none, 16-byte aligned logits (and outputs without a fold, selection loss with one).
bool router_biased_eligible(int experts, int scoring, int fold, const RouterParams& p);
cudaError_t launch_router_biased(int fold, const RouterParams& p, cudaStream_t s);
cudaError_t launch_fold(int w_dtype, int id_dtype, int variant, const FoldParams& p, cudaStream_t s);
cudaError_t launch_decode(int w_dtype, int id_dtype, const DecodeParams& p, cudaStream_t s);
// Decode with the merged routes of the expert layer: fp32 weights, int32 ids, experts <=
// kDecodeAlignMaxExperts, routes <= kDecodeAlignMaxRoutes (moe_align and the gather of the layer
// then run in one align_gather launch), top_k <= 8
constexpr int kDecodeAlignMaxExperts = 256;
constexpr int kDecodeAlignMaxRoutes = 8192;
cudaError_t launch_decode_merge(const DecodeParams& p, cudaStream_t s);
cudaError_t launch_importance(int w_dtype, int id_dtype, const void* w, const void* ids,
                              int64_t routes, int experts, const float* norms, int64_t* imp,
                              cudaStream_t s);
cudaError_t launch_static_table(const float* norms, const float* coeff, const float* loss, int E,
                                int D, int32_t* target, float* scale, cudaStream_t s);
cudaError_t launch_static_remap(int w_dtype, int id_dtype, void* w, void* ids, int64_t routes,
                                int experts, const int32_t* target, const float* scale,
                                cudaStream_t s);
cudaError_t launch_align(int id_dtype, const AlignParams& p, cudaStream_t s);
// moe_align of int32 ids fused with the gather of token rows for the expert layer:
// xs[slot] = x[sorted_ids[slot] / top_k] (bf16 rows of `hidden`) for every placed route; at most
// align_gather_max_numel() routes.  zero[0, zero_n) is set to 0 as well (may be null / 0).
int64_t align_gather_max_numel();
cudaError_t launch_align_gather(const AlignParams& p, const void* x, int top_k, int hidden,
                                void* xs, int32_t* zero, int zero_n, cudaStream_t s);
cudaError_t launch_calib_update(int out_dtype, int id_dtype, const void* out, const void* ids,
                                int64_t tokens, int K, int H, int E, double* dot, double* tsq,
                                double* ssq, double* nsum, double* ncnt, cudaStream_t s);
cudaError_t launch_calib_finalize(const double* dot, const double* tsq, const double* ssq, int E,
                                  double ridge, double lo, double hi, float* coeff, float* loss,
                                  int32_t* nonfinite, cudaStream_t s);
cudaError_t launch_calib_norms(const double* nsum, const double* ncnt, int E, float* norms,
                               cudaStream_t s);
int64_t align_workspace_bytes(int64_t numel, int experts);
int align_max_experts();
int64_t align_static_table_ints();
cudaError_t launch_align_static(int id_dtype, AlignParams p, cudaStream_t s);

}  // namespace exf
