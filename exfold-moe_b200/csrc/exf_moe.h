// Grouped SwiGLU expert computation: parameter blocks and host entry (internal).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "exf_kernels.h"

namespace exf {

struct ExpertGemmParams {
  const int32_t* num_post_pad;
  const int32_t* expert_ids;   // [capacity / 128]
  const int32_t* sorted_ids;   // [capacity]
  int experts;
  int numel;                   // routes = tokens * top_k
  int hidden;
  int k;                       // reduction length of this GEMM
  int n_total;                 // GEMM-1: intermediate size; GEMM-2: hidden size
  int n_tiles;                 // output tiles per 128-row block
  int m_blocks;                // 128-row blocks of the capacity (those past the padded count
                               // are skipped on the device)
  int* status;                 // set to 1 if a pipeline wait timed out (may be null)
  __nv_bfloat16* act;          // GEMM-1 output [capacity][intermediate]
  const float* route_w;        // GEMM-2: [numel] routing weights
  __nv_bfloat16* out;          // GEMM-2 output [numel][hidden]
};

struct MoeArgs {
  const void* x;               // bf16 [tokens][hidden]
  const float* topk_w;         // fp32 [tokens][top_k]
  const int32_t* topk_ids;     // int32 [tokens][top_k]
  int64_t tokens;
  int top_k;
  const void* w13;             // bf16 [experts][2 * inter][hidden]  (gate rows, then up rows)
  const void* w2;              // bf16 [experts][hidden][inter]
  int experts;
  int hidden;
  int inter;
  void* y;                     // bf16 [tokens][hidden]
  int* status;
};

struct MoeWorkspace {
  int64_t capacity;
  int32_t* sorted_ids;
  int32_t* expert_ids;
  int32_t* num_post_pad;
  void* align_ws;
  int64_t align_bytes;
  __nv_bfloat16* xs;
  __nv_bfloat16* act;
  __nv_bfloat16* out;
  // the decode expert layer kernel's counters: [0] the next tile to hand out, [1 + b] the GEMM-1
  // tiles of route block b finished (zeroed by the gather before each layer)
  int32_t* layer_sync;
  int layer_sync_ints;
  int64_t bytes;
};

int64_t moe_capacity(int64_t numel, int experts);
// Carves the workspace at `base` (null: sizes only).
MoeWorkspace moe_workspace(int64_t tokens, int top_k, int experts, int hidden, int inter,
                           void* base);
cudaError_t launch_moe_experts(const MoeArgs& a, const MoeWorkspace& w, cudaStream_t s);
// Decode expert budget (d: the exf_decode parameters; fp32 weights, int32 ids) followed by the
// expert layer over its routes, with moe_align done inside the decode launch and duplicate
// (token, expert) routes merged.  The workspace holds a MoeWorkspace then the merged routes.
int64_t decode_moe_workspace_bytes(int64_t tokens, int top_k, int experts, int hidden,
                                   int inter);
cudaError_t launch_decode_moe_experts(DecodeParams d, const MoeArgs& a, void* workspace,
                                      cudaStream_t s);

}  // namespace exf
