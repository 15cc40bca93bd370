/*
 * exfold_b200.h - C ABI of the B200 (sm_100a) ExFold routing-transform library
 * (libexfold_b200.so).
 *
 * Every entry point takes raw device pointers, sizes and enums, launches its
 * kernels on `stream` (a cudaStream_t; NULL = the legacy default stream) and
 * returns EXF_OK or a negative code; exf_last_error() then holds a message
 * for the calling thread.  No entry point allocates device memory, copies to
 * the host or synchronises: callers own every output and workspace buffer, so
 * the calls can be captured in CUDA graphs.  The first launch of a kernel that
 * uses more than 48 KB of shared memory raises its shared-memory limit once per
 * device (cudaFuncSetAttribute), so make one eager call of an entry point, with
 * the shapes it will be captured with, before capturing it.  Calibration tables are fp32,
 * row-major [source][target], `experts` x `experts`.  Routing tensors are
 * row-major [tokens][top_k].
 *
 * Reference interfaces (paths relative to the reference project root):
 *   exfold/qwen3/kernels.py                    Triton kernels + host wrappers
 *   exfold/deepseek_v4/csrc/exfold_kernels.cu  CUDA kernels + ATen launchers
 *   exfold/deepseek_v4/csrc/exfold_ops.cpp     torch.ops.dsv4_exfold schemas
 *   vLLM fused_topk / fused_topk_bias / moe_align_block_size, called from
 *   exfold/qwen3/vllm_patch.py:98-109 and exfold/deepseek_v4/vllm_patch.py:175-209
 */
#ifndef EXFOLD_B200_H_
#define EXFOLD_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define EXF_API __attribute__((visibility("default")))
#else
#define EXF_API
#endif

/* Same type as cudaStream_t, declared here so this header needs no CUDA headers. */
typedef struct CUstream_st* exf_stream_t;

enum exf_status {
  EXF_OK = 0,
  EXF_ERR_INVALID = -1,     /* bad argument: shape, size, null pointer, alignment */
  EXF_ERR_UNSUPPORTED = -2, /* valid request outside the compiled shapes / dtypes */
  EXF_ERR_CUDA = -3         /* a CUDA runtime call or kernel launch failed */
};

enum exf_weight_dtype { EXF_F32 = 0, EXF_BF16 = 1, EXF_F16 = 2 };
enum exf_index_dtype { EXF_I32 = 0, EXF_I64 = 1 };
enum exf_scoring { EXF_SOFTMAX = 0, EXF_SIGMOID = 1, EXF_SQRTSOFTPLUS = 2 };

/* Fold / decode semantics:
 *   EXF_QWEN3: exfold/qwen3/kernels.py (retain the first P slots as given, drop a transfer whose
 *              minimum loss is >= 1e30; decode subset may hold zero-importance experts)
 *   EXF_DSV4:  exfold/deepseek_v4/csrc/exfold_kernels.cu (stable sort by weight, argmin below
 *              FLT_MAX, renorm modes; decode keeps only positive-importance experts) */
enum exf_variant { EXF_QWEN3 = 0, EXF_DSV4 = 1 };
/* EXF_DSV4 prefill renorm_mode (exfold_kernels.cu:94-110) */
enum exf_renorm { EXF_RENORM_NONE = 0, EXF_RENORM_ROUTER_L2 = 1, EXF_RENORM_SIMILARITY_BLEND = 2 };

EXF_API int exf_abi_version(void);
EXF_API const char* exf_last_error(void);

/* Router kernel choice.  The tile kernels (one token per lane over bulk-copied logit tiles, for
 * E = 128 softmax and E = 256 biased sigmoid) are the fastest on large launches; below
 * `rows` = tokens x layers (default 32768; 4x that for the biased kernel without a fold) the
 * generic kernel (a token per E/32 lanes) has the lower latency.  Both give identical results.
 * Sets the threshold for every later call in the process and returns the previous one; a
 * negative `rows` only returns it. */
EXF_API int64_t exf_router_tile_min_rows(int64_t rows);

/* Router scoring + top-k.  Replaces vLLM fused_topk (softmax; exfold/qwen3/vllm_patch.py:98-109)
 * and fused_topk_bias (sigmoid or sqrtsoftplus + selection bias; exfold/deepseek_v4/
 * vllm_patch.py:175-209).  logits [tokens][experts] of logit_dtype (EXF_F32, EXF_BF16 or EXF_F16:
 * vLLM hands the router the gate output in the model dtype), 16-byte aligned; 16-bit logits are
 * converted to fp32 exactly, so the results equal those for logits.float(); bias [experts] or NULL
 * (sigmoid and sqrtsoftplus only).  Slots are ordered by selection key descending, ties by lower
 * expert id.  Weights: softmax over the selected experts (renormalize) or over all experts; the
 * unbiased sigmoid / sqrt(softplus) of the selected experts, divided by their sum when
 * renormalize (the sqrtsoftplus sum clamped at 1e-20); then times `scaling`.
 * experts in {64, 128, 256, 512}; 1 <= top_k <= 8. */
EXF_API int exf_router_topk(const void* logits, int logit_dtype, int64_t tokens, int experts,
                            int top_k, int scoring, const float* bias, int renormalize,
                            float scaling, float* out_w, int32_t* out_ids, exf_stream_t stream);

/* Hash routing of DeepSeek-V4's hash-MoE layers: replaces vLLM fused_topk_bias with
 * hash_indices_table = gate.tid2eid and input_tokens (exfold/deepseek_v4/vllm_patch.py:175-209).
 * The routes of token t are table[token_ids[t]][0..top_k) in table order, weights the unbiased
 * scores (scoring EXF_SIGMOID or EXF_SQRTSOFTPLUS; EXF_SOFTMAX is EXF_ERR_UNSUPPORTED) of those
 * experts, divided by their sum when renormalize (sqrtsoftplus: sum clamped at 1e-20), times
 * `scaling`.  logits [tokens][experts] of logit_dtype (as exf_router_topk); token_ids [tokens]
 * (id_dtype); table
 * [table_rows][top_k] int32; outputs [tokens][top_k].  A token id outside the table gives ids -1
 * and weights 0; a table entry outside [0, experts) keeps its id with weight 0. */
EXF_API int exf_router_hash(const void* logits, int logit_dtype, int64_t tokens, int experts,
                            int top_k, int scoring, const void* token_ids, int id_dtype,
                            const int32_t* table, int64_t table_rows, int renormalize,
                            float scaling, float* out_w, int32_t* out_ids, exf_stream_t stream);

/* Router + prefill fold in one pass over the logits: the B200 form of the patched prefill router
 * (exfold/qwen3/vllm_patch.py:166-176 -> kernels.py:97-151; exfold/deepseek_v4/vllm_patch.py:
 * 262-284 -> exfold_kernels.cu:228-278).  `layers` independent layers are processed in one
 * launch: logits [layers][tokens][experts] of logit_dtype (as exf_router_topk), bias
 * [layers][experts], tables
 * [layers][experts][experts], outputs [layers][tokens][target_k].  conf_loss is used by
 * EXF_DSV4 with EXF_RENORM_SIMILARITY_BLEND only (may be NULL otherwise). */
EXF_API int exf_router_fold_prefill(const void* logits, int logit_dtype, int64_t tokens,
                                    int layers, int experts, int top_k, int scoring,
                                    const float* bias, int renormalize,
                                    float scaling, int target_k, int variant, int renorm_mode,
                                    const float* coeff, const float* sel_loss,
                                    const float* conf_loss, float* out_w, int32_t* out_ids,
                                    exf_stream_t stream);

/* Prefill fold of precomputed top-k routes.
 * EXF_QWEN3 replaces project_prefill_topk / _project_prefill_kernel (exfold/qwen3/kernels.py:
 * 97-151, 9-94); EXF_DSV4 replaces exfold_prefill_cuda / prefill_kernel (exfold/deepseek_v4/
 * csrc/exfold_kernels.cu:228-278, 17-118).  w [tokens][top_k] (w_dtype), ids [tokens][top_k]
 * (id_dtype); outputs [tokens][target_k] in the same dtypes.  1 <= target_k <= top_k <= 8
 * (target_k == top_k folds nothing; EXF_DSV4 still sorts by weight and renormalises). */
EXF_API int exf_fold_prefill(const void* w, int w_dtype, const void* ids, int id_dtype,
                             int64_t tokens, int top_k, int target_k, int experts, int variant,
                             int renorm_mode, const float* coeff, const float* sel_loss,
                             const float* conf_loss, void* out_w, void* out_ids,
                             exf_stream_t stream);

/* Decode expert budget in one launch: importance (2^-32 fixed-point, order independent), top-D
 * select, per-expert target table, apply.
 * EXF_QWEN3 replaces select_and_reroute_decode (exfold/qwen3/kernels.py:423-491, 4 launches);
 * EXF_DSV4 replaces exfold_decode_cuda / fused_importance_select_and_apply_kernel
 * (exfold_kernels.cu:280-322, 120-201).  out_subset [budget] int32 or NULL receives the selected
 * experts in importance order.  experts <= 1024, 1 <= budget <= experts. */
EXF_API int exf_decode(const void* w, int w_dtype, const void* ids, int id_dtype, int64_t batch,
                       int top_k, int experts, int budget, int variant, const float* norms,
                       const float* coeff, const float* loss, void* out_w, void* out_ids,
                       int32_t* out_subset, exf_stream_t stream);

/* Split decode for a batch sharded over GPUs: each rank adds its routes' fixed-point importance
 * into `importance` [experts] int64 (zeroed by the caller), the ranks sum the vectors (one
 * all-reduce of `experts` int64), then every rank runs exf_decode_apply on its own routes.
 * Results equal exf_decode on the unsharded batch bit for bit. */
EXF_API int exf_decode_importance(const void* w, int w_dtype, const void* ids, int id_dtype,
                                  int64_t routes, int experts, const float* norms,
                                  int64_t* importance, exf_stream_t stream);
EXF_API int exf_decode_apply(const int64_t* importance, const void* w, int w_dtype,
                             const void* ids, int id_dtype, int64_t batch, int top_k,
                             int experts, int budget, int variant, const float* coeff,
                             const float* loss, void* out_w, void* out_ids, int32_t* out_subset,
                             exf_stream_t stream);

/* Sharded decode in one launch per layer, the importance exchanged over NVLink peer memory
 * instead of an all-reduce between two launches.  Each of `world` <= 8 ranks (one process per
 * GPU) holds its shard [batch][top_k] of the decode batch and one exchange buffer of
 * exf_decode_exchange_bytes(experts, world) bytes, zeroed before first use and 64-byte aligned;
 * `peers` (host array of `world` device pointers) gives every rank's buffer as mapped in this
 * process (peers[rank] = its own; the others from exf_ipc_import).  The launch adds this shard's
 * fixed-point importance, writes it into every rank's buffer as 8-byte words that each carry the
 * call number beside half a value (so a word that shows the current call is complete: no fence
 * or flag round trip), waits until every rank's words of this call have arrived, and sums the
 * vectors in rank order, then selects, builds the table and applies it to its own routes:
 * results equal exf_decode on the unsharded batch bit for bit.  Like a collective, every rank must make the same sequence of
 * calls on its buffer (same experts, world, budget and variant), each on one stream.
 * A wait is bounded by wait_ns (0: 2 s); when it runs out, *status (device int32, may be NULL)
 * is set to 1, the result uses this rank's importance only, and the buffers must be rebuilt.
 * Replaces exf_decode_importance + an all-reduce + exf_decode_apply. */
EXF_API int64_t exf_decode_exchange_bytes(int experts, int world);
EXF_API int exf_decode_sharded(const void* w, int w_dtype, const void* ids, int id_dtype,
                               int64_t batch, int top_k, int experts, int budget, int variant,
                               const float* norms, const float* coeff, const float* loss,
                               int world, int rank, void* const* peers, uint64_t wait_ns,
                               void* out_w, void* out_ids, int32_t* out_subset, int32_t* status,
                               exf_stream_t stream);

/* CUDA IPC of a device buffer between the processes of one node (cudaIpcGetMemHandle /
 * cudaIpcOpenMemHandle with lazy peer access): export gives a 64-byte handle of the cudaMalloc
 * allocation holding `ptr` and ptr's offset in it; import maps another process's allocation and
 * returns the mapped address plus that offset; release unmaps an imported address.  The buffer
 * must come from cudaMalloc (or an allocator built on it), not from virtual-memory mappings. */
#define EXF_IPC_HANDLE_BYTES 64
EXF_API int exf_ipc_export(const void* ptr, void* handle, int64_t* offset);
EXF_API int exf_ipc_import(const void* handle, int64_t offset, void** ptr);
EXF_API int exf_ipc_release(void* ptr, int64_t offset);

/* Reroute to an explicit subset (importance order given by the caller): replaces
 * reroute_decode_subset / _reroute_decode_kernel (exfold/qwen3/kernels.py:235-292, 154-232).
 * subset [subset_size] int32 expert ids. */
EXF_API int exf_reroute_subset(const void* w, int w_dtype, const void* ids, int id_dtype,
                               int64_t batch, int top_k, int experts, const int32_t* subset,
                               int subset_size, const float* coeff, const float* loss,
                               void* out_w, void* out_ids, exf_stream_t stream);

/* Static decode table from calibrated norms: replaces the host-side table build of
 * exfold/qwen3/vllm_patch.py:130-143.  target [experts] int32, scale [experts] fp32. */
EXF_API int exf_static_table(const float* norms, const float* coeff, const float* loss,
                             int experts, int budget, int32_t* target, float* scale,
                             exf_stream_t stream);

/* In-place static remap ids = target[ids], w = w * scale[ids]: replaces remap_decode_static /
 * _static_decode_remap_kernel (exfold/qwen3/kernels.py:322-356, 295-319). */
EXF_API int exf_static_remap(void* w, int w_dtype, void* ids, int id_dtype, int64_t routes,
                             int experts, const int32_t* target, const float* scale,
                             exf_stream_t stream);

/* moe_align / permute: replaces vLLM moe_align_block_size (vllm/model_executor/layers/
 * fused_moe/moe_align_block_size.py:11-93) as used by fused_experts after the ExFold transform.
 * capacity = exf_moe_align_capacity(); sorted_ids [capacity], expert_ids [ceil(capacity /
 * block_size)], num_post_pad [1].  Routes of one expert keep ascending flat order; padding
 * holds `numel`; unused blocks hold expert -1.  `workspace` (exf_moe_align_workspace_bytes
 * bytes, any contents) may be NULL when that size is 0.  Offsets are int32: the padded total
 * numel + experts * (block_size - 1) and the capacity must be below 2^31 (EXF_ERR_INVALID). */
EXF_API int64_t exf_moe_align_capacity(int64_t numel, int experts, int block_size,
                                       int pad_sorted);
EXF_API int64_t exf_moe_align_workspace_bytes(int64_t numel, int experts);
EXF_API int exf_moe_align(const void* ids, int id_dtype, int64_t numel, int experts,
                          int block_size, int64_t capacity, int32_t* sorted_ids,
                          int32_t* expert_ids, int32_t* num_post_pad, void* workspace,
                          int64_t workspace_bytes, exf_stream_t stream);

/* Grouped SwiGLU expert layer on the tcgen05 tensor cores: replaces vLLM fused_experts
 * (vllm/model_executor/layers/fused_moe/fused_moe.py:1587-1630) as called after the ExFold
 * transform.  y[t] = sum_j w[t,j] * W2[e] (silu(W1[e] x[t]) * (W3[e] x[t])), e = ids[t,j].
 * x bf16 [tokens][hidden]; topk_w fp32 and topk_ids int32 [tokens][top_k]; w13 bf16
 * [experts][2*inter][hidden] (rows [0, inter) gate W1, rows [inter, 2*inter) up W3); w2 bf16
 * [experts][hidden][inter]; y bf16 [tokens][hidden].  The intermediate activation is rounded to
 * bf16 (as vLLM's intermediate cache).  workspace: exf_fused_experts_workspace_bytes(), 16-byte
 * aligned.  status: optional device int32, set to 1 if a pipeline wait timed out.
 * hidden % 256 == 0, inter % 128 == 0, experts <= 512, 1 <= top_k <= 8; routes whose id is
 * outside [0, experts) contribute nothing. */
EXF_API int64_t exf_fused_experts_workspace_bytes(int64_t tokens, int top_k, int experts,
                                                  int hidden, int inter);
EXF_API int exf_fused_experts(const void* x, const float* topk_w, const int32_t* topk_ids,
                              int64_t tokens, int top_k, const void* w13, const void* w2,
                              int experts, int hidden, int inter, void* y, void* workspace,
                              int64_t workspace_bytes, int32_t* status, exf_stream_t stream);

/* Decode expert budget followed by the expert layer: select_and_reroute_decode /
 * exfold_decode_cuda (exfold/qwen3/kernels.py:423-491; exfold_kernels.cu:280-322), then vLLM
 * moe_align_block_size (moe_align_block_size.py:11-93) and fused_experts (fused_moe.py:1587)
 * over the remapped routes.  The decode launch also merges the routes of a token that the table
 * sent to the same expert (their weights summed in slot order, the expert computed once); the
 * layer is then one launch for moe_align and the gather of token rows, one for both GEMMs and
 * one for the combine.
 * out_w / out_ids [batch][top_k] receive exf_decode's outputs bit for bit; y bf16
 * [batch][hidden] equals exf_fused_experts over them within bf16 rounding (a merged route's
 * output is rounded once instead of twice).  w fp32, ids int32; experts <= 256, top_k <= 8,
 * batch * top_k <= 8192; other arguments as exf_decode and exf_fused_experts.  workspace:
 * exf_decode_fused_experts_workspace_bytes(), 16-byte aligned. */
EXF_API int64_t exf_decode_fused_experts_workspace_bytes(int64_t batch, int top_k, int experts,
                                                        int hidden, int inter);
EXF_API int exf_decode_fused_experts(const void* x, const float* w, const int32_t* ids,
                                     int64_t batch, int top_k, int experts, int budget,
                                     int variant, const float* norms, const float* coeff,
                                     const float* loss, const void* w13, const void* w2,
                                     int hidden, int inter, float* out_w, int32_t* out_ids,
                                     void* y, void* workspace, int64_t workspace_bytes,
                                     int32_t* status, exf_stream_t stream);

/* Calibration statistics (offline): the GPU form of PairwiseScalarStats
 * (exfold/qwen3/calibration.py:9-140), which builds the [E][E] coefficient / loss tables and the
 * expert norms that the folds above read.
 * exf_calibration_update (PairwiseScalarStats.update, calibration.py:49-95): outputs
 * [tokens][top_k][hidden] unweighted expert outputs (out_dtype; 16-byte aligned, hidden a
 * multiple of 8), ids [tokens][top_k].  For each token and ordered pair of its routes with
 * different experts (s, d), with w_s = ||u_s||, adds w_s <u_s, u_d>, w_s ||u_d||^2 and
 * w_s ||u_s||^2 (each formed in fp32) to dot, target_sq, source_sq at [e_s][e_d] (fp64 [E][E],
 * caller-zeroed at the start of a calibration); adds ||u|| and 1 to norm_sum, norm_count [E]
 * for every route.  Routes with an expert id outside [0, experts) are skipped.  Accumulation is
 * by fp64 atomics, so the low bits depend on their order, as with the reference's index_add_.
 * exf_calibration_finalize (finalize, calibration.py:97-126): coeff, loss fp32 [E][E]; sets
 * *nonfinite (device int32, may be NULL) to 1 when a statistic is not finite (the reference
 * raises RuntimeError; the caller reads the flag).
 * exf_calibration_norms (expert_norms, calibration.py:128-140): norms fp32 [E], the mean output
 * norm of each routed expert, the lower median of those for the others (1 when none was routed).
 * 2 <= experts <= 1024; 1 <= top_k <= 8. */
EXF_API int exf_calibration_update(const void* outputs, int out_dtype, const void* ids,
                                   int id_dtype, int64_t tokens, int top_k, int hidden,
                                   int experts, double* dot, double* target_sq,
                                   double* source_sq, double* norm_sum, double* norm_count,
                                   exf_stream_t stream);
EXF_API int exf_calibration_finalize(const double* dot, const double* target_sq,
                                     const double* source_sq, int experts, double ridge,
                                     double clip_min, double clip_max, float* coeff, float* loss,
                                     int32_t* nonfinite, exf_stream_t stream);
EXF_API int exf_calibration_norms(const double* norm_sum, const double* norm_count, int experts,
                                  float* norms, exf_stream_t stream);

/* exf_moe_align for callers that cannot allocate device memory at call time.  This entry point
 * has no counterpart in the reference.
 *
 * Who needs it: exf_moe_align wants a caller workspace above 8192 routes.  Some callers have no
 * way to provide one per call: an inference-engine plugin whose execute step may not allocate,
 * a host whose device memory all belongs to another runtime's pool, or code that must not call
 * cudaMalloc/cudaFree because they synchronise the device.  This variant allocates nothing: the
 * caller passes only the inputs and outputs, and the [chunks][experts] count table lives in a
 * fixed 1 MiB array inside the library (262144 int32 entries, held on every GPU that loads the
 * library until the process exits).
 *
 * Limit: ceil(numel / 2048) * experts <= 262144, i.e. at most 2048 * floor(262144 / experts)
 * routes (4,194,304 at 128 experts, 2,097,152 at 256); larger inputs are rejected with
 * EXF_ERR_INVALID and a message, never truncated.
 * Set-up: the first call on each device looks up the array's device address (one
 * cudaGetSymbolAddress with that device current); make that first call before any stream
 * capture.  The address is kept for the life of the process: after cudaDeviceReset (or
 * anything else that destroys the device's primary context) do not call this entry point on
 * that device again.
 * Sharing: all calls on a device use the same array and it keeps the last call's contents (each
 * call rewrites every entry it reads, so nothing needs clearing).  Calls whose kernels overlap on
 * the GPU (different streams, or concurrent graphs) race on the array; serialise them.
 * Outputs and errors are those of exf_moe_align. */
EXF_API int exf_moe_align_noalloc(const void* ids, int id_dtype, int64_t numel, int experts,
                                  int block_size, int64_t capacity, int32_t* sorted_ids,
                                  int32_t* expert_ids, int32_t* num_post_pad,
                                  exf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* EXFOLD_B200_H_ */
