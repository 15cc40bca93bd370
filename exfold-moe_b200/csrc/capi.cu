// extern "C" entry points of libexfold_b200.so: argument checks, error reporting, dispatch.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <unordered_map>

#include "exf_common.cuh"
#include "exf_kernels.h"
#include "exf_launch.h"
#include "exf_moe.h"

namespace exf {



// ---- launch helpers -----------------------------------------------------------------------
static std::mutex g_grid_mu;
static std::unordered_map<uint64_t, int> g_grid_cache;

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

int persistent_grid(const void* kernel, int threads, size_t smem) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const uint64_t key = (reinterpret_cast<uint64_t>(kernel) << 8) ^ (uint64_t)dev;
  {
    std::lock_guard<std::mutex> lk(g_grid_mu);
    auto it = g_grid_cache.find(key);
    if (it != g_grid_cache.end()) return it->second;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess)
    return 0;
  const int grid = per_sm * sm_count();
  std::lock_guard<std::mutex> lk(g_grid_mu);
  g_grid_cache[key] = grid;
  return grid;
}

}  // namespace exf

using namespace exf;

// ---- error reporting ------------------------------------------------------------------------
static thread_local char g_err[512] = "";

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) {
    g_err[0] = 0;
    return EXF_OK;
  }
  if (e == cudaErrorNotSupported) return fail(EXF_ERR_UNSUPPORTED, "%s: shape not compiled", what);
  return fail(EXF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define EXF_REQUIRE(cond, ...)                                 \
  do {                                                         \
    if (!(cond)) return fail(EXF_ERR_INVALID, __VA_ARGS__);    \
  } while (0)

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static bool good_wdtype(int d) { return d == EXF_F32 || d == EXF_BF16 || d == EXF_F16; }
static bool good_idtype(int d) { return d == EXF_I32 || d == EXF_I64; }

// ---- entry points ---------------------------------------------------------------------------
extern "C" {

EXF_API int exf_abi_version(void) { return 3; }

EXF_API int64_t exf_router_tile_min_rows(int64_t rows) { return router_tile_min_rows(rows); }

EXF_API const char* exf_last_error(void) { return g_err; }

static int router_common(const char* name, const void* logits, int logit_dtype, int64_t tokens,
                         int layers, int experts, int top_k, int scoring, const float* out_w,
                         const int32_t* out_ids) {
  EXF_REQUIRE(good_wdtype(logit_dtype), "%s: logits must be EXF_F32, EXF_BF16 or EXF_F16", name);
  EXF_REQUIRE(tokens >= 0 && layers >= 1, "%s: tokens must be >= 0 and layers >= 1", name);
  EXF_REQUIRE(top_k >= 1 && top_k <= 8, "%s: top_k must be in [1, 8], got %d", name, top_k);
  EXF_REQUIRE(experts >= top_k, "%s: experts (%d) < top_k (%d)", name, experts, top_k);
  EXF_REQUIRE(scoring == EXF_SOFTMAX || scoring == EXF_SIGMOID || scoring == EXF_SQRTSOFTPLUS,
              "%s: unknown scoring %d", name, scoring);
  if (experts != 64 && experts != 128 && experts != 256 && experts != 512)
    return fail(EXF_ERR_UNSUPPORTED, "%s: experts must be one of 64, 128, 256, 512 (got %d)", name,
                experts);
  if (tokens > 0) {
    EXF_REQUIRE(logits && out_w && out_ids, "%s: null pointer", name);
    EXF_REQUIRE(aligned16(logits), "%s: logits must be 16-byte aligned", name);
  }
  return EXF_OK;
}

EXF_API int exf_router_topk(const void* logits, int logit_dtype, int64_t tokens, int experts,
                            int top_k, int scoring, const float* bias, int renormalize,
                            float scaling, float* out_w, int32_t* out_ids, exf_stream_t stream) {
  int rc = router_common("exf_router_topk", logits, logit_dtype, tokens, 1, experts, top_k,
                         scoring, out_w, out_ids);
  if (rc != EXF_OK) return rc;
  if (tokens == 0) return EXF_OK;
  EXF_REQUIRE(!bias || aligned16(bias), "exf_router_topk: bias must be 16-byte aligned");
  RouterParams p{logits, tokens, 1, top_k, bias, renormalize, scaling, top_k, 0,
                 nullptr, nullptr, nullptr, out_w, out_ids, logit_dtype};
  return cuda_status(launch_router(experts, scoring, 0, p, (cudaStream_t)stream), "exf_router_topk");
}

EXF_API int exf_router_hash(const void* logits, int logit_dtype, int64_t tokens, int experts,
                            int top_k, int scoring, const void* token_ids, int id_dtype,
                            const int32_t* table, int64_t table_rows, int renormalize,
                            float scaling, float* out_w, int32_t* out_ids, exf_stream_t stream) {
  const char* name = "exf_router_hash";
  EXF_REQUIRE(tokens >= 0, "%s: tokens must be >= 0", name);
  EXF_REQUIRE(top_k >= 1 && top_k <= 8, "%s: top_k must be in [1, 8], got %d", name, top_k);
  EXF_REQUIRE(experts >= 1, "%s: experts must be >= 1", name);
  EXF_REQUIRE(good_idtype(id_dtype), "%s: unsupported token id dtype", name);
  EXF_REQUIRE(good_wdtype(logit_dtype), "%s: logits must be EXF_F32, EXF_BF16 or EXF_F16", name);
  EXF_REQUIRE(table_rows >= 1, "%s: the hash table needs at least one row", name);
  if (scoring == EXF_SOFTMAX)
    return fail(EXF_ERR_UNSUPPORTED, "%s: hash routing takes sigmoid or sqrtsoftplus scores", name);
  EXF_REQUIRE(scoring == EXF_SIGMOID || scoring == EXF_SQRTSOFTPLUS, "%s: unknown scoring %d",
              name, scoring);
  if (tokens == 0) return EXF_OK;
  EXF_REQUIRE(logits && token_ids && table && out_w && out_ids, "%s: null pointer", name);
  return cuda_status(launch_router_hash(logits, logit_dtype, tokens, experts, top_k, scoring,
                                        token_ids,
                                        id_dtype, table, table_rows, renormalize, scaling, out_w,
                                        out_ids, (cudaStream_t)stream),
                     name);
}

EXF_API int exf_router_fold_prefill(const void* logits, int logit_dtype, int64_t tokens,
                                    int layers, int experts, int top_k, int scoring,
                                    const float* bias, int renormalize,
                                    float scaling, int target_k, int variant, int renorm_mode,
                                    const float* coeff, const float* sel_loss,
                                    const float* conf_loss, float* out_w, int32_t* out_ids,
                                    exf_stream_t stream) {
  const char* name = "exf_router_fold_prefill";
  int rc = router_common(name, logits, logit_dtype, tokens, layers, experts, top_k, scoring,
                         out_w, out_ids);
  if (rc != EXF_OK) return rc;
  EXF_REQUIRE(variant == EXF_QWEN3 || variant == EXF_DSV4, "%s: unknown variant %d", name, variant);
  EXF_REQUIRE(target_k >= 1 && target_k <= top_k, "%s: target_k must be in [1, top_k]", name);
  EXF_REQUIRE(renorm_mode >= 0 && renorm_mode <= 2, "%s: renorm_mode must be 0, 1 or 2", name);
  EXF_REQUIRE(variant == EXF_DSV4 || renorm_mode == 0, "%s: renorm_mode needs EXF_DSV4", name);
  if (tokens == 0) return EXF_OK;
  EXF_REQUIRE(coeff && sel_loss, "%s: null calibration table", name);
  EXF_REQUIRE(renorm_mode != 2 || conf_loss, "%s: similarity_blend needs conf_loss", name);
  EXF_REQUIRE(!bias || aligned16(bias), "%s: bias must be 16-byte aligned", name);
  RouterParams p{logits, tokens, layers, top_k, bias, renormalize, scaling, target_k, renorm_mode,
                 coeff, sel_loss, conf_loss, out_w, out_ids, logit_dtype};
  return cuda_status(launch_router(experts, scoring, variant == EXF_QWEN3 ? 1 : 2, p,
                                   (cudaStream_t)stream),
                     name);
}

EXF_API int exf_fold_prefill(const void* w, int w_dtype, const void* ids, int id_dtype,
                             int64_t tokens, int top_k, int target_k, int experts, int variant,
                             int renorm_mode, const float* coeff, const float* sel_loss,
                             const float* conf_loss, void* out_w, void* out_ids,
                             exf_stream_t stream) {
  const char* name = "exf_fold_prefill";
  EXF_REQUIRE(good_wdtype(w_dtype) && good_idtype(id_dtype), "%s: unsupported dtype", name);
  EXF_REQUIRE(tokens >= 0, "%s: tokens must be >= 0", name);
  EXF_REQUIRE(top_k >= 1 && top_k <= 8, "%s: top_k must be in [1, 8], got %d", name, top_k);
  EXF_REQUIRE(target_k >= 1 && target_k <= top_k, "%s: target_k must be in [1, top_k]", name);
  EXF_REQUIRE(experts >= 1, "%s: experts must be >= 1", name);
  EXF_REQUIRE(variant == EXF_QWEN3 || variant == EXF_DSV4, "%s: unknown variant %d", name, variant);
  EXF_REQUIRE(renorm_mode >= 0 && renorm_mode <= 2, "%s: renorm_mode must be 0, 1 or 2", name);
  if (tokens == 0) return EXF_OK;
  EXF_REQUIRE(w && ids && out_w && out_ids && coeff && sel_loss, "%s: null pointer", name);
  EXF_REQUIRE(variant != EXF_DSV4 || renorm_mode != 2 || conf_loss,
              "%s: similarity_blend needs conf_loss", name);
  FoldParams p{w, ids, tokens, top_k, target_k, experts, variant == EXF_DSV4 ? renorm_mode : 0,
               coeff, sel_loss, conf_loss, out_w, out_ids};
  return cuda_status(launch_fold(w_dtype, id_dtype, variant, p, (cudaStream_t)stream), name);
}

static int decode_checks(const char* name, int w_dtype, int id_dtype, int64_t batch, int top_k,
                         int experts, int budget, int variant) {
  EXF_REQUIRE(good_wdtype(w_dtype) && good_idtype(id_dtype), "%s: unsupported dtype", name);
  EXF_REQUIRE(batch >= 0 && top_k >= 1, "%s: bad routing shape", name);
  EXF_REQUIRE(experts >= 1 && experts <= 1024, "%s: experts must be in [1, 1024]", name);
  EXF_REQUIRE(budget >= 1 && budget <= experts, "%s: budget must be in [1, experts]", name);
  EXF_REQUIRE(variant == EXF_QWEN3 || variant == EXF_DSV4, "%s: unknown variant %d", name, variant);
  return EXF_OK;
}

EXF_API int exf_decode(const void* w, int w_dtype, const void* ids, int id_dtype, int64_t batch,
                       int top_k, int experts, int budget, int variant, const float* norms,
                       const float* coeff, const float* loss, void* out_w, void* out_ids,
                       int32_t* out_subset, exf_stream_t stream) {
  const char* name = "exf_decode";
  int rc = decode_checks(name, w_dtype, id_dtype, batch, top_k, experts, budget, variant);
  if (rc != EXF_OK) return rc;
  EXF_REQUIRE(norms && coeff && loss, "%s: null calibration table", name);
  EXF_REQUIRE(batch == 0 || (w && ids && out_w && out_ids), "%s: null routing pointer", name);
  DecodeParams p{w, ids, batch * top_k, experts, budget, variant, 0 /*from routes*/, norms,
                 nullptr, nullptr, coeff, loss, out_w, out_ids, out_subset};
  return cuda_status(launch_decode(w_dtype, id_dtype, p, (cudaStream_t)stream), name);
}

EXF_API int exf_decode_importance(const void* w, int w_dtype, const void* ids, int id_dtype,
                                  int64_t routes, int experts, const float* norms,
                                  int64_t* importance, exf_stream_t stream) {
  const char* name = "exf_decode_importance";
  EXF_REQUIRE(good_wdtype(w_dtype) && good_idtype(id_dtype), "%s: unsupported dtype", name);
  EXF_REQUIRE(routes >= 0 && experts >= 1 && experts <= 1024, "%s: bad shape", name);
  EXF_REQUIRE(norms && importance, "%s: null pointer", name);
  if (routes == 0) return EXF_OK;
  EXF_REQUIRE(w && ids, "%s: null routing pointer", name);
  return cuda_status(launch_importance(w_dtype, id_dtype, w, ids, routes, experts, norms,
                                       importance, (cudaStream_t)stream),
                     name);
}

EXF_API int exf_decode_apply(const int64_t* importance, const void* w, int w_dtype,
                             const void* ids, int id_dtype, int64_t batch, int top_k,
                             int experts, int budget, int variant, const float* coeff,
                             const float* loss, void* out_w, void* out_ids, int32_t* out_subset,
                             exf_stream_t stream) {
  const char* name = "exf_decode_apply";
  int rc = decode_checks(name, w_dtype, id_dtype, batch, top_k, experts, budget, variant);
  if (rc != EXF_OK) return rc;
  EXF_REQUIRE(importance && coeff && loss, "%s: null pointer", name);
  EXF_REQUIRE(batch == 0 || (w && ids && out_w && out_ids), "%s: null routing pointer", name);
  DecodeParams p{w, ids, batch * top_k, experts, budget, variant, 1 /*importance given*/,
                 nullptr, importance, nullptr, coeff, loss, out_w, out_ids, out_subset};
  return cuda_status(launch_decode(w_dtype, id_dtype, p, (cudaStream_t)stream), name);
}

// ---- sharded decode with the importance exchanged over peer memory ---------------------------
EXF_API int64_t exf_decode_exchange_bytes(int experts, int world) {
  if (experts < 1 || experts > 1024 || world < 1 || world > kMaxPeers) return -1;
  return exchange_longs(experts, world) * (int64_t)sizeof(int64_t);
}

// cuMemGetAddressRange through the runtime's driver entry point (no link against libcuda)
typedef int (*exf_get_range_fn)(unsigned long long*, size_t*, unsigned long long);

static cudaError_t allocation_base(const void* ptr, uintptr_t* base) {
  static exf_get_range_fn fn = nullptr;
  static std::once_flag once;
  static cudaError_t lookup = cudaSuccess;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    lookup = cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q);
    if (lookup == cudaSuccess && (q != cudaDriverEntryPointSuccess || f == nullptr))
      lookup = cudaErrorSymbolNotFound;
    fn = reinterpret_cast<exf_get_range_fn>(f);
  });
  if (lookup != cudaSuccess) return lookup;
  unsigned long long b = 0;
  size_t size = 0;
  if (fn(&b, &size, reinterpret_cast<unsigned long long>(ptr)) != 0)
    return cudaErrorInvalidDevicePointer;
  *base = static_cast<uintptr_t>(b);
  return cudaSuccess;
}

EXF_API int exf_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  const char* name = "exf_ipc_export";
  EXF_REQUIRE(ptr && handle && offset, "%s: null pointer", name);
  uintptr_t base = 0;
  cudaError_t e = allocation_base(ptr, &base);
  if (e != cudaSuccess) return cuda_status(e, name);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_status(e, name);
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - base);
  return EXF_OK;
}

EXF_API int exf_ipc_import(const void* handle, int64_t offset, void** ptr) {
  const char* name = "exf_ipc_import";
  EXF_REQUIRE(handle && ptr && offset >= 0, "%s: bad argument", name);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_status(e, name);
  *ptr = static_cast<uint8_t*>(base) + offset;
  return EXF_OK;
}

EXF_API int exf_ipc_release(void* ptr, int64_t offset) {
  const char* name = "exf_ipc_release";
  EXF_REQUIRE(ptr && offset >= 0, "%s: bad argument", name);
  return cuda_status(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset), name);
}

EXF_API int exf_decode_sharded(const void* w, int w_dtype, const void* ids, int id_dtype,
                               int64_t batch, int top_k, int experts, int budget, int variant,
                               const float* norms, const float* coeff, const float* loss,
                               int world, int rank, void* const* peers, uint64_t wait_ns,
                               void* out_w, void* out_ids, int32_t* out_subset, int32_t* status,
                               exf_stream_t stream) {
  const char* name = "exf_decode_sharded";
  int rc = decode_checks(name, w_dtype, id_dtype, batch, top_k, experts, budget, variant);
  if (rc != EXF_OK) return rc;
  EXF_REQUIRE(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world,
              "%s: world must be in [1, %d] and 0 <= rank < world", name, kMaxPeers);
  EXF_REQUIRE(norms && coeff && loss && peers, "%s: null pointer", name);
  EXF_REQUIRE(batch == 0 || (w && ids && out_w && out_ids), "%s: null routing pointer", name);
  DecodeParams p{w, ids, batch * top_k, experts, budget, variant, kImportanceExchanged, norms,
                 nullptr, nullptr, coeff, loss, out_w, out_ids, out_subset};
  p.world = world;
  p.rank = rank;
  for (int r = 0; r < world; ++r) {
    EXF_REQUIRE(peers[r] && (reinterpret_cast<uintptr_t>(peers[r]) & 63u) == 0,
                "%s: exchange buffer of rank %d is null or not 64-byte aligned", name, r);
    p.peers[r] = static_cast<int64_t*>(peers[r]);
  }
  p.status = status;
  p.wait_ns = wait_ns;
  return cuda_status(launch_decode(w_dtype, id_dtype, p, (cudaStream_t)stream), name);
}

EXF_API int exf_reroute_subset(const void* w, int w_dtype, const void* ids, int id_dtype,
                               int64_t batch, int top_k, int experts, const int32_t* subset,
                               int subset_size, const float* coeff, const float* loss,
                               void* out_w, void* out_ids, exf_stream_t stream) {
  const char* name = "exf_reroute_subset";
  EXF_REQUIRE(subset_size >= 1 && subset_size <= experts, "%s: subset_size must be in [1, experts]",
              name);
  int rc = decode_checks(name, w_dtype, id_dtype, batch, top_k, experts, subset_size, EXF_QWEN3);
  if (rc != EXF_OK) return rc;
  EXF_REQUIRE(subset && coeff && loss, "%s: null pointer", name);
  if (batch == 0) return EXF_OK;
  EXF_REQUIRE(w && ids && out_w && out_ids, "%s: null routing pointer", name);
  DecodeParams p{w, ids, batch * top_k, experts, subset_size, EXF_QWEN3, 2 /*subset given*/,
                 nullptr, nullptr, subset, coeff, loss, out_w, out_ids, nullptr};
  return cuda_status(launch_decode(w_dtype, id_dtype, p, (cudaStream_t)stream), name);
}

EXF_API int exf_static_table(const float* norms, const float* coeff, const float* loss,
                             int experts, int budget, int32_t* target, float* scale,
                             exf_stream_t stream) {
  const char* name = "exf_static_table";
  EXF_REQUIRE(experts >= 1 && experts <= 1024, "%s: experts must be in [1, 1024]", name);
  EXF_REQUIRE(budget >= 1 && budget <= experts, "%s: budget must be in [1, experts]", name);
  EXF_REQUIRE(norms && coeff && loss && target && scale, "%s: null pointer", name);
  return cuda_status(launch_static_table(norms, coeff, loss, experts, budget, target, scale,
                                         (cudaStream_t)stream),
                     name);
}

EXF_API int exf_static_remap(void* w, int w_dtype, void* ids, int id_dtype, int64_t routes,
                             int experts, const int32_t* target, const float* scale,
                             exf_stream_t stream) {
  const char* name = "exf_static_remap";
  EXF_REQUIRE(good_wdtype(w_dtype) && good_idtype(id_dtype), "%s: unsupported dtype", name);
  EXF_REQUIRE(routes >= 0 && experts >= 1, "%s: bad shape", name);
  if (routes == 0) return EXF_OK;
  EXF_REQUIRE(w && ids && target && scale, "%s: null pointer", name);
  return cuda_status(launch_static_remap(w_dtype, id_dtype, w, ids, routes, experts, target, scale,
                                         (cudaStream_t)stream),
                     name);
}

EXF_API int64_t exf_moe_align_capacity(int64_t numel, int experts, int block_size, int pad_sorted) {
  if (numel < 0 || experts < 1 || block_size < 1) return -1;
  int64_t cap = numel + (int64_t)experts * (block_size - 1);
  if (pad_sorted) cap = (cap + block_size - 1) / block_size * block_size;
  if (numel < experts && numel * block_size < cap) cap = numel * block_size;
  return cap;
}

EXF_API int64_t exf_moe_align_workspace_bytes(int64_t numel, int experts) {
  if (numel < 0 || experts < 1) return -1;
  return align_workspace_bytes(numel, experts);
}

// Checks shared by the two moe_align entry points.  The kernels keep expert offsets, the padded
// total and block starts in int32, so the padded total (at most the capacity formula) and the
// capacity must stay below 2^31.
static int align_checks(const char* name, const void* ids, int id_dtype, int64_t numel,
                        int experts, int block_size, int64_t capacity, const int32_t* sorted_ids,
                        const int32_t* expert_ids, const int32_t* num_post_pad) {
  EXF_REQUIRE(good_idtype(id_dtype), "%s: unsupported id dtype", name);
  EXF_REQUIRE(numel >= 0 && numel < (int64_t)1 << 31, "%s: numel out of range", name);
  EXF_REQUIRE(block_size >= 1, "%s: block_size must be >= 1", name);
  if (experts < 1 || experts > align_max_experts())
    return fail(EXF_ERR_UNSUPPORTED, "%s: experts must be in [1, %d]", name, align_max_experts());
  const int64_t padded = exf_moe_align_capacity(numel, experts, block_size, 0);
  EXF_REQUIRE(padded < ((int64_t)1 << 31) && capacity < ((int64_t)1 << 31),
              "%s: %lld routes over %d experts in blocks of %d (capacity %lld) exceed the int32 "
              "offsets: the padded total and the capacity must be below 2^31",
              name, (long long)numel, experts, block_size, (long long)capacity);
  EXF_REQUIRE(capacity >= padded || capacity >= numel * (int64_t)block_size,
              "%s: capacity too small", name);
  EXF_REQUIRE(num_post_pad && (capacity == 0 || (sorted_ids && expert_ids)), "%s: null output",
              name);
  EXF_REQUIRE(numel == 0 || ids, "%s: null ids", name);
  return EXF_OK;
}

EXF_API int exf_moe_align(const void* ids, int id_dtype, int64_t numel, int experts,
                          int block_size, int64_t capacity, int32_t* sorted_ids,
                          int32_t* expert_ids, int32_t* num_post_pad, void* workspace,
                          int64_t workspace_bytes, exf_stream_t stream) {
  const char* name = "exf_moe_align";
  const int rc = align_checks(name, ids, id_dtype, numel, experts, block_size, capacity,
                              sorted_ids, expert_ids, num_post_pad);
  if (rc != EXF_OK) return rc;
  const int64_t need = align_workspace_bytes(numel, experts);
  EXF_REQUIRE(need == 0 || (workspace && workspace_bytes >= need),
              "%s: workspace of %lld bytes required", name, (long long)need);
  AlignParams p{ids, numel, experts, block_size, capacity, sorted_ids, expert_ids, num_post_pad,
                static_cast<int32_t*>(workspace), 0};
  return cuda_status(launch_align(id_dtype, p, (cudaStream_t)stream), name);
}

EXF_API int64_t exf_fused_experts_workspace_bytes(int64_t tokens, int top_k, int experts,
                                                  int hidden, int inter) {
  if (tokens < 0 || top_k < 1 || experts < 1 || hidden < 1 || inter < 1) return -1;
  return moe_workspace(tokens, top_k, experts, hidden, inter, nullptr).bytes;
}

EXF_API int exf_fused_experts(const void* x, const float* topk_w, const int32_t* topk_ids,
                              int64_t tokens, int top_k, const void* w13, const void* w2,
                              int experts, int hidden, int inter, void* y, void* workspace,
                              int64_t workspace_bytes, int32_t* status, exf_stream_t stream) {
  const char* name = "exf_fused_experts";
  EXF_REQUIRE(tokens >= 0 && top_k >= 1 &&
                  tokens * top_k + (int64_t)experts * 127 < ((int64_t)1 << 31),
              "%s: bad routing shape (routes plus block padding must stay below 2^31)", name);
  if (top_k > 8) return fail(EXF_ERR_UNSUPPORTED, "%s: top_k must be at most 8, got %d", name, top_k);
  if (experts < 1 || experts > align_max_experts())
    return fail(EXF_ERR_UNSUPPORTED, "%s: experts must be in [1, %d]", name, align_max_experts());
  if (hidden % 256 != 0 || inter % 128 != 0)
    return fail(EXF_ERR_UNSUPPORTED,
                "%s: hidden must be a multiple of 256 and intermediate a multiple of 128", name);
  if (tokens == 0) return EXF_OK;
  EXF_REQUIRE(x && topk_w && topk_ids && w13 && w2 && y && workspace, "%s: null pointer", name);
  EXF_REQUIRE(aligned16(x) && aligned16(w13) && aligned16(w2) && aligned16(y) &&
                  aligned16(workspace),
              "%s: tensors must be 16-byte aligned", name);
  MoeWorkspace ws = moe_workspace(tokens, top_k, experts, hidden, inter, workspace);
  EXF_REQUIRE(workspace_bytes >= ws.bytes, "%s: workspace of %lld bytes required", name,
              (long long)ws.bytes);
  MoeArgs a{x, topk_w, topk_ids, tokens, top_k, w13, w2, experts, hidden, inter, y, status};
  return cuda_status(launch_moe_experts(a, ws, (cudaStream_t)stream), name);
}

EXF_API int64_t exf_decode_fused_experts_workspace_bytes(int64_t batch, int top_k, int experts,
                                                        int hidden, int inter) {
  if (batch < 0 || top_k < 1 || experts < 1) return -1;
  return decode_moe_workspace_bytes(batch, top_k, experts, hidden, inter);
}

EXF_API int exf_decode_fused_experts(const void* x, const float* w, const int32_t* ids,
                                     int64_t batch, int top_k, int experts, int budget,
                                     int variant, const float* norms, const float* coeff,
                                     const float* loss, const void* w13, const void* w2,
                                     int hidden, int inter, float* out_w, int32_t* out_ids,
                                     void* y, void* workspace, int64_t workspace_bytes,
                                     int32_t* status, exf_stream_t stream) {
  const char* name = "exf_decode_fused_experts";
  int rc = decode_checks(name, EXF_F32, EXF_I32, batch, top_k, experts, budget, variant);
  if (rc != EXF_OK) return rc;
  if (experts > kDecodeAlignMaxExperts || top_k > 8 ||
      batch * top_k > (int64_t)kDecodeAlignMaxRoutes)
    return fail(EXF_ERR_UNSUPPORTED,
                "%s: at most %d experts, top_k <= 8 and %d routes (batch * top_k)", name,
                kDecodeAlignMaxExperts, kDecodeAlignMaxRoutes);
  if (hidden % 256 != 0 || inter % 128 != 0)
    return fail(EXF_ERR_UNSUPPORTED,
                "%s: hidden must be a multiple of 256 and intermediate a multiple of 128", name);
  if (batch == 0) return EXF_OK;
  EXF_REQUIRE(norms && coeff && loss, "%s: null calibration table", name);
  EXF_REQUIRE(x && w && ids && w13 && w2 && out_w && out_ids && y && workspace,
              "%s: null pointer", name);
  EXF_REQUIRE(aligned16(x) && aligned16(w13) && aligned16(w2) && aligned16(y) &&
                  aligned16(workspace),
              "%s: tensors must be 16-byte aligned", name);
  const int64_t need = decode_moe_workspace_bytes(batch, top_k, experts, hidden, inter);
  EXF_REQUIRE(workspace_bytes >= need, "%s: workspace of %lld bytes required", name,
              (long long)need);
  DecodeParams d{w, ids, batch * top_k, experts, budget, variant, 0 /*from routes*/, norms,
                 nullptr, nullptr, coeff, loss, out_w, out_ids, nullptr};
  MoeArgs a{x, out_w, out_ids, batch, top_k, w13, w2, experts, hidden, inter, y, status};
  return cuda_status(launch_decode_moe_experts(d, a, workspace, (cudaStream_t)stream), name);
}

// moe_align without any device allocation: the chunk-count table lives in the library's fixed
// scratch array (exf::g_align_static_table) instead of a caller workspace.
EXF_API int exf_moe_align_noalloc(const void* ids, int id_dtype, int64_t numel, int experts,
                                  int block_size, int64_t capacity, int32_t* sorted_ids,
                                  int32_t* expert_ids, int32_t* num_post_pad,
                                  exf_stream_t stream) {
  const char* name = "exf_moe_align_noalloc";
  const int rc = align_checks(name, ids, id_dtype, numel, experts, block_size, capacity,
                              sorted_ids, expert_ids, num_post_pad);
  if (rc != EXF_OK) return rc;
  const int64_t entries = align_workspace_bytes(numel, experts) / (int64_t)sizeof(int32_t);
  const int64_t limit = align_static_table_ints();
  if (entries > limit) {
    const int64_t max_numel = (limit / experts) * 2048;
    return fail(EXF_ERR_INVALID,
                "%s: %lld routes over %d experts need %lld scratch entries but the fixed scratch "
                "holds %lld; at most %lld routes for %d experts (use exf_moe_align with a "
                "workspace for larger inputs)",
                name, (long long)numel, experts, (long long)entries, (long long)limit,
                (long long)max_numel, experts);
  }
  AlignParams p{ids, numel, experts, block_size, capacity, sorted_ids, expert_ids, num_post_pad,
                nullptr, 0};
  return cuda_status(launch_align_static(id_dtype, p, (cudaStream_t)stream), name);
}

// ---- calibration statistics (offline) ------------------------------------------------------
EXF_API int exf_calibration_update(const void* outputs, int out_dtype, const void* ids,
                                   int id_dtype, int64_t tokens, int top_k, int hidden,
                                   int experts, double* dot, double* target_sq,
                                   double* source_sq, double* norm_sum, double* norm_count,
                                   exf_stream_t stream) {
  const char* name = "exf_calibration_update";
  EXF_REQUIRE(good_wdtype(out_dtype) && good_idtype(id_dtype), "%s: unsupported dtype", name);
  EXF_REQUIRE(tokens >= 0, "%s: tokens must be >= 0", name);
  EXF_REQUIRE(top_k >= 1 && top_k <= 8, "%s: top_k must be in [1, 8], got %d", name, top_k);
  EXF_REQUIRE(hidden >= 8 && hidden % 8 == 0, "%s: hidden must be a positive multiple of 8", name);
  EXF_REQUIRE(experts >= 2 && experts <= 1024, "%s: experts must be in [2, 1024]", name);
  if (tokens == 0) return EXF_OK;
  EXF_REQUIRE(outputs && ids && dot && target_sq && source_sq && norm_sum && norm_count,
              "%s: null pointer", name);
  EXF_REQUIRE(aligned16(outputs), "%s: outputs must be 16-byte aligned", name);
  return cuda_status(launch_calib_update(out_dtype, id_dtype, outputs, ids, tokens, top_k, hidden,
                                         experts, dot, target_sq, source_sq, norm_sum, norm_count,
                                         (cudaStream_t)stream),
                     name);
}

EXF_API int exf_calibration_finalize(const double* dot, const double* target_sq,
                                     const double* source_sq, int experts, double ridge,
                                     double clip_min, double clip_max, float* coeff, float* loss,
                                     int32_t* nonfinite, exf_stream_t stream) {
  const char* name = "exf_calibration_finalize";
  EXF_REQUIRE(experts >= 2 && experts <= 1024, "%s: experts must be in [2, 1024]", name);
  EXF_REQUIRE(ridge > 0, "%s: ridge must be positive", name);
  EXF_REQUIRE(clip_min < clip_max, "%s: clip_min must be smaller than clip_max", name);
  EXF_REQUIRE(dot && target_sq && source_sq && coeff && loss, "%s: null pointer", name);
  return cuda_status(launch_calib_finalize(dot, target_sq, source_sq, experts, ridge, clip_min,
                                           clip_max, coeff, loss, nonfinite, (cudaStream_t)stream),
                     name);
}

EXF_API int exf_calibration_norms(const double* norm_sum, const double* norm_count, int experts,
                                  float* norms, exf_stream_t stream) {
  const char* name = "exf_calibration_norms";
  EXF_REQUIRE(experts >= 2 && experts <= 1024, "%s: experts must be in [2, 1024]", name);
  EXF_REQUIRE(norm_sum && norm_count && norms, "%s: null pointer", name);
  return cuda_status(launch_calib_norms(norm_sum, norm_count, experts, norms, (cudaStream_t)stream),
                     name);
}

}  // extern "C"
