// Device helpers of the tile router kernel (router_tpt.cu): mbarrier waits and
// bulk copies of logit tiles into shared memory, and the register sorting networks of the
// top-8 selection.
#pragma once

#include <stdint.h>

namespace exf {
namespace tile {

constexpr uint32_t kSpinLimit = 1u << 20;

__device__ __forceinline__ uint32_t saddr(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}
__device__ __forceinline__ void bar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool bar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for a tile; false if the copy did not complete within the limit.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (bar_test(bar, parity)) return true;
    if (i > 16) __nanosleep(32);
  }
  return false;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(bar))
      : "memory");
}

// max that returns NaN when either input is NaN
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// three-input max (PTX 8.8, sm_100): NaN when any input is NaN / the largest non-NaN input
__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ void cx32(uint32_t& a, uint32_t& b) {
  const uint32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}
__device__ __forceinline__ void cxs32(int32_t& a, int32_t& b) {
  const int32_t hi = max(a, b), lo = min(a, b);
  a = hi;
  b = lo;
}
__device__ __forceinline__ void cx64(uint64_t& a, uint64_t& b) {
  const bool swap = a < b;
  const uint64_t hi = swap ? b : a, lo = swap ? a : b;
  a = hi;
  b = lo;
}
// Optimal 19-comparator network for 8 inputs, descending.
template <typename T, void (*CX)(T&, T&)>
__device__ __forceinline__ void sort8(T* v) {
  CX(v[0], v[2]); CX(v[1], v[3]); CX(v[4], v[6]); CX(v[5], v[7]);
  CX(v[0], v[4]); CX(v[1], v[5]); CX(v[2], v[6]); CX(v[3], v[7]);
  CX(v[0], v[1]); CX(v[2], v[3]); CX(v[4], v[5]); CX(v[6], v[7]);
  CX(v[2], v[4]); CX(v[3], v[5]);
  CX(v[1], v[4]); CX(v[3], v[6]);
  CX(v[1], v[2]); CX(v[3], v[4]); CX(v[5], v[6]);
}
// a, b sorted descending -> a = the 8 largest of both, sorted descending; dmax = the largest of
// the values dropped so far (over a whole merge tree: the 9th largest input)
__device__ __forceinline__ void merge8(uint32_t* a, const uint32_t* b, uint32_t& dmax) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    dmax = max(dmax, min(a[i], b[7 - i]));
    a[i] = max(a[i], b[7 - i]);
  }
  cx32(a[0], a[4]); cx32(a[1], a[5]); cx32(a[2], a[6]); cx32(a[3], a[7]);
  cx32(a[0], a[2]); cx32(a[1], a[3]); cx32(a[4], a[6]); cx32(a[5], a[7]);
  cx32(a[0], a[1]); cx32(a[2], a[3]); cx32(a[4], a[5]); cx32(a[6], a[7]);
}
// merge8 on signed keys
__device__ __forceinline__ void merge8s(int32_t* a, const int32_t* b, int32_t& dmax) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    dmax = max(dmax, min(a[i], b[7 - i]));
    a[i] = max(a[i], b[7 - i]);
  }
  cxs32(a[0], a[4]); cxs32(a[1], a[5]); cxs32(a[2], a[6]); cxs32(a[3], a[7]);
  cxs32(a[0], a[2]); cxs32(a[1], a[3]); cxs32(a[4], a[6]); cxs32(a[5], a[7]);
  cxs32(a[0], a[1]); cxs32(a[2], a[3]); cxs32(a[4], a[5]); cxs32(a[6], a[7]);
}
// Insert v into T (sorted descending), dropping the smallest.
__device__ __forceinline__ void insert8(uint64_t (&T)[8], uint64_t v) {
#pragma unroll
  for (int q = 0; q < 8; ++q) cx64(T[q], v);
}
// (key desc, column asc) as one unsigned 64-bit order: the key, then the complemented column.
__device__ __forceinline__ uint64_t pack(uint32_t key, int col) {
  return (static_cast<uint64_t>(key) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(col));
}

}  // namespace tile
}  // namespace exf
