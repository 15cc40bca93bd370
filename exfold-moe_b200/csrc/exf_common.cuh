// Shared device helpers for the ExFold routing-transform kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "exfold_b200.h"

namespace exf {

// ---------------------------------------------------------------------------------------------
// Element types of the routing tensors.  Computation is fp32; weights are read and written in
// their own type, ids as int32 or int64.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// ---------------------------------------------------------------------------------------------
// Exact elementwise math.  These functions are defined by their operation sequence: every step
// is one IEEE binary32 operation with round-to-nearest-even (explicit _rn intrinsics, no
// contraction), so a scalar C restatement performing the same steps returns the same bits.
//
// exp(x): Cody-Waite reduction x = n*ln2 + r with ln2 split into a 15-bit head (n*ln2_hi exact)
// and a tail, the degree-7 Taylor polynomial of e^r on |r| <= ln2/2 by Horner with fused
// multiply-adds (truncation error below 6e-9 relative), and scaling by 2^n through the exponent
// field.  Inputs are clamped to [-87, 88] (NaN to -87) so that 2^n stays a normal number.
constexpr float kLog2e = 0x1.715476p+0f;
constexpr float kLn2Hi = 0x1.62e4p-1f;
constexpr float kLn2Lo = 0x1.7f7d1cp-20f;

__device__ __forceinline__ float exact_exp(float x) {
  x = (x > -87.0f) ? x : -87.0f;
  x = (x > 88.0f) ? 88.0f : x;
  const float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fmaf_rn(n, -kLn2Hi, x);
  r = __fmaf_rn(n, -kLn2Lo, r);
  float p = 0x1.a01a02p-13f;          // 1/7!
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);  // 1/6!
  p = __fmaf_rn(p, r, 0x1.111112p-7f);   // 1/5!
  p = __fmaf_rn(p, r, 0x1.555556p-5f);   // 1/4!
  p = __fmaf_rn(p, r, 0x1.555556p-3f);   // 1/3!
  p = __fmaf_rn(p, r, 0x1p-1f);          // 1/2!
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = __float2int_rz(n);
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// exact_exp for arguments that are never above 88 (differences from a row maximum, or NaN):
// the same operations without the upper clamp, so the same bits.
__device__ __forceinline__ float exact_exp_le88(float x) {
  x = (x > -87.0f) ? x : -87.0f;
  const float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fmaf_rn(n, -kLn2Hi, x);
  r = __fmaf_rn(n, -kLn2Lo, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0x1p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = __float2int_rz(n);
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

__device__ __forceinline__ float exact_sigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exact_exp(-x)));
}

// Fast sigmoid used only to pre-select candidates; its error is far below kSigmoidMargin, and
// every candidate is then re-ranked with exact_sigmoid.
// fminf maps NaN to 88, matching exact_sigmoid (whose exp clamp sends NaN to sigmoid(88)).
__device__ __forceinline__ float approx_sigmoid(float x) {
  x = fminf(x, 88.0f);
  return __fdividef(1.0f, 1.0f + __expf(-x));
}
// sqrt(softplus(x)), the "sqrtsoftplus" router score: softplus(x) = max(x, 0) + log1p(exp(-|x|))
// with exact_exp (NaN goes to its lower clamp), log1p(y) for 0 < y <= 1 as 2 atanh(u), u =
// y / (2 + y) <= 1/3: 2u (1 + u^2/3 + ... + u^14/15) by Horner in u^2 with fused multiply-adds
// (truncation below 2e-9 relative), then the IEEE square root.
__device__ __forceinline__ float exact_log1p_unit(float y) {
  const float u = __fdiv_rn(y, __fadd_rn(2.0f, y));
  const float s = __fmul_rn(u, u);
  float q = 0x1.111112p-4f;           // 1/15
  q = __fmaf_rn(q, s, 0x1.3b13b2p-4f);  // 1/13
  q = __fmaf_rn(q, s, 0x1.745d18p-4f);  // 1/11
  q = __fmaf_rn(q, s, 0x1.c71c72p-4f);  // 1/9
  q = __fmaf_rn(q, s, 0x1.24924ap-3f);  // 1/7
  q = __fmaf_rn(q, s, 0x1.99999ap-3f);  // 1/5
  q = __fmaf_rn(q, s, 0x1.555556p-2f);  // 1/3
  q = __fmaf_rn(q, s, 1.0f);
  return __fmul_rn(__fmul_rn(2.0f, u), q);
}
__device__ __forceinline__ float exact_sqrtsoftplus(float x) {
  const float e = exact_exp(-fabsf(x));
  return __fsqrt_rn(__fadd_rn(fmaxf(x, 0.0f), exact_log1p_unit(e)));
}
// Fast version for candidate preselection; NaN is mapped as in the exact version.
__device__ __forceinline__ float approx_sqrtsoftplus(float x) {
  float t = -fabsf(x);
  t = t > -87.0f ? t : -87.0f;
  return sqrtf(fmaxf(x, 0.0f) + __logf(1.0f + __expf(t)));
}

// Bound on |approx score + b - (exact score + b)| (sigmoid and sqrtsoftplus) with a wide safety
// factor.
constexpr float kSigmoidMargin = 1.0e-4f;

// The biased-score routers: EXF_SIGMOID or EXF_SQRTSOFTPLUS.
template <int SCORING>
__device__ __forceinline__ float exact_score(float x) {
  return SCORING == EXF_SQRTSOFTPLUS ? exact_sqrtsoftplus(x) : exact_sigmoid(x);
}
template <int SCORING>
__device__ __forceinline__ float approx_score(float x) {
  return SCORING == EXF_SQRTSOFTPLUS ? approx_sqrtsoftplus(x) : approx_sigmoid(x);
}

// Keys: floats mapped to unsigned ints in IEEE 754 totalOrder (-NaN < -inf < ... < -0 < +0 <
// ... < +inf < +NaN), two instructions.  key_of additionally ranks -0 equal to +0, which is
// the order every comparison of the reference sees for finite values.
constexpr uint32_t kKeyPosZero = 0x80000000u;
constexpr uint32_t kKeyNegZero = 0x7FFFFFFFu;

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
}
__device__ __forceinline__ uint32_t key_of(float x) {
  const uint32_t k = order_key(x);
  return k == kKeyNegZero ? kKeyPosZero : k;
}
__device__ __forceinline__ float float_of_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// (key desc, index asc) order
__device__ __forceinline__ bool ranks_before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Decode importance in 2^-32 fixed point: fp32 product, a NaN product counts 0, clamp to
// |p| <= 2^24 (so one route adds at most 2^56), round to nearest even.  Integer sums are exact
// and wrap modulo 2^64, so an expert's importance is exact, whatever the summation order or the
// split of the batch over GPUs, while its true total stays below 2^31 in magnitude.
__device__ __forceinline__ long long fixed_point(float p) {
  if (p != p) return 0;
  p = fminf(fmaxf(p, -16777216.0f), 16777216.0f);
  return __float2ll_rn(__fmul_rn(p, 4294967296.0f));
}

// ---------------------------------------------------------------------------------------------
// Router logits come as fp32, bf16 or fp16 (the model's gate output dtype).  Each logit is
// converted to fp32 exactly (bf16: the 16 bits become the high half of the float; fp16: the
// exact half-to-float conversion), and selection and weights run on the converted values, so the
// results equal the fp32 path on logits.float().  Four consecutive logits are 16 bytes (fp32) or
// 8 bytes (16-bit): one load either way.
template <typename LT>
__device__ __forceinline__ float logit_f32(LT v);
template <>
__device__ __forceinline__ float logit_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float logit_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __uint_as_float(static_cast<uint32_t>(__bfloat16_as_ushort(v)) << 16);
}
template <>
__device__ __forceinline__ float logit_f32<__half>(__half v) { return __half2float(v); }

// Two packed 16-bit logits (low half first) as two floats.
template <typename LT>
__device__ __forceinline__ float2 logit2_f32(uint32_t u);
template <>
__device__ __forceinline__ float2 logit2_f32<__nv_bfloat16>(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ float2 logit2_f32<__half>(uint32_t u) {
  return make_float2(__half2float(__ushort_as_half(static_cast<unsigned short>(u & 0xFFFFu))),
                     __half2float(__ushort_as_half(static_cast<unsigned short>(u >> 16))));
}

// logits p[0..3] as a float4; p is 16-byte (fp32) / 8-byte (16-bit) aligned.  Plain load (global
// or shared memory).
template <typename LT>
__device__ __forceinline__ float4 load_logits4(const LT* p) {
  if constexpr (sizeof(LT) == 4) {
    return *reinterpret_cast<const float4*>(p);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = logit2_f32<LT>(u.x), b = logit2_f32<LT>(u.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
}

// Streaming 16-byte load that does not allocate in L1 (router logits are read exactly once).
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
// load_logits4 from global memory through the non-allocating streaming path
template <typename LT>
__device__ __forceinline__ float4 ld_stream_logits4(const LT* p) {
  if constexpr (sizeof(LT) == 4) {
    return ld_stream_f4(reinterpret_cast<const float*>(p));
  } else {
    uint32_t x, y;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(x), "=r"(y)
                 : "l"(p));
    const float2 a = logit2_f32<LT>(x), b = logit2_f32<LT>(y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
}

}  // namespace exf
