// Exhaustive check of the approximate sigmoid that router_biased.cu preselects with:
// 0.5 * tanh.approx(x / 2) + 0.5 (the same operation sequence, c = 0.5), against a
// double-precision sigmoid, over every finite fp32 x; and the error of exact_sigmoid.  Prints
// "approx <max abs err> exact <max abs err> inf <approx(+inf)> <approx(-inf)>".  Test
// infrastructure: built and run by tests/test_gpu_approx_bound.py.
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#include "exf_common.cuh"

__device__ __forceinline__ float approx_sigmoid_tanh(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(__fmul_rn(0.5f, x)));
  return __fmaf_rn(0.5f, t, 0.5f);
}

__global__ void sweep(unsigned long long* worst, float* inf_out) {
  unsigned long long wa = 0, we = 0;
  const uint64_t n = 1ull << 32;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const float x = __uint_as_float(static_cast<uint32_t>(i));
    if (!isfinite(x)) continue;
    const double s = 1.0 / (1.0 + exp(-static_cast<double>(x)));
    const double ea = fabs(static_cast<double>(approx_sigmoid_tanh(x)) - s);
    const double ee = fabs(static_cast<double>(exf::exact_sigmoid(x)) - s);
    wa = max(wa, static_cast<unsigned long long>(__double_as_longlong(ea)));
    we = max(we, static_cast<unsigned long long>(__double_as_longlong(ee)));
  }
  atomicMax(&worst[0], wa);
  atomicMax(&worst[1], we);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    inf_out[0] = approx_sigmoid_tanh(__int_as_float(0x7F800000));
    inf_out[1] = approx_sigmoid_tanh(__int_as_float(static_cast<int>(0xFF800000u)));
  }
}

int main() {
  unsigned long long* w = nullptr;
  float* f = nullptr;
  if (cudaMalloc(&w, 16) != cudaSuccess || cudaMalloc(&f, 8) != cudaSuccess) return 2;
  cudaMemset(w, 0, 16);
  sweep<<<148 * 8, 256>>>(w, f);
  if (cudaDeviceSynchronize() != cudaSuccess) return 3;
  unsigned long long h[2];
  float hf[2];
  cudaMemcpy(h, w, 16, cudaMemcpyDeviceToHost);
  cudaMemcpy(hf, f, 8, cudaMemcpyDeviceToHost);
  double a, e;
  std::memcpy(&a, &h[0], 8);
  std::memcpy(&e, &h[1], 8);
  std::printf("approx %.9e exact %.9e inf %.9g %.9g\n", a, e, hf[0], hf[1]);
  return 0;
}
