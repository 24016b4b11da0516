// common.cuh -- shared device helpers for the RACE B200 library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace race {

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Hyperplane sign of corner r for bit p of a P-bit table: +1 iff bit (P-1-p)
// of r is set (itertools.product([-1,+1], repeat=P) order).
__device__ __forceinline__ float corner_sign(int r, int p, int P) {
  return ((r >> (P - 1 - p)) & 1) ? 1.f : -1.f;
}

__host__ __device__ __forceinline__ size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace race
