// Shared helpers for the B200 Cut Cross-Entropy kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cce_b200.h"

namespace cce {

// Rows per filter block; the vocabulary side of a block is CCE_STAT_TILE.
constexpr int kRowBlock = 128;
constexpr int kStatTile = CCE_STAT_TILE;

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// log2(e), the base change used with exp2f (exp(x) = 2^(x * log2(e))).
constexpr float kLog2e = 1.4426950408889634f;

}  // namespace cce
