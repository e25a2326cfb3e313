// Shared device helpers for the Mesh GPT sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {

constexpr uint32_t kIgnoreTarget = 0xFFFFFFFFu;  // src/gpt/mod.rs:26
constexpr float kRmsEpsilon = 1e-5f;              // src/gpt/mod.rs:39
constexpr float kXsaEpsilon = 1e-12f;             // src/gpt/mod.rs:41

// ELU with alpha 1, written like the reference kernel (src/gpt/gpu.rs:135-139).
__device__ __forceinline__ float elu(float z) { return z < 0.0f ? expf(z) - 1.0f : z; }

// ELU derivative from the activated output y (src/gpt/gpu.rs:28-34).
__device__ __forceinline__ float elu_slope(float y) { return y >= 0.0f ? 1.0f : y + 1.0f; }

__device__ __forceinline__ float2 operator+(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 operator-(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 operator*(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

template <int LANES>
__device__ __forceinline__ float group_sum(float v) {
  // Butterfly sum over aligned groups of LANES consecutive lanes (LANES | 32).
#pragma unroll
  for (int o = LANES / 2; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float2 shfl_xor2(float2 v, int o) {
  return make_float2(__shfl_xor_sync(0xffffffffu, v.x, o), __shfl_xor_sync(0xffffffffu, v.y, o));
}

}  // namespace mb
