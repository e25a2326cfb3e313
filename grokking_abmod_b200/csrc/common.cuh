// Shared device helpers for the Mesh GPT sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {

constexpr uint32_t kIgnoreTarget = 0xFFFFFFFFu;  // src/gpt/mod.rs:26
constexpr float kRmsEpsilon = 1e-5f;              // src/gpt/mod.rs:39
constexpr float kXsaEpsilon = 1e-12f;             // src/gpt/mod.rs:41

// ELU with alpha 1 as in the reference kernel (src/gpt/gpu.rs:135-139):
// exp(z) - 1 for z < 0.  The exponential is the __expf intrinsic (one
// multiply and the hardware base-2 exponential); its error, a few ulp of
// exp(z) on the negative branch, sits far inside the model's tolerances and
// keeps the mesh layers' instruction count low.
__device__ __forceinline__ float elu(float z) { return z < 0.0f ? __expf(z) - 1.0f : z; }

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
