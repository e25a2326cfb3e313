// Shared device helpers for the Mesh GPT sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {

constexpr uint32_t kIgnoreTarget = 0xFFFFFFFFu;  // src/gpt/mod.rs:26
constexpr float kRmsEpsilon = 1e-5f;              // src/gpt/mod.rs:39
constexpr float kXsaEpsilon = 1e-12f;             // src/gpt/mod.rs:41

// Packed two-lane FP32 arithmetic (sm_100 f32x2 instructions): one issue
// slot for a channel pair, each lane rounded exactly like its scalar form.
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }

__device__ __forceinline__ float2 operator+(float2 a, float2 b) { return add2(a, b); }
__device__ __forceinline__ float2 operator-(float2 a, float2 b) { return add2(a, make_float2(-b.x, -b.y)); }
__device__ __forceinline__ float2 operator*(float2 a, float s) { return mul2(a, splat2(s)); }

// 2^x on the hardware exponential unit (PTX ex2.approx.ftz.f32); results
// below 2^-126 flush to zero.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// ELU with alpha 1 as in the reference kernel (src/gpt/gpu.rs:135-139):
// exp(z) - 1 for z < 0, with e^z evaluated as 2^(z log2 e).  Its error, a
// few ulp of e^z on the negative branch, sits far inside the model's
// tolerances and keeps the mesh layers' instruction count low.
__device__ __forceinline__ float2 elu2(float2 z) {
  const float2 t = mul2(z, splat2(kLog2e));
  const float2 em1 = add2(make_float2(ex2_ftz(t.x), ex2_ftz(t.y)), splat2(-1.0f));
  return make_float2(z.x < 0.0f ? em1.x : z.x, z.y < 0.0f ? em1.y : z.y);
}
__device__ __forceinline__ float elu(float z) { return z < 0.0f ? ex2_ftz(z * kLog2e) - 1.0f : z; }

// ELU derivative from the activated output y (src/gpt/gpu.rs:28-34).
__device__ __forceinline__ float elu_slope(float y) { return y >= 0.0f ? 1.0f : y + 1.0f; }
__device__ __forceinline__ float2 elu_slope2(float2 y) {
  const float2 s = add2(y, splat2(1.0f));
  return make_float2(y.x >= 0.0f ? 1.0f : s.x, y.y >= 0.0f ? 1.0f : s.y);
}

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
