// FP32-accurate GEMM on the sm_100a tensor cores (tcgen05, 3xTF32):
// C[M][N] = A[M][K] . B[N][K]^T, all row-major FP32.  This is the dense
// contraction of the reference's register-blocked FP32 GEMMs
// (src/simple/dense_tiled.rs:161-232, blocked_product) and the building-block
// check of the tcgen05 path used by the attention kernels.
//
// A CTA of 128 threads owns a 128 x 64 tile of C in TMEM (128 lanes x 64
// FP32 columns).  Per 32-wide K block every thread loads and splits one slice
// of A and B into hi/lo TF32 shared tiles; thread 0 issues 4 K-steps x 3
// MMAs and commits them to an mbarrier that all threads wait on (bounded).

#include <string>

#include "host.h"
#include "tc05.cuh"

namespace mb {

namespace {

constexpr int kGemmBM = 128, kGemmBN = 64, kGemmBK = 32;

// Loads rows [r0, r0+R) x cols [k0, k0+BK) of a row-major [rows][K] matrix,
// splitting each value into hi / lo blocked tiles (zero outside the matrix).
template <int R>
__device__ __forceinline__ void load_split_rows(float* hi, float* lo, const float* __restrict__ g, int r0, int rows,
                                                int k0, int K) {
  constexpr int C4 = kGemmBK / 4;
  for (int i = threadIdx.x; i < R * C4; i += blockDim.x) {
    const int rl = i & 7, c4 = (i >> 3) % C4, rh = (i >> 3) / C4;
    const int r = rh * 8 + rl, c = c4 * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    const int gr = r0 + r, gc = k0 + c;
    if (gr < rows) {
      const float* p = g + (size_t)gr * K + gc;
      if (gc + 3 < K && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
        v = *reinterpret_cast<const float4*>(p);
      } else {
        v.x = gc < K ? p[0] : 0.f;
        v.y = gc + 1 < K ? p[1] : 0.f;
        v.z = gc + 2 < K ? p[2] : 0.f;
        v.w = gc + 3 < K ? p[3] : 0.f;
      }
    }
    const float4 h = make_float4(tc::tf32_hi(v.x), tc::tf32_hi(v.y), tc::tf32_hi(v.z), tc::tf32_hi(v.w));
    const int off = tc::blk(r, c, kGemmBK);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

// B [K][N] row-major -> transposed hi/lo blocked tiles [BN rows][BK cols]
// (K-major).  An MN-major TF32 descriptor would avoid the transpose, but on
// sm_100a TF32 MMAs with an MN-major (transposed) operand read it as zeros,
// so every operand here is staged K-major.
__device__ __forceinline__ void load_split_cols(float* hi, float* lo, const float* __restrict__ g, int k0, int K,
                                                int n0, int N) {
  for (int i = threadIdx.x; i < kGemmBK * kGemmBN; i += blockDim.x) {
    const int n = i % kGemmBN, kk = i / kGemmBN;
    const float x = (k0 + kk < K && n0 + n < N) ? g[(size_t)(k0 + kk) * N + n0 + n] : 0.f;
    const float h = tc::tf32_hi(x);
    const int off = tc::blk(n, kk, kGemmBK);
    hi[off] = h;
    lo[off] = x - h;
  }
}

__global__ void __launch_bounds__(128, 1)
    gemm_tf32x3_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M, int N,
                       int K, int mode, int* __restrict__ err) {
  extern __shared__ __align__(128) float sm[];
  float* Ah = sm;
  float* Al = Ah + kGemmBM * kGemmBK;
  float* Bh = Al + kGemmBM * kGemmBK;
  float* Bl = Bh + kGemmBN * kGemmBK;
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * kGemmBN;
  if (warp == 0) tc::tmem_alloc(&tmem_base, 128);
  if (tid == 0) {
    tc::bar_init(&bar, 1);
    tc::bar_init_fence();
    failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = tc::idesc_tf32(kGemmBM, kGemmBN, false, false);
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  uint32_t phase = 0;
  const int nk = (K + kGemmBK - 1) / kGemmBK;
  for (int kb = 0; kb < nk; ++kb) {
    if (mode == 2) {
      // This thread's row of the A block, split and stored to TMEM columns
      // [64, 96) (hi) and [96, 128) (lo) of its lane.
      float hi[16], lo[16];
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int r = m0 + tid, c = kb * kGemmBK + half * 16 + j;
          const float x = (r < M && c < K) ? A[(size_t)r * K + c] : 0.f;
          hi[j] = tc::tf32_hi(x);
          lo[j] = x - hi[j];
        }
        tc::tmem_st16(tmem + lane_off + 64 + half * 16, hi);
        tc::tmem_st16(tmem + lane_off + 96 + half * 16, lo);
      }
      tc::tmem_st_wait();
    } else {
      load_split_rows<kGemmBM>(Ah, Al, A, m0, M, kb * kGemmBK, K);
    }
    if (mode == 1)
      load_split_cols(Bh, Bl, B, kb * kGemmBK, K, n0, N);
    else
      load_split_rows<kGemmBN>(Bh, Bl, B, n0, N, kb * kGemmBK, K);
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after_sync();
#pragma unroll
      for (int s = 0; s < kGemmBK / 8; ++s) {
        const uint64_t ah = tc::desc_kmajor(Ah, kGemmBK, s), al = tc::desc_kmajor(Al, kGemmBK, s);
        const uint64_t bh = tc::desc_kmajor(Bh, kGemmBK, s), bl = tc::desc_kmajor(Bl, kGemmBK, s);
        const uint32_t acc = (kb > 0 || s > 0) ? 1u : 0u;
        if (mode == 2) {
          tc::mma_ts(tmem, tmem + 64 + 8 * s, bh, idesc, acc);
          tc::mma_ts(tmem, tmem + 64 + 8 * s, bl, idesc, 1u);
          tc::mma_ts(tmem, tmem + 96 + 8 * s, bh, idesc, 1u);
        } else {
          tc::mma_ss(tmem, ah, bh, idesc, acc);
          tc::mma_ss(tmem, ah, bl, idesc, 1u);
          tc::mma_ss(tmem, al, bh, idesc, 1u);
        }
      }
      tc::commit(&bar);
    }
    if (!tc::bar_wait(&bar, phase)) failed = 1;
    phase ^= 1;
    __syncthreads();
    if (failed) break;
  }
  tc::fence_after_sync();
  if (!failed) {
    const int r = m0 + tid;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll
    for (int c0 = 0; c0 < kGemmBN; c0 += 16) {
      float v[16];
      tc::tmem_ld16(lane_base + c0, v);
      tc::tmem_ld_wait();
      if (r < M) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (n0 + c0 + j < N) C[(size_t)r * N + n0 + c0 + j] = v[j];
      }
    }
  } else if (tid == 0) {
    atomicExch(err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 128);
}

}  // namespace

void launch_gemm_tf32x3(const float* A, const float* B, float* C, int M, int N, int K, int mode, int* err,
                        cudaStream_t st) {
  const size_t smem = (size_t)(2 * kGemmBM * kGemmBK + 2 * kGemmBN * kGemmBK) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(&gemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) throw Error(MB_ERR_CUDA, std::string("gemm attribute: ") + cudaGetErrorString(e));
  dim3 grid((M + kGemmBM - 1) / kGemmBM, (N + kGemmBN - 1) / kGemmBN);
  gemm_tf32x3_kernel<<<grid, 128, smem, st>>>(A, B, C, M, N, K, mode, err);
  e = cudaGetLastError();
  if (e != cudaSuccess) throw Error(MB_ERR_CUDA, std::string("gemm launch: ") + cudaGetErrorString(e));
}

}  // namespace mb

extern "C" int mb_op_gemm_tf32x3(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                                 uint32_t layout, int* d_status, void* stream) {
  return mb::guarded([&] {
    mb::need(a, "a");
    mb::need(b, "b");
    mb::need(c, "c");
    mb::need(d_status, "status");
    mb::require(m >= 1 && n >= 1 && k >= 1, "GEMM dimensions must be positive");
    mb::require(layout <= 2, "layout must be 0 (B [n][k]), 1 (B [k][n]) or 2 (B [n][k], A through TMEM)");
    mb::launch_gemm_tf32x3(a, b, c, (int)m, (int)n, (int)k, (int)layout, d_status, (cudaStream_t)stream);
  });
}
