// FP32-accurate GEMM on the sm_100a tensor cores (tcgen05, 3xTF32):
// C[M][N] = A . B^T over K with A an M x K and B an N x K operand, each
// stored either K-major ([rows][K], row stride ld) or K-outer ([K][rows],
// e.g. the activations of a weight gradient).  This is the dense contraction
// of the reference's register-blocked FP32 GEMMs (src/simple/dense_tiled.rs:
// 161-232 forward / input gradient, :234-318 weight gradient) and the
// building-block check of the tcgen05 path used by the attention kernels.
//
// A CTA of 128 threads owns a 128 x 64 tile of C in TMEM (128 lanes x 64
// FP32 columns).  Per 32-wide K block every thread loads and splits one slice
// of A and B into hi/lo TF32 shared tiles (K-major: a K-outer operand is
// transposed while staging, since TF32 MMAs read a transposed descriptor as
// zeros here); thread 0 issues 4 K-steps x 3 MMAs and commits them to the
// stage's mbarrier.  Two stages alternate, so the next block loads while the
// current block's MMAs run; all waits are bounded.  Long reductions (K = batch
// rows in a weight gradient) split K over grid.z; each chunk writes its own
// partial tile and a second kernel sums the chunks in a fixed order, so the
// result is bitwise reproducible.

#include <string>

#include "gemm_tc.h"
#include "host.h"
#include "tc05.cuh"

namespace mb {

namespace {

constexpr int kGemmBM = 128, kGemmBN = 64, kGemmBK = 32;
constexpr int kGemmStages = 2;
constexpr int kGemmStageFloats = 2 * kGemmBM * kGemmBK + 2 * kGemmBN * kGemmBK;  // A hi/lo, B hi/lo

// Rows [r0, r0+R) x K columns [k0, k0+BK) of a K-major operand
// (element (r, k) at g[r * ld + k]) into hi / lo blocked tiles, zero outside.
template <int R>
__device__ __forceinline__ void load_kmajor(float* hi, float* lo, const float* __restrict__ g, int ld, int r0,
                                            int rows, int k0, int K) {
  constexpr int C4 = kGemmBK / 4;
  for (int i = threadIdx.x; i < R * C4; i += blockDim.x) {
    const int rl = i & 7, c4 = (i >> 3) % C4, rh = (i >> 3) / C4;
    const int r = rh * 8 + rl, c = c4 * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    const int gr = r0 + r, gc = k0 + c;
    if (gr < rows) {
      const float* p = g + (size_t)gr * ld + gc;
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

// The same from a K-outer operand (element (r, k) at g[k * ld + r]): reads
// coalesce along r and the tile is transposed into K-major blocks.
template <int R>
__device__ __forceinline__ void load_kouter(float* hi, float* lo, const float* __restrict__ g, int ld, int r0,
                                            int rows, int k0, int K) {
  for (int i = threadIdx.x; i < kGemmBK * R; i += blockDim.x) {
    const int r = i % R, kk = i / R;
    const float x = (k0 + kk < K && r0 + r < rows) ? g[(size_t)(k0 + kk) * ld + r0 + r] : 0.f;
    const float h = tc::tf32_hi(x);
    const int off = tc::blk(r, kk, kGemmBK);
    hi[off] = h;
    lo[off] = x - h;
  }
}

__global__ void __launch_bounds__(128, 1)
    gemm_tf32x3_kernel(GemmOperand A, GemmOperand B, float* __restrict__ C, int ldc, size_t chunk_stride, int M,
                       int N, int K, int k_chunk, bool a_tmem, int* __restrict__ err) {
  extern __shared__ __align__(128) float sm[];
  __shared__ uint64_t bar[kGemmStages];
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * kGemmBN;
  const int kbeg = blockIdx.z * k_chunk, kend = min(K, kbeg + k_chunk);
  const int nb = kend > kbeg ? (kend - kbeg + kGemmBK - 1) / kGemmBK : 0;
  C += blockIdx.z * chunk_stride;  // split-K: this chunk's own partial tile
  // TMEM: the 64-column accumulator, then per stage 32 hi + 32 lo columns of
  // a TMEM-staged A block.
  if (warp == 0) tc::tmem_alloc(&tmem_base, 256);
  if (tid == 0) {
    for (int st = 0; st < kGemmStages; ++st) tc::bar_init(&bar[st], 1);
    tc::bar_init_fence();
    failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = tc::idesc_tf32(kGemmBM, kGemmBN, false, false);
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  // K block i into stage st (shared-memory tiles, or TMEM columns for A).
  auto load = [&](int i, int st) {
    const int k0 = kbeg + i * kGemmBK;
    float* Ah = sm + st * kGemmStageFloats;
    float* Al = Ah + kGemmBM * kGemmBK;
    float* Bh = Al + kGemmBM * kGemmBK;
    float* Bl = Bh + kGemmBN * kGemmBK;
    if (a_tmem) {
      // This thread's row of the A block, split and stored to the stage's
      // TMEM columns of its lane.
      float hi[16], lo[16];
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int r = m0 + tid, c = k0 + half * 16 + j;
          const float x = (r < M && c < kend) ? A.p[(size_t)r * A.ld + c] : 0.f;
          hi[j] = tc::tf32_hi(x);
          lo[j] = x - hi[j];
        }
        tc::tmem_st16(tmem + lane_off + 64 + 64 * st + half * 16, hi);
        tc::tmem_st16(tmem + lane_off + 96 + 64 * st + half * 16, lo);
      }
      tc::tmem_st_wait();
    } else if (A.k_outer) {
      load_kouter<kGemmBM>(Ah, Al, A.p, A.ld, m0, M, k0, kend);
    } else {
      load_kmajor<kGemmBM>(Ah, Al, A.p, A.ld, m0, M, k0, kend);
    }
    if (B.k_outer)
      load_kouter<kGemmBN>(Bh, Bl, B.p, B.ld, n0, N, k0, kend);
    else
      load_kmajor<kGemmBN>(Bh, Bl, B.p, B.ld, n0, N, k0, kend);
    tc::fence_async_smem();
    tc::fence_before_sync();
  };
  // Two stages: block i + 1 is loaded while block i's MMAs run.  A stage is
  // refilled only after the MMAs that read it (block i - 1) have completed.
  uint32_t phase[kGemmStages] = {0, 0};
  if (nb > 0) load(0, 0);
  __syncthreads();
  for (int i = 0; i < nb; ++i) {
    const int st = i & 1;
    if (tid == 0) {
      tc::fence_after_sync();
      const float* Ah = sm + st * kGemmStageFloats;
      const float* Al = Ah + kGemmBM * kGemmBK;
      const float* Bh = Al + kGemmBM * kGemmBK;
      const float* Bl = Bh + kGemmBN * kGemmBK;
#pragma unroll
      for (int s = 0; s < kGemmBK / 8; ++s) {
        const uint64_t ah = tc::desc_kmajor(Ah, kGemmBK, s), al = tc::desc_kmajor(Al, kGemmBK, s);
        const uint64_t bh = tc::desc_kmajor(Bh, kGemmBK, s), bl = tc::desc_kmajor(Bl, kGemmBK, s);
        const uint32_t acc = (i > 0 || s > 0) ? 1u : 0u;
        if (a_tmem) {
          const uint32_t a0 = tmem + 64 + 64 * st;
          tc::mma_ts(tmem, a0 + 8 * s, bh, idesc, acc);
          tc::mma_ts(tmem, a0 + 8 * s, bl, idesc, 1u);
          tc::mma_ts(tmem, a0 + 32 + 8 * s, bh, idesc, 1u);
        } else {
          tc::mma_ss(tmem, ah, bh, idesc, acc);
          tc::mma_ss(tmem, ah, bl, idesc, 1u);
          tc::mma_ss(tmem, al, bh, idesc, 1u);
        }
      }
      tc::commit(&bar[st]);
    }
    if (i + 1 < nb) {
      const int nx = st ^ 1;
      if (i >= 1) {
        if (!tc::bar_wait(&bar[nx], phase[nx])) failed = 1;
        phase[nx] ^= 1;
        tc::fence_after_sync();
      }
      load(i + 1, nx);
    }
    __syncthreads();
    if (failed) break;
  }
  // The last block's commit covers every MMA this thread issued.
  if (nb > 0 && !failed) {
    const int st = (nb - 1) & 1;
    if (!tc::bar_wait(&bar[st], phase[st])) failed = 1;
  }
  tc::fence_after_sync();
  __syncthreads();
  if (!failed) {
    const int r = m0 + tid;
    const uint32_t lane_base = tmem + lane_off;
    // An empty K range (a trailing chunk) never wrote TMEM: its tile is zero.
    const bool empty = nb == 0;
#pragma unroll
    for (int c0 = 0; c0 < kGemmBN; c0 += 16) {
      float v[16];
      tc::tmem_ld16(lane_base + c0, v);
      if (r < M) {
        float* dst = C + (size_t)r * ldc + n0 + c0;
        if (n0 + c0 + 16 <= N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            reinterpret_cast<float4*>(dst)[q] = empty ? make_float4(0.f, 0.f, 0.f, 0.f)
                                                      : make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (n0 + c0 + j < N) dst[j] = empty ? 0.f : v[j];
        }
      }
    }
  } else if (tid == 0) {
    atomicExch(err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

// C[m][n] = sum over chunks (in order) of partial[chunk][m][n].
__global__ void gemm_reduce_chunks(const float* __restrict__ partial, int chunks, int M, int N,
                                   float* __restrict__ C, int ldc) {
  const size_t mn = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < mn; i += (size_t)gridDim.x * blockDim.x) {
    float s = partial[i];
    for (int c = 1; c < chunks; ++c) s += partial[(size_t)c * mn + i];
    C[(i / N) * (size_t)ldc + i % N] = s;
  }
}

size_t gemm_smem() { return (size_t)kGemmStages * kGemmStageFloats * sizeof(float); }

}  // namespace

void gemm_prepare() {
  cudaError_t e =
      cudaFuncSetAttribute(&gemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem());
  if (e != cudaSuccess) throw Error(MB_ERR_CUDA, std::string("gemm attribute: ") + cudaGetErrorString(e));
}

int gemm_chunks(int K, int k_chunk) { return k_chunk <= 0 || k_chunk >= K ? 1 : (K + k_chunk - 1) / k_chunk; }

size_t gemm_partial_floats(int M, int N, int K, int k_chunk) {
  const int chunks = gemm_chunks(K, k_chunk);
  return chunks > 1 ? (size_t)chunks * M * N : 0;
}

int gemm_launches(int K, int k_chunk) { return gemm_chunks(K, k_chunk) > 1 ? 2 : 1; }

void launch_gemm(const GemmOperand& A, const GemmOperand& B, float* C, int ldc, int M, int N, int K, int k_chunk,
                 float* partial, int* err, cudaStream_t st, bool a_tmem) {
  require(!(a_tmem && A.k_outer), "an A operand staged through TMEM must be K-major");
  const int chunks = gemm_chunks(K, k_chunk);
  const int kc = chunks > 1 ? k_chunk : K;
  require(chunks == 1 || kc % kGemmBK == 0, "split-K chunks must be multiples of 32");
  require(chunks == 1 || partial != nullptr, "split-K needs a partial buffer");
  dim3 grid((M + kGemmBM - 1) / kGemmBM, (N + kGemmBN - 1) / kGemmBN, chunks);
  if (chunks == 1) {
    gemm_tf32x3_kernel<<<grid, 128, gemm_smem(), st>>>(A, B, C, ldc, 0, M, N, K, kc, a_tmem, err);
  } else {
    gemm_tf32x3_kernel<<<grid, 128, gemm_smem(), st>>>(A, B, partial, N, (size_t)M * N, M, N, K, kc, a_tmem,
                                                       err);
    const size_t mn = (size_t)M * N;
    const int blocks = (int)std::min<size_t>((mn + 255) / 256, 148 * 8);
    gemm_reduce_chunks<<<blocks, 256, 0, st>>>(partial, chunks, M, N, C, ldc);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw Error(MB_ERR_CUDA, std::string("gemm launch: ") + cudaGetErrorString(e));
}

}  // namespace mb

// layout bits: 1 = B stored [k][n], 2 = A staged through TMEM, 4 = A stored [k][m].
extern "C" int mb_op_gemm_tf32x3(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                                 uint32_t layout, int* d_status, void* stream) {
  return mb::guarded([&] {
    mb::need(a, "a");
    mb::need(b, "b");
    mb::need(c, "c");
    mb::need(d_status, "status");
    mb::require(m >= 1 && n >= 1 && k >= 1, "GEMM dimensions must be positive");
    mb::require(layout <= 7 && layout != 6 && layout != 7,
                "layout bits: 1 = B [k][n], 2 = A through TMEM, 4 = A [k][m] (not with 2)");
    const bool b_outer = layout & 1, a_tmem = layout & 2, a_outer = layout & 4;
    mb::gemm_prepare();
    const mb::GemmOperand A{a, a_outer ? (int)m : (int)k, a_outer};
    const mb::GemmOperand B{b, b_outer ? (int)n : (int)k, b_outer};
    mb::launch_gemm(A, B, c, (int)n, (int)m, (int)n, (int)k, 0, nullptr, d_status, (cudaStream_t)stream, a_tmem);
  });
}
