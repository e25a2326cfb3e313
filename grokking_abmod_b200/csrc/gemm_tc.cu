// FP32-accurate GEMM on the sm_100a tensor cores (tcgen05, 3xTF32):
// C[M][N] = A . B^T over K with A an M x K and B an N x K operand, each
// stored either K-major ([rows][K], row stride ld) or K-outer ([K][rows],
// e.g. the activations of a weight gradient).  This is the dense contraction
// of the reference's register-blocked FP32 GEMMs (src/simple/dense_tiled.rs:
// 161-232 forward / input gradient, :234-318 weight gradient) and the
// building-block check of the tcgen05 path used by the attention kernels.
//
// A CTA of 256 threads owns a 128 x 64 tile of C in TMEM (128 lanes x 64
// FP32 columns).  The raw fp32 tiles of each 32-wide K block of A and B are
// copied into shared memory four blocks ahead by TMA tensor copies (cp.async
// pieces where an operand's alignment rules a tensor map out).  Worker warps
// split a landed block into hi/lo TF32: A rows straight into TMEM columns
// (one lane per row), B into K-major shared tiles (a K-outer operand is
// transposed while splitting, since TF32 MMAs read a transposed descriptor
// as zeros here).  A separate MMA warp issues 4 K-steps x 3 MMAs (A from
// TMEM, B from shared memory) per block.  Two hi/lo stages alternate, so one
// block is split while the previous block's MMAs run; all waits are bounded.  Long reductions (K = batch
// rows in a weight gradient) split K over grid.z; each chunk writes its own
// partial tile and a second kernel sums the chunks in a fixed order, so the
// result is bitwise reproducible.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <string>

#include "gemm_tc.h"
#include "host.h"
#include "tc05.cuh"

namespace mb {

namespace {

constexpr int kGemmBM = 128, kGemmBN = 64, kGemmBK = 32;
constexpr int kGemmStages = 2;
constexpr int kGemmStageFloats = 2 * kGemmBN * kGemmBK;  // B hi/lo (A hi/lo live in TMEM)

// Eight warps: the copy and split work of a K block is spread over all of
// them; warp w reads TMEM lane quarter w % 4, column half w / 4.
constexpr int kGemmThreads = 256;
// Raw fp32 operand tiles staged ahead of the split: kGemmRaw stages, all in
// flight while the tensor cores work on earlier blocks.  A K-major tile is
// raw[r][BK] with the 16-byte pieces of row r at piece c ^ (r & 7) (the TMA
// 128-byte swizzle, so the split's row-wise reads are conflict-free); a
// K-outer tile is raw[k][R].  Tiles come from TMA tensor copies where the
// operand allows one (16-byte aligned base and row stride), else cp.async.
constexpr int kGemmRaw = 4;
constexpr int kRawFloats = (kGemmBM + kGemmBN) * kGemmBK;
constexpr int kTmaA = 1, kTmaB = 2;

__device__ __forceinline__ int raw_kmajor(int r, int c) { return r * kGemmBK + (((c >> 2) ^ (r & 7)) << 2); }

// One 2D tensor copy (box at coordinates x inner, y outer) into shared
// memory, completing its bytes on the mbarrier.  x is a multiple of 32
// (K-major) or of 64 (K-outer) elements: every copy starts 16-byte aligned.
__device__ __forceinline__ void tma_load_2d(float* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(tc::smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void cp_async16(float* dst, const float* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tc::smem_addr(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src, int bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(tc::smem_addr(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Starts the copy of rows [r0, r0+R) x K columns [k0, k0+BK) of an operand
// into a raw tile; bytes outside the matrix are zero-filled (and not read).
// `vec`: 16-byte copies are aligned (base 16-byte aligned, ld a multiple of 4).
template <int R>
__device__ __forceinline__ void stage_raw(float* raw, const GemmOperand& op, bool vec, int r0, int rows, int k0,
                                          int K) {
  constexpr int kPer = R * (kGemmBK / 4) / kGemmThreads;
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int i = threadIdx.x + u * kGemmThreads;
    int gr, gk, rlim, klim;
    float* dst;
    if (!op.k_outer) {  // 16-byte pieces along k
      const int r = i >> 3, c = (i & 7) * 4;
      gr = r0 + r;
      gk = k0 + c;
      dst = raw + raw_kmajor(r, c);
      rlim = gr < rows ? 1 : 0;
      klim = K - gk;
    } else {  // 16-byte pieces along r
      const int kk = i / (R / 4), r = (i % (R / 4)) * 4;
      gr = r0 + r;
      gk = k0 + kk;
      dst = raw + kk * R + r;
      rlim = rows - gr;
      klim = gk < K ? 1 : 0;
    }
    const int n = op.k_outer ? (klim > 0 ? min(4, max(0, rlim)) : 0) : (rlim > 0 ? min(4, max(0, klim)) : 0);
    const float* src = n > 0 ? op.p + (op.k_outer ? (size_t)gk * op.ld + gr : (size_t)gr * op.ld + gk) : op.p;
    if (vec) {
      cp_async16(dst, src, 4 * n);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) cp_async4(dst + j, j < n ? src + j : op.p, j < n ? 4 : 0);
    }
  }
}

// Splits a landed raw tile into hi / lo TF32 K-major blocked tiles.  A
// thread takes one row and one 4-wide K group; consecutive threads take
// consecutive rows, so the 16-byte stores of a quarter warp fill one
// contiguous core-matrix run and the raw reads are conflict-free.
template <int R, int T>
__device__ __forceinline__ void split_raw(float* hi, float* lo, const float* raw, bool k_outer, int t) {
  constexpr int kPer = R * (kGemmBK / 4) / T;
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int i = t + u * T;
    int r, c;
    float4 v;
    if (!k_outer) {
      r = (i >> 3) / (kGemmBK / 4) * 8 + (i & 7);
      c = ((i >> 3) % (kGemmBK / 4)) * 4;
      v = *reinterpret_cast<const float4*>(raw + raw_kmajor(r, c));
    } else {
      r = i % R;
      c = (i / R) * 4;
      v = make_float4(raw[c * R + r], raw[(c + 1) * R + r], raw[(c + 2) * R + r], raw[(c + 3) * R + r]);
    }
    const float4 h = make_float4(tc::tf32_hi(v.x), tc::tf32_hi(v.y), tc::tf32_hi(v.z), tc::tf32_hi(v.w));
    const int off = tc::blk(r, c, kGemmBK);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

// Splits row r of a landed raw A tile into hi / lo TF32 and stores them to
// this thread's TMEM lane: 32 hi columns at col_hi, 32 lo columns at col_lo.
__device__ __forceinline__ void split_a_row(const float* raw, bool k_outer, int r, uint32_t col_hi,
                                            uint32_t col_lo) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float x[16], hi[16], lo[16];
    if (!k_outer) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(raw + raw_kmajor(r, half * 16 + q * 4));
        x[4 * q] = v.x;
        x[4 * q + 1] = v.y;
        x[4 * q + 2] = v.z;
        x[4 * q + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = raw[(half * 16 + j) * kGemmBM + r];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      hi[j] = tc::tf32_hi(x[j]);
      lo[j] = x[j] - hi[j];
    }
    tc::tmem_st16(col_hi + half * 16, hi);
    tc::tmem_st16(col_lo + half * 16, lo);
  }
  tc::tmem_st_wait();
}

// Bounded wait on an mbarrier phase (`rounds` rounds of four polls) that
// also gives up as soon as another warp of the CTA has flagged a failure.
constexpr uint32_t kWaitRounds = 1u << 22;
__device__ __forceinline__ bool wait_or_failed(uint64_t* bar, uint32_t parity, volatile int* failed,
                                               uint32_t rounds) {
  for (uint32_t i = 0; i < rounds; ++i) {
    if (tc::bar_wait(bar, parity, 4)) return true;
    if (*failed) return false;
  }
  return false;
}

// Named barrier 1 over the worker warps only (the MMA warp never joins it);
// workers_any also ORs a flag over them, so all workers take the same branch.
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kGemmThreads) : "memory"); }
__device__ __forceinline__ bool workers_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kGemmThreads)
      : "memory");
  return r != 0;
}

// Warps 0-7 (workers) stage raw tiles, split them into hi/lo stages and run
// the epilogue; warp 8 issues the MMAs.  Per hi/lo stage st: ready[st] (one
// arrival per worker warp) publishes a split block to the MMA warp, and
// done[st] (tcgen05.commit) hands the stage back once its MMAs completed.
__global__ void __launch_bounds__(kGemmThreads + 32, 1)
    gemm_tf32x3_kernel(GemmOperand A, GemmOperand B, const __grid_constant__ CUtensorMap tma_a,
                       const __grid_constant__ CUtensorMap tma_b, int tma, float* __restrict__ C, int ldc,
                       size_t chunk_stride, int M, int N, int K, int k_chunk, int* __restrict__ err,
                       int lost_block, uint32_t wait_rounds) {
  wait_prior_grids();
  extern __shared__ __align__(1024) float sm[];
  __shared__ uint64_t ready[kGemmStages], done[kGemmStages];
  __shared__ uint64_t full[kGemmRaw];  // TMA completion per raw stage
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  constexpr int kWorkerWarps = kGemmThreads / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * kGemmBN;
  const int kbeg = blockIdx.z * k_chunk, kend = min(K, kbeg + k_chunk);
  const int nb = kend > kbeg ? (kend - kbeg + kGemmBK - 1) / kGemmBK : 0;
  C += blockIdx.z * chunk_stride;  // split-K: this chunk's own partial tile
  // TMEM: the 64-column accumulator, then per stage 32 hi + 32 lo columns of
  // a TMEM-staged A block.
  if (warp == 0) tc::tmem_alloc(&tmem_base, 256);
  if (tid == 0) {
    for (int st = 0; st < kGemmStages; ++st) {
      tc::bar_init(&ready[st], kWorkerWarps);
      tc::bar_init(&done[st], 1);
    }
    for (int st = 0; st < kGemmRaw; ++st) tc::bar_init(&full[st], 1);
    tc::bar_init_fence();
    failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  // Raw tiles start on a 1024-byte boundary (the 128-byte swizzle's period).
  float* raw_base = sm + kGemmStages * kGemmStageFloats;
  raw_base += ((1024u - (tc::smem_addr(raw_base) & 1023u)) & 1023u) / 4;
  volatile int* vfailed = &failed;

  if (warp < kWorkerWarps) {
    const bool vec_a = A.ld % 4 == 0 && (reinterpret_cast<uintptr_t>(A.p) & 15) == 0;
    const bool vec_b = B.ld % 4 == 0 && (reinterpret_cast<uintptr_t>(B.p) & 15) == 0;
    const bool cp_a = !(tma & kTmaA), cp_b = !(tma & kTmaB);
    // Starts the copies of K block i into raw stage i % kGemmRaw: thread 0
    // issues the tensor copies, every worker its cp.async pieces (one commit
    // group per block, empty past the end so the group count stays uniform).
    auto stage = [&](int i) {
      if (i < nb) {
        const int s = i % kGemmRaw;
        float* raw = raw_base + s * kRawFloats;
        const int k0 = kbeg + i * kGemmBK;
        if (tma && tid == 0) {
          const uint32_t bytes =
              ((tma & kTmaA) ? kGemmBM * kGemmBK * 4 : 0) + ((tma & kTmaB) ? kGemmBN * kGemmBK * 4 : 0);
          tc::bar_expect_tx(&full[s], bytes);
          if (tma & kTmaA) tma_load_2d(raw, &tma_a, A.k_outer ? m0 : k0, A.k_outer ? k0 : m0, &full[s]);
          if (tma & kTmaB)
            tma_load_2d(raw + kGemmBM * kGemmBK, &tma_b, B.k_outer ? n0 : k0, B.k_outer ? k0 : n0, &full[s]);
        }
        if (cp_a) stage_raw<kGemmBM>(raw, A, vec_a, m0, M, k0, kend);
        if (cp_b) stage_raw<kGemmBN>(raw + kGemmBM * kGemmBK, B, vec_b, n0, N, k0, kend);
      }
      cp_async_commit();
    };
    uint32_t full_phase = 0, done_phase = 0;  // bit s: parity of the barrier's next completion
    int landed = 0;                           // blocks whose tensor copies have been waited for
    for (int p = 0; p < kGemmRaw; ++p) stage(p);
    for (int i = 0; i < nb; ++i) {
      const int st = i & 1, s = i % kGemmRaw;
      cp_async_wait<kGemmRaw - 1>();  // this thread's pieces of block i have landed
      bool bad = false;
      if (tma) {
        // A wait cut short (own limit, or another warp's failure) leaves
        // block i's copy in flight: it stays with the drain below.
        if (wait_or_failed(&full[s], (full_phase >> s) & 1u, vfailed, wait_rounds)) {
          full_phase ^= 1u << s;
          landed = i + 1;
        } else {
          bad = true;
        }
      }
      // hi/lo stage st was last read by the MMAs of block i - 2.
      if (i >= 2) {
        bad |= !wait_or_failed(&done[st], (done_phase >> st) & 1u, vfailed, wait_rounds);
        done_phase ^= 1u << st;
        tc::fence_after_sync();
      }
      // One decision for all workers (and every worker's cp.async pieces
      // have landed once all have passed this barrier).
      if (workers_any(bad || *vfailed)) {
        failed = 1;
        break;
      }
      const float* raw = raw_base + s * kRawFloats;
      float* Bh = sm + st * kGemmStageFloats;
      float* Bl = Bh + kGemmBN * kGemmBK;
      // Warps 0-3: A row tid into TMEM lane tid (stage st's hi/lo columns);
      // warps 4-7: the B tile into shared hi/lo tiles.
      if (warp < 4)
        split_a_row(raw, A.k_outer, tid, tmem + lane_off + 64 + 64 * st, tmem + lane_off + 96 + 64 * st);
      else
        split_raw<kGemmBN, kGemmThreads / 2>(Bh, Bl, raw + kGemmBM * kGemmBK, B.k_outer, tid - kGemmThreads / 2);
      tc::fence_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      // lost_block (a test hook, -1 in every product launch) withholds warp
      // 0's arrival for that K block, so the MMA warp's wait must give up.
      if (lane == 0 && !(warp == 0 && i == lost_block)) tc::bar_arrive(&ready[st]);
      // Every worker has read raw stage s: refill it with block i + kGemmRaw.
      workers_sync();
      stage(i + kGemmRaw);
    }
    cp_async_wait<0>();
    // After a failure, let the tensor copies still in flight land (bounded)
    // before the shared memory is released.
    if (tma) {
      const int issued = min(nb, landed + kGemmRaw - 1);
      for (int j = landed; j < issued; ++j) {
        const int s = j % kGemmRaw;
        tc::bar_wait(&full[s], (full_phase >> s) & 1u);
        full_phase ^= 1u << s;
      }
    }
  } else {
    // MMA warp: block i's 4 K-steps x 3 MMAs (hi.hi + hi.lo + lo.hi) once its
    // stage is split, committed to done[st]; then the last commit is awaited
    // (it covers every MMA this thread issued) before the epilogue.
    const uint32_t idesc = tc::idesc_tf32(kGemmBM, kGemmBN, false, false);
    uint32_t ready_phase = 0;
    int committed = 0;
    for (int i = 0; lane == 0 && i < nb; ++i) {
      const int st = i & 1;
      if (!wait_or_failed(&ready[st], (ready_phase >> st) & 1u, vfailed, wait_rounds)) {
        failed = 1;
        break;
      }
      ready_phase ^= 1u << st;
      tc::fence_after_sync();
      {
        const float* Bh = sm + st * kGemmStageFloats;
        const float* Bl = Bh + kGemmBN * kGemmBK;
        const uint32_t a0 = tmem + 64 + 64 * st;  // A hi at a0, lo at a0 + 32
#pragma unroll
        for (int s = 0; s < kGemmBK / 8; ++s) {
          const uint64_t bh = tc::desc_kmajor(Bh, kGemmBK, s), bl = tc::desc_kmajor(Bl, kGemmBK, s);
          const uint32_t acc = (i > 0 || s > 0) ? 1u : 0u;
          tc::mma_ts(tmem, a0 + 8 * s, bh, idesc, acc);
          tc::mma_ts(tmem, a0 + 8 * s, bl, idesc, 1u);
          tc::mma_ts(tmem, a0 + 32 + 8 * s, bh, idesc, 1u);
        }
        tc::commit(&done[st]);
      }
      committed = i + 1;
    }
    // The k-th commit on done[st] completes the barrier's phase k (parity k & 1).
    if (committed > 0) {
      const int j = committed - 1;
      if (!tc::bar_wait(&done[j & 1], (uint32_t)(j >> 1) & 1u)) failed = 1;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp < kWorkerWarps && !failed) {
    const int r = m0 + (warp & 3) * 32 + lane;
    const uint32_t lane_base = tmem + lane_off;
    // An empty K range (a trailing chunk) never wrote TMEM: its tile is zero.
    const bool empty = nb == 0;
#pragma unroll
    for (int h = 0; h < kGemmBN / 32; ++h) {
      const int c0 = (warp >> 2) * (kGemmBN / 2) + h * 16;
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
  } else if (tid == 0 && failed) {
    atomicExch(err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

// C[m][n] = sum over chunks (in order) of partial[chunk][m][n].
__global__ void gemm_reduce_chunks(const float* __restrict__ partial, int chunks, int M, int N,
                                   float* __restrict__ C, int ldc) {
  wait_prior_grids();
  const size_t mn = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < mn; i += (size_t)gridDim.x * blockDim.x) {
    float s = partial[i];
    for (int c = 1; c < chunks; ++c) s += partial[(size_t)c * mn + i];
    C[(i / N) * (size_t)ldc + i % N] = s;
  }
}

size_t gemm_smem() {
  return ((size_t)kGemmStages * kGemmStageFloats + (size_t)kGemmRaw * kRawFloats) * sizeof(float) + 1024;
}

// cuTensorMapEncodeTiled from the driver (null if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor map of an operand's (rows x K) matrix with an R x BK box: K-major as
// [rows][K] with the 128-byte swizzle, K-outer as [K][rows] unswizzled.
// False (the kernel then stages with cp.async) when the operand's base or
// row stride is not 16-byte aligned or the driver refuses the map.
bool encode_operand(CUtensorMap* map, const GemmOperand& op, int rows, int K, int R) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr || (reinterpret_cast<uintptr_t>(op.p) & 15) != 0 || op.ld % 4 != 0) return false;
  cuuint64_t dims[2];
  cuuint32_t box[2];
  const cuuint32_t elem[2] = {1, 1};
  if (op.k_outer) {
    dims[0] = (cuuint64_t)rows;
    dims[1] = (cuuint64_t)K;
    box[0] = (cuuint32_t)R;
    box[1] = kGemmBK;
  } else {
    dims[0] = (cuuint64_t)K;
    dims[1] = (cuuint64_t)rows;
    box[0] = kGemmBK;
    box[1] = (cuuint32_t)R;
  }
  const cuuint64_t stride[1] = {(cuuint64_t)op.ld * sizeof(float)};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(op.p), dims, stride, box,
                            elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            op.k_outer ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool encode_rows_map(CUtensorMap* map, const float* p, int rows, int width, int box_rows) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) != 0 || width % 4 != 0) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const cuuint64_t stride[1] = {(cuuint64_t)width * sizeof(float)};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, stride, box, elem,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

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
                 float* partial, int* err, cudaStream_t st, bool a_tmem, int lost_block, uint32_t wait_rounds) {
  (void)a_tmem;  // A is always staged through tensor memory
  const int chunks = gemm_chunks(K, k_chunk);
  const int kc = chunks > 1 ? k_chunk : K;
  require(chunks == 1 || kc % kGemmBK == 0, "split-K chunks must be multiples of 32");
  require(chunks == 1 || partial != nullptr, "split-K needs a partial buffer");
  dim3 grid((M + kGemmBM - 1) / kGemmBM, (N + kGemmBN - 1) / kGemmBN, chunks);
  CUtensorMap ta{}, tb{};
  int tma = 0;
  if (encode_operand(&ta, A, M, K, kGemmBM)) tma |= kTmaA;
  if (encode_operand(&tb, B, N, K, kGemmBN)) tma |= kTmaB;
  if (chunks == 1) {
    gemm_tf32x3_kernel<<<grid, kGemmThreads + 32, gemm_smem(), st>>>(A, B, ta, tb, tma, C, ldc, 0, M, N, K, kc, err,
                                                                lost_block, wait_rounds);
  } else {
    gemm_tf32x3_kernel<<<grid, kGemmThreads + 32, gemm_smem(), st>>>(A, B, ta, tb, tma, partial, N, (size_t)M * N, M, N,
                                                                K, kc, err, lost_block, wait_rounds);
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

// Test hook for the bounded waits: one K-major GEMM whose K block
// `lost_block` is never published to the MMA warp, with waits of
// `wait_rounds` rounds, so every CTA gives up, drains its copies, skips its
// epilogue and sets *d_status.  Not a product path.
extern "C" int mb_test_gemm_lost_arrival(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                                         uint32_t lost_block, uint32_t wait_rounds, int* d_status, void* stream) {
  return mb::guarded([&] {
    mb::need(a, "a");
    mb::need(b, "b");
    mb::need(c, "c");
    mb::need(d_status, "status");
    mb::require(m >= 1 && n >= 1 && k >= 1, "GEMM dimensions must be positive");
    mb::require(lost_block < (k + 31) / 32, "lost_block must name one of the K blocks");
    mb::require(wait_rounds >= 1 && wait_rounds <= mb::kWaitRounds, "wait_rounds must be in 1..2^22");
    mb::gemm_prepare();
    const mb::GemmOperand A{a, (int)k, false};
    const mb::GemmOperand B{b, (int)k, false};
    mb::launch_gemm(A, B, c, (int)n, (int)m, (int)n, (int)k, 0, nullptr, d_status, (cudaStream_t)stream, false,
                    (int)lost_block, wait_rounds);
  });
}
