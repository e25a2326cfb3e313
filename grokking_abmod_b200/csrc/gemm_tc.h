// Host interface of the tcgen05 3xTF32 GEMM (gemm_tc.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace mb {

// First statement of every grok-simple and GEMM kernel: waits until the
// grids this one depends on through a programmatic graph edge have completed
// and their writes are visible (PTX griddepcontrol.wait).  A kernel launched
// without such an edge returns from it at once.
__device__ __forceinline__ void wait_prior_grids() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// One GEMM operand of `rows` (M or N) x K: element (r, k) is p[r * ld + k]
// (K-major) or, with k_outer, p[k * ld + r].
struct GemmOperand {
  const float* p;
  int ld;
  bool k_outer;
};

// Sets the kernel's shared-memory limit; call once per device before the
// first launch (and before any stream capture).
void gemm_prepare();
// C[M][N] (row stride ldc) = A . B^T over K.  k_chunk > 0 and < K splits K
// into chunks of that many (a multiple of 32) with partial tiles in
// `partial` (gemm_partial_floats floats) summed in chunk order.  `err` is a
// device flag set if an mbarrier wait gave up.  A is always staged through
// tensor memory; `a_tmem` is accepted for callers that ask for it.
// lost_block and wait_rounds are the bounded-wait test hook of
// mb_test_gemm_lost_arrival; every product call keeps the defaults.
void launch_gemm(const GemmOperand& A, const GemmOperand& B, float* C, int ldc, int M, int N, int K, int k_chunk,
                 float* partial, int* err, cudaStream_t st, bool a_tmem = false, int lost_block = -1,
                 uint32_t wait_rounds = 1u << 22);
int gemm_chunks(int K, int k_chunk);
size_t gemm_partial_floats(int M, int N, int K, int k_chunk);
// Kernel launches of one launch_gemm call.
int gemm_launches(int K, int k_chunk);

// TMA map of a row-major [rows][width] FP32 tensor whose boxes are box_rows
// rows x 32 columns (128 bytes) with the 128-byte swizzle: 16-byte piece c of
// box row r lands at piece c ^ (r % 8).  False when the base or the row
// stride is not 16-byte aligned or the driver refuses the map.
bool encode_rows_map(CUtensorMap* map, const float* p, int rows, int width, int box_rows);

}  // namespace mb
