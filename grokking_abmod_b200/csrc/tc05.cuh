// Blackwell (sm_100a) tensor-core building blocks: tcgen05.mma with TF32
// operands, TMEM allocation / loads / stores, mbarrier waits with bounded
// spins, and the shared-memory operand layout they consume.
//
// FP32 accuracy from TF32 tensor cores ("3xTF32"): each FP32 operand x is
// split into hi = rna_tf32(x) and lo = x - hi (exact in FP32), and a product
// a.b is accumulated as hi_a.hi_b + hi_a.lo_b + lo_a.hi_b in FP32 (TMEM).
// The dropped lo_a.lo_b term and TF32 truncation of lo leave a relative error
// near 2^-21 per product, the level of FP32 accumulation itself.
//
// Operand tiles live in shared memory without swizzling, blocked into 8 x 4
// "core matrices" of 128 contiguous bytes: element (r, c) of an R x C tile is
// at float offset ((r / 8) * (C / 4) + c / 4) * 32 + (r % 8) * 4 + c % 4.
// Tiles are K-major operands (rows = M or N, columns = K); fields per the PTX
// ISA tcgen05 shared memory descriptor (CUTLASS cute/arch/mma_sm100_desc.hpp
// documents them).  TF32 operands are never given MN-major: measured on this
// sm_100a pool, a TF32 MMA with the transpose bit set for B reads zeros, so a
// TF32 operand needed with its rows along N is stored transposed instead.
// FP16 B operands may be MN-major (desc_mn16), which lets one FP16 tile
// serve both as the K-major B of one product and the MN-major B of another.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {
namespace tc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Float offset of element (r, c) in a blocked tile with C columns.
__device__ __forceinline__ int blk(int r, int c, int C) { return ((r >> 3) * (C >> 2) + (c >> 2)) * 32 + (r & 7) * 4 + (c & 3); }

// Shared-memory matrix descriptor, no swizzle, sm_100 version field = 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// K-major operand: rows = M (or N), K along columns.  Step s covers K
// columns [8s, 8s+8) (two core matrices, 128 B apart).
__device__ __forceinline__ uint64_t desc_kmajor(const float* tile, int C, int s) {
  return sdesc(smem_addr(tile) + (uint32_t)s * 256u, 128u, (uint32_t)(C / 4) * 128u);
}


// Instruction descriptor: FP32 accumulator, TF32 A and B, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (TMEM) (+)= A (smem) * B (smem)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

// D (TMEM) (+)= A (TMEM, K-major, lane = row) * B (smem)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Arrives on the mbarrier once every tcgen05 operation this thread issued so
// far has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes become visible to the tensor cores.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Arrival that also announces `bytes` of bulk-copy transactions to wait for.
__device__ __forceinline__ void bar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// Bulk (non-tensor, non-multicast) copy global -> this CTA's shared memory,
// completing `bytes` transactions on the mbarrier.  Both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// One arrival (release semantics) on an mbarrier.
__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Waits for the mbarrier phase with the given parity.  Gives up after
// `limit` polls (returns false) so a lost arrival can never hang the GPU.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity, uint32_t limit = (1u << 24)) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// TMEM allocation by one full warp; the base address lands in *dst (smem).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// Loads of this thread's TMEM lane (warp w reads lanes 32w..32w+31; the
// caller adds (32w) << 16 to the address).  tcgen05.ld is asynchronous: its
// destination registers are valid only after tcgen05.wait::ld, so each load
// and its wait form one asm statement and the compiler never reads the
// registers early.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive columns, load and wait in one statement.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 16-column loads (e.g. S and dP of the same lane) behind one wait, so
// their round trips overlap.
__device__ __forceinline__ void tmem_ld16_pair(uint32_t ta, float (&a)[16], uint32_t tb, float (&b)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    a[i] = __uint_as_float(r[i]);
    b[i] = __uint_as_float(r[16 + i]);
  }
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TF32 hi part (round to nearest, ties away from zero) of a finite FP32
// value: adding half a TF32 ulp (bit 12) to the magnitude bits and clearing
// the 13 dropped bits is exactly cvt.rna.tf32.f32 for every finite input
// (carries into the exponent round up a binade; the sign bit is untouched).
// Integer ALU work instead of a conversion on the XU pipe, which the softmax
// loops already load with ex2.
__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// ---------------------------------------------------------------- f16 forms
// Three-term FP16 products ("3xF16"): a finite FP32 value x, first scaled by
// a power of two s that puts the operand's largest magnitude near 2^13, is
// split into hi = FP16(x s) and lo = FP16(x s - hi); a product
// is accumulated as hi.hi + hi.lo + lo.hi in FP32 (TMEM) on kind::f16 MMAs,
// which run at twice the kind::tf32 rate.  The relative error per product is
// near 2^-21 as with 3xTF32; the scaling keeps hi within FP16's range, and
// magnitudes below 2^-16 of the operand's largest lose low bits of lo only,
// an absolute error near 2^-38 of that largest magnitude.
//
// FP16 operand tiles use the same unswizzled blocked layout with 8 x 8 core
// matrices of 128 contiguous bytes: half-element (r, c) of an R x C tile is
// at half offset ((r / 8) * (C / 8) + c / 8) * 64 + (r % 8) * 8 + c % 8; a K
// step of 16 elements is again two core matrices 128 B apart.  In tensor
// memory an FP16 A operand packs two consecutive K elements per 32-bit
// column (the lower index in the low half), so K step s reads columns
// [8s, 8s + 8).
__device__ __forceinline__ int blk16(int r, int c, int C) {
  return ((r >> 3) * (C >> 3) + (c >> 3)) * 64 + (r & 7) * 8 + (c & 7);
}

// K-major FP16 operand with C columns (half elements); step s covers K
// columns [16s, 16s + 16).
__device__ __forceinline__ uint64_t desc_kmajor16(const void* tile, int C, int s) {
  return sdesc(smem_addr(tile) + (uint32_t)s * 256u, 128u, (uint32_t)(C / 8) * 128u);
}

// MN-major FP16 B operand read from a blocked tile whose rows run along K
// and whose C columns run along N (the bytes of the K-major tile of the
// transposed product): K step s covers tile rows [16s, 16s + 16).  LBO is
// the stride between 8-row groups along K, SBO the stride between 8-column
// groups along N (checked against a CPU product on sm_100a, kind::f16).
__device__ __forceinline__ uint64_t desc_mn16(const void* tile, int C, int s) {
  const uint32_t kgroup = (uint32_t)(C / 8) * 128u;
  return sdesc(smem_addr(tile) + (uint32_t)s * 2u * kgroup, kgroup, 128u);
}

// Instruction descriptor: FP32 accumulator, FP16 A and B, M x N, A K-major,
// B K-major or (b_mn) MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn = false) {
  return (1u << 4) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (TMEM) (+)= A (TMEM, FP16 pairs, lane = row) * B (smem, FP16)
__device__ __forceinline__ void mma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

// D (TMEM) (+)= A (smem, FP16) * B (smem, FP16)
__device__ __forceinline__ void mma_ss_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

// The power of two 2^(13 - e), 2^(e-1) <= max_abs < 2^e: scales an operand
// whose largest magnitude is max_abs into [2^12, 2^13).  1 for an all-zero
// operand; clamped so that the scale and its inverse stay normal FP32.
__device__ __forceinline__ float f16_scale(float max_abs) {
  if (!(max_abs > 0.f)) return 1.0f;
  int e;
  frexpf(max_abs, &e);  // max_abs = m 2^e, 0.5 <= m < 1
  int k = 13 - e;
  k = k > 120 ? 120 : (k < -120 ? -120 : k);
  return __int_as_float((k + 127) << 23);
}

// hi/lo FP16 parts of x (already scaled) packed with those of y: the pair
// (x, y) in one 32-bit word each, x in the low half.  lo is taken from the
// FP16 hi itself (x - hi is exact in FP32), so subnormal hi parts stay exact.
__device__ __forceinline__ void split_f16x2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

}  // namespace tc
}  // namespace mb
