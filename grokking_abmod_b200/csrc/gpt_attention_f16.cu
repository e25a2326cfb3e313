// Causal flash attention on the sm_100a tensor cores with three-term FP16
// products (tcgen05 kind::f16, "3xF16"; tc05.cuh): softmax(Q K^T / sqrt(hd)) V
// with a causal, same-sequence mask over the flattened token rows, base-2
// LSE, and dQ and dK/dV as separate kernels (no atomics, bitwise
// reproducible) - the semantics and statistics of the reference's FA2
// kernels (src/gpt/gpu.rs:381-750) and of gpt_attention.cu's FP32 SIMT
// kernels, at FP32-level accuracy with twice the MMA rate of 3xTF32.
//
// Scaling.  FP16 holds magnitudes in [2^-24, 65504], so every operand is
// scaled by a power of two before it is split, and the scale is divided out
// of the FP32 result exactly:
//  * Q: per query row (the thread that owns the row splits it into TMEM);
//  * K and V: per 64-key tile, chosen by the format pass and stored in the
//    tile's header; a score is S_tmem / (s_q(row) s_k(tile));
//  * P (the unnormalised probabilities, at most 2^8 under the lazy rescale)
//    is stored as P c_j with c_j = C / s_v(j), C = 2^7 min_j s_v(j) over the
//    CTA's key tiles, so every step's P.V product carries the same factor C
//    and O = O_tmem / (C L).  c_j <= 2^7 keeps P c_j <= 2^15; a tile whose
//    values are smaller than the largest by more than 2^7 has c_j < 1, which
//    costs precision only in products far below the accumulated magnitude.
//
// Roles (every CTA): compute warps (8 in the forward, 16 in dQ and dK/dV;
// thread i owns TMEM lane / row i % 128 and one column slice of each step), a
// producer thread that streams operand tiles into shared-memory rings with
// cp.async.bulk (plain, no multicast; completion counted on mbarriers), and
// two MMA issuer threads in separate warps, each committing its own MMAs to
// mbarriers, so one issuer's waits overlap the other's MMAs.  All waits are
// bounded and report through `err` instead of hanging.  Operand tiles are
// written once per use by format passes in the unswizzled FP16 blocked
// layout of tc05.cuh, [64 rows][HD]: the same tile is the K-major B operand
// of one product (Q K^T) and the MN-major B operand of another (P V).  The
// CTA's own 128 rows move between global memory and TMEM through shared
// memory with coalesced accesses.  CTAs are ordered by causal work, longest
// first.

#include <cuda.h>

#include "common.cuh"
#include "tc05.cuh"

namespace mb {

constexpr int kTcRows = 128;     // CTA tile rows = TMEM lanes
constexpr int kTcK = 64;         // key-tile rows (forward, dQ)
constexpr int kTcQ = 64;         // query-tile rows (dK/dV)
// Forward: 8 compute warps (row = tid % 128, column half = tid / 128), a
// producer warp (thread 256), two MMA issuers in separate warps (threads 288
// and 320) and a loader warp (352).
constexpr int kTcCompute = 256, kTcProducer = 256, kTcIssuer = 288, kTcIssuer2 = 320;
// dQ and dK/dV: 16 compute warps (row = tid % 128, 16-column block of a step
// = tid / 128), a producer warp (thread 512), two issuers (544, 576) and a
// loader warp (608).
constexpr int kKvCompute = 512, kKvProducer = 512, kKvIssuer = 544, kKvIssuer2 = 576;

constexpr int kFmtThreads = 256;  // threads of the format kernels

// Rows [row0, row0 + R) of head h of two row-major [rows][W] tensors into
// shared memory ([R][HD], stride HD + 2), zero past the last row.  Every
// load of the thread is issued before the first store, so a CTA keeps all
// of its 2 R HD floats in flight.
template <int R, int HD>
__device__ __forceinline__ void load_rows2(float* xa, const float* __restrict__ ga, float* xb,
                                           const float* __restrict__ gb, int row0, int rows, int W, int h) {
  constexpr int XS = HD + 2, PER = R * HD / 4 / kFmtThreads;
  static_assert(PER * kFmtThreads * 4 == R * HD, "tile must split evenly over the threads");
  float4 va[PER], vb[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = threadIdx.x + kFmtThreads * j, r = i / (HD / 4), c = (i % (HD / 4)) * 4, row = row0 + r;
    const size_t off = (size_t)row * W + h * HD + c;
    va[j] = row < rows ? __ldg(reinterpret_cast<const float4*>(ga + off)) : make_float4(0.f, 0.f, 0.f, 0.f);
    vb[j] = row < rows ? __ldg(reinterpret_cast<const float4*>(gb + off)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = threadIdx.x + kFmtThreads * j, r = i / (HD / 4), c = (i % (HD / 4)) * 4;
    float* a = xa + r * XS + c;
    float* b = xb + r * XS + c;
    a[0] = va[j].x, a[1] = va[j].y, a[2] = va[j].z, a[3] = va[j].w;
    b[0] = vb[j].x, b[1] = vb[j].y, b[2] = vb[j].z, b[3] = vb[j].w;
  }
}

// The 128-row tile CTA b works on, ordered by causal work (most first) so the
// last wave of the grid holds the shortest CTAs.  With sequences made of
// whole tiles, all sequences' tiles at one position come together; a query
// tile's work grows with its position (more keys before it), a key tile's
// shrinks (fewer queries after it).  Other shapes keep a plain order.
__device__ __forceinline__ int tile_by_work(int b, int nt, int rows, int T, bool queries) {
  if (T % kTcRows != 0 || rows % T != 0) return queries ? nt - 1 - b : b;
  const int per_seq = T / kTcRows, nseq = nt / per_seq;
  const int i = b / nseq, seq = b % nseq;
  return seq * per_seq + (queries ? per_seq - 1 - i : i);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


struct TcShared {
  uint32_t tmem_base;
  int failed;
};


// Inside a role loop: a wait that gives up marks the CTA failed and leaves.
#define F16_WAIT_OR_FAIL(bar, parity)    \
  if (!tc::bar_wait((bar), (parity))) {  \
    sh.failed = 1;                       \
    break;                               \
  }

template <int HD>
struct F16Fmt {
  static constexpr int PART_BYTES = kTcK * HD * 2;  // one 64 x HD FP16 part
  static constexpr int HEADER_BYTES = 128;          // scales (and room to keep tiles 128-byte aligned)
  static constexpr int KTILE_BYTES = 4 * PART_BYTES + HEADER_BYTES;
  // parts: K, K', V, V' ([64 keys][HD] each; K-major B operands of Q K^T and
  // dO V^T, MN-major B operands of P V and dS K); header floats: s_k, s_v,
  // the largest row norm of V, the largest |V|
  static constexpr int K_HI = 0, V_HI = 2, HEADER_OFF = 4 * PART_BYTES;
};

constexpr int kMaxKeyTiles = 72;  // key tiles one query CTA visits: (4096 + 128) / 64 + 2

// Writes the FP16 hi/lo parts p, p + 1 of one operand tile in the blocked
// layout ([R rows][HD columns]) from a shared-memory copy x ([R][HD], row
// stride HD + 2), scaled by `scale`.  Each thread writes whole 16-byte
// core-matrix rows, contiguous across a warp.
template <int R, int HD>
__device__ __forceinline__ void store_parts16(uint8_t* __restrict__ tile, int p, const float* x, float scale) {
  constexpr int XS = HD + 2, PB = F16Fmt<HD>::PART_BYTES;
  uint4* hi = reinterpret_cast<uint4*>(tile + (size_t)p * PB);
  uint4* lo = reinterpret_cast<uint4*>(tile + (size_t)(p + 1) * PB);
  for (int q = threadIdx.x; q < R * HD / 8; q += kFmtThreads) {
    const int rl = q & 7, c8 = (q >> 3) % (HD / 8), rg = (q >> 3) / (HD / 8);
    const int r = rg * 8 + rl, c = c8 * 8;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = x[r * XS + c + e] * scale;
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) tc::split_f16x2(v[2 * e], v[2 * e + 1], h[e], l[e]);
    hi[q] = make_uint4(h[0], h[1], h[2], h[3]);
    lo[q] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// Key tiles of K and V in FP16 parts with their scales: grid
// (ceil(rows/64), H), kFmtThreads threads.
template <int HD>
__global__ void __launch_bounds__(kFmtThreads) attention_format_keys_f16(int rows, int W, const float* __restrict__ k,
                                                                   const float* __restrict__ v,
                                                                   uint8_t* __restrict__ fmt) {
  using F = F16Fmt<HD>;
  constexpr int XS = HD + 2, NW = kFmtThreads / 32;
  __shared__ float xk[kTcK * XS], xv[kTcK * XS];
  __shared__ float red[3][NW];
  const int t = blockIdx.x, h = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t* tile = fmt + ((size_t)h * gridDim.x + t) * F::KTILE_BYTES;
  load_rows2<kTcK, HD>(xk, k, xv, v, t * kTcK, rows, W, h);
  __syncthreads();
  float mk = 0.f, mv = 0.f, nv = 0.f;
  for (int i = threadIdx.x; i < kTcK * HD; i += kFmtThreads) {
    const int r = i / HD, c = i % HD;
    mk = fmaxf(mk, fabsf(xk[r * XS + c]));
    mv = fmaxf(mv, fabsf(xv[r * XS + c]));
  }
  if (threadIdx.x < kTcK) {
    float s = 0.f;
    for (int c = 0; c < HD; ++c) s += xv[threadIdx.x * XS + c] * xv[threadIdx.x * XS + c];
    nv = sqrtf(s);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
    mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
    nv = fmaxf(nv, __shfl_xor_sync(0xffffffffu, nv, o));
  }
  if (lane == 0) {
    red[0][warp] = mk;
    red[1][warp] = mv;
    red[2][warp] = nv;
  }
  __syncthreads();
  mk = mv = nv = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    mk = fmaxf(mk, red[0][w]);
    mv = fmaxf(mv, red[1][w]);
    nv = fmaxf(nv, red[2][w]);
  }
  const float sk = tc::f16_scale(mk), sv = tc::f16_scale(mv);
  store_parts16<kTcK, HD>(tile, F::K_HI, xk, sk);
  store_parts16<kTcK, HD>(tile, F::V_HI, xv, sv);
  if (threadIdx.x == 0) *reinterpret_cast<float4*>(tile + F::HEADER_OFF) = make_float4(sk, sv, nv, mv);
}

// Named barrier ID over NT threads.
template <int ID, int NT>
__device__ __forceinline__ void named_sync() {
  asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(NT) : "memory");
}

// D (+)= A . B^T with A = FP16 hi/lo TMEM columns and B a K-major FP16 hi/lo
// shared tile with KC columns, over K steps [s0, s0 + NSTEP) of 16 elements:
// three MMAs per step.
// MN: B is MN-major and C is the tile's column count (N) instead of its K
// column count.
template <int C, int NSTEP, bool MN = false>
__device__ __forceinline__ void mma16_tmem_a(uint32_t d, uint32_t ah, uint32_t al, const void* bh, const void* bl,
                                             uint32_t idesc, bool accumulate, int s0) {
#pragma unroll
  for (int i = 0; i < NSTEP; ++i) {
    const int s = s0 + i;
    const uint64_t b_h = MN ? tc::desc_mn16(bh, C, s) : tc::desc_kmajor16(bh, C, s);
    const uint64_t b_l = MN ? tc::desc_mn16(bl, C, s) : tc::desc_kmajor16(bl, C, s);
    tc::mma_ts_f16(d, ah + 8 * s, b_h, idesc, (accumulate || i > 0) ? 1u : 0u);
    tc::mma_ts_f16(d, ah + 8 * s, b_l, idesc, 1u);
    tc::mma_ts_f16(d, al + 8 * s, b_h, idesc, 1u);
  }
}

// NC values scaled by `scale`, split into FP16 hi/lo pairs and stored to
// NC / 2 packed TMEM columns each.
template <int NC>
__device__ __forceinline__ void tc_st_split16(uint32_t thi, uint32_t tlo, const float* v, float scale) {
#pragma unroll
  for (int c = 0; c < NC; c += 32) {
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) tc::split_f16x2(v[c + 2 * e] * scale, v[c + 2 * e + 1] * scale, hi[e], lo[e]);
    tc::tmem_st16u(thi + c / 2, hi);
    tc::tmem_st16u(tlo + c / 2, lo);
  }
}

// D (+)= A . B^T over K steps [s0, s0 + NSTEP) of 16 elements with A's FP16
// hi and lo parts interleaved in TMEM: step s reads hi columns [16s, 16s + 8)
// and lo columns [16s + 8, 16s + 16) of `a`.  B is MN-major (tc05.cuh
// desc_mn16) from a tile with NC columns along N.
template <int NC, int NSTEP>
__device__ __forceinline__ void mma16_tmem_a_il(uint32_t d, uint32_t a, const void* bh, const void* bl,
                                                uint32_t idesc, bool accumulate, int s0) {
#pragma unroll
  for (int i = 0; i < NSTEP; ++i) {
    const int s = s0 + i;
    const uint64_t b_h = tc::desc_mn16(bh, NC, s), b_l = tc::desc_mn16(bl, NC, s);
    tc::mma_ts_f16(d, a + 16 * s, b_h, idesc, (accumulate || i > 0) ? 1u : 0u);
    tc::mma_ts_f16(d, a + 16 * s, b_l, idesc, 1u);
    tc::mma_ts_f16(d, a + 16 * s + 8, b_h, idesc, 1u);
  }
}

// ------------------------------------------------------------------- dK/dV
// Query tiles in FP16 parts: Q, Q', dO, dO' ([64 queries][HD] each) and a header with the 64 rows' LSE and delta, the tile's scales
// s_q and s_do, its largest dO row norm and its largest |delta|.
template <int HD>
struct F16Q {
  static constexpr int PART_BYTES = kTcQ * HD * 2;
  static constexpr int HEADER_BYTES = 1024;
  static constexpr int QTILE_BYTES = 4 * PART_BYTES + HEADER_BYTES;
  static constexpr int Q_HI = 0, D_HI = 2, HEADER_OFF = 4 * PART_BYTES;
  static constexpr int LSE = 0, DELTA = kTcQ, SCALES = 2 * kTcQ;  // header floats
};

// Query tiles of Q and dO with LSE and delta: grid (ceil(rows/64), H).
template <int HD>
__global__ void __launch_bounds__(kFmtThreads) attention_format_queries_f16(int rows, int W, const float* __restrict__ q,
                                                                      const float* __restrict__ dout,
                                                                      const float* __restrict__ lse2,
                                                                      const float* __restrict__ delta,
                                                                      uint8_t* __restrict__ fmt) {
  using G = F16Q<HD>;
  constexpr int XS = HD + 2, NW = kFmtThreads / 32;
  __shared__ float xq[kTcQ * XS], xd[kTcQ * XS];
  __shared__ float red[4][NW];
  const int t = blockIdx.x, h = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t* tile = fmt + ((size_t)h * gridDim.x + t) * G::QTILE_BYTES;
  float* hdr = reinterpret_cast<float*>(tile + G::HEADER_OFF);
  load_rows2<kTcQ, HD>(xq, q, xd, dout, t * kTcQ, rows, W, h);
  __syncthreads();
  float mq = 0.f, md = 0.f, nd = 0.f, mdl = 0.f;
  for (int i = threadIdx.x; i < kTcQ * HD; i += kFmtThreads) {
    const int r = i / HD, c = i % HD;
    mq = fmaxf(mq, fabsf(xq[r * XS + c]));
    md = fmaxf(md, fabsf(xd[r * XS + c]));
  }
  if (threadIdx.x < kTcQ) {
    const int row = t * kTcQ + threadIdx.x;
    float ss = 0.f;
    for (int c = 0; c < HD; ++c) ss += xd[threadIdx.x * XS + c] * xd[threadIdx.x * XS + c];
    nd = sqrtf(ss);
    const float L = row < rows ? lse2[(size_t)h * rows + row] : 0.f;
    const float dl = row < rows ? delta[(size_t)h * rows + row] : 0.f;
    hdr[G::LSE + threadIdx.x] = L;
    hdr[G::DELTA + threadIdx.x] = dl;
    mdl = fabsf(dl);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
    md = fmaxf(md, __shfl_xor_sync(0xffffffffu, md, o));
    nd = fmaxf(nd, __shfl_xor_sync(0xffffffffu, nd, o));
    mdl = fmaxf(mdl, __shfl_xor_sync(0xffffffffu, mdl, o));
  }
  if (lane == 0) {
    red[0][warp] = mq;
    red[1][warp] = md;
    red[2][warp] = nd;
    red[3][warp] = mdl;
  }
  __syncthreads();
  mq = md = nd = mdl = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    mq = fmaxf(mq, red[0][w]);
    md = fmaxf(md, red[1][w]);
    nd = fmaxf(nd, red[2][w]);
    mdl = fmaxf(mdl, red[3][w]);
  }
  const float sq = tc::f16_scale(mq), sd = tc::f16_scale(md);
  store_parts16<kTcQ, HD>(tile, G::Q_HI, xq, sq);
  store_parts16<kTcQ, HD>(tile, G::D_HI, xd, sd);
  if (threadIdx.x == 0) *reinterpret_cast<float4*>(hdr + G::SCALES) = make_float4(sq, sd, nd, mdl);
}

// Persistent dK/dV: each CTA (one per SM) walks a fixed list of key tiles
// (128 keys of one head; the grid-wide order puts the longest causal work
// first and deals it to the CTAs in snake order) and, for each, their
// queries 64 at a time through a ring of query tiles that runs on across key
// tiles.  K and V sit in TMEM split into FP16 hi/lo columns with per-row
// scales; dV and dK accumulate in TMEM; S^T/dP^T are double-buffered.
// Per step i (buffer b = i & 1, i counted over the CTA's whole list):
// threads 544 and 512 issue S^T = K Q^T and dP^T = V dO^T (keys on lanes,
// N = 64 queries); all 16 compute warps (thread (row, quarter) owns query
// columns [16 quarter, +16)) form P^T = exp2(S^T scale - lse) and store it
// over the S^T columns they have read (FP16 hi/lo interleaved), then
// dS^T = P^T (dP^T - delta) scale over the dP^T columns; thread 576 issues
// dV += P^T dO and dK += dS^T Q.  Thread 512 also streams the query tiles.
// The MMAs come from three warps because a warp issues at most one MMA per
// ~48 cycles (~100 beside busy compute warps), while the tensor pipe
// finishes an N = 64 MMA in 32: a single issuing warp would set the pace.
// A loader warp (608) works one key tile ahead in a shared staging area: it
// reads the scales of the next tile's query tiles and brings its FP32 K and
// V rows in with TMA box copies; after a key tile it writes the tile's dK
// and dV out of the staging area with TMA box stores (dV as a TMA reduce-add
// onto the XSA term when that is given).  Between two key tiles compute
// warps 0-7 split the staged K and V rows into TMEM (once the last S^T/dP^T
// of the previous tile have been read) and release the issuer, while warps
// 8-15 move the previous tile's dK and dV from TMEM into the staging area.
// Scales: K rows s_K(k), V rows s_V(k); query tiles s_q(i), s_do(i).  P^T is
// stored as P c_i, c_i = 2^13 min_i s_do / s_do(i) (P <= 1), so
// dV = dV_tmem / (2^13 min_i s_do); dS^T as dS r(k) min_i s_q / s_q(i) with
// r(k) = f16_scale((max|dO_q| |V_k| + max|delta|) scale), a bound on
// |dS_k.|, so dK = dK_tmem / (r(k) min_i s_q); minima and maxima run over
// the key tile's query tiles.
// TMEM: K hi | K lo | V hi | V lo (32 each) | dV | dK (64 each) |
// S^T0 | dP^T0 | S^T1 | dP^T1 (64 each) = 512.
constexpr int kBoxBytes = kTcRows * 32 * 4;  // a TMA box: 128 rows x 32 FP32 columns

template <int HD>
struct F16Kv {
  using G = F16Q<HD>;
  static constexpr int STAGES = 4;
  // Staging: the K (t = 0) and V (t = 1) rows of a key tile on the way in,
  // its dK and dV rows on the way out, as TMA boxes of 128 rows x 32 FP32
  // columns with the 128-byte swizzle (1024-byte aligned; one slack KB).
  static constexpr int BOX_BYTES = kBoxBytes;
  static constexpr size_t STAGING_OFF = (size_t)STAGES * G::QTILE_BYTES;
  static constexpr size_t smem = STAGING_OFF + 2 * (HD / 32) * (size_t)BOX_BYTES + 1024;
};

// Float4 chunk c of staged row r of tensor t (0: K/dK, 1: V/dV): box
// (t, c / 8), 16-byte piece (c % 8) ^ (r % 8) of the box's 128-byte row r.
template <int HD>
__device__ __forceinline__ float4* staged_chunk(uint8_t* staging, int t, int r, int c) {
  return reinterpret_cast<float4*>(staging + (t * (HD / 32) + (c >> 3)) * kBoxBytes + r * 128 +
                                   (((c & 7) ^ (r & 7)) << 4));
}

// TMA tensor copies of one 2D box (x: first column, a multiple of 32 FP32
// columns, so every copy starts 16-byte aligned; y: first row >= 0).
__device__ __forceinline__ void tma_load_box(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(tc::smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_box(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(tc::smem_addr(src))
               : "memory");
}
// global += box, element-wise (one addition per element: exact order-free).
__device__ __forceinline__ void tma_add_box(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(tc::smem_addr(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Threads of the persistent dK/dV kernel: 16 compute warps, then one warp
// each for the query-tile producer, the two issuers and the key-row loader.
constexpr int kKvLoader = 608, kKvThreadsP = 640;

// Key tile `item` of the grid-wide work list: its first key and head.
__device__ __forceinline__ void kv_item(int item, int rows, int T, int H, int& k0, int& h) {
  const int nt = (rows + kTcRows - 1) / kTcRows;
  h = item % H;
  k0 = tile_by_work(item / H, nt, rows, T, false) * kTcRows;
}

// The CTA's k-th work item in snake order over a grid of G CTAs (-1: none).
__device__ __forceinline__ int snake_item(int k, int G, int items) {
  const int g = k * G + ((k & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
  return g < items ? g : -1;
}

// Query steps of the key tile starting at k0: its keys' sequences to the end.
__device__ __forceinline__ int kv_steps(int k0, int rows, int T) {
  const int last = min(rows, k0 + kTcRows) - 1;
  const int qend = min(rows, (last / T + 1) * T);
  return (qend - k0 + kTcQ - 1) / kTcQ;
}

template <int HD>
__global__ void __launch_bounds__(kKvThreadsP, 1)
    attention_backward_dkdv_f16(int rows, int T, int H, float scale, const __grid_constant__ CUtensorMap map_k,
                                const __grid_constant__ CUtensorMap map_v, const uint8_t* __restrict__ qfmt,
                                const __grid_constant__ CUtensorMap map_dk, const __grid_constant__ CUtensorMap map_dv,
                                int dv_add, int* __restrict__ err) {
  using G = F16Q<HD>;
  using KV = F16Kv<HD>;
  constexpr int NS = KV::STAGES;
  extern __shared__ __align__(128) uint8_t sm8[];
  __shared__ uint64_t q_full[NS], q_empty[NS], s_full[2], dp_full[2], p_full[2], ds_full[2][2], dv_done[2],
      dk_done[2];
  __shared__ uint64_t staged, kv_ready, drained;
  __shared__ TcShared sh;
  __shared__ float kscale[2][kTcRows], vscale[2][kTcRows], vnorm[2][kTcRows];  // by item parity
  __shared__ float2 tscale[2][kMaxKeyTiles];  // (s_q, s_do) of each query tile of a key tile, by item parity
  __shared__ float4 tmin[2];                  // (min s_q, min s_do, max dO row norm, max |delta|), by item parity
  const int tid = threadIdx.x, warp = tid >> 5;
  const int items = ((rows + kTcRows - 1) / kTcRows) * H;
  const int nqt = (rows + kTcQ - 1) / kTcQ;
  uint8_t* staging = sm8 + KV::STAGING_OFF;
  staging += (1024u - (tc::smem_addr(staging) & 1023u)) & 1023u;  // the swizzle's period
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, 512);
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) {
      tc::bar_init(&q_full[b], 1);
      tc::bar_init(&q_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&s_full[b], 1);
      tc::bar_init(&dp_full[b], 1);
      tc::bar_init(&p_full[b], kKvCompute);
      tc::bar_init(&ds_full[b][0], kKvCompute / 2);
      tc::bar_init(&ds_full[b][1], kKvCompute / 2);
      tc::bar_init(&dv_done[b], 1);
      tc::bar_init(&dk_done[b], 1);
    }
    tc::bar_init(&staged, 1);
    tc::bar_init(&kv_ready, kKvCompute);
    tc::bar_init(&drained, kKvCompute);
    tc::bar_init_fence();
    sh.failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t t0 = sh.tmem_base;
  const uint32_t tKh = t0, tKl = t0 + 32, tVh = t0 + 64, tVl = t0 + 96, tdV = t0 + 128, tdK = t0 + 192,
                 tS = t0 + 256;  // buffer b: S^T at tS + 128 b, dP^T at tS + 128 b + 64
  // A wait that gives up marks the CTA failed; once failed, waits return
  // at once, so every role runs its loops to the end (the compute warps'
  // named barriers stay matched) and the kernel leaves quickly.
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (sh.failed) return false;
    if (tc::bar_wait(bar, parity)) return true;
    sh.failed = 1;
    return false;
  };

  if (tid < kKvCompute) {
    // ---------------------------------------------------------- compute warps
    const int row = tid & (kTcRows - 1), quarter = tid >> 7;
    const int col = 16 * quarter;  // query columns [col, col + 16) of each step
    const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
    int it = 0;                    // steps so far over the CTA's list
    float p_ov = 0.f, p_ok = 0.f;  // output scales of the previous key tile
    // Warps 8-15 carry the previous key tile's dK (warps 8-11) or dV
    // (warps 12-15) rows from TMEM into staging, where the loader writes them
    // out: the first half of each row waits in registers while warps 0-7
    // still read the staged K and V rows.  Warp-uniform waits: the TMEM loads
    // are .aligned.
    const int half8 = (warp >> 2) & 1;  // for warps 8-15: 0 = dK, 1 = dV
    const uint32_t dsrc = (half8 ? tdV : tdK) + lane;
    float g[HD / 2];  // the first half of the row until staging is free
    auto drain_load = [&]() {
      uint64_t* done = half8 ? &dv_done[(it - 1) & 1] : &dk_done[(it - 1) & 1];
      const bool ok = __all_sync(0xffffffffu, wait(done, ((it - 1) >> 1) & 1));
      tc::fence_after_sync();
      if (ok) {
#pragma unroll
        for (int c = 0; c < HD / 2; c += 16) {
          float a16[16];
          tc::tmem_ld16(dsrc + c, a16);
#pragma unroll
          for (int e = 0; e < 16; ++e) g[c + e] = a16[e];
        }
      }
      return ok;
    };
    auto drain_store = [&](bool ok) {
      if (!ok) return;
      const float mul = half8 ? p_ov : p_ok;
#pragma unroll
      for (int c = 0; c < HD / 2; c += 4)
        *staged_chunk<HD>(staging, half8, row, c / 4) = make_float4(g[c] * mul, g[c + 1] * mul, g[c + 2] * mul,
                                                                    g[c + 3] * mul);
#pragma unroll
      for (int c = HD / 2; c < HD; c += 16) {
        float a16[16];
        tc::tmem_ld16(dsrc + c, a16);
#pragma unroll
        for (int e = 0; e < 16; e += 4)
          *staged_chunk<HD>(staging, half8, row, (c + e) / 4) =
              make_float4(a16[e] * mul, a16[e + 1] * mul, a16[e + 2] * mul, a16[e + 3] * mul);
      }
      tc::fence_async_smem();  // the loader's TMA stores read these rows
    };
    int kk = 0;
    for (;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int k0, h;
      kv_item(item, rows, T, H, k0, h);
      const int n = kv_steps(k0, rows, T);
      const int pb_ = kk & 1;
      // Warps 0-7: the key tile's staged FP32 K (warps 0-3) and V (4-7) rows
      // -> FP16 hi/lo TMEM columns with per-row scales (the K, V columns are
      // free: every S^T / dP^T of the previous tile has been read).
      // Warps 8-15 meanwhile take the previous tile's dK / dV out of TMEM.
      bool dok = false;
      if (warp < 8) {
        const bool staged_ok = __all_sync(0xffffffffu, wait(&staged, kk & 1));
        if (staged_ok) {
          const bool isv = warp >= 4;
          // Two passes over the staged row (its largest magnitude and norm,
          // then the split), so the row is never held in registers whole.
          float m = 0.f, ss = 0.f;  // rows past `rows` arrive as zeros (TMA fill)
#pragma unroll
          for (int c = 0; c < HD / 4; ++c) {
            const float4 t4 = *staged_chunk<HD>(staging, isv, row, c);
            m = fmaxf(fmaxf(m, fmaxf(fabsf(t4.x), fabsf(t4.y))), fmaxf(fabsf(t4.z), fabsf(t4.w)));
            ss += t4.x * t4.x + t4.y * t4.y + t4.z * t4.z + t4.w * t4.w;
          }
          const float sc = tc::f16_scale(m);
          const uint32_t thi = (isv ? tVh : tKh) + lane, tlo = (isv ? tVl : tKl) + lane;
#pragma unroll
          for (int c = 0; c < HD; c += 32) {
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float4 t4 = *staged_chunk<HD>(staging, isv, row, (c + 2 * e) / 4);
              tc::split_f16x2(t4.x * sc, t4.y * sc, hi[e], lo[e]);
              tc::split_f16x2(t4.z * sc, t4.w * sc, hi[e + 1], lo[e + 1]);
            }
            tc::tmem_st16u(thi + c / 2, hi);
            tc::tmem_st16u(tlo + c / 2, lo);
          }
          if (isv) {
            vscale[pb_][row] = sc;
            vnorm[pb_][row] = sqrtf(ss);
          } else {
            kscale[pb_][row] = sc;
          }
          tc::tmem_st_wait();
        }
      } else if (kk > 0) {
        dok = drain_load();
      }
      tc::fence_before_sync();
      named_sync<2, kKvCompute>();  // staged rows read; scales visible
      tc::bar_arrive(&kv_ready);    // the issuer may start this key tile
      if (warp >= 8 && kk > 0) drain_store(dok);
      tc::bar_arrive(&drained);  // staging holds the previous tile's dK and dV (or nothing)
      // This tile's per-row constants.
      const float4 mn = tmin[pb_];
      const float scale2 = scale * 1.4426950408889634f / kscale[pb_][row];
      const float vinv = 1.0f / vscale[pb_][row];
      const float sqmin = mn.x, pv_e = 8192.0f * mn.y;
      const float rk = tc::f16_scale((mn.z * vnorm[pb_][row] + mn.w) * scale);
      p_ov = 1.0f / pv_e;
      p_ok = 1.0f / (rk * sqmin);
      const int kr = k0 + row;
      const int ke = (kr / T + 1) * T;  // end of the key's sequence
      const int kseq_end = (k0 / T + 1) * T;
      const bool one_seq = (k0 + kTcRows - 1) / T == k0 / T && k0 + kTcRows <= rows;
      const float2* tsc = tscale[pb_];
      for (int i = 0; i < n; ++i, ++it) {
        const int st = it % NS, b = it & 1, pb = (it >> 1) & 1;
        const float2 ts = tsc[i];
        const float coef = scale2 / ts.x;              // S^T_tmem -> log2 units
        const float dcoef = vinv / ts.y;               // dP^T_tmem -> dP
        const float pc = pv_e / ts.y;                  // P -> stored P
        const float gc = scale * rk * (sqmin / ts.x);  // (dP - delta) P -> stored dS
        const float* hdr = reinterpret_cast<const float*>(sm8 + st * G::QTILE_BYTES + G::HEADER_OFF);
        const uint32_t tSb = tS + 128 * b;
        wait(&q_full[st], (it / NS) & 1);
        wait(&s_full[b], pb);
        tc::fence_after_sync();
        float pv[16];
        {
          float sv[16];
          tc::tmem_ld16(tSb + col + lane, sv);
          const int qh = k0 + i * kTcQ + col;
          const bool full = one_seq && qh >= k0 + kTcRows - 1 && qh + 16 <= min(kseq_end, rows);
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(hdr + G::LSE + col + c);
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
              const float2 lv = u == 0 ? make_float2(l4.x, l4.y) : make_float2(l4.z, l4.w);
              const int q0j = qh + c + u;
              const float2 t = fma2(make_float2(sv[c + u], sv[c + u + 1]), splat2(coef), make_float2(-lv.x, -lv.y));
              const bool ok0 = full || (q0j >= kr && q0j < ke && q0j < rows && kr < rows);
              const bool ok1 = full || (q0j + 1 >= kr && q0j + 1 < ke && q0j + 1 < rows && kr < rows);
              pv[c + u] = ok0 ? ex2(t.x) : 0.f;
              pv[c + u + 1] = ok1 ? ex2(t.y) : 0.f;
            }
          }
          uint32_t hl[16];  // hi parts, then lo parts
#pragma unroll
          for (int e = 0; e < 8; ++e) tc::split_f16x2(pv[2 * e] * pc, pv[2 * e + 1] * pc, hl[e], hl[8 + e]);
          tc::tmem_st16u(tSb + col + lane, hl);  // P^T over the S^T columns just read
        }
        tc::tmem_st_wait();
        tc::fence_before_sync();
        tc::bar_arrive(&p_full[b]);
        wait(&dp_full[b], pb);
        tc::fence_after_sync();
        {
          float dp[16];
          tc::tmem_ld16(tSb + 64 + col + lane, dp);
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const float4 e4 = *reinterpret_cast<const float4*>(hdr + G::DELTA + col + c);
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
              const float2 ev = u == 0 ? make_float2(e4.x, e4.y) : make_float2(e4.z, e4.w);
              const float2 pp = make_float2(pv[c + u], pv[c + u + 1]);
              const float2 g = mul2(pp, fma2(make_float2(dp[c + u], dp[c + u + 1]), splat2(dcoef),
                                             make_float2(-ev.x, -ev.y)));
              dp[c + u] = g.x;
              dp[c + u + 1] = g.y;
            }
          }
          uint32_t hl[16];
#pragma unroll
          for (int e = 0; e < 8; ++e) tc::split_f16x2(dp[2 * e] * gc, dp[2 * e + 1] * gc, hl[e], hl[8 + e]);
          tc::tmem_st16u(tSb + 64 + col + lane, hl);  // dS^T over the dP^T columns just read
          tc::tmem_st_wait();
          tc::fence_before_sync();
          tc::bar_arrive(&ds_full[b][quarter >> 1]);  // query columns [0, 32) or [32, 64)
        }
      }
    }
    if (kk > 0) {
      // The last key tile, once the loader has written out the one before.
      bool dok = false;
      if (warp >= 8) {
        wait(&staged, kk & 1);
        dok = drain_load();
        drain_store(dok);
      }
      tc::bar_arrive(&drained);
    }
  } else if (tid == kKvIssuer || tid == kKvProducer) {
    // ---------------------------------------------------------- S^T / dP^T issuers
    // Thread 544: S^T = K Q^T into buffer b's first 64 columns (free once dV
    // of step it - 2 has read P^T there); thread 512: dP^T = V dO^T into its
    // last 64 (free once dK of step it - 2 has read dS^T).  Separate warps,
    // so the two products issue concurrently.
    const bool dp = tid == kKvProducer;
    constexpr uint32_t idS = tc::idesc_f16(kTcRows, kTcQ);
    uint64_t* full = dp ? dp_full : s_full;
    uint64_t* freed = dp ? dk_done : dv_done;
    const uint32_t ah = dp ? tVh : tKh, al = dp ? tVl : tKl, col = dp ? 64u : 0u;
    const int part = dp ? G::D_HI : G::Q_HI;
    // Thread 512 also streams the query tiles, NS - 1 steps ahead: the tile
    // of step j goes into stage j % NS once dV and dK of step j - NS have
    // read that stage.  It issues the load for step it + NS - 1 after its
    // dP^T of step it, so the wait for step it - 1's release holds up only
    // dP^T of step it + 1, which waits for dK of step it - 1 anyway.
    int lk = 0, li = 0, lsteps = 0, lh = 0, lq0 = 0, lj = 0;  // the load cursor
    auto load_next = [&]() {
      while (li == lsteps) {  // the cursor's work item is done: take the next
        const int item = snake_item(lk, gridDim.x, items);
        if (item < 0) return;
        int k0;
        kv_item(item, rows, T, H, k0, lh);
        lsteps = kv_steps(k0, rows, T);
        lq0 = k0 / kTcQ;
        li = 0;
        ++lk;
      }
      const int st = lj % NS;
      const bool ok = lj < NS || wait(&q_empty[st], ((lj - NS) / NS) & 1);
      if (ok && !sh.failed) {
        tc::bar_expect_tx(&q_full[st], G::QTILE_BYTES);
        tc::bulk_g2s(sm8 + st * G::QTILE_BYTES, qfmt + ((size_t)lh * nqt + lq0 + li) * G::QTILE_BYTES,
                     G::QTILE_BYTES, &q_full[st]);
      }
      ++li;
      ++lj;
    };
    if (dp)
      for (int j = 0; j < NS - 1; ++j) load_next();
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int k0, h;
      kv_item(item, rows, T, H, k0, h);
      const int n = kv_steps(k0, rows, T);
      wait(&kv_ready, kk & 1);  // this key tile's K and V are in TMEM
      for (int i = 0; i < n; ++i, ++it) {
        const int st = it % NS, b = it & 1;
        const uint8_t* stage = sm8 + st * G::QTILE_BYTES;
        wait(&q_full[st], (it / NS) & 1);
        if (it >= 2) wait(&freed[b], ((it - 2) >> 1) & 1);
        tc::fence_after_sync();
        if (!sh.failed) {
          mma16_tmem_a<HD, HD / 16>(tS + 128 * b + col, ah, al, stage + part * G::PART_BYTES,
                                    stage + (part + 1) * G::PART_BYTES, idS, false, 0);
          tc::commit(&full[b]);
        }
        if (dp) load_next();
      }
    }
  } else if (tid == kKvIssuer2) {
    // ---------------------------------------------------------- dV / dK issuer
    constexpr uint32_t idG = tc::idesc_f16(kTcRows, HD, true);
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int k0, h;
      kv_item(item, rows, T, H, k0, h);
      const int n = kv_steps(k0, rows, T);
      for (int i = 0; i < n; ++i, ++it) {
        const int st = it % NS, b = it & 1, pb = (it >> 1) & 1;
        const uint8_t* stage = sm8 + st * G::QTILE_BYTES;
        const uint32_t tSb = tS + 128 * b;
        wait(&q_full[st], (it / NS) & 1);
        wait(&p_full[b], pb);
        tc::fence_after_sync();
        // dV += P^T dO over the step's 64 queries (B = the dO tile [64 queries][HD], MN-major)
        if (!sh.failed) {
          mma16_tmem_a_il<HD, 4>(tdV, tSb, stage + G::D_HI * G::PART_BYTES, stage + (G::D_HI + 1) * G::PART_BYTES,
                                 idG, i > 0, 0);
          tc::commit(&dv_done[b]);
        }
        for (int q2 = 0; q2 < 2; ++q2) {
          wait(&ds_full[b][q2], pb);
          tc::fence_after_sync();
          // dK += dS^T Q over queries [32 q2, 32 q2 + 32) (B = the Q tile [64 queries][HD], MN-major)
          if (!sh.failed)
            mma16_tmem_a_il<HD, 2>(tdK, tSb + 64, stage + G::Q_HI * G::PART_BYTES,
                                   stage + (G::Q_HI + 1) * G::PART_BYTES, idG, i > 0 || q2 > 0, 2 * q2);
        }
        if (sh.failed) continue;
        tc::commit(&dk_done[b]);
        tc::commit(&q_empty[st]);  // both products of the step have read the stage
      }
    }
  } else if (warp == kKvLoader / 32) {
    // ---------------------------------------------------------- key-row loader
    const int ln = tid & 31;
    // dK and dV of work item j (TMEM -> staging by the compute warps) out to
    // its rows with TMA box stores; dV is added onto the XSA term instead
    // when one is given.  Rows past `rows` are clipped by the TMA.  Lane 0.
    auto write_out = [&](int j) {
      int k0, h;
      kv_item(snake_item(j, gridDim.x, items), rows, T, H, k0, h);
      if (!sh.failed) {
#pragma unroll
        for (int half = 0; half < HD / 32; ++half) {
          const int x = h * HD + 32 * half;
          tma_store_box(&map_dk, x, k0, staging + half * KV::BOX_BYTES);
          const uint8_t* vb = staging + (HD / 32 + half) * KV::BOX_BYTES;
          if (dv_add) {
            tma_add_box(&map_dv, x, k0, vb);
          } else {
            tma_store_box(&map_dv, x, k0, vb);
          }
        }
      }
      bulk_commit();
    };
    // Work item kk: the scales of its query tiles (all lanes), then its K and
    // V rows as TMA boxes (lane 0; rows past `rows` fill with zeros).
    auto load = [&](int kk) {
      int k0, h;
      kv_item(snake_item(kk, gridDim.x, items), rows, T, H, k0, h);
      const int n = kv_steps(k0, rows, T), qt0 = k0 / kTcQ, pb = kk & 1;
      float sqm = INFINITY, sdm = INFINITY, ndm = 0.f, dlm = 0.f;
      for (int i = ln; i < n; i += 32) {
        const float4 sc = __ldg(reinterpret_cast<const float4*>(qfmt + ((size_t)h * nqt + qt0 + i) * G::QTILE_BYTES +
                                                                G::HEADER_OFF + G::SCALES * 4));
        tscale[pb][i] = make_float2(sc.x, sc.y);
        sqm = fminf(sqm, sc.x);
        sdm = fminf(sdm, sc.y);
        ndm = fmaxf(ndm, sc.z);
        dlm = fmaxf(dlm, sc.w);
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        sqm = fminf(sqm, __shfl_xor_sync(0xffffffffu, sqm, off));
        sdm = fminf(sdm, __shfl_xor_sync(0xffffffffu, sdm, off));
        ndm = fmaxf(ndm, __shfl_xor_sync(0xffffffffu, ndm, off));
        dlm = fmaxf(dlm, __shfl_xor_sync(0xffffffffu, dlm, off));
      }
      if (ln == 0) tmin[pb] = make_float4(sqm, sdm, ndm, dlm);
      __syncwarp();
      if (ln == 0) {
        // arrive (releasing the scales) and expect the boxes' bytes
        tc::bar_expect_tx(&staged, sh.failed ? 0u : (uint32_t)(2 * (HD / 32) * KV::BOX_BYTES));
        if (!sh.failed) {
#pragma unroll
          for (int half = 0; half < HD / 32; ++half) {
            tma_load_box(staging + half * KV::BOX_BYTES, &map_k, h * HD + 32 * half, k0, &staged);
            tma_load_box(staging + (HD / 32 + half) * KV::BOX_BYTES, &map_v, h * HD + 32 * half, k0, &staged);
          }
        }
      }
    };
    int ni = 0;
    while (snake_item(ni, gridDim.x, items) >= 0) ++ni;
    for (int kk = 0; kk < ni; ++kk) {
      if (kk >= 1) wait(&drained, (kk - 1) & 1);  // rows kk - 1 are in TMEM; staging holds dK/dV of kk - 2
      __syncwarp();
      if (kk >= 2 && ln == 0) {
        write_out(kk - 2);
        bulk_wait_read();  // the stores have read staging before it is refilled
      }
      __syncwarp();
      load(kk);
    }
    if (ni > 0) {
      wait(&drained, (ni - 1) & 1);
      if (ln == 0) {
        if (ni >= 2) {
          write_out(ni - 2);
          bulk_wait_read();
        }
        tc::bar_arrive(&staged);  // staging is free for the last tile's dK and dV
      }
      wait(&drained, ni & 1);
      if (ln == 0) {
        write_out(ni - 1);
        bulk_wait_all();  // every store done before the CTA leaves
      }
      __syncwarp();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (sh.failed && tid == 0) atomicExch(err, 1);
  if (warp == 0) tc::tmem_dealloc(t0, 512);
}

// ---------------------------------------------------------------------- dQ
// Persistent dQ, built like the persistent dK/dV: each CTA (one per SM)
// walks a fixed list of query tiles (128 rows of one head, the longest
// causal work first, dealt in snake order) and, for each, its key tiles 64 at
// a time through a ring that runs on across query tiles.  Q and dO sit in
// TMEM split into FP16 hi/lo columns with per-row scales; dQ accumulates in
// TMEM; S/dP are double-buffered.  Per step j (buffer b = j & 1, j counted
// over the CTA's list): thread 544 issues S = Q K^T and dP = dO V^T; all 16
// compute warps (thread (row, quarter) owns key columns [16 quarter, +16))
// form dS = P (dP - delta) scale over the S columns they have read (FP16
// hi/lo interleaved: hi in S columns [16m, 16m + 8), lo in [16m + 8,
// 16m + 16) for keys [16m, 16m + 16)), each 32-key half handed to thread 576
// for dQ += dS K (B = the K tile, MN-major) as soon as it is stored.
// The loader warp (608) works one query tile ahead: the scales of its key
// tiles, its rows' LSE and delta, and its FP32 Q and dO rows as TMA boxes;
// after a query tile it stores the tile's dQ rows with TMA.  Between two
// query tiles compute warps 0-7 split the staged Q and dO rows into TMEM
// (once the last S/dP of the previous tile have been read) while warps 8-15
// move the previous tile's dQ from TMEM into the staging area.
// Scales: Q rows s_q(i), dO rows t(i); key tiles s_k(j), s_v(j); dS_ij is
// stored as dS_ij r(i) d(j) with r(i) = f16_scale(2 |dO_i| max|V_row| scale),
// a bound on |dS_i.| (|dP| and |delta| are at most |dO_i| max|V_row|), and
// d(j) = min_j s_k / s_k(j), so dQ_i = dQ_tmem / (r(i) min_j s_k); the
// minima and maxima run over the query tile's key tiles.
// TMEM: Q hi | Q lo | dO hi | dO lo (32 each) | S0 | dP0 | S1 | dP1 (64 each) |
// dQ (64) = 448 (512 allocated).
template <int HD>
struct F16Dq {
  using F = F16Fmt<HD>;
  static constexpr int STAGES = 4;
  static constexpr int STAGE_BYTES = 4 * F::PART_BYTES;  // K, K', V, V'
  // Staging: Q (t = 0) and dO (t = 1) rows in, dQ rows (t = 0) out, as
  // 128 x 32 swizzled TMA boxes (staged_chunk), 1024-byte aligned.
  static constexpr size_t STAGING_OFF = (size_t)STAGES * STAGE_BYTES;
  static constexpr size_t smem = STAGING_OFF + 2 * (HD / 32) * (size_t)kBoxBytes + 1024;
};

// Query tile `item` of the grid-wide work list: its first row and head.
__device__ __forceinline__ void dq_item(int item, int rows, int T, int H, int& q0, int& h) {
  const int nt = (rows + kTcRows - 1) / kTcRows;
  h = item % H;
  q0 = tile_by_work(item / H, nt, rows, T, true) * kTcRows;
}
// Its key tiles: from the 64-aligned start of its first row's sequence.
__device__ __forceinline__ void dq_keys(int q0, int rows, int T, int& kbeg, int& n) {
  kbeg = ((q0 - q0 % T) / kTcK) * kTcK;
  const int kend = min(rows, q0 + kTcRows);
  n = (kend - kbeg + kTcK - 1) / kTcK;
}

template <int HD>
__global__ void __launch_bounds__(kKvThreadsP, 1)
    attention_backward_dq_f16(int rows, int T, int H, float scale, const __grid_constant__ CUtensorMap map_q,
                              const __grid_constant__ CUtensorMap map_do, const uint8_t* __restrict__ kfmt,
                              const float* __restrict__ lse2, const float* __restrict__ delta,
                              const __grid_constant__ CUtensorMap map_dq, int* __restrict__ err) {
  using A = F16Dq<HD>;
  using F = F16Fmt<HD>;
  constexpr int NS = A::STAGES;
  extern __shared__ __align__(128) uint8_t sm8[];
  __shared__ uint64_t kv_full[NS], kv_empty[NS], s_full[2], d_full[2][2], q_done[2];
  __shared__ uint64_t staged, qo_ready, drained;
  __shared__ TcShared sh;
  __shared__ float qscale[2][kTcRows], oscale[2][kTcRows], onorm[2][kTcRows];  // by item parity
  __shared__ float lrow[2][kTcRows], drow[2][kTcRows];                        // LSE and delta, by item parity
  __shared__ float2 tscale[2][kMaxKeyTiles];  // (s_k, s_v) of each key tile of a query tile, by item parity
  __shared__ float2 tmin[2];                  // (min s_k, max V row norm), by item parity
  const int tid = threadIdx.x, warp = tid >> 5;
  const int items = ((rows + kTcRows - 1) / kTcRows) * H;
  const int nkt = (rows + kTcK - 1) / kTcK;
  uint8_t* staging = sm8 + A::STAGING_OFF;
  staging += (1024u - (tc::smem_addr(staging) & 1023u)) & 1023u;  // the swizzle's period
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, 512);
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) {
      tc::bar_init(&kv_full[b], 1);
      tc::bar_init(&kv_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&s_full[b], 1);
      tc::bar_init(&d_full[b][0], kKvCompute / 2);
      tc::bar_init(&d_full[b][1], kKvCompute / 2);
      tc::bar_init(&q_done[b], 1);
    }
    tc::bar_init(&staged, 1);
    tc::bar_init(&qo_ready, kKvCompute);
    tc::bar_init(&drained, kKvCompute);
    tc::bar_init_fence();
    sh.failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t t0 = sh.tmem_base;
  const uint32_t tQh = t0, tQl = t0 + 32, tDh = t0 + 64, tDl = t0 + 96, tS = t0 + 128, tG = t0 + 384;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (sh.failed) return false;
    if (tc::bar_wait(bar, parity)) return true;
    sh.failed = 1;
    return false;
  };

  if (tid < kKvCompute) {
    // ---------------------------------------------------------- compute warps
    const int row = tid & (kTcRows - 1), quarter = tid >> 7;
    const int col = 16 * quarter;  // key columns [col, col + 16) of each step
    const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
    int it = 0;
    float p_out = 0.f;  // output scale of the previous query tile
    // Warps 8-15: the previous tile's dQ rows (lane quarter warp % 4,
    // column half (warp / 4) % 2) from TMEM into staging box area t = 0.
    const int half8 = (warp >> 2) & 1;
    float g[HD / 2];
    auto drain_load = [&]() {
      const bool ok = __all_sync(0xffffffffu, wait(&q_done[(it - 1) & 1], ((it - 1) >> 1) & 1));
      tc::fence_after_sync();
      if (ok) {
#pragma unroll
        for (int c = 0; c < HD / 2; c += 16) {
          float a16[16];
          tc::tmem_ld16(tG + lane + half8 * (HD / 2) + c, a16);
#pragma unroll
          for (int e = 0; e < 16; ++e) g[c + e] = a16[e];
        }
      }
      return ok;
    };
    auto drain_store = [&](bool ok) {
      if (ok) {
#pragma unroll
        for (int c = 0; c < HD / 2; c += 4)
          *staged_chunk<HD>(staging, 0, row, (half8 * (HD / 2) + c) / 4) =
              make_float4(g[c] * p_out, g[c + 1] * p_out, g[c + 2] * p_out, g[c + 3] * p_out);
      }
      tc::fence_async_smem();  // the loader's TMA stores read these rows
    };
    int kk = 0;
    for (;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      const int pb_ = kk & 1;
      bool dok = false;
      if (warp < 8) {
        // Staged FP32 Q (warps 0-3) and dO (4-7) rows -> FP16 hi/lo TMEM
        // columns with per-row scales, two passes over the row.
        const bool staged_ok = __all_sync(0xffffffffu, wait(&staged, kk & 1));
        if (staged_ok) {
          const int t = warp >= 4 ? 1 : 0;
          float m = 0.f, ss = 0.f;  // rows past `rows` arrive as zeros (TMA fill)
#pragma unroll
          for (int c = 0; c < HD / 4; ++c) {
            const float4 t4 = *staged_chunk<HD>(staging, t, row, c);
            m = fmaxf(fmaxf(m, fmaxf(fabsf(t4.x), fabsf(t4.y))), fmaxf(fabsf(t4.z), fabsf(t4.w)));
            ss += t4.x * t4.x + t4.y * t4.y + t4.z * t4.z + t4.w * t4.w;
          }
          const float sc = tc::f16_scale(m);
          const uint32_t thi = (t ? tDh : tQh) + lane, tlo = (t ? tDl : tQl) + lane;
#pragma unroll
          for (int c = 0; c < HD; c += 32) {
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float4 t4 = *staged_chunk<HD>(staging, t, row, (c + 2 * e) / 4);
              tc::split_f16x2(t4.x * sc, t4.y * sc, hi[e], lo[e]);
              tc::split_f16x2(t4.z * sc, t4.w * sc, hi[e + 1], lo[e + 1]);
            }
            tc::tmem_st16u(thi + c / 2, hi);
            tc::tmem_st16u(tlo + c / 2, lo);
          }
          if (t) {
            oscale[pb_][row] = sc;
            onorm[pb_][row] = sqrtf(ss);
          } else {
            qscale[pb_][row] = sc;
          }
          tc::tmem_st_wait();
        }
      } else if (kk > 0) {
        dok = drain_load();
      }
      tc::fence_before_sync();
      named_sync<2, kKvCompute>();  // staged rows read; scales visible
      tc::bar_arrive(&qo_ready);    // the issuer may start this query tile
      if (warp >= 8 && kk > 0) drain_store(dok);
      tc::bar_arrive(&drained);  // staging holds the previous tile's dQ (or nothing)
      // This tile's per-row constants.
      const float2 mn = tmin[pb_];
      const float sq_inv = 1.0f / qscale[pb_][row], so_inv = 1.0f / oscale[pb_][row];
      const float rg = tc::f16_scale(2.0f * onorm[pb_][row] * mn.y * scale);  // |dO_row| bounds dS
      const float scale2 = scale * 1.4426950408889634f * sq_inv;
      const float kmin = mn.x;
      const float L = lrow[pb_][row], dl = drow[pb_][row];
      p_out = 1.0f / (rg * kmin);
      const int qr = q0 + row, qs = qr - qr % T;
      const int seq0 = q0 - q0 % T;
      const bool one_seq = (q0 + kTcRows - 1) / T == q0 / T && q0 + kTcRows <= rows;
      const float2* tsc = tscale[pb_];
      for (int j = 0; j < n; ++j, ++it) {
        const int b = it & 1;
        const float2 ts = tsc[j];
        const float coef = scale2 / ts.x;                // S_tmem -> log2 units
        const float dcoef = so_inv / ts.y;               // dP_tmem -> dP
        const float gcoef = scale * rg * (kmin / ts.x);  // dS -> stored dS
        const uint32_t tSb = tS + 128 * b;
        wait(&s_full[b], (it >> 1) & 1);
        tc::fence_after_sync();
        const int kh = kbeg + j * kTcK + col;
        float sv[16], dp[16];
        tc::tmem_ld16_pair(tSb + col + lane, sv, tSb + 64 + col + lane, dp);
        const bool full = one_seq && kh >= seq0 && kh + 15 <= q0;
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          const float2 t = fma2(make_float2(sv[c], sv[c + 1]), splat2(coef), splat2(-L));
          const bool ok0 = full || (kh + c <= qr && kh + c >= qs && kh + c < rows);
          const bool ok1 = full || (kh + c + 1 <= qr && kh + c + 1 >= qs && kh + c + 1 < rows);
          const float2 p = make_float2(ok0 ? ex2(t.x) : 0.f, ok1 ? ex2(t.y) : 0.f);
          const float2 gg = mul2(p, fma2(make_float2(dp[c], dp[c + 1]), splat2(dcoef), splat2(-dl)));
          sv[c] = gg.x;
          sv[c + 1] = gg.y;
        }
        uint32_t hl[16];  // hi parts, then lo parts
#pragma unroll
        for (int e = 0; e < 8; ++e) tc::split_f16x2(sv[2 * e] * gcoef, sv[2 * e + 1] * gcoef, hl[e], hl[8 + e]);
        tc::tmem_st16u(tSb + col + lane, hl);  // over the S columns just read
        tc::tmem_st_wait();
        tc::fence_before_sync();
        tc::bar_arrive(&d_full[b][quarter >> 1]);  // key columns [0, 32) or [32, 64)
      }
    }
    if (kk > 0) {
      // The last query tile, once the loader has stored the one before.
      bool dok = false;
      if (warp >= 8) {
        wait(&staged, kk & 1);
        dok = drain_load();
        drain_store(dok);
      }
      tc::bar_arrive(&drained);
    }
  } else if (tid == kKvProducer) {
    // ---------------------------------------------------------- key tiles
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      const int kt0 = kbeg / kTcK;
      for (int j = 0; j < n; ++j, ++it) {
        const int st = it % NS;
        if (it >= NS && !wait(&kv_empty[st], ((it - NS) / NS) & 1)) continue;
        if (sh.failed) continue;
        tc::bar_expect_tx(&kv_full[st], A::STAGE_BYTES);
        tc::bulk_g2s(sm8 + st * A::STAGE_BYTES, kfmt + ((size_t)h * nkt + kt0 + j) * F::KTILE_BYTES, A::STAGE_BYTES,
                     &kv_full[st]);  // K, K', V, V'
      }
    }
  } else if (tid == kKvIssuer) {
    // ---------------------------------------------------------- S / dP issuer
    constexpr uint32_t idS = tc::idesc_f16(kTcRows, kTcK);
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      wait(&qo_ready, kk & 1);  // this query tile's Q and dO are in TMEM
      for (int j = 0; j < n; ++j, ++it) {
        const int st = it % NS, b = it & 1;
        const uint8_t* stage = sm8 + st * A::STAGE_BYTES;
        wait(&kv_full[st], (it / NS) & 1);
        if (it >= 2) wait(&q_done[b], ((it - 2) >> 1) & 1);  // dQ of step it - 2 has read this buffer's dS
        tc::fence_after_sync();
        if (sh.failed) continue;
        const uint32_t tSb = tS + 128 * b;
        mma16_tmem_a<HD, HD / 16>(tSb, tQh, tQl, stage + F::K_HI * F::PART_BYTES,
                                  stage + (F::K_HI + 1) * F::PART_BYTES, idS, false, 0);  // S = Q K^T
        mma16_tmem_a<HD, HD / 16>(tSb + 64, tDh, tDl, stage + F::V_HI * F::PART_BYTES,
                                  stage + (F::V_HI + 1) * F::PART_BYTES, idS, false, 0);  // dP = dO V^T
        tc::commit(&s_full[b]);
      }
    }
  } else if (tid == kKvIssuer2) {
    // ---------------------------------------------------------- dQ issuer
    constexpr uint32_t idG = tc::idesc_f16(kTcRows, HD, true);
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      for (int j = 0; j < n; ++j, ++it) {
        const int st = it % NS, b = it & 1;
        const uint8_t* stage = sm8 + st * A::STAGE_BYTES;
        const uint32_t tSb = tS + 128 * b;
        wait(&kv_full[st], (it / NS) & 1);
        for (int k2 = 0; k2 < 2; ++k2) {
          wait(&d_full[b][k2], (it >> 1) & 1);
          tc::fence_after_sync();
          // dQ += dS K over keys [32 k2, 32 k2 + 32): K steps 2 k2, 2 k2 + 1
          // of the K tile [64 keys][HD], MN-major
          if (!sh.failed)
            mma16_tmem_a_il<HD, 2>(tG, tSb, stage + F::K_HI * F::PART_BYTES, stage + (F::K_HI + 1) * F::PART_BYTES,
                                   idG, j > 0 || k2 > 0, 2 * k2);
        }
        if (sh.failed) continue;
        tc::commit(&q_done[b]);
        tc::commit(&kv_empty[st]);
      }
    }
  } else if (warp == kKvLoader / 32) {
    // ---------------------------------------------------------- query-row loader
    const int ln = tid & 31;
    auto write_out = [&](int j, const CUtensorMap* map) {  // lane 0
      int q0, h;
      dq_item(snake_item(j, gridDim.x, items), rows, T, H, q0, h);
      if (!sh.failed)
#pragma unroll
        for (int half = 0; half < HD / 32; ++half) tma_store_box(map, h * HD + 32 * half, q0, staging + half * kBoxBytes);
      bulk_commit();
    };
    auto load = [&](int kk) {
      int q0, h, kbeg, n;
      dq_item(snake_item(kk, gridDim.x, items), rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      const int kt0 = kbeg / kTcK, pb = kk & 1;
      float kmn = INFINITY, vn = 0.f;
      for (int j = ln; j < n; j += 32) {
        const float4 hd4 = __ldg(reinterpret_cast<const float4*>(kfmt + ((size_t)h * nkt + kt0 + j) * F::KTILE_BYTES +
                                                                 F::HEADER_OFF));
        tscale[pb][j] = make_float2(hd4.x, hd4.y);
        kmn = fminf(kmn, hd4.x);
        vn = fmaxf(vn, hd4.z);
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        kmn = fminf(kmn, __shfl_xor_sync(0xffffffffu, kmn, off));
        vn = fmaxf(vn, __shfl_xor_sync(0xffffffffu, vn, off));
      }
      if (ln == 0) tmin[pb] = make_float2(kmn, vn);
      for (int r = ln; r < kTcRows; r += 32) {
        const int qr = q0 + r;
        lrow[pb][r] = qr < rows ? __ldg(lse2 + (size_t)h * rows + qr) : 0.f;
        drow[pb][r] = qr < rows ? __ldg(delta + (size_t)h * rows + qr) : 0.f;
      }
      __syncwarp();
      if (ln == 0) {
        // arrive (releasing the values above) and expect the boxes' bytes
        tc::bar_expect_tx(&staged, sh.failed ? 0u : (uint32_t)(2 * (HD / 32) * kBoxBytes));
        if (!sh.failed) {
#pragma unroll
          for (int half = 0; half < HD / 32; ++half) {
            tma_load_box(staging + half * kBoxBytes, &map_q, h * HD + 32 * half, q0, &staged);
            tma_load_box(staging + (HD / 32 + half) * kBoxBytes, &map_do, h * HD + 32 * half, q0, &staged);
          }
        }
      }
    };
    int ni = 0;
    while (snake_item(ni, gridDim.x, items) >= 0) ++ni;
    for (int kk = 0; kk < ni; ++kk) {
      if (kk >= 1) wait(&drained, (kk - 1) & 1);  // rows kk - 1 are in TMEM; staging holds dQ of kk - 2
      __syncwarp();
      if (kk >= 2 && ln == 0) {
        write_out(kk - 2, &map_dq);
        bulk_wait_read();  // the stores have read staging before it is refilled
      }
      __syncwarp();
      load(kk);
    }
    if (ni > 0) {
      wait(&drained, (ni - 1) & 1);
      if (ln == 0) {
        if (ni >= 2) {
          write_out(ni - 2, &map_dq);
          bulk_wait_read();
        }
        tc::bar_arrive(&staged);  // staging is free for the last tile's dQ
      }
      wait(&drained, ni & 1);
      if (ln == 0) {
        write_out(ni - 1, &map_dq);
        bulk_wait_all();  // every store done before the CTA leaves
      }
      __syncwarp();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (sh.failed && tid == 0) atomicExch(err, 1);
  if (warp == 0) tc::tmem_dealloc(t0, 512);
}

// ------------------------------------------------------------------ forward
// Persistent forward, built like the persistent backward kernels: each CTA
// (one per SM) walks a fixed list of query tiles (128 rows of one head, the
// longest causal work first, dealt in snake order) and, for each, its key
// tiles 64 at a time through a ring that runs on across query tiles.
// Compute threads 0-255: row = tid % 128 = TMEM lane, half = tid / 128 takes
// keys [32 half, 32 half + 32) of each 64-key step with its own
// online-softmax stream and O accumulator; thread 256 streams key tiles,
// thread 288 issues S = Q K^T and thread 320 P.V; the loader warp (352)
// works one query tile ahead (the scales of its key tiles, its FP32 Q rows as
// TMA boxes) and stores each finished tile's O rows with TMA.  S and P are
// double-buffered (buffer j & 1 for step j, counted over the CTA's list):
// the softmax of step j + 1 runs while P.V of step j executes, and writing P
// waits only for P.V of step j - 2 to have read that buffer.  A lazy O
// rescale at step j waits for P.V of step j - 1, so O is stable.  Between two
// query tiles warps 0-3 split the staged Q rows into TMEM (once the last S of
// the previous tile has been read), then all compute warps merge the
// previous tile's two streams into staging.
// TMEM columns: Q hi | Q lo (32 each) | S0 | S1 (64 each) | P0 hi | P0 lo |
// P1 hi | P1 lo (32 each) | O0 | O1 (64 each) = 448.
template <int HD>
struct F16Att {
  using F = F16Fmt<HD>;
  static constexpr int FWD_STAGES = 4;
  static constexpr int FWD_STAGE_BYTES = 4 * F::PART_BYTES;  // K, K', V, V'
  // Staging: Q rows in, O rows out (staged_chunk box area t = 0), 1024-byte aligned.
  static constexpr size_t STAGING_OFF = (size_t)FWD_STAGES * FWD_STAGE_BYTES;
  static constexpr size_t smem_forward = STAGING_OFF + (HD / 32) * (size_t)kBoxBytes + 1024;
};
constexpr int kFwdLoader = 352, kFwdThreads = 384;

template <int HD>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attention_forward_f16(int rows, int T, int H, float scale, const __grid_constant__ CUtensorMap map_q,
                          const uint8_t* __restrict__ kfmt, const __grid_constant__ CUtensorMap map_o,
                          float* __restrict__ lse2, int* __restrict__ err) {
  using A = F16Att<HD>;
  using F = F16Fmt<HD>;
  constexpr int NS = A::FWD_STAGES;
  extern __shared__ __align__(128) uint8_t sm8[];
  __shared__ uint64_t kv_full[NS], kv_empty[NS], s_full[2], s_empty[2], p_full[2], o_done[2];
  __shared__ uint64_t staged, q_ready, drained;
  __shared__ TcShared sh;
  __shared__ float xm[2][kTcRows], xl[2][kTcRows], qscale[2][kTcRows];
  __shared__ float2 tscale[2][kMaxKeyTiles];  // (s_k, s_v) of each key tile of a query tile, by item parity
  __shared__ float vmin[2];                   // the smallest V scale over them, by item parity
  const int tid = threadIdx.x, warp = tid >> 5;
  const int items = ((rows + kTcRows - 1) / kTcRows) * H;
  const int nkt = (rows + kTcK - 1) / kTcK;
  uint8_t* staging = sm8 + A::STAGING_OFF;
  staging += (1024u - (tc::smem_addr(staging) & 1023u)) & 1023u;  // the swizzle's period
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, 512);
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) {
      tc::bar_init(&kv_full[b], 1);
      tc::bar_init(&kv_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&s_full[b], 1);
      tc::bar_init(&s_empty[b], kTcCompute);
      tc::bar_init(&p_full[b], kTcCompute);
      tc::bar_init(&o_done[b], 1);
    }
    tc::bar_init(&staged, 1);
    tc::bar_init(&q_ready, kTcCompute);
    tc::bar_init(&drained, kTcCompute);
    tc::bar_init_fence();
    sh.failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t t0 = sh.tmem_base;
  // P buffer b: hi at tP + 64 b, lo at tP + 64 b + 32
  const uint32_t tQh = t0, tQl = t0 + 32, tS = t0 + 64, tP = t0 + 192, tO = t0 + 320;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (sh.failed) return false;
    if (tc::bar_wait(bar, parity)) return true;
    sh.failed = 1;
    return false;
  };

  if (tid < kTcCompute) {
    // ---------------------------------------------------------- softmax
    const int row = tid & (kTcRows - 1), half = tid >> 7;
    const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t myO = tO + 64 * half + lane;
    int it = 0;
    float m = -INFINITY, l = 0.f;     // this thread's stream of the current tile
    float p_pvc = 0.f;                // C of the previous tile
    int p_q0 = 0, p_h = 0;            // the previous tile
    // The previous tile's two streams merged into staging (rows of box area
    // t = 0): O = (O0 2^(m0-M) + O1 2^(m1-M)) / (C L), and its LSE.  Needs
    // xm / xl of both halves (a named barrier before).  Warp-uniform: the
    // TMEM loads are .aligned.
    auto merge = [&](bool ok) {
      if (__all_sync(0xffffffffu, ok)) {
        const float m0 = xm[0][row], m1 = xm[1][row];
        const float mt = fmaxf(m0, m1);
        const float f0 = m0 == -INFINITY ? 0.f : ex2(m0 - mt), f1 = m1 == -INFINITY ? 0.f : ex2(m1 - mt);
        const float L = xl[0][row] * f0 + xl[1][row] * f1;
        const float inv = L > 0.f ? 1.0f / (L * p_pvc) : 0.f;
#pragma unroll
        for (int c = 0; c < HD / 2; c += 16) {
          const int col = (HD / 2) * half + c;
          float a[16], bb[16];
          tc::tmem_ld16_pair(tO + lane + col, a, tO + 64 + lane + col, bb);
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *staged_chunk<HD>(staging, 0, row, (col + e) / 4) =
                make_float4((a[e] * f0 + bb[e] * f1) * inv, (a[e + 1] * f0 + bb[e + 1] * f1) * inv,
                            (a[e + 2] * f0 + bb[e + 2] * f1) * inv, (a[e + 3] * f0 + bb[e + 3] * f1) * inv);
        }
        const int qr = p_q0 + row;
        if (qr < rows && half == 0) lse2[(size_t)p_h * rows + qr] = mt + log2f(L);
      }
      tc::fence_async_smem();  // the loader's TMA stores read these rows
    };
    // The previous tile's last P.V done, its streams' (m, l) published.
    // Every thread passed its wait for P.V of step it - 3, so the parity
    // wait is exact.
    auto finish = [&]() {
      const bool ok = wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1);
      tc::fence_after_sync();
      xm[half][row] = m;
      xl[half][row] = l;
      return ok;
    };
    int kk = 0;
    for (;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      const int pb_ = kk & 1;
      const bool fin = kk > 0 ? finish() : true;
      if (warp < 4) {
        // Staged FP32 Q rows -> FP16 hi/lo TMEM columns with per-row scales
        // (the Q columns are free: the previous tile's last S has been read).
        const bool staged_ok = __all_sync(0xffffffffu, wait(&staged, kk & 1));
        if (staged_ok) {
          float mq = 0.f;  // rows past `rows` arrive as zeros (TMA fill)
#pragma unroll
          for (int c = 0; c < HD / 4; ++c) {
            const float4 t4 = *staged_chunk<HD>(staging, 0, row, c);
            mq = fmaxf(fmaxf(mq, fmaxf(fabsf(t4.x), fabsf(t4.y))), fmaxf(fabsf(t4.z), fabsf(t4.w)));
          }
          const float sc = tc::f16_scale(mq);
#pragma unroll
          for (int c = 0; c < HD; c += 32) {
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float4 t4 = *staged_chunk<HD>(staging, 0, row, (c + 2 * e) / 4);
              tc::split_f16x2(t4.x * sc, t4.y * sc, hi[e], lo[e]);
              tc::split_f16x2(t4.z * sc, t4.w * sc, hi[e + 1], lo[e + 1]);
            }
            tc::tmem_st16u(tQh + lane + c / 2, hi);
            tc::tmem_st16u(tQl + lane + c / 2, lo);
          }
          qscale[pb_][row] = sc;
          tc::tmem_st_wait();
        }
      }
      tc::fence_before_sync();
      named_sync<2, kTcCompute>();  // staged rows read; scales and (m, l) visible
      tc::bar_arrive(&q_ready);     // the issuer may start this query tile
      if (kk > 0) merge(fin);
      tc::bar_arrive(&drained);  // staging holds the previous tile's O (or nothing)
      // This tile's constants.
      const float pv_c = 128.0f * vmin[pb_];  // C: every step's P.V carries this factor
      p_pvc = pv_c;
      p_q0 = q0;
      p_h = h;
      const float scale2 = scale * 1.4426950408889634f / qscale[pb_][row];
      const int qr = q0 + row, qs = qr - qr % T;
      const int seq0 = q0 - q0 % T;
      const bool one_seq = (q0 + kTcRows - 1) / T == q0 / T && q0 + kTcRows <= rows;
      const float2* tsc = tscale[pb_];
      m = -INFINITY;
      l = 0.f;
      for (int j = 0; j < n; ++j, ++it) {
        const int b = it & 1;
        const float2 ts = tsc[j];
        const float coef = scale2 / ts.x;  // scaled score -> log2 units
        wait(&s_full[b], (it >> 1) & 1);
        tc::fence_after_sync();
        float sv[32];
        tc::tmem_ld32(tS + 64 * b + 32 * half + lane, sv);
        tc::fence_before_sync();
        tc::bar_arrive(&s_empty[b]);
        const int kt = kbeg + j * kTcK;
        const bool full = one_seq && kt >= seq0 && kt + kTcK - 1 <= q0;
        const int kh = kt + 32 * half;
        if (!full) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int kr = kh + c;
            sv[c] = (kr <= qr && kr >= qs && kr < rows) ? sv[c] : -INFINITY;
          }
        }
        float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int c = 4; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], sv[c]);
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        mx *= coef;
        const bool need = mx > m + 8.0f;  // false while every key so far is masked
        float alpha = 1.0f;
        if (need) {
          alpha = ex2(m - mx);  // 0 when m = -inf
          m = mx;
        }
        const float nm = m == -INFINITY ? 0.f : -m;
        float2 rs2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float2 t = fma2(make_float2(sv[c], sv[c + 1]), splat2(coef), splat2(nm));
          sv[c] = ex2(t.x);  // ex2(-inf) = 0 for masked keys
          sv[c + 1] = ex2(t.y);
          rs2 = add2(rs2, make_float2(sv[c], sv[c + 1]));
        }
        l = l * alpha + (rs2.x + rs2.y);
        if (it >= 2) {
          // P.V of step it - 2 has read this P buffer.
          wait(&o_done[b], ((it - 2) >> 1) & 1);
          tc::fence_after_sync();
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // P.V of step it - 1 complete: O is stable for the rescale.
          const bool ok = __all_sync(0xffffffffu, wait(&o_done[b ^ 1], ((it - 1) >> 1) & 1));
          tc::fence_after_sync();
          if (ok) {
#pragma unroll
            for (int c = 0; c < HD; c += 16) {
              float ov[16];
              tc::tmem_ld16(myO + c, ov);
#pragma unroll
              for (int e = 0; e < 16; ++e) ov[e] *= alpha;
              tc::tmem_st16(myO + c, ov);
            }
          }
        }
        const uint32_t tPb = tP + 64 * b;
        tc_st_split16<32>(tPb + 16 * half + lane, tPb + 32 + 16 * half + lane, sv, pv_c / ts.y);
        tc::tmem_st_wait();
        tc::fence_before_sync();
        tc::bar_arrive(&p_full[b]);
      }
    }
    if (kk > 0) {
      // The last query tile, once the loader has stored the one before.
      const bool fin = finish();
      wait(&staged, kk & 1);
      named_sync<2, kTcCompute>();  // (m, l) of both halves visible
      merge(fin);
      tc::bar_arrive(&drained);
    }
  } else if (tid == kTcProducer) {
    // ---------------------------------------------------------- producer
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      const int kt0 = kbeg / kTcK;
      for (int j = 0; j < n; ++j, ++it) {
        const int st = it % NS;
        if (it >= NS && !wait(&kv_empty[st], ((it - NS) / NS) & 1)) continue;
        if (sh.failed) continue;
        tc::bar_expect_tx(&kv_full[st], A::FWD_STAGE_BYTES);
        tc::bulk_g2s(sm8 + st * A::FWD_STAGE_BYTES, kfmt + ((size_t)h * nkt + kt0 + j) * F::KTILE_BYTES,
                     A::FWD_STAGE_BYTES, &kv_full[st]);
      }
    }
  } else if (tid == kTcIssuer) {
    // ---------------------------------------------------------- S issuer
    constexpr uint32_t idS = tc::idesc_f16(kTcRows, kTcK);
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      wait(&q_ready, kk & 1);  // this query tile's Q is in TMEM
      for (int j = 0; j < n; ++j, ++it) {
        const int st = it % NS, b = it & 1;
        const uint8_t* stage = sm8 + st * A::FWD_STAGE_BYTES;
        wait(&kv_full[st], (it / NS) & 1);
        if (it >= 2) wait(&s_empty[b], ((it - 2) >> 1) & 1);
        tc::fence_after_sync();
        if (sh.failed) continue;
        // S_j = Q K_j^T over HD / 16 steps
        mma16_tmem_a<HD, HD / 16>(tS + 64 * b, tQh, tQl, stage, stage + F::PART_BYTES, idS, false, 0);
        tc::commit(&s_full[b]);
      }
    }
  } else if (tid == kTcIssuer2) {
    // ---------------------------------------------------------- P.V issuer
    constexpr uint32_t idO = tc::idesc_f16(kTcRows, HD, true);
    int it = 0;
    for (int kk = 0;; ++kk) {
      const int item = snake_item(kk, gridDim.x, items);
      if (item < 0) break;
      int q0, h, kbeg, n;
      dq_item(item, rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      for (int j = 0; j < n; ++j, ++it) {
        const int st = it % NS, b = it & 1;
        const uint8_t* stage = sm8 + st * A::FWD_STAGE_BYTES;
        wait(&p_full[b], (it >> 1) & 1);
        wait(&kv_full[st], (it / NS) & 1);
        tc::fence_after_sync();
        if (sh.failed) continue;
        // O_half += P[:, half keys] V[half keys]  (B = the V tile [64 keys][HD],
        // MN-major; K steps of 16 keys: half 0 steps 0-1, half 1 steps 2-3)
        const uint8_t* vh = stage + F::V_HI * F::PART_BYTES;
        const uint8_t* vl = stage + (F::V_HI + 1) * F::PART_BYTES;
        const uint32_t tPb = tP + 64 * b;
        mma16_tmem_a<HD, 2, true>(tO, tPb, tPb + 32, vh, vl, idO, j > 0, 0);
        mma16_tmem_a<HD, 2, true>(tO + 64, tPb, tPb + 32, vh, vl, idO, j > 0, 2);
        tc::commit(&o_done[b]);
        tc::commit(&kv_empty[st]);
      }
    }
  } else if (warp == kFwdLoader / 32) {
    // ---------------------------------------------------------- query-row loader
    const int ln = tid & 31;
    auto write_out = [&](int j) {  // lane 0
      int q0, h;
      dq_item(snake_item(j, gridDim.x, items), rows, T, H, q0, h);
      if (!sh.failed)
#pragma unroll
        for (int half = 0; half < HD / 32; ++half)
          tma_store_box(&map_o, h * HD + 32 * half, q0, staging + half * kBoxBytes);
      bulk_commit();
    };
    auto load = [&](int kk) {
      int q0, h, kbeg, n;
      dq_item(snake_item(kk, gridDim.x, items), rows, T, H, q0, h);
      dq_keys(q0, rows, T, kbeg, n);
      const int kt0 = kbeg / kTcK, pb = kk & 1;
      float mn = INFINITY;
      for (int j = ln; j < n; j += 32) {
        const float4 hd4 = __ldg(reinterpret_cast<const float4*>(kfmt + ((size_t)h * nkt + kt0 + j) * F::KTILE_BYTES +
                                                                 F::HEADER_OFF));
        tscale[pb][j] = make_float2(hd4.x, hd4.y);
        mn = fminf(mn, hd4.y);
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
      if (ln == 0) vmin[pb] = mn;
      __syncwarp();
      if (ln == 0) {
        // arrive (releasing the scales) and expect the boxes' bytes
        tc::bar_expect_tx(&staged, sh.failed ? 0u : (uint32_t)((HD / 32) * kBoxBytes));
        if (!sh.failed)
#pragma unroll
          for (int half = 0; half < HD / 32; ++half)
            tma_load_box(staging + half * kBoxBytes, &map_q, h * HD + 32 * half, q0, &staged);
      }
    };
    int ni = 0;
    while (snake_item(ni, gridDim.x, items) >= 0) ++ni;
    for (int kk = 0; kk < ni; ++kk) {
      if (kk >= 1) wait(&drained, (kk - 1) & 1);  // rows kk - 1 are in TMEM; staging holds O of kk - 2
      __syncwarp();
      if (kk >= 2 && ln == 0) {
        write_out(kk - 2);
        bulk_wait_read();  // the stores have read staging before it is refilled
      }
      __syncwarp();
      load(kk);
    }
    if (ni > 0) {
      wait(&drained, (ni - 1) & 1);
      if (ln == 0) {
        if (ni >= 2) {
          write_out(ni - 2);
          bulk_wait_read();
        }
        tc::bar_arrive(&staged);  // staging is free for the last tile's O
      }
      wait(&drained, ni & 1);
      if (ln == 0) {
        write_out(ni - 1);
        bulk_wait_all();  // every store done before the CTA leaves
      }
      __syncwarp();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (sh.failed && tid == 0) atomicExch(err, 1);
  if (warp == 0) tc::tmem_dealloc(t0, 512);
}

#undef F16_WAIT_OR_FAIL

}  // namespace mb
