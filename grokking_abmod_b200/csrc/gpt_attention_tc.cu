// Causal flash attention on the sm_100a tensor cores (tcgen05, 3xTF32).
//
// Same semantics and statistics as the FP32 SIMT kernels in
// gpt_attention.cu (and the reference's FA2 kernels, src/gpt/gpu.rs:381-750):
// softmax(Q K^T / sqrt(hd)) V with a causal, same-sequence mask over 128-row
// tiles of the flattened token rows; base-2 LSE; dQ and dK/dV as separate
// kernels (no atomics, bitwise reproducible).
//
// Every product runs on tcgen05.mma kind::tf32 with each FP32 operand split
// into hi/lo TF32 parts (hi.hi + hi.lo + lo.hi), accumulated in FP32 in
// tensor memory (TMEM).
//
// Data movement, B200-first:
//  * A format pass writes, per head and per tile of rows, the hi/lo parts of
//    every shared-memory operand as contiguous UMMA-canonical tiles
//    (tc05.cuh's blocked layout): one key tile is 8 parts x 64 rows x hd;
//    one query tile (dK/dV) is 8 parts x 32 rows x hd plus its LSE and delta.
//    Operands needed with rows along N are stored transposed (K-major), since
//    TF32 MMAs read a transposed (MN-major) operand as zeros here.
//  * Producer threads stream each step's tile into multi-stage shared-memory
//    rings with cp.async.bulk (plain, no multicast); the tiles arrive as
//    mbarrier transactions.
//  * The 128-row operand owned by the CTA (Q in the forward, Q and dO in dQ,
//    K in dK/dV) is split by the compute threads into TMEM and used through
//    the A-from-TMEM form (dK/dV keeps V in shared memory); score /
//    probability tiles also live in TMEM (thread i of the compute warps owns
//    lane i = row i).
//  * One thread issues all MMAs and commits them to mbarriers; all waits are
//    bounded and report through `err` instead of hanging.

#include "common.cuh"
#include "tc05.cuh"

namespace mb {

constexpr int kTcRows = 128;     // CTA tile rows = TMEM lanes
constexpr int kTcK = 64;         // key-tile rows (forward, dQ)
constexpr int kTcQ = 64;         // query-tile rows (dK/dV)
constexpr int kTcCompute = 256;  // compute threads: row = tid % 128, column half = tid / 128
// Forward and dQ: 8 compute warps, a producer warp (thread 256), and two MMA
// issuers in separate warps (threads 288 and 320).
constexpr int kTcProducer = 256, kTcIssuer = 288;
constexpr int kTcThreads2 = 352, kTcIssuer2 = 320;

template <int HD>
struct TcFmt {
  static constexpr int KPART = kTcK * HD;             // floats per key-tile part
  static constexpr int KTILE = 8 * KPART;             // K, K', Vt, Vt', V, V', Kt, Kt'
  static constexpr int QPART = kTcQ * HD;             // floats per query-tile part
  static constexpr int QTILE = 8 * QPART + 2 * kTcQ;  // Q, Q', dO, dO', Qt, Qt', dOt, dOt', lse2, delta
  static constexpr int K_HI = 0, K_LO = 1, VT_HI = 2, VT_LO = 3, V_HI = 4, V_LO = 5, KT_HI = 6, KT_LO = 7;
  static constexpr int Q_HI = 0, Q_LO = 1, D_HI = 2, D_LO = 3, QT_HI = 4, QT_LO = 5, DT_HI = 6, DT_LO = 7;
  static_assert(QT_HI == 4 && DT_HI == 6, "dK/dV streams parts 0-3 and 4-7 (+ lse2, delta) as two rings");
};

constexpr int kFmtThreads = 256;  // threads of the format kernels

// Writes parts of one operand tile in the blocked K-major layout from a
// shared-memory copy `x` ([R][HD], row stride HD + 2).  Part kind 0 is the
// tile itself ([R rows][HD columns]), kind 1 its transpose ([HD rows][R
// columns]); each part is written as its TF32 hi and lo halves (parts `p`,
// `p + 1` of `tile`).  Every thread writes whole 16-byte groups of the
// blocked layout (4 consecutive columns of one core-matrix row), so the
// stores of a warp cover contiguous 512-byte runs.
template <int R, int HD>
__device__ __forceinline__ void store_parts(float* __restrict__ tile, int part_floats, int p, bool transposed,
                                            const float* x) {
  constexpr int XS = HD + 2;
  const int rows = transposed ? HD : R, cols = transposed ? R : HD;
  float* hi = tile + (size_t)p * part_floats;
  float* lo = hi + part_floats;
#pragma unroll
  for (int q = threadIdx.x; q < R * HD / 4; q += kFmtThreads) {
    const int rl = q & 7, c4 = (q >> 3) % (cols / 4), rg = (q >> 3) / (cols / 4);
    const int r = rg * 8 + rl, c = c4 * 4;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = transposed ? x[(c + e) * XS + r] : x[r * XS + c + e];
    float4 h, l;
    h.x = tc::tf32_hi(v[0]);
    h.y = tc::tf32_hi(v[1]);
    h.z = tc::tf32_hi(v[2]);
    h.w = tc::tf32_hi(v[3]);
    l = make_float4(v[0] - h.x, v[1] - h.y, v[2] - h.z, v[3] - h.w);
    reinterpret_cast<float4*>(hi)[q] = h;
    reinterpret_cast<float4*>(lo)[q] = l;
  }
}

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

// Key tiles of K and V: grid (ceil(rows/64), H), 256 threads.  `parts` is a
// bit mask over the hi parts of TcFmt's key tile (K_HI, VT_HI, V_HI, KT_HI):
// only the parts the following kernel reads are written.
template <int HD>
__global__ void __launch_bounds__(kFmtThreads) attention_format_keys(int rows, int W, const float* __restrict__ k,
                                                               const float* __restrict__ v, float* __restrict__ fmt,
                                                               unsigned parts) {
  using F = TcFmt<HD>;
  __shared__ float xk[kTcK * (HD + 2)], xv[kTcK * (HD + 2)];
  const int t = blockIdx.x, h = blockIdx.y;
  float* tile = fmt + ((size_t)h * gridDim.x + t) * F::KTILE;
  load_rows2<kTcK, HD>(xk, k, xv, v, t * kTcK, rows, W, h);
  __syncthreads();
  if (parts & (1u << F::K_HI)) store_parts<kTcK, HD>(tile, F::KPART, F::K_HI, false, xk);
  if (parts & (1u << F::VT_HI)) store_parts<kTcK, HD>(tile, F::KPART, F::VT_HI, true, xv);
  if (parts & (1u << F::V_HI)) store_parts<kTcK, HD>(tile, F::KPART, F::V_HI, false, xv);
  if (parts & (1u << F::KT_HI)) store_parts<kTcK, HD>(tile, F::KPART, F::KT_HI, true, xk);
}

// Query tiles of Q and dO with their LSE and delta: grid (ceil(rows/32), H).
template <int HD>
__global__ void __launch_bounds__(kFmtThreads) attention_format_queries(int rows, int W, const float* __restrict__ q,
                                                                  const float* __restrict__ dout,
                                                                  const float* __restrict__ lse2,
                                                                  const float* __restrict__ delta,
                                                                  float* __restrict__ fmt) {
  using F = TcFmt<HD>;
  __shared__ float xq[kTcQ * (HD + 2)], xd[kTcQ * (HD + 2)];
  const int t = blockIdx.x, h = blockIdx.y;
  float* tile = fmt + ((size_t)h * gridDim.x + t) * F::QTILE;
  load_rows2<kTcQ, HD>(xq, q, xd, dout, t * kTcQ, rows, W, h);
  __syncthreads();
  store_parts<kTcQ, HD>(tile, F::QPART, F::Q_HI, false, xq);
  store_parts<kTcQ, HD>(tile, F::QPART, F::D_HI, false, xd);
  store_parts<kTcQ, HD>(tile, F::QPART, F::QT_HI, true, xq);
  store_parts<kTcQ, HD>(tile, F::QPART, F::DT_HI, true, xd);
  if (threadIdx.x < kTcQ) {
    const int row = t * kTcQ + threadIdx.x;
    tile[8 * F::QPART + threadIdx.x] = row < rows ? lse2[(size_t)h * rows + row] : 0.f;
    tile[8 * F::QPART + kTcQ + threadIdx.x] = row < rows ? delta[(size_t)h * rows + row] : 0.f;
  }
}

// The CTA's 128 rows of head h, loaded by all `nthreads` threads with
// coalesced float4 reads into a staging area ([128][HD + 4]) of shared memory.
template <int HD>
__device__ __forceinline__ void stage_rows(float* stage, const float* __restrict__ g, int row0, int rows, int W,
                                           int h, int nthreads) {
  constexpr int XS = HD + 4, PER = kTcRows * HD / 4;
  for (int i = threadIdx.x; i < PER; i += nthreads) {
    const int r = i / (HD / 4), c = (i % (HD / 4)) * 4;
    const float4 x = row0 + r < rows ? __ldg(reinterpret_cast<const float4*>(g + (size_t)(row0 + r) * W + h * HD + c))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(stage + r * XS + c) = x;
  }
}

// Row `r` of a staging area split into hi/lo TMEM columns of this thread's
// lane (threads 0-127, row = TMEM lane).
template <int HD>
__device__ __forceinline__ void staged_row_to_tmem(const float* stage, int r, uint32_t thi, uint32_t tlo) {
  constexpr int XS = HD + 4;
#pragma unroll
  for (int c = 0; c < HD; c += 16) {
    float hi[16], lo[16];
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 x = *reinterpret_cast<const float4*>(stage + r * XS + c + e);
      const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        hi[e + u] = tc::tf32_hi(xs[u]);
        lo[e + u] = xs[u] - hi[e + u];
      }
    }
    tc::tmem_st16(thi + c, hi);
    tc::tmem_st16(tlo + c, lo);
  }
}

// This thread's row (HD floats, row-major) split into hi/lo TMEM columns.
template <int HD>
__device__ __forceinline__ void row_to_tmem(const float* __restrict__ g, int row, int rows, int W, int h,
                                            uint32_t thi, uint32_t tlo) {
#pragma unroll
  for (int c = 0; c < HD; c += 16) {
    float hi[16], lo[16];
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 x = row < rows ? __ldg(reinterpret_cast<const float4*>(g + (size_t)row * W + h * HD + c + e))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
      const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        hi[e + u] = tc::tf32_hi(xs[u]);
        lo[e + u] = xs[u] - hi[e + u];
      }
    }
    tc::tmem_st16(thi + c, hi);
    tc::tmem_st16(tlo + c, lo);
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

// Named barrier over the 256 compute threads.
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// NC consecutive TMEM columns of this thread's lane.
template <int NC>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
#pragma unroll
  for (int c = 0; c < NC; c += 32) tc::tmem_ld32(taddr + c, v + c);
}

// Stores hi/lo TF32 parts of NC values into two TMEM column ranges.
template <int NC>
__device__ __forceinline__ void tc_st_split(uint32_t thi, uint32_t tlo, const float* v) {
#pragma unroll
  for (int c = 0; c < NC; c += 16) {
    float hi[16], lo[16];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      hi[j] = tc::tf32_hi(v[c + j]);
      hi[j + 1] = tc::tf32_hi(v[c + j + 1]);
      const float2 l2 = add2(make_float2(v[c + j], v[c + j + 1]), make_float2(-hi[j], -hi[j + 1]));
      lo[j] = l2.x;
      lo[j + 1] = l2.y;
    }
    tc::tmem_st16(thi + c, hi);
    tc::tmem_st16(tlo + c, lo);
  }
}

// D (+)= A . B^T with A = hi/lo TMEM columns (KC of them, K-major) and B a
// K-major hi/lo shared tile [N rows][KC columns]: 3 MMAs per 8-wide K step.
template <int KC>
__device__ __forceinline__ void mma_tmem_a(uint32_t d, uint32_t ah, uint32_t al, const float* bh, const float* bl,
                                           uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int s = 0; s < KC / 8; ++s) {
    const uint64_t b_h = tc::desc_kmajor(bh, KC, s), b_l = tc::desc_kmajor(bl, KC, s);
    tc::mma_ts(d, ah + 8 * s, b_h, idesc, (accumulate || s > 0) ? 1u : 0u);
    tc::mma_ts(d, ah + 8 * s, b_l, idesc, 1u);
    tc::mma_ts(d, al + 8 * s, b_h, idesc, 1u);
  }
}

// The same over K steps [s0, s0 + NSTEP) of a B tile with KC columns (A
// columns 8s of the TMEM ranges).
template <int KC, int NSTEP>
__device__ __forceinline__ void mma_tmem_a_steps(uint32_t d, uint32_t ah, uint32_t al, const float* bh,
                                                 const float* bl, uint32_t idesc, bool accumulate, int s0) {
#pragma unroll
  for (int i = 0; i < NSTEP; ++i) {
    const int s = s0 + i;
    const uint64_t b_h = tc::desc_kmajor(bh, KC, s), b_l = tc::desc_kmajor(bl, KC, s);
    tc::mma_ts(d, ah + 8 * s, b_h, idesc, (accumulate || i > 0) ? 1u : 0u);
    tc::mma_ts(d, ah + 8 * s, b_l, idesc, 1u);
    tc::mma_ts(d, al + 8 * s, b_h, idesc, 1u);
  }
}

template <int HD>
struct TcAtt {
  using F = TcFmt<HD>;
  static constexpr int FWD_STAGES = 3;
  static constexpr int FWD_STAGE = 4 * F::KPART;  // K, K', Vt, Vt'
  static constexpr int DQ_STAGES = 2;
  static constexpr int DQ_STAGE = 6 * F::KPART;  // K, K', V, V', Kt, Kt'
  static constexpr size_t smem_forward = (size_t)FWD_STAGES * FWD_STAGE * sizeof(float);
  static constexpr size_t smem_dq = (size_t)DQ_STAGES * DQ_STAGE * sizeof(float);
};

struct TcShared {
  uint32_t tmem_base;
  int failed;
};

// Inside a role loop: a wait that gives up marks the CTA failed and leaves.
#define TC_WAIT_OR_FAIL(bar, parity)     \
  if (!tc::bar_wait((bar), (parity))) {  \
    sh.failed = 1;                       \
    break;                               \
  }

// ------------------------------------------------------------------ forward
// Threads 0-255 compute (row r = tid % 128 owns TMEM lane r; half = tid / 128
// takes keys [32 half, 32 half + 32) of every 64-key step and keeps its own
// online-softmax stream with its own O accumulator), thread 256 producer,
// thread 288 issues the S = Q K^T MMAs and thread 320 (an eleventh warp) the
// P.V MMAs: with TMEM loads and stores of the softmax warps in flight every
// mbarrier wait of an issuing thread takes hundreds of cycles, and two
// issuers let one keep the tensor pipe fed while the other waits.  The two
// softmax streams merge once at the end, so no
// per-step cross-warp reduction is needed.  O is rescaled lazily (only when a
// row's running maximum grows by more than 2^8), as in FlashAttention-4.
// TMEM: Q hi | Q lo | S0 | S1 | P hi | P lo | O0 | O1   (64 columns each).
// mbarriers (parity = use index & 1): kv_full/kv_empty per stage, s_full /
// s_empty per S buffer, p_full (256 arrivals), o_done (commit after P.V).
template <int HD>
__global__ void __launch_bounds__(kTcThreads2, 1)
    attention_forward_tc(int rows, int W, int T, float scale, const float* __restrict__ q,
                         const float* __restrict__ kfmt, float* __restrict__ o, float* __restrict__ lse2,
                         int* __restrict__ err) {
  using A = TcAtt<HD>;
  using F = TcFmt<HD>;
  constexpr int NS = A::FWD_STAGES;
  extern __shared__ __align__(128) float sm[];
  __shared__ uint64_t kv_full[NS], kv_empty[NS], s_full[2], s_empty[2], p_full, o_done;
  __shared__ TcShared sh;
  __shared__ float xm[2][kTcRows], xl[2][kTcRows];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nt = (rows + kTcRows - 1) / kTcRows;
  const int q0 = tile_by_work(blockIdx.x, nt, rows, T, true) * kTcRows;  // longest causal spans first
  const int h = blockIdx.y;
  const int nkt = (rows + kTcK - 1) / kTcK;
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, 512);
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) {
      tc::bar_init(&kv_full[b], 1);
      tc::bar_init(&kv_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&s_full[b], 1);
      tc::bar_init(&s_empty[b], kTcCompute);
    }
    tc::bar_init(&p_full, kTcCompute);
    tc::bar_init(&o_done, 1);
    tc::bar_init_fence();
    sh.failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t t0 = sh.tmem_base;
  const uint32_t tQh = t0, tQl = t0 + 64, tS = t0 + 128, tPh = t0 + 256, tPl = t0 + 320, tO = t0 + 384;
  const int kbeg = ((q0 - q0 % T) / kTcK) * kTcK;  // 64-aligned start of the first sequence
  const int kend = min(rows, q0 + kTcRows);
  const int n = (kend - kbeg + kTcK - 1) / kTcK;
  const int kt0 = kbeg / kTcK;
  if (warp < 4) {
    const uint32_t lane = (uint32_t)(warp * 32) << 16;
    row_to_tmem<HD>(q, q0 + tid, rows, W, h, tQh + lane, tQl + lane);
    tc::tmem_st_wait();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (tid < kTcCompute) {
    // ---------------------------------------------------------- softmax
    const int row = tid & (kTcRows - 1), half = tid >> 7;
    const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t myO = tO + 64 * half + lane;
    const float scale2 = scale * 1.4426950408889634f;
    const int qr = q0 + row, qs = qr - qr % T;
    // Every query row of the CTA in one sequence: steps wholly below the
    // diagonal need no mask.
    const int seq0 = q0 - q0 % T;
    const bool one_seq = (q0 + kTcRows - 1) / T == q0 / T && q0 + kTcRows <= rows;
    float m = -INFINITY, l = 0.f;
    bool done = false;
    for (int j = 0; j < n; ++j) {
      const int b = j & 1;
      TC_WAIT_OR_FAIL(&s_full[b], (j >> 1) & 1);
      tc::fence_after_sync();
      float s[32];
      tc::tmem_ld32(tS + 64 * b + 32 * half + lane, s);
      tc::fence_before_sync();
      tc::bar_arrive(&s_empty[b]);
      const int kt = kbeg + j * kTcK;
      const bool full = one_seq && kt >= seq0 && kt + kTcK - 1 <= q0;
      const int kh = kt + 32 * half;
      if (!full) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int kr = kh + c;
          s[c] = (kr <= qr && kr >= qs && kr < rows) ? s[c] : -INFINITY;
        }
      }
      // Row maximum over four independent chains (max is exact in any order).
      float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int c = 4; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], s[c]);
      float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      mx *= scale2;
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
        const float2 t = fma2(make_float2(s[c], s[c + 1]), splat2(scale2), splat2(nm));
        s[c] = ex2(t.x);  // ex2(-inf) = 0 for masked keys
        s[c + 1] = ex2(t.y);
        rs2 = add2(rs2, make_float2(s[c], s[c + 1]));
      }
      l = l * alpha + (rs2.x + rs2.y);
      if (j > 0) {
        // P.V of step j-1 complete: O is stable and the P buffer is free.
        TC_WAIT_OR_FAIL(&o_done, (j - 1) & 1);
        tc::fence_after_sync();
        if (__any_sync(0xffffffffu, need)) {
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
      tc_st_split<32>(tPh + 32 * half + lane, tPl + 32 * half + lane, s);
      tc::tmem_st_wait();
      tc::fence_before_sync();
      tc::bar_arrive(&p_full);
      if (j + 1 == n) done = true;
    }
    if (done && !tc::bar_wait(&o_done, (n - 1) & 1)) sh.failed = 1;
    tc::fence_after_sync();
    xm[half][row] = m;
    xl[half][row] = l;
    compute_sync();
    if (done && !sh.failed) {
      // Merge the two streams: O = (O0 2^(m0-M) + O1 2^(m1-M)) / L.
      const float m0 = xm[0][row], m1 = xm[1][row];
      const float mt = fmaxf(m0, m1);
      const float f0 = m0 == -INFINITY ? 0.f : ex2(m0 - mt), f1 = m1 == -INFINITY ? 0.f : ex2(m1 - mt);
      const float L = xl[0][row] * f0 + xl[1][row] * f1;
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      const uint32_t o0 = tO + lane, o1 = tO + 64 + lane;
#pragma unroll
      for (int c = 0; c < HD / 2; c += 16) {
        const int col = (HD / 2) * half + c;
        float a[16], bb[16];
        tc::tmem_ld16_pair(o0 + col, a, o1 + col, bb);
        if (qr < rows) {
          float4* dst = reinterpret_cast<float4*>(o + (size_t)qr * W + h * HD + col);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            dst[e] = make_float4((a[4 * e] * f0 + bb[4 * e] * f1) * inv, (a[4 * e + 1] * f0 + bb[4 * e + 1] * f1) * inv,
                                 (a[4 * e + 2] * f0 + bb[4 * e + 2] * f1) * inv,
                                 (a[4 * e + 3] * f0 + bb[4 * e + 3] * f1) * inv);
        }
      }
      if (qr < rows && half == 0) lse2[(size_t)h * rows + qr] = mt + log2f(L);
    }
  } else if (tid == kTcProducer) {
    // ---------------------------------------------------------- producer
    for (int j = 0; j < n; ++j) {
      const int st = j % NS;
      if (j >= NS) {
        TC_WAIT_OR_FAIL(&kv_empty[st], ((j - NS) / NS) & 1);
      }
      tc::bar_expect_tx(&kv_full[st], A::FWD_STAGE * 4);
      tc::bulk_g2s(sm + st * A::FWD_STAGE, kfmt + ((size_t)h * nkt + kt0 + j) * F::KTILE, A::FWD_STAGE * 4,
                   &kv_full[st]);
    }
  } else if (tid == kTcIssuer) {
    // ---------------------------------------------------------- S issuer
    constexpr uint32_t idS = tc::idesc_tf32(kTcRows, kTcK, false, false);
    for (int j = 0; j < n; ++j) {
      const int st = j % NS, b = j & 1;
      const float* stage = sm + st * A::FWD_STAGE;
      TC_WAIT_OR_FAIL(&kv_full[st], (j / NS) & 1);
      if (j >= 2) {
        TC_WAIT_OR_FAIL(&s_empty[b], ((j - 2) >> 1) & 1);
      }
      tc::fence_after_sync();
      // S_j = Q K_j^T
      mma_tmem_a<HD>(tS + 64 * b, tQh, tQl, stage + F::K_HI * F::KPART, stage + F::K_LO * F::KPART, idS, false);
      tc::commit(&s_full[b]);
    }
  } else if (tid == kTcIssuer2) {
    // ---------------------------------------------------------- P.V issuer
    constexpr uint32_t idO = tc::idesc_tf32(kTcRows, HD, false, false);
    for (int j = 0; j < n; ++j) {
      const int st = j % NS;
      const float* stage = sm + st * A::FWD_STAGE;
      TC_WAIT_OR_FAIL(&p_full, j & 1);
      // Already complete (S_j read this stage); observed here as well so
      // the Vt bytes are ordered before this thread's MMAs.
      TC_WAIT_OR_FAIL(&kv_full[st], (j / NS) & 1);
      tc::fence_after_sync();
      // O_half += P[:, half] V[half keys]   (B = V^T tile, K-major over keys)
      const float* vh = stage + F::VT_HI * F::KPART;
      const float* vl = stage + F::VT_LO * F::KPART;
      mma_tmem_a_steps<kTcK, 4>(tO, tPh, tPl, vh, vl, idO, j > 0, 0);
      mma_tmem_a_steps<kTcK, 4>(tO + 64, tPh, tPl, vh, vl, idO, j > 0, 4);
      tc::commit(&o_done);
      tc::commit(&kv_empty[st]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (sh.failed && tid == 0) atomicExch(err, 1);
  if (warp == 0) tc::tmem_dealloc(t0, 512);
}

// ---------------------------------------------------------------------- dQ
// TMEM: Q hi | Q lo | dO hi | dO lo | S | dP then dS hi | dS lo | dQ
// Per key step: S = Q K^T, dP = dO V^T; dS = P (dP - delta) scale; dQ += dS K.
// dS hi overwrites dP, so S_{j+1} is issued as soon as the compute warps have
// read S_j, ahead of dQ_j's second half completing; only dP_{j+1} waits for
// dQ_j.  Thread 288 issues S and dP, thread 320 (an eleventh warp) dQ, so
// each issuer's mbarrier waits overlap the other's MMAs.
template <int HD>
__global__ void __launch_bounds__(kTcThreads2, 1)
    attention_backward_dq_tc(int rows, int W, int T, float scale, const float* __restrict__ q,
                             const float* __restrict__ dout, const float* __restrict__ kfmt,
                             const float* __restrict__ lse2, const float* __restrict__ delta, float* __restrict__ dq,
                             int* __restrict__ err) {
  using A = TcAtt<HD>;
  using F = TcFmt<HD>;
  constexpr int NS = A::DQ_STAGES;
  extern __shared__ __align__(128) float sm[];
  __shared__ uint64_t kv_full[NS], kv_empty[NS], s_full, d_full[2], q_done;
  __shared__ TcShared sh;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nt = (rows + kTcRows - 1) / kTcRows;
  const int q0 = tile_by_work(blockIdx.x, nt, rows, T, true) * kTcRows;
  const int h = blockIdx.y;
  const int nkt = (rows + kTcK - 1) / kTcK;
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, 512);
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) {
      tc::bar_init(&kv_full[b], 1);
      tc::bar_init(&kv_empty[b], 1);
    }
    tc::bar_init(&s_full, 1);
    tc::bar_init(&d_full[0], kTcCompute);
    tc::bar_init(&d_full[1], kTcCompute);
    tc::bar_init(&q_done, 1);
    tc::bar_init_fence();
    sh.failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t t0 = sh.tmem_base;
  const uint32_t tQh = t0, tQl = t0 + 64, tDh = t0 + 128, tDl = t0 + 192, tS = t0 + 256, tP = t0 + 320,
                 tSl = t0 + 384, tG = t0 + 448;
  const int kbeg = ((q0 - q0 % T) / kTcK) * kTcK;
  const int kend = min(rows, q0 + kTcRows);
  const int n = (kend - kbeg + kTcK - 1) / kTcK;
  const int kt0 = kbeg / kTcK;
  if (warp < 4) {
    const uint32_t lane = (uint32_t)(warp * 32) << 16;
    row_to_tmem<HD>(q, q0 + tid, rows, W, h, tQh + lane, tQl + lane);
    row_to_tmem<HD>(dout, q0 + tid, rows, W, h, tDh + lane, tDl + lane);
    tc::tmem_st_wait();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (tid < kTcCompute) {
    // Thread (row, half) handles key columns [32 half, 32 half + 32).
    const int row = tid & (kTcRows - 1), half = tid >> 7;
    const uint32_t lane = (uint32_t)((warp & 3) * 32) << 16;
    const float scale2 = scale * 1.4426950408889634f;
    const int qr = q0 + row, qs = qr - qr % T;
    const int seq0 = q0 - q0 % T;
    const bool one_seq = (q0 + kTcRows - 1) / T == q0 / T && q0 + kTcRows <= rows;
    const bool in = qr < rows;
    const float L = in ? lse2[(size_t)h * rows + qr] : 0.f;
    const float dl = in ? delta[(size_t)h * rows + qr] : 0.f;
    bool done = false;
    for (int j = 0; j < n; ++j) {
      TC_WAIT_OR_FAIL(&s_full, j & 1);
      tc::fence_after_sync();
      const int kt = kbeg + j * kTcK;
      // Key columns [32 k2 + 16 half, +16): the first 32 keys are handed to
      // the MMA thread (dQ += dS K) while the second 32 are computed.
      for (int k2 = 0; k2 < 2; ++k2) {
        const int col = 32 * k2 + 16 * half;
        float s[16], dp[16];
        tc::tmem_ld16_pair(tS + col + lane, s, tP + col + lane, dp);
        const bool full = one_seq && kt + 32 * k2 >= seq0 && kt + 32 * k2 + 31 <= q0;
        const int kh = kt + col;
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          const float2 t = fma2(make_float2(s[c], s[c + 1]), splat2(scale2), splat2(-L));
          const bool ok0 = full || (kh + c <= qr && kh + c >= qs && kh + c < rows);
          const bool ok1 = full || (kh + c + 1 <= qr && kh + c + 1 >= qs && kh + c + 1 < rows);
          const float2 p = make_float2(ok0 ? ex2(t.x) : 0.f, ok1 ? ex2(t.y) : 0.f);
          const float2 g = mul2(mul2(p, add2(make_float2(dp[c], dp[c + 1]), splat2(-dl))), splat2(scale));
          s[c] = g.x;
          s[c + 1] = g.y;
        }
        tc_st_split<16>(tP + col + lane, tSl + col + lane, s);  // dS hi over dP
        tc::tmem_st_wait();
        tc::fence_before_sync();
        tc::bar_arrive(&d_full[k2]);
      }
      if (j + 1 == n) done = true;
    }
    if (done && !tc::bar_wait(&q_done, (n - 1) & 1)) sh.failed = 1;
    tc::fence_after_sync();
    if (done && !sh.failed) {
#pragma unroll
      for (int c = 0; c < HD / 2; c += 16) {
        const int col = (HD / 2) * half + c;
        float gv[16];
        tc::tmem_ld16(tG + lane + col, gv);
        if (in) {
          float4* dst = reinterpret_cast<float4*>(dq + (size_t)qr * W + h * HD + col);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = make_float4(gv[4 * e], gv[4 * e + 1], gv[4 * e + 2], gv[4 * e + 3]);
        }
      }
    }
  } else if (tid == kTcProducer) {
    for (int j = 0; j < n; ++j) {
      const int st = j % NS;
      if (j >= NS) {
        TC_WAIT_OR_FAIL(&kv_empty[st], ((j - NS) / NS) & 1);
      }
      const float* tile = kfmt + ((size_t)h * nkt + kt0 + j) * F::KTILE;
      float* stage = sm + st * A::DQ_STAGE;
      tc::bar_expect_tx(&kv_full[st], A::DQ_STAGE * 4);
      tc::bulk_g2s(stage, tile + F::K_HI * F::KPART, 2 * F::KPART * 4, &kv_full[st]);                 // K, K'
      tc::bulk_g2s(stage + 2 * F::KPART, tile + F::V_HI * F::KPART, 4 * F::KPART * 4, &kv_full[st]);  // V, V', Kt, Kt'
    }
  } else if (tid == kTcIssuer) {
    // ---------------------------------------------------------- S / dP issuer
    constexpr uint32_t idS = tc::idesc_tf32(kTcRows, kTcK, false, false);
    for (int j = 0; j < n; ++j) {
      const int st = j % NS;
      const float* stage = sm + st * A::DQ_STAGE;  // K, K', V, V', Kt, Kt'
      TC_WAIT_OR_FAIL(&kv_full[st], (j / NS) & 1);
      if (j > 0) {
        TC_WAIT_OR_FAIL(&d_full[1], (j - 1) & 1);  // the compute warps have read S_{j-1}
      }
      tc::fence_after_sync();
      mma_tmem_a<HD>(tS, tQh, tQl, stage, stage + F::KPART, idS, false);  // S_j = Q K_j^T
      if (j > 0) {
        TC_WAIT_OR_FAIL(&q_done, (j - 1) & 1);  // dQ_{j-1} has read dS_{j-1} hi (the dP columns)
      }
      tc::fence_after_sync();
      mma_tmem_a<HD>(tP, tDh, tDl, stage + 2 * F::KPART, stage + 3 * F::KPART, idS, false);  // dP_j = dO V_j^T
      tc::commit(&s_full);
    }
  } else if (tid == kTcIssuer2) {
    // ---------------------------------------------------------- dQ issuer
    constexpr uint32_t idG = tc::idesc_tf32(kTcRows, HD, false, false);
    for (int j = 0; j < n; ++j) {
      const int st = j % NS;
      const float* stage = sm + st * A::DQ_STAGE;
      // Complete since S_j read this stage; observed so the Kt bytes are
      // ordered before this thread's MMAs.
      TC_WAIT_OR_FAIL(&kv_full[st], (j / NS) & 1);
      bool ok = true;
      for (int k2 = 0; k2 < 2 && ok; ++k2) {
        ok = tc::bar_wait(&d_full[k2], j & 1);
        tc::fence_after_sync();
        // dQ += dS K over keys [32 k2, 32 k2 + 32) (K steps 4 k2 .. 4 k2 + 3)
        if (ok)
          mma_tmem_a_steps<kTcK, 4>(tG, tP, tSl, stage + 4 * F::KPART, stage + 5 * F::KPART, idG,
                                    j > 0 || k2 > 0, 4 * k2);
      }
      if (!ok) {
        sh.failed = 1;
        break;
      }
      tc::commit(&q_done);
      tc::commit(&kv_empty[st]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (sh.failed && tid == 0) atomicExch(err, 1);
  if (warp == 0) tc::tmem_dealloc(t0, 512);
}

// ------------------------------------------------------------------- dK/dV
// A CTA owns 128 keys of one head and walks the later queries 64 at a time.
// Threads 0-255 compute (key row = tid % 128 = TMEM lane; thread half
// tid / 128 takes 16 of each 32-query half), warp 8 streams the A tile
// (Q, dO), warp 9 issues S^T and dP^T, warp 10 streams the B tile (Q^T,
// dO^T, LSE, delta), warp 11 issues dV and dK (two issuers, so each one's
// mbarrier waits overlap the other's MMAs).  K lives in TMEM, V in shared memory.  Per query step the
// tensor pipe runs S^T = K Q^T, dP^T = V dO^T (keys on lanes, N = 64
// queries), dV += P^T dO and dK += dS^T Q, and the softmax hides behind it:
//   * the P phase (P^T from S^T and LSE) runs while dP^T executes;
//   * the dS phase (dS^T from P^T, dP^T and delta, two 32-query halves)
//     runs while dV and the first half's dK execute;
//   * dV and dK complete on separate barriers, so the next step's S^T (over
//     the P^T columns) queues behind dK and only dP^T (over the dS^T
//     columns) waits for dK.
// TMEM: K hi | K lo | dV | dK | S^T then P^T hi | dP^T then dS^T hi | P^T lo
// | dS^T lo (64 columns each).
constexpr int kTcKvThreads = 384;
constexpr int kKvProducerA = 256, kKvIssuer = 288, kKvProducerB = 320, kKvIssuer2 = 352;

template <int HD>
struct TcKv {
  using F = TcFmt<HD>;
  static constexpr int A_FLOATS = 4 * F::QPART;             // Q, Q', dO, dO'
  static constexpr int B_FLOATS = 4 * F::QPART + 2 * kTcQ;  // Q^T, Q^T', dO^T, dO^T', lse2, delta
  static constexpr int V_FLOATS = 2 * kTcRows * HD;         // V hi, V lo
  static constexpr size_t smem = (size_t)(V_FLOATS + A_FLOATS + B_FLOATS) * sizeof(float);
};

// D (+)= A . B^T with A a K-major hi/lo shared tile [128 rows][KC columns].
template <int KC>
__device__ __forceinline__ void mma_smem_a(uint32_t d, const float* ah, const float* al, const float* bh,
                                           const float* bl, uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int s = 0; s < KC / 8; ++s) {
    const uint64_t a_h = tc::desc_kmajor(ah, KC, s), a_l = tc::desc_kmajor(al, KC, s);
    const uint64_t b_h = tc::desc_kmajor(bh, KC, s), b_l = tc::desc_kmajor(bl, KC, s);
    tc::mma_ss(d, a_h, b_h, idesc, (accumulate || s > 0) ? 1u : 0u);
    tc::mma_ss(d, a_h, b_l, idesc, 1u);
    tc::mma_ss(d, a_l, b_h, idesc, 1u);
  }
}

template <int HD>
__global__ void __launch_bounds__(kTcKvThreads, 1)
    attention_backward_dkdv_tc(int rows, int W, int T, float scale, const float* __restrict__ k,
                               const float* __restrict__ v, const float* __restrict__ qfmt,
                               const float* __restrict__ dv_add, float* __restrict__ dk, float* __restrict__ dv,
                               int* __restrict__ err) {
  using F = TcFmt<HD>;
  using S = TcKv<HD>;
  extern __shared__ __align__(128) float sm[];
  float* Vh = sm;
  float* Vl = sm + kTcRows * HD;
  float* tile_a = sm + S::V_FLOATS;
  float* tile_b = tile_a + S::A_FLOATS;
  __shared__ uint64_t a_full, a_empty, b_full, b_empty, s_full, dp_full, p_full, ds_full[2], v_done, g_done;
  __shared__ TcShared sh;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int k0 = tile_by_work(blockIdx.x, gridDim.x, rows, T, false) * kTcRows;
  const int h = blockIdx.y;
  const int nqt = (rows + kTcQ - 1) / kTcQ;
  if (warp == 0) tc::tmem_alloc(&sh.tmem_base, 512);
  if (tid == 0) {
    tc::bar_init(&a_full, 1);
    tc::bar_init(&a_empty, 1);
    tc::bar_init(&b_full, 1);
    tc::bar_init(&b_empty, 1);
    tc::bar_init(&s_full, 1);
    tc::bar_init(&dp_full, 1);
    tc::bar_init(&p_full, kTcCompute);
    tc::bar_init(&ds_full[0], kTcCompute);
    tc::bar_init(&ds_full[1], kTcCompute);
    tc::bar_init(&v_done, 1);
    tc::bar_init(&g_done, 1);
    tc::bar_init_fence();
    sh.failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t t0 = sh.tmem_base;
  const uint32_t tKh = t0, tKl = t0 + 64, tdV = t0 + 128, tdK = t0 + 192, tS = t0 + 256, tP = t0 + 320,
                 tPl = t0 + 384, tSl = t0 + 448;
  const int last = min(rows, k0 + kTcRows) - 1;
  const int qend = min(rows, (last / T + 1) * T);
  const int n = (qend - k0 + kTcQ - 1) / kTcQ;
  const int qt0 = k0 / kTcQ;
  // K through the (still idle) A tile into TMEM.
  stage_rows<HD>(tile_a, k, k0, rows, W, h, kTcKvThreads);
  __syncthreads();
  if (warp < 4) {
    const uint32_t lane = (uint32_t)(warp * 32) << 16;
    staged_row_to_tmem<HD>(tile_a, tid, tKh + lane, tKl + lane);
    tc::tmem_st_wait();
  }
  if (tid < kTcCompute) {
    // V rows of the CTA, split and stored in the blocked K-major layout.  All
    // loads are issued before the first shared-memory store, so they overlap.
    constexpr int PER = kTcRows * HD / 4 / kTcCompute;  // float4 per thread
    float4 x[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid + kTcCompute * j, r = i / (HD / 4), c = (i % (HD / 4)) * 4;
      x[j] = k0 + r < rows ? __ldg(reinterpret_cast<const float4*>(v + (size_t)(k0 + r) * W + h * HD + c))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = tid + kTcCompute * j, r = i / (HD / 4), c = (i % (HD / 4)) * 4;
      const float4 hv = make_float4(tc::tf32_hi(x[j].x), tc::tf32_hi(x[j].y), tc::tf32_hi(x[j].z),
                                    tc::tf32_hi(x[j].w));
      *reinterpret_cast<float4*>(Vh + tc::blk(r, c, HD)) = hv;
      *reinterpret_cast<float4*>(Vl + tc::blk(r, c, HD)) =
          make_float4(x[j].x - hv.x, x[j].y - hv.y, x[j].z - hv.z, x[j].w - hv.w);
    }
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (tid < kTcCompute) {
    // ---------------------------------------------------------- softmax
    const int row = tid & (kTcRows - 1), half = tid >> 7;
    const uint32_t lane = (uint32_t)(((tid >> 5) & 3) * 32) << 16;
    const float scale2 = scale * 1.4426950408889634f;
    const int kr = k0 + row;
    const int ke = (kr / T + 1) * T;  // end of the key's sequence
    // Every key row of the CTA in one sequence, so query halves wholly above
    // the diagonal and inside the sequence need no mask.
    const int kseq_end = (k0 / T + 1) * T;
    const bool one_seq = (k0 + kTcRows - 1) / T == k0 / T && k0 + kTcRows <= rows;
    const float* Ls0 = tile_b + 4 * F::QPART;  // lse2 of the query step
    const float* Es0 = Ls0 + kTcQ;             // delta of the query step
    bool done = false;
    for (int j = 0; j < n; ++j) {
      // P phase: P^T = exp2(S^T scale - lse) as soon as S^T is done, while
      // the tensor cores run dP^T; P stays in registers for the dS phase.
      TC_WAIT_OR_FAIL(&s_full, j & 1);
      TC_WAIT_OR_FAIL(&b_full, j & 1);
      tc::fence_after_sync();
      float pv[32];
      for (int q2 = 0; q2 < 2; ++q2) {
        // Columns [32 q2 + 16 half, +16) of this query step.
        const int col = 32 * q2 + 16 * half;
        const float* Ls = Ls0 + col;
        float s[16];
        tc::tmem_ld16(tS + col + lane, s);
        const int qh = k0 + j * kTcQ + col;
        const bool full = one_seq && k0 + j * kTcQ + 32 * q2 >= k0 + kTcRows - 1 &&
                          k0 + j * kTcQ + 32 * q2 + 32 <= min(kseq_end, rows);
#pragma unroll
        for (int c = 0; c < 16; c += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(Ls + c);
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            const float2 lv = u == 0 ? make_float2(l4.x, l4.y) : make_float2(l4.z, l4.w);
            const int q0j = qh + c + u;
            const float2 t = fma2(make_float2(s[c + u], s[c + u + 1]), splat2(scale2), make_float2(-lv.x, -lv.y));
            const bool ok0 = full || (q0j >= kr && q0j < ke && q0j < rows && kr < rows);
            const bool ok1 = full || (q0j + 1 >= kr && q0j + 1 < ke && q0j + 1 < rows && kr < rows);
            s[c + u] = ok0 ? ex2(t.x) : 0.f;
            s[c + u + 1] = ok1 ? ex2(t.y) : 0.f;
          }
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) pv[16 * q2 + c] = s[c];
        tc_st_split<16>(tS + col + lane, tPl + col + lane, s);  // P^T hi over S^T
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      tc::bar_arrive(&p_full);
      // dS phase: dS^T = P^T (dP^T - delta) scale, one 32-query half at a
      // time, while the tensor cores run dV and the first half's dK.
      TC_WAIT_OR_FAIL(&dp_full, j & 1);
      tc::fence_after_sync();
      for (int q2 = 0; q2 < 2; ++q2) {
        const int col = 32 * q2 + 16 * half;
        const float* Es = Es0 + col;
        float dp[16];
        tc::tmem_ld16(tP + col + lane, dp);
#pragma unroll
        for (int c = 0; c < 16; c += 4) {
          const float4 e4 = *reinterpret_cast<const float4*>(Es + c);
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            const float2 ev = u == 0 ? make_float2(e4.x, e4.y) : make_float2(e4.z, e4.w);
            const float2 pp = make_float2(pv[16 * q2 + c + u], pv[16 * q2 + c + u + 1]);
            const float2 g = mul2(mul2(pp, add2(make_float2(dp[c + u], dp[c + u + 1]), make_float2(-ev.x, -ev.y))),
                                  splat2(scale));
            dp[c + u] = g.x;
            dp[c + u + 1] = g.y;
          }
        }
        tc_st_split<16>(tP + col + lane, tSl + col + lane, dp);  // dS^T hi over dP^T
        tc::tmem_st_wait();
        tc::fence_before_sync();
        tc::bar_arrive(&ds_full[q2]);
      }
      if (j + 1 == n) done = true;
    }
    // dV and dK of the last step complete before the accumulators are read.
    if (done && !tc::bar_wait(&g_done, (n - 1) & 1)) sh.failed = 1;
    tc::fence_after_sync();
    if (done && !sh.failed) {
      const bool in = kr < rows;
#pragma unroll
      for (int c = 0; c < HD / 2; c += 16) {
        const int col = (HD / 2) * half + c;
        float gk[16], gv[16];
        tc::tmem_ld16_pair(tdK + lane + col, gk, tdV + lane + col, gv);
        if (in) {
          const size_t base = (size_t)kr * W + h * HD + col;  // 16-float aligned
          float4* dk4 = reinterpret_cast<float4*>(dk + base);
          float4* dv4 = reinterpret_cast<float4*>(dv + base);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float4 a = make_float4(gv[4 * e], gv[4 * e + 1], gv[4 * e + 2], gv[4 * e + 3]);
            if (dv_add != nullptr) {
              const float4 x = __ldg(reinterpret_cast<const float4*>(dv_add + base) + e);
              a = make_float4(a.x + x.x, a.y + x.y, a.z + x.z, a.w + x.w);
            }
            dk4[e] = make_float4(gk[4 * e], gk[4 * e + 1], gk[4 * e + 2], gk[4 * e + 3]);
            dv4[e] = a;
          }
        }
      }
    }
  } else if (tid == kKvProducerA) {
    // ---------------------------------------------------------- A tile: Q, dO
    for (int j = 0; j < n; ++j) {
      if (j >= 1) {
        TC_WAIT_OR_FAIL(&a_empty, (j - 1) & 1);
      }
      tc::bar_expect_tx(&a_full, S::A_FLOATS * 4);
      tc::bulk_g2s(tile_a, qfmt + ((size_t)h * nqt + qt0 + j) * F::QTILE, S::A_FLOATS * 4, &a_full);
    }
  } else if (tid == kKvProducerB) {
    // ---------------------------------------------------------- B tile: Q^T, dO^T, lse2, delta
    for (int j = 0; j < n; ++j) {
      if (j >= 1) {
        TC_WAIT_OR_FAIL(&b_empty, (j - 1) & 1);
      }
      tc::bar_expect_tx(&b_full, S::B_FLOATS * 4);
      tc::bulk_g2s(tile_b, qfmt + ((size_t)h * nqt + qt0 + j) * F::QTILE + 4 * F::QPART, S::B_FLOATS * 4,
                   &b_full);
    }
  } else if (tid == kKvIssuer) {
    // ---------------------------------------------------------- S^T / dP^T issuer
    constexpr uint32_t idS = tc::idesc_tf32(kTcRows, kTcQ, false, false);
    for (int j = 0; j < n; ++j) {
      TC_WAIT_OR_FAIL(&a_full, j & 1);
      if (j >= 1) {
        TC_WAIT_OR_FAIL(&v_done, (j - 1) & 1);  // dV of step j-1 has read P^T (the S^T columns)
      }
      tc::fence_after_sync();
      mma_tmem_a<HD>(tS, tKh, tKl, tile_a + F::Q_HI * F::QPART, tile_a + F::Q_LO * F::QPART, idS, false);  // S^T
      tc::commit(&s_full);
      if (j >= 1) {
        TC_WAIT_OR_FAIL(&g_done, (j - 1) & 1);  // dK of step j-1 has read dS^T (the dP^T columns)
      }
      tc::fence_after_sync();
      mma_smem_a<HD>(tP, Vh, Vl, tile_a + F::D_HI * F::QPART, tile_a + F::D_LO * F::QPART, idS, false);    // dP^T
      tc::commit(&dp_full);
      tc::commit(&a_empty);
    }
  } else if (tid == kKvIssuer2) {
    // ---------------------------------------------------------- dV / dK issuer
    constexpr uint32_t idG = tc::idesc_tf32(kTcRows, HD, false, false);
    const float* qt = tile_b;                   // Q^T, Q^T'
    const float* dot = tile_b + 2 * F::QPART;   // dO^T, dO^T'
    for (int j = 0; j < n; ++j) {
      TC_WAIT_OR_FAIL(&b_full, j & 1);
      TC_WAIT_OR_FAIL(&p_full, j & 1);
      tc::fence_after_sync();
      // dV += P^T dO over the step's 64 queries
      mma_tmem_a_steps<kTcQ, 8>(tdV, tS, tPl, dot, dot + F::QPART, idG, j > 0, 0);
      tc::commit(&v_done);
      bool ok = true;
      for (int q2 = 0; q2 < 2 && ok; ++q2) {
        ok = tc::bar_wait(&ds_full[q2], j & 1);
        tc::fence_after_sync();
        // dK += dS^T Q over queries [32 q2, 32 q2 + 32) (K steps 4 q2 .. 4 q2 + 3)
        if (ok) mma_tmem_a_steps<kTcQ, 4>(tdK, tP, tSl, qt, qt + F::QPART, idG, j > 0 || q2 > 0, 4 * q2);
      }
      if (!ok) {
        sh.failed = 1;
        break;
      }
      tc::commit(&g_done);
      tc::commit(&b_empty);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (sh.failed && tid == 0) atomicExch(err, 1);
  if (warp == 0) tc::tmem_dealloc(t0, 512);
}

#undef TC_WAIT_OR_FAIL

}  // namespace mb
