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
// tensor memory.  One thread per tile row: thread i of the 128-thread CTA owns
// TMEM lane i, so score rows are read with tcgen05.ld and softmax needs no
// shuffles.  The probability (or dS) tile is written back to TMEM as hi/lo
// parts and used directly as the A operand of the next MMA (A from TMEM).
// Shared-memory operand tiles use the blocked layout of tc05.cuh and are all
// K-major: an operand needed with its rows along N (V and K as the B of
// P.V / dS.K, Q and dO as the B of the dK / dV products) is stored
// transposed while it is split.  Thread 0
// issues the MMAs and commits them to an mbarrier; all waits are bounded and
// report through `err` instead of hanging.

#include "tc05.cuh"

namespace mb {

constexpr int kTcRows = 128;  // tile rows = TMEM lanes
constexpr int kTcCols = 64;   // keys per step (forward, dQ)
constexpr int kTcQ = 32;      // queries per step (dK/dV)

// Rows [r0, r0+R) of head h (columns h*hd .. h*hd+HD) -> hi/lo blocked tiles
// with HD columns; zero outside the matrix.
// (128 threads; every load is issued before the first split so the L2
// latencies overlap.)
template <int R, int HD>
__device__ __forceinline__ void tc_load_split(float* hi, float* lo, const float* __restrict__ g, int r0, int rows,
                                              int W, int h) {
  constexpr int C4 = HD / 4;
  constexpr int N = R * C4 / 128;
  float4 v[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    const int i = threadIdx.x + n * 128;
    const int rl = i & 7, c4 = (i >> 3) % C4, rh = (i >> 3) / C4;
    const int r = rh * 8 + rl;
    v[n] = r0 + r < rows ? __ldg(reinterpret_cast<const float4*>(g + (size_t)(r0 + r) * W + h * HD) + c4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int n = 0; n < N; ++n) {
    const int i = threadIdx.x + n * 128;
    const int rl = i & 7, c4 = (i >> 3) % C4, rh = (i >> 3) / C4;
    const int r = rh * 8 + rl;
    const float4 hv = make_float4(tc::tf32_hi(v[n].x), tc::tf32_hi(v[n].y), tc::tf32_hi(v[n].z), tc::tf32_hi(v[n].w));
    const int off = tc::blk(r, c4 * 4, HD);
    *reinterpret_cast<float4*>(hi + off) = hv;
    *reinterpret_cast<float4*>(lo + off) =
        make_float4(v[n].x - hv.x, v[n].y - hv.y, v[n].z - hv.z, v[n].w - hv.w);
  }
}

// Rows [r0, r0+R) of head h -> hi/lo blocked tiles of the TRANSPOSE
// ([HD rows][R columns]); zero outside the matrix.
template <int R, int HD>
__device__ __forceinline__ void tc_load_split_t(float* hi, float* lo, const float* __restrict__ g, int r0, int rows,
                                                int W, int h) {
  constexpr int C4 = HD / 4;
  constexpr int N = R * C4 / 128;
  float4 v[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    const int i = threadIdx.x + n * 128;
    const int r = i % R, c4 = i / R;
    v[n] = r0 + r < rows ? __ldg(reinterpret_cast<const float4*>(g + (size_t)(r0 + r) * W + h * HD) + c4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int n = 0; n < N; ++n) {
    const int i = threadIdx.x + n * 128;
    const int r = i % R, c4 = i / R;
    const float x[4] = {v[n].x, v[n].y, v[n].z, v[n].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float hv = tc::tf32_hi(x[j]);
      const int off = tc::blk(c4 * 4 + j, r, R);
      hi[off] = hv;
      lo[off] = x[j] - hv;
    }
  }
}

// 64 TMEM columns of this thread's lane.
__device__ __forceinline__ void tc_ld64(uint32_t taddr, float (&v)[64]) {
  tc::tmem_ld32(taddr, v);
  tc::tmem_ld32(taddr + 32, v + 32);
}

// Stores hi/lo TF32 parts of NC values into two TMEM column ranges.
template <int NC>
__device__ __forceinline__ void tc_st_split(uint32_t thi, uint32_t tlo, const float* v) {
#pragma unroll
  for (int c = 0; c < NC; c += 16) {
    float hi[16], lo[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      hi[j] = tc::tf32_hi(v[c + j]);
      lo[j] = v[c + j] - hi[j];
    }
    tc::tmem_st16(thi + c, hi);
    tc::tmem_st16(tlo + c, lo);
  }
}

// S (+)= A . B^T for K-major hi/lo tiles with HD columns (3 MMAs per K step).
template <int HD>
__device__ __forceinline__ void tc_mma_nt(uint32_t d, const float* ah, const float* al, const float* bh,
                                          const float* bl, uint32_t idesc) {
#pragma unroll
  for (int s = 0; s < HD / 8; ++s) {
    const uint64_t a_h = tc::desc_kmajor(ah, HD, s), a_l = tc::desc_kmajor(al, HD, s);
    const uint64_t b_h = tc::desc_kmajor(bh, HD, s), b_l = tc::desc_kmajor(bl, HD, s);
    tc::mma_ss(d, a_h, b_h, idesc, s > 0 ? 1u : 0u);
    tc::mma_ss(d, a_h, b_l, idesc, 1u);
    tc::mma_ss(d, a_l, b_h, idesc, 1u);
  }
}

// D (+)= A(TMEM hi/lo, KC K columns) . B^T, B given transposed as a K-major
// smem hi/lo tile [N rows][KC columns].
template <int KC>
__device__ __forceinline__ void tc_mma_tn(uint32_t d, uint32_t ah, uint32_t al, const float* bh, const float* bl,
                                          uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int s = 0; s < KC / 8; ++s) {
    const uint64_t b_h = tc::desc_kmajor(bh, KC, s), b_l = tc::desc_kmajor(bl, KC, s);
    tc::mma_ts(d, ah + 8 * s, b_h, idesc, (accumulate || s > 0) ? 1u : 0u);
    tc::mma_ts(d, ah + 8 * s, b_l, idesc, 1u);
    tc::mma_ts(d, al + 8 * s, b_h, idesc, 1u);
  }
}

template <int HD>
struct TcAtt {
  static constexpr int BIG = kTcRows * HD;    // floats of a 128-row operand tile
  static constexpr int SMALL = kTcCols * HD;  // floats of a 64-row operand tile
  static constexpr int QT = kTcQ * HD;        // floats of a 32-row operand tile
  static constexpr size_t smem_forward = (size_t)(2 * BIG + 4 * SMALL) * sizeof(float);
  static constexpr size_t smem_dq = (size_t)(4 * BIG + 6 * SMALL) * sizeof(float);
  static constexpr size_t smem_dkdv = (size_t)(4 * BIG + 8 * QT + 2 * kTcQ) * sizeof(float);
};

// ------------------------------------------------------------------ forward
template <int HD>
__global__ void __launch_bounds__(128, 1)
    attention_forward_tc(int rows, int W, int T, float scale, const float* __restrict__ q,
                         const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ o,
                         float* __restrict__ lse2, int* __restrict__ err) {
  using A = TcAtt<HD>;
  extern __shared__ __align__(128) float sm[];
  float* Qh = sm;
  float* Ql = Qh + A::BIG;
  float* Kh = Ql + A::BIG;
  float* Kl = Kh + A::SMALL;
  float* Vh = Kl + A::SMALL;
  float* Vl = Vh + A::SMALL;
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nt = (rows + kTcRows - 1) / kTcRows;
  const int q0 = (nt - 1 - (int)blockIdx.x) * kTcRows;  // longest causal spans first
  const int h = blockIdx.y;
  if (warp == 0) tc::tmem_alloc(&tmem_base, 256);
  if (tid == 0) {
    tc::bar_init(&bar_s, 1);
    tc::bar_init(&bar_o, 1);
    tc::bar_init_fence();
    failed = 0;
  }
  tc_load_split<kTcRows, HD>(Qh, Ql, q, q0, rows, W, h);
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t lane = (uint32_t)(warp * 32) << 16;
  const uint32_t tS = tmem_base, tPh = tS + 64, tPl = tS + 128, tO = tS + 192;
  constexpr uint32_t idS = tc::idesc_tf32(kTcRows, kTcCols, false, false);
  constexpr uint32_t idO = tc::idesc_tf32(kTcRows, HD, false, false);
  const float scale2 = scale * 1.4426950408889634f;
  const int qr = q0 + tid, qs = qr - qr % T;
  float m = -INFINITY, l = 0.f;
  const int kbeg = q0 - q0 % T, kend = min(rows, q0 + kTcRows);
  uint32_t ph_s = 0, ph_o = 0;
  bool first = true;
  for (int kt = kbeg; kt < kend; kt += kTcCols) {
    if (!first) {
      if (!tc::bar_wait(&bar_o, ph_o)) failed = 1;  // P.V of the previous step done
      ph_o ^= 1;
    }
    tc_load_split<kTcCols, HD>(Kh, Kl, k, kt, rows, W, h);
    tc_load_split_t<kTcCols, HD>(Vh, Vl, v, kt, rows, W, h);  // V^T [HD][64]
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (failed) break;
    if (tid == 0) {
      tc::fence_after_sync();
      tc_mma_nt<HD>(tS, Qh, Ql, Kh, Kl, idS);
      tc::commit(&bar_s);
    }
    if (!tc::bar_wait(&bar_s, ph_s)) failed = 1;
    ph_s ^= 1;
    tc::fence_after_sync();
    float s[64];
    tc_ld64(tS + lane, s);
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const int kr = kt + j;
      const bool ok = kr <= qr && kr >= qs && kr < rows;
      s[j] = ok ? s[j] * scale2 : -INFINITY;
      mx = fmaxf(mx, s[j]);
    }
    const float mn = fmaxf(m, mx);
    const float alpha = mn == -INFINITY ? 1.0f : exp2f(m - mn);
    float rs = 0.f;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      s[j] = mn == -INFINITY ? 0.f : exp2f(s[j] - mn);
      rs += s[j];
    }
    l = l * alpha + rs;
    m = mn;
    if (!first) {
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        float ov[16];
        tc::tmem_ld16(tO + lane + c, ov);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) ov[j] *= alpha;
        tc::tmem_st16(tO + lane + c, ov);
      }
    }
    tc_st_split<64>(tPh + lane, tPl + lane, s);
    tc::tmem_st_wait();
    tc::fence_before_sync();
    __syncthreads();
    if (failed) break;
    if (tid == 0) {
      tc::fence_after_sync();
      tc_mma_tn<kTcCols>(tO, tPh, tPl, Vh, Vl, idO, !first);
      tc::commit(&bar_o);
    }
    first = false;
  }
  if (!first && !failed) {
    if (!tc::bar_wait(&bar_o, ph_o)) failed = 1;
  }
  tc::fence_after_sync();
  __syncthreads();
  if (!failed) {
    const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
    for (int c = 0; c < HD; c += 16) {
      float ov[16];
      tc::tmem_ld16(tO + lane + c, ov);
      tc::tmem_ld_wait();
      if (qr < rows && !first) {
        float4* dst = reinterpret_cast<float4*>(o + (size_t)qr * W + h * HD + c);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] = make_float4(ov[4 * j] * inv, ov[4 * j + 1] * inv, ov[4 * j + 2] * inv, ov[4 * j + 3] * inv);
      }
    }
    if (qr < rows) lse2[(size_t)h * rows + qr] = m + log2f(l);
  } else if (tid == 0) {
    atomicExch(err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem_base, 256);
}

// ---------------------------------------------------------------------- dQ
template <int HD>
__global__ void __launch_bounds__(128, 1)
    attention_backward_dq_tc(int rows, int W, int T, float scale, const float* __restrict__ q,
                             const float* __restrict__ k, const float* __restrict__ v,
                             const float* __restrict__ dout, const float* __restrict__ lse2,
                             const float* __restrict__ delta, float* __restrict__ dq, int* __restrict__ err) {
  using A = TcAtt<HD>;
  extern __shared__ __align__(128) float sm[];
  float* Qh = sm;
  float* Ql = Qh + A::BIG;
  float* Dh = Ql + A::BIG;  // dO
  float* Dl = Dh + A::BIG;
  float* Kh = Dl + A::BIG;
  float* Kl = Kh + A::SMALL;
  float* Vh = Kl + A::SMALL;
  float* Vl = Vh + A::SMALL;
  float* Th = Vl + A::SMALL;  // K^T [HD][64]
  float* Tl = Th + A::SMALL;
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int nt = (rows + kTcRows - 1) / kTcRows;
  const int q0 = (nt - 1 - (int)blockIdx.x) * kTcRows;
  const int h = blockIdx.y;
  if (warp == 0) tc::tmem_alloc(&tmem_base, 512);
  if (tid == 0) {
    tc::bar_init(&bar_s, 1);
    tc::bar_init(&bar_o, 1);
    tc::bar_init_fence();
    failed = 0;
  }
  tc_load_split<kTcRows, HD>(Qh, Ql, q, q0, rows, W, h);
  tc_load_split<kTcRows, HD>(Dh, Dl, dout, q0, rows, W, h);
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t lane = (uint32_t)(warp * 32) << 16;
  const uint32_t tS = tmem_base, tP = tS + 64, tSh = tS + 128, tSl = tS + 192, tQ = tS + 256;
  constexpr uint32_t idS = tc::idesc_tf32(kTcRows, kTcCols, false, false);
  constexpr uint32_t idQ = tc::idesc_tf32(kTcRows, HD, false, false);
  const float scale2 = scale * 1.4426950408889634f;
  const int qr = q0 + tid, qs = qr - qr % T;
  const bool in = qr < rows;
  const float L = in ? lse2[(size_t)h * rows + qr] : 0.f;
  const float dl = in ? delta[(size_t)h * rows + qr] : 0.f;
  const int kbeg = q0 - q0 % T, kend = min(rows, q0 + kTcRows);
  uint32_t ph_s = 0, ph_o = 0;
  bool first = true;
  for (int kt = kbeg; kt < kend; kt += kTcCols) {
    if (!first) {
      if (!tc::bar_wait(&bar_o, ph_o)) failed = 1;
      ph_o ^= 1;
    }
    tc_load_split<kTcCols, HD>(Kh, Kl, k, kt, rows, W, h);
    tc_load_split<kTcCols, HD>(Vh, Vl, v, kt, rows, W, h);
    tc_load_split_t<kTcCols, HD>(Th, Tl, k, kt, rows, W, h);
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (failed) break;
    if (tid == 0) {
      tc::fence_after_sync();
      tc_mma_nt<HD>(tS, Qh, Ql, Kh, Kl, idS);  // S  = Q K^T
      tc_mma_nt<HD>(tP, Dh, Dl, Vh, Vl, idS);  // dP = dO V^T
      tc::commit(&bar_s);
    }
    if (!tc::bar_wait(&bar_s, ph_s)) failed = 1;
    ph_s ^= 1;
    tc::fence_after_sync();
    float s[64], dp[64];
    tc_ld64(tS + lane, s);
    tc_ld64(tP + lane, dp);
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const int kr = kt + j;
      const bool ok = kr <= qr && kr >= qs && kr < rows;
      const float p = ok ? exp2f(s[j] * scale2 - L) : 0.f;
      s[j] = p * (dp[j] - dl) * scale;
    }
    tc_st_split<64>(tSh + lane, tSl + lane, s);
    tc::tmem_st_wait();
    tc::fence_before_sync();
    __syncthreads();
    if (failed) break;
    if (tid == 0) {
      tc::fence_after_sync();
      tc_mma_tn<kTcCols>(tQ, tSh, tSl, Th, Tl, idQ, !first);  // dQ += dS K
      tc::commit(&bar_o);
    }
    first = false;
  }
  if (!first && !failed) {
    if (!tc::bar_wait(&bar_o, ph_o)) failed = 1;
  }
  tc::fence_after_sync();
  __syncthreads();
  if (!failed) {
#pragma unroll
    for (int c = 0; c < HD; c += 16) {
      float ov[16];
      tc::tmem_ld16(tQ + lane + c, ov);
      tc::tmem_ld_wait();
      if (in && !first) {
        float4* dst = reinterpret_cast<float4*>(dq + (size_t)qr * W + h * HD + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[j] = make_float4(ov[4 * j], ov[4 * j + 1], ov[4 * j + 2], ov[4 * j + 3]);
      }
    }
  } else if (tid == 0) {
    atomicExch(err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------- dK/dV
// A CTA owns 128 keys of one head and walks the later queries 32 at a time:
// S^T = K Q^T and dP^T = V dO^T (keys on TMEM lanes), P^T and dS^T go back to
// TMEM as hi/lo parts, then dV += P^T dO and dK += dS^T Q with Q^T / dO^T
// staged transposed.
template <int HD>
__global__ void __launch_bounds__(128, 1)
    attention_backward_dkdv_tc(int rows, int W, int T, float scale, const float* __restrict__ q,
                               const float* __restrict__ k, const float* __restrict__ v,
                               const float* __restrict__ dout, const float* __restrict__ lse2,
                               const float* __restrict__ delta, const float* __restrict__ dv_add,
                               float* __restrict__ dk, float* __restrict__ dv, int* __restrict__ err) {
  using A = TcAtt<HD>;
  extern __shared__ __align__(128) float sm[];
  float* Kh = sm;
  float* Kl = Kh + A::BIG;
  float* Vh = Kl + A::BIG;
  float* Vl = Vh + A::BIG;
  float* Qh = Vl + A::BIG;    // Q   [32][HD]
  float* Ql = Qh + A::QT;
  float* Dh = Ql + A::QT;     // dO  [32][HD]
  float* Dl = Dh + A::QT;
  float* Qth = Dl + A::QT;    // Q^T [HD][32]
  float* Qtl = Qth + A::QT;
  float* Dth = Qtl + A::QT;   // dO^T [HD][32]
  float* Dtl = Dth + A::QT;
  float* Ls = Dtl + A::QT;    // lse2 of the query step
  float* Es = Ls + kTcQ;      // delta of the query step
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int k0 = blockIdx.x * kTcRows;
  const int h = blockIdx.y;
  if (warp == 0) tc::tmem_alloc(&tmem_base, 512);
  if (tid == 0) {
    tc::bar_init(&bar_s, 1);
    tc::bar_init(&bar_o, 1);
    tc::bar_init_fence();
    failed = 0;
  }
  tc_load_split<kTcRows, HD>(Kh, Kl, k, k0, rows, W, h);
  tc_load_split<kTcRows, HD>(Vh, Vl, v, k0, rows, W, h);
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t lane = (uint32_t)(warp * 32) << 16;
  // S^T then P^T hi | dP^T then dS^T hi | P^T lo | dS^T lo | dV | dK
  const uint32_t tS = tmem_base, tP = tS + 32, tPl = tS + 64, tSl = tS + 96, tV = tS + 128, tK = tS + 128 + HD;
  constexpr uint32_t idS = tc::idesc_tf32(kTcRows, kTcQ, false, false);
  constexpr uint32_t idG = tc::idesc_tf32(kTcRows, HD, false, false);
  const float scale2 = scale * 1.4426950408889634f;
  const int kr = k0 + tid;
  const int ke = (kr / T + 1) * T;  // end of the key's sequence
  const int last = min(rows, k0 + kTcRows) - 1;
  const int qend = min(rows, (last / T + 1) * T);
  uint32_t ph_s = 0, ph_o = 0;
  bool first = true;
  for (int qt = k0; qt < qend; qt += kTcQ) {
    if (!first) {
      if (!tc::bar_wait(&bar_o, ph_o)) failed = 1;
      ph_o ^= 1;
    }
    tc_load_split<kTcQ, HD>(Qh, Ql, q, qt, rows, W, h);
    tc_load_split<kTcQ, HD>(Dh, Dl, dout, qt, rows, W, h);
    tc_load_split_t<kTcQ, HD>(Qth, Qtl, q, qt, rows, W, h);
    tc_load_split_t<kTcQ, HD>(Dth, Dtl, dout, qt, rows, W, h);
    if (tid < kTcQ) {
      const int r = qt + tid;
      Ls[tid] = r < rows ? lse2[(size_t)h * rows + r] : 0.f;
      Es[tid] = r < rows ? delta[(size_t)h * rows + r] : 0.f;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (failed) break;
    if (tid == 0) {
      tc::fence_after_sync();
      tc_mma_nt<HD>(tS, Kh, Kl, Qh, Ql, idS);  // S^T  = K Q^T
      tc_mma_nt<HD>(tP, Vh, Vl, Dh, Dl, idS);  // dP^T = V dO^T
      tc::commit(&bar_s);
    }
    if (!tc::bar_wait(&bar_s, ph_s)) failed = 1;
    ph_s ^= 1;
    tc::fence_after_sync();
    float s[kTcQ], dp[kTcQ];
    tc::tmem_ld32(tS + lane, s);
    tc::tmem_ld32(tP + lane, dp);
#pragma unroll
    for (int j = 0; j < kTcQ; ++j) {
      const int qj = qt + j;
      const bool ok = qj >= kr && qj < ke && qj < rows && kr < rows;
      const float p = ok ? exp2f(s[j] * scale2 - Ls[j]) : 0.f;
      s[j] = p;
      dp[j] = p * (dp[j] - Es[j]) * scale;
    }
    tc_st_split<kTcQ>(tS + lane, tPl + lane, s);   // P^T hi over S^T
    tc_st_split<kTcQ>(tP + lane, tSl + lane, dp);  // dS^T hi over dP^T
    tc::tmem_st_wait();
    tc::fence_before_sync();
    __syncthreads();
    if (failed) break;
    if (tid == 0) {
      tc::fence_after_sync();
      tc_mma_tn<kTcQ>(tV, tS, tPl, Dth, Dtl, idG, !first);  // dV += P^T dO
      tc_mma_tn<kTcQ>(tK, tP, tSl, Qth, Qtl, idG, !first);  // dK += dS^T Q
      tc::commit(&bar_o);
    }
    first = false;
  }
  if (!first && !failed) {
    if (!tc::bar_wait(&bar_o, ph_o)) failed = 1;
  }
  tc::fence_after_sync();
  __syncthreads();
  if (!failed) {
    const bool in = kr < rows && !first;
#pragma unroll
    for (int c = 0; c < HD; c += 16) {
      float gk[16], gv[16];
      tc::tmem_ld16(tK + lane + c, gk);
      tc::tmem_ld16(tV + lane + c, gv);
      if (in) {
        const size_t base = (size_t)kr * W + h * HD + c;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          dk[base + j] = gk[j];
          dv[base + j] = gv[j] + (dv_add != nullptr ? dv_add[base + j] : 0.f);
        }
      }
    }
  } else if (tid == 0) {
    atomicExch(err, 1);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem_base, 512);
}

}  // namespace mb
