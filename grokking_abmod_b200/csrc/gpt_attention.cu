// FP32 causal flash attention (forward, dQ, dK/dV) for Mesh GPT on sm_100a.
//
// Semantics follow the reference's FA2 kernels (src/gpt/gpu.rs:381-750) and
// its f64 verifier (src/gpt/reference.rs:510-554): softmax(Q K^T / sqrt(hd))
// V with a causal mask that includes the diagonal, per sequence and head.
// Statistics are kept in base 2: lse2 = max(s log2e) + log2(sum), so backward
// recomputes P = exp2(s log2e - lse2).
//
// Tiling.  A CTA of 256 threads owns a 64-row tile of the flattened token
// rows for one head (tiles may span several short sequences; the mask tests
// "same sequence and key <= query").  Q/K/V/dO tiles sit in padded shared
// memory; each thread owns a 4 x 4 patch of the 64 x 64 score tile (rows
// ty*4+i, columns tx+16j) and a 4 x HD/16 patch of the 64 x HD output.  dQ and
// dK/dV run as separate kernels so no gradient needs atomics: results are
// bitwise reproducible.

#include "common.cuh"

namespace mb {

template <int HD>
struct Att {
  static constexpr int B = 64;          // rows per tile
  static constexpr int NT = 256;
  static constexpr int LD = HD + 4;     // padded stride of Q/K/V/dO tiles
  static constexpr int LP = B + 4;      // padded stride of P / dS tiles
  static constexpr int OC = HD / 16;    // output columns per thread
  static constexpr int TILE = B * LD;   // floats per operand tile
};

// Loads rows [r0, r0+64) of head h (columns h*hd .. h*hd+hd) into s[64][LD],
// zero-filling rows >= rows and columns >= hd.
template <int HD>
__device__ __forceinline__ void load_tile(float* s, const float* __restrict__ g, int r0, int rows, int W, int h,
                                          int hd) {
  using A = Att<HD>;
  constexpr int P2 = HD / 2;  // float2 per padded row
  for (int i = threadIdx.x; i < A::B * P2; i += A::NT) {
    const int r = i / P2, c2 = i % P2;
    float2 v = make_float2(0.f, 0.f);
    if (r0 + r < rows && 2 * c2 < hd) v = __ldg(reinterpret_cast<const float2*>(g + (size_t)(r0 + r) * W + h * hd) + c2);
    *reinterpret_cast<float2*>(s + r * A::LD + 2 * c2) = v;
  }
}

// acc[i][j] += sum_d a[ty*4+i][d] * b[tx+16j][d]
template <int HD>
__device__ __forceinline__ void tile_qk(float (&acc)[4][4], const float* a, const float* b, int ty, int tx) {
  using A = Att<HD>;
#pragma unroll 4
  for (int d = 0; d < HD; d += 4) {
    float4 av[4], bv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) av[i] = *reinterpret_cast<const float4*>(a + (ty * 4 + i) * A::LD + d);
#pragma unroll
    for (int j = 0; j < 4; ++j) bv[j] = *reinterpret_cast<const float4*>(b + (tx + 16 * j) * A::LD + d);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = fmaf(av[i].x, bv[j].x, acc[i][j]);
        acc[i][j] = fmaf(av[i].y, bv[j].y, acc[i][j]);
        acc[i][j] = fmaf(av[i].z, bv[j].z, acc[i][j]);
        acc[i][j] = fmaf(av[i].w, bv[j].w, acc[i][j]);
      }
  }
}

// out[i][c] += sum_j p[ty*4+i][j] * v[j][tx*OC+c]
template <int HD>
__device__ __forceinline__ void tile_pv(float (&out)[4][Att<HD>::OC], const float* p, const float* v, int ty,
                                        int tx) {
  using A = Att<HD>;
  constexpr int OC = A::OC;
#pragma unroll 2
  for (int j = 0; j < A::B; j += 4) {
    float4 pv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4*>(p + (ty * 4 + i) * A::LP + j);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      float vv[OC];
      const float* vr = v + (j + jj) * A::LD + tx * OC;
      if constexpr (OC % 4 == 0) {
#pragma unroll
        for (int c = 0; c < OC; c += 4) {
          const float4 t = *reinterpret_cast<const float4*>(vr + c);
          vv[c] = t.x; vv[c + 1] = t.y; vv[c + 2] = t.z; vv[c + 3] = t.w;
        }
      } else if constexpr (OC == 2) {
        float2 t = *reinterpret_cast<const float2*>(vr);
        vv[0] = t.x; vv[1] = t.y;
      } else {
        vv[0] = vr[0];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pj = jj == 0 ? pv[i].x : jj == 1 ? pv[i].y : jj == 2 ? pv[i].z : pv[i].w;
#pragma unroll
        for (int c = 0; c < OC; ++c) out[i][c] = fmaf(pj, vv[c], out[i][c]);
      }
    }
  }
}

template <int HD>
__device__ __forceinline__ void store_rows(float* g, const float (&o)[4][Att<HD>::OC], int r0,
                                           int rows, int W, int h, int hd, int ty, int tx, float scale_row[4],
                                           const float* add) {  // may alias g (element-wise in place)
  constexpr int OC = Att<HD>::OC;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= rows) continue;
#pragma unroll
    for (int c = 0; c < OC; ++c) {
      const int col = tx * OC + c;
      if (col < hd) {
        const size_t idx = (size_t)r * W + h * hd + col;
        float val = o[i][c] * scale_row[i];
        if (add != nullptr) val += add[idx];
        g[idx] = val;
      }
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(256)
    attention_forward(int rows, int W, int T, int hd, float scale, const float* __restrict__ q,
                      const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ o,
                      float* __restrict__ lse2) {
  using A = Att<HD>;
  constexpr int OC = A::OC;
  extern __shared__ float4 smem4[];
  float* Qs = reinterpret_cast<float*>(smem4);
  float* Ks = Qs + A::TILE;
  float* Vs = Ks + A::TILE;
  float* Ps = Vs + A::TILE;
  const int nt = (rows + A::B - 1) / A::B;
  const int q0 = (nt - 1 - blockIdx.x) * A::B;  // longest causal spans first
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ty = warp * 2 + lane / 16, tx = lane % 16;
  const float scale2 = scale * 1.4426950408889634f;
  load_tile<HD>(Qs, q, q0, rows, W, h, hd);
  int qr[4], qs[4];
  float m[4], l[4], out[4][OC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    qr[i] = q0 + ty * 4 + i;
    qs[i] = qr[i] - qr[i] % T;
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < OC; ++c) out[i][c] = 0.f;
  }
  const int kbeg = q0 - q0 % T;
  const int kend = min(rows, q0 + A::B);
  for (int kt = kbeg; kt < kend; kt += A::B) {
    __syncthreads();
    load_tile<HD>(Ks, k, kt, rows, W, h, hd);
    load_tile<HD>(Vs, v, kt, rows, W, h, hd);
    __syncthreads();
    float s[4][4] = {};
    tile_qk<HD>(s, Qs, Ks, ty, tx);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kr = kt + tx + 16 * j;
        const bool ok = kr <= qr[i] && kr >= qs[i] && kr < rows;
        s[i][j] = ok ? s[i][j] * scale2 : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[i], mx);
      const float alpha = mn == -INFINITY ? 1.0f : exp2f(m[i] - mn);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = mn == -INFINITY ? 0.f : exp2f(s[i][j] - mn);
        s[i][j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * alpha + rs;
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < OC; ++c) out[i][c] *= alpha;
#pragma unroll
      for (int j = 0; j < 4; ++j) Ps[(ty * 4 + i) * A::LP + tx + 16 * j] = s[i][j];
    }
    __syncthreads();
    tile_pv<HD>(out, Ps, Vs, ty, tx);
  }
  float inv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    inv[i] = l[i] > 0.f ? 1.0f / l[i] : 0.f;
    if (tx == 0 && qr[i] < rows) lse2[(size_t)h * rows + qr[i]] = m[i] + log2f(l[i]);
  }
  store_rows<HD>(o, out, q0, rows, W, h, hd, ty, tx, inv, nullptr);
}

template <int HD>
__global__ void __launch_bounds__(256)
    attention_backward_dq(int rows, int W, int T, int hd, float scale, const float* __restrict__ q,
                          const float* __restrict__ k, const float* __restrict__ v, const float* __restrict__ dout,
                          const float* __restrict__ lse2, const float* __restrict__ delta, float* __restrict__ dq) {
  using A = Att<HD>;
  constexpr int OC = A::OC;
  extern __shared__ float4 smem4[];
  float* Qs = reinterpret_cast<float*>(smem4);
  float* Ds = Qs + A::TILE;   // dO
  float* Ks = Ds + A::TILE;
  float* Vs = Ks + A::TILE;
  float* Ss = Vs + A::TILE;   // dS
  const int nt = (rows + A::B - 1) / A::B;
  const int q0 = (nt - 1 - blockIdx.x) * A::B;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ty = warp * 2 + lane / 16, tx = lane % 16;
  const float scale2 = scale * 1.4426950408889634f;
  load_tile<HD>(Qs, q, q0, rows, W, h, hd);
  load_tile<HD>(Ds, dout, q0, rows, W, h, hd);
  int qr[4], qs[4];
  float L[4], dl[4], acc[4][OC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    qr[i] = q0 + ty * 4 + i;
    qs[i] = qr[i] - qr[i] % T;
    const bool in = qr[i] < rows;
    L[i] = in ? lse2[(size_t)h * rows + qr[i]] : 0.f;
    dl[i] = in ? delta[(size_t)h * rows + qr[i]] : 0.f;
#pragma unroll
    for (int c = 0; c < OC; ++c) acc[i][c] = 0.f;
  }
  const int kbeg = q0 - q0 % T;
  const int kend = min(rows, q0 + A::B);
  for (int kt = kbeg; kt < kend; kt += A::B) {
    __syncthreads();
    load_tile<HD>(Ks, k, kt, rows, W, h, hd);
    load_tile<HD>(Vs, v, kt, rows, W, h, hd);
    __syncthreads();
    float s[4][4] = {}, dp[4][4] = {};
    tile_qk<HD>(s, Qs, Ks, ty, tx);
    tile_qk<HD>(dp, Ds, Vs, ty, tx);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kr = kt + tx + 16 * j;
        const bool ok = kr <= qr[i] && kr >= qs[i] && kr < rows;
        const float p = ok ? exp2f(s[i][j] * scale2 - L[i]) : 0.f;
        Ss[(ty * 4 + i) * A::LP + tx + 16 * j] = p * (dp[i][j] - dl[i]) * scale;
      }
    __syncthreads();
    tile_pv<HD>(acc, Ss, Ks, ty, tx);
  }
  float one[4] = {1.f, 1.f, 1.f, 1.f};
  store_rows<HD>(dq, acc, q0, rows, W, h, hd, ty, tx, one, nullptr);
}

template <int HD>
__global__ void __launch_bounds__(256)
    attention_backward_dkdv(int rows, int W, int T, int hd, float scale, const float* __restrict__ q,
                            const float* __restrict__ k, const float* __restrict__ v,
                            const float* __restrict__ dout, const float* __restrict__ lse2,
                            const float* __restrict__ delta, const float* dv_add, float* __restrict__ dk,
                            float* dv) {
  using A = Att<HD>;
  constexpr int OC = A::OC;
  extern __shared__ float4 smem4[];
  float* Ks = reinterpret_cast<float*>(smem4);
  float* Vs = Ks + A::TILE;
  float* Qs = Vs + A::TILE;
  float* Ds = Qs + A::TILE;
  float* Ps = Ds + A::TILE;
  float* Ss = Ps + A::B * A::LP;
  float* Ls = Ss + A::B * A::LP;  // lse2 of the query tile
  float* Es = Ls + A::B;          // delta of the query tile
  const int k0 = blockIdx.x * A::B;  // short causal spans are the later tiles: launch early tiles first
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ty = warp * 2 + lane / 16, tx = lane % 16;
  const float scale2 = scale * 1.4426950408889634f;
  load_tile<HD>(Ks, k, k0, rows, W, h, hd);
  load_tile<HD>(Vs, v, k0, rows, W, h, hd);
  int kr[4], ke[4];
  float gk[4][OC], gv[4][OC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    kr[i] = k0 + ty * 4 + i;
    ke[i] = (kr[i] / T + 1) * T;  // end of the key's sequence
#pragma unroll
    for (int c = 0; c < OC; ++c) gk[i][c] = gv[i][c] = 0.f;
  }
  const int last = min(rows, k0 + A::B) - 1;
  const int qend = min(rows, (last / T + 1) * T);
  for (int qt = k0; qt < qend; qt += A::B) {
    __syncthreads();
    load_tile<HD>(Qs, q, qt, rows, W, h, hd);
    load_tile<HD>(Ds, dout, qt, rows, W, h, hd);
    if (threadIdx.x < A::B) {
      const int r = qt + threadIdx.x;
      Ls[threadIdx.x] = r < rows ? lse2[(size_t)h * rows + r] : 0.f;
      Es[threadIdx.x] = r < rows ? delta[(size_t)h * rows + r] : 0.f;
    }
    __syncthreads();
    float s[4][4] = {}, dp[4][4] = {};
    tile_qk<HD>(s, Ks, Qs, ty, tx);
    tile_qk<HD>(dp, Vs, Ds, ty, tx);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tx + 16 * j;
      const int qrow = qt + c;
      const float Lq = Ls[c], Eq = Es[c];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool ok = qrow >= kr[i] && qrow < ke[i] && qrow < rows && kr[i] < rows;
        const float p = ok ? exp2f(s[i][j] * scale2 - Lq) : 0.f;
        Ps[(ty * 4 + i) * A::LP + c] = p;
        Ss[(ty * 4 + i) * A::LP + c] = p * (dp[i][j] - Eq) * scale;
      }
    }
    __syncthreads();
    tile_pv<HD>(gv, Ps, Ds, ty, tx);
    tile_pv<HD>(gk, Ss, Qs, ty, tx);
  }
  float one[4] = {1.f, 1.f, 1.f, 1.f};
  store_rows<HD>(dk, gk, k0, rows, W, h, hd, ty, tx, one, nullptr);
  store_rows<HD>(dv, gv, k0, rows, W, h, hd, ty, tx, one, dv_add);
}

template <int HD>
struct AttentionKernels {
  using A = Att<HD>;
  static size_t smem_forward() { return (size_t)(3 * A::TILE + A::B * A::LP) * sizeof(float); }
  static size_t smem_dq() { return (size_t)(4 * A::TILE + A::B * A::LP) * sizeof(float); }
  static size_t smem_dkdv() { return (size_t)(4 * A::TILE + 2 * A::B * A::LP + 2 * A::B) * sizeof(float); }
};

}  // namespace mb
