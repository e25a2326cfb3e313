// Fused Mesh GPT block kernels (forward and backward) for sm_100a.
//
// Per block the reference launches ~4A+F mesh layers, five RMSNorms, two
// RoPEs, XSA and five gradient additions as separate kernels, each making a
// full HBM round trip (src/gpt/gpu.rs:2177-2278, :2351-2502).  Here one
// row-tile kernel runs each row-local span of the block, keeping every
// intermediate in registers and shared memory:
//
//   qkv_forward    x -> RMSNorm -> {Q,K,V} meshes -> QK-Norm -> RoPE
//   post_forward   (O, V, x) -> XSA -> O mesh -> +x -> RMSNorm -> FFN mesh -> +x_mid
//   post_backward  recomputes the FFN and O meshes, backpropagates through
//                  them, RMSNorm and XSA, and emits dO, dV(XSA), dx_mid and
//                  the attention row statistic delta = dO . O
//   qkv_backward   recomputes Q/K/V meshes and QK-Norm, inverse RoPE,
//                  backpropagates to dx
//
// Mesh layers follow src/gpt/gpu.rs:103-146 (forward/backward) and
// :1087-1149 (edge gradients); RMSNorm :65-94/:1035-1077; RoPE :175-208;
// XSA :781-897.

#include "gpt_rows.cuh"

namespace mb {

template <class T>
__device__ __forceinline__ float2 ld2(const float* p, int row, int rows, int W, int cp) {
  if (row < rows) return __ldg(reinterpret_cast<const float2*>(p + (size_t)row * W) + cp);
  return make_float2(0.f, 0.f);
}

__device__ __forceinline__ void st2(float* p, int row, int rows, int W, int cp, float2 v) {
  if (row < rows) reinterpret_cast<float2*>(p + (size_t)row * W)[cp] = v;
}

// Per-head RMS (QK-Norm) of row k's pair: returns 1/rms of the pair's head,
// and the normalized pair in v.  inv_hw = 1 / head width.  Every thread of
// the CTA calls it at the same point (wide heads reduce through `red`).
template <bool WIDE, class T>
__device__ __forceinline__ float head_rmsnorm(const Ctx<T>& c, float2& v, int hp, float inv_hw, int k, float* red,
                                              int& phase) {
  float s = head_sum_any<WIDE, T>(c, v.x * v.x + v.y * v.y, hp, k, red, phase);
  float inv = rms_scale(s, inv_hw);
  v = v * inv;
  return inv;
}

// XSA's 1 / max(|v|, eps) from |v|^2 (src/gpt/gpu.rs:781-822).
__device__ __forceinline__ float xsa_scale(float sq) {
  return sq >= kXsaEpsilon * kXsaEpsilon ? rsqrtf(sq) : 1.0f / kXsaEpsilon;
}

template <int W, int RPT, class S>
__global__ void __launch_bounds__(RowTile<W, RPT>::NT)
    qkv_forward(Dims d, const float* __restrict__ x, const uint32_t* __restrict__ tokens,
                const float* __restrict__ emb, float* __restrict__ x_out, const float* __restrict__ wq,
                const float* __restrict__ wk, const float* __restrict__ wv, const float2* __restrict__ rope_cs,
                float* __restrict__ q_out, float* __restrict__ k_out, float* __restrict__ v_out) {
  using T = RowTile<W, RPT>;
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  float* bufs = smem;               // 2 exchange buffers
  float* red = smem + 2 * T::BUF;   // 2 * TR * WPR
  Ctx<T> c;
  int phase = 0;
  const int hp = S::head_pairs(d);
  const float inv_hw = 1.0f / (float)d.head_width;
  const RopeLane rope(c.cp, hp);
  const int ntiles = (d.rows + T::TR - 1) / T::TR;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float2 n[RPT];
    float inv[RPT];
    int pos[RPT];
    prefetch_next_tile<W, T::TR>(c.tid, tile, d.rows, tokens != nullptr ? nullptr : x, nullptr);
    tile_positions<T>(c, tile, d.sequence, pos);
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      const int r = tile * T::TR + c.row(k);
      if (tokens != nullptr) {
        // Block 0: the embedding lookup (src/gpt/gpu.rs:41-56) is fused here.
        n[k] = make_float2(0.f, 0.f);
        if (r < d.rows) {
          uint32_t t = __ldg(tokens + r);
          t = t < (uint32_t)d.vocab ? t : 0u;
          n[k] = __ldg(reinterpret_cast<const float2*>(emb + (size_t)t * W) + c.cp);
          if (x_out != nullptr) st2(x_out, r, d.rows, W, c.cp, n[k]);
        }
      } else {
        n[k] = ld2<T>(x, r, d.rows, W, c.cp);
      }
    }
    rmsnorm_rows<T>(c, n, inv, red, phase, W);
#pragma unroll 1
    for (int m = 0; m < 3; ++m) {
      // Selected, not indexed: a pointer array indexed by m would live in local memory.
      const float4* wg = reinterpret_cast<const float4*>(m == 0 ? wq : (m == 1 ? wk : wv));
      float* out = m == 0 ? q_out : (m == 1 ? k_out : v_out);
      float2 a[RPT];
#pragma unroll
      for (int k = 0; k < RPT; ++k) a[k] = n[k];
      mesh_forward<W, T, S::A, S::CONN>(c, d, a, wg, S::attn(d), bufs, false);
#pragma unroll
      for (int k = 0; k < RPT; ++k) {
        const int r = tile * T::TR + c.row(k);
        float2 v = a[k];
        if (m < 2) {
          head_rmsnorm<S::WIDE, T>(c, v, hp, inv_hw, k, red, phase);
          v = rope_any<S::WIDE, T>(c, rope, v, k, pos[k], rope_cs, false, bufs);
        }
        st2(out, r, d.rows, W, c.cp, v);
      }
      __syncthreads();
    }
  }
}

template <int W, int RPT, class S>
__global__ void __launch_bounds__(RowTile<W, RPT>::NT)
    post_forward(Dims d, const float* __restrict__ o, const float* __restrict__ v, const float* __restrict__ x,
                 const float* __restrict__ wo, const float* __restrict__ wf, float* __restrict__ xmid_out,
                 float* __restrict__ xnext_out) {
  using T = RowTile<W, RPT>;
  extern __shared__ float4 smem4[];
  float* smem = reinterpret_cast<float*>(smem4);
  float* bufs = smem;
  float* red = smem + 2 * T::BUF;
  Ctx<T> c;
  int phase = 0;
  const int hp = S::head_pairs(d);
  const int ntiles = (d.rows + T::TR - 1) / T::TR;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float2 a[RPT], res[RPT];
    prefetch_next_tile<W, T::TR>(c.tid, tile, d.rows, o, v, x);
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      const int r = tile * T::TR + c.row(k);
      float2 y = ld2<T>(o, r, d.rows, W, c.cp);
      float2 vv = ld2<T>(v, r, d.rows, W, c.cp);
      res[k] = ld2<T>(x, r, d.rows, W, c.cp);
      // XSA: z = y - (y.u)u, u = v / max(|v|, eps)   (src/gpt/gpu.rs:829-853)
      float sq = head_sum_any<S::WIDE, T>(c, vv.x * vv.x + vv.y * vv.y, hp, k, red, phase);
      float iv = xsa_scale(sq);
      float2 u = vv * iv;
      float proj = head_sum_any<S::WIDE, T>(c, y.x * u.x + y.y * u.y, hp, k, red, phase);
      a[k] = make_float2(y.x - proj * u.x, y.y - proj * u.y);
    }
    mesh_forward<W, T, S::A, S::CONN>(c, d, a, reinterpret_cast<const float4*>(wo), S::attn(d), bufs, false);
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      res[k] = res[k] + a[k];
      st2(xmid_out, tile * T::TR + c.row(k), d.rows, W, c.cp, res[k]);
      a[k] = res[k];
    }
    float inv[RPT];
    __syncthreads();
    rmsnorm_rows<T>(c, a, inv, red, phase, W);
    mesh_forward<W, T, S::F, S::CONN>(c, d, a, reinterpret_cast<const float4*>(wf), S::ffn(d), bufs, false);
#pragma unroll
    for (int k = 0; k < RPT; ++k) st2(xnext_out, tile * T::TR + c.row(k), d.rows, W, c.cp, res[k] + a[k]);
    __syncthreads();
  }
}

// Writes the per-thread edge-gradient slots of one mesh stack as the partial
// of (CTA, row lane): layout [slot][depth][W][2].
template <class T>
__device__ __forceinline__ void flush_partials(const Ctx<T>& c, const float4* acc, int depth, float* partial) {
  if (partial == nullptr) return;
  const int slot = blockIdx.x * T::RL + c.rl;
  float4* out = reinterpret_cast<float4*>(partial) + (size_t)slot * depth * T::PAIRS;
  for (int l = 0; l < depth; ++l) out[l * T::PAIRS + c.cp] = slot_to_params(acc[l * T::NT + c.tid]);
}

template <class T>
__device__ __forceinline__ void zero_slots(const Ctx<T>& c, float4* acc, int layers) {
  for (int l = 0; l < layers; ++l) acc[l * T::NT + c.tid] = make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int W, int RPT, class S>
__global__ void __launch_bounds__(RowTile<W, RPT>::NT, 3)
    post_backward(Dims d, const float* __restrict__ dxn, const float* __restrict__ xmid, const float* __restrict__ o,
                  const float* __restrict__ v, const float* __restrict__ wo, const float* __restrict__ wf,
                  float* __restrict__ do_out, float* __restrict__ dvx_out, float* __restrict__ dxm_out,
                  float* __restrict__ delta_out, float* __restrict__ part_o, float* __restrict__ part_f) {
  using T = RowTile<W, RPT>;
  extern __shared__ float4 smem4[];
  const int A = S::attn(d), F = S::ffn(d);
  const int dmax = F > A ? F : A;
  float4* acc_f = smem4;                 // F * NT slots
  float4* acc_o = smem4 + F * T::NT;     // A * NT slots
  float* smem = reinterpret_cast<float*>(smem4 + (F + A) * T::NT);
  float* bufs = smem;                              // dmax activation buffers
  float* xch = smem + dmax * T::BUF;               // 2 exchange buffers
  float* red = xch + 2 * T::BUF;
  Ctx<T> c;
  zero_slots<T>(c, acc_f, F);
  zero_slots<T>(c, acc_o, A);
  int phase = 0;
  const int hp = S::head_pairs(d);
  const int ntiles = (d.rows + T::TR - 1) / T::TR;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float2 g[RPT], n2[RPT], dy[RPT];
    float inv2[RPT];
    prefetch_next_tile<W, T::TR>(c.tid, tile, d.rows, dxn, xmid, o, v);
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      const int r = tile * T::TR + c.row(k);
      g[k] = ld2<T>(dxn, r, d.rows, W, c.cp);
      n2[k] = ld2<T>(xmid, r, d.rows, W, c.cp);
    }
    // FFN: x_next = x_mid + FFN(RMSNorm(x_mid)).
    rmsnorm_rows<T>(c, n2, inv2, red, phase, W);
    KeptInputs<T, S::F, S::CONN> kept_f;
    {
      float2 a[RPT];
#pragma unroll
      for (int k = 0; k < RPT; ++k) a[k] = n2[k];
      mesh_forward_kept<W, T, S::F, S::CONN>(c, d, a, reinterpret_cast<const float4*>(wf), F, bufs, kept_f);
    }
    // O and V of the attention path, in flight during the FFN backward.
    float2 y[RPT], vv[RPT];
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      const int r = tile * T::TR + c.row(k);
      y[k] = ld2<T>(o, r, d.rows, W, c.cp);
      vv[k] = ld2<T>(v, r, d.rows, W, c.cp);
      dy[k] = g[k];
    }
    mesh_backward_kept<W, T, S::F, S::CONN>(c, d, dy, reinterpret_cast<const float4*>(wf), F, bufs, xch, acc_f,
                                            kept_f);
    rmsnorm_rows_backward<T>(c, n2, inv2, dy, red, phase, W);
#pragma unroll
    for (int k = 0; k < RPT; ++k) g[k] = g[k] + dy[k];  // dx_mid
    // Attention output path: x_mid = x + Omesh(XSA(O, V)).
    float2 u[RPT];
    float proj[RPT], iv[RPT], sq[RPT];
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      sq[k] = head_sum_any<S::WIDE, T>(c, vv[k].x * vv[k].x + vv[k].y * vv[k].y, hp, k, red, phase);
      iv[k] = xsa_scale(sq[k]);
      u[k] = vv[k] * iv[k];
      proj[k] = head_sum_any<S::WIDE, T>(c, y[k].x * u[k].x + y[k].y * u[k].y, hp, k, red, phase);
    }
    __syncthreads();  // the FFN backward may still read bufs
    KeptInputs<T, S::A, S::CONN> kept_o;
    {
      float2 a[RPT];
#pragma unroll
      for (int k = 0; k < RPT; ++k) a[k] = make_float2(y[k].x - proj[k] * u[k].x, y[k].y - proj[k] * u[k].y);
      mesh_forward_kept<W, T, S::A, S::CONN>(c, d, a, reinterpret_cast<const float4*>(wo), A, bufs, kept_o);
    }
#pragma unroll
    for (int k = 0; k < RPT; ++k) dy[k] = g[k];
    mesh_backward_kept<W, T, S::A, S::CONN>(c, d, dy, reinterpret_cast<const float4*>(wo), A, bufs, xch, acc_o,
                                            kept_o);
    // XSA backward (src/gpt/gpu.rs:861-897); dy is dL/dz.
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      const int r = tile * T::TR + c.row(k);
      float gp = head_sum_any<S::WIDE, T>(c, dy[k].x * u[k].x + dy[k].y * u[k].y, hp, k, red, phase);
      float2 dO = make_float2(dy[k].x - gp * u[k].x, dy[k].y - gp * u[k].y);
      float2 dv;
      const bool above = sq[k] >= kXsaEpsilon * kXsaEpsilon;
      dv.x = -gp * y[k].x - proj[k] * dy[k].x;
      dv.y = -gp * y[k].y - proj[k] * dy[k].y;
      if (above) {
        dv.x += 2.0f * proj[k] * gp * u[k].x;
        dv.y += 2.0f * proj[k] * gp * u[k].y;
      }
      dv = dv * iv[k];
      float delta = head_sum_any<S::WIDE, T>(c, dO.x * y[k].x + dO.y * y[k].y, hp, k, red, phase);
      st2(do_out, r, d.rows, W, c.cp, dO);
      st2(dvx_out, r, d.rows, W, c.cp, dv);
      st2(dxm_out, r, d.rows, W, c.cp, g[k]);
      if ((c.cp % hp) == 0 && r < d.rows) delta_out[(size_t)(c.cp / hp) * d.rows + r] = delta;
    }
    __syncthreads();
  }
  flush_partials<T>(c, acc_f, F, part_f);
  flush_partials<T>(c, acc_o, A, part_o);
}

// Register budget: shared memory limits the backward kernels to three CTAs
// of 256 threads per SM at width 512, so ptxas gets the registers three CTAs
// allow (85) instead of spilling to fit CTAs that shared memory would not admit.
template <int W, int RPT, class S>
__global__ void __launch_bounds__(RowTile<W, RPT>::NT, 3)
    qkv_backward(Dims d, const float* __restrict__ dq, const float* __restrict__ dk, const float* __restrict__ dv,
                 const float* __restrict__ x, const float* __restrict__ dxm, const float* __restrict__ wq,
                 const float* __restrict__ wk, const float* __restrict__ wv, const float2* __restrict__ rope_cs,
                 float* __restrict__ dx_out, float* __restrict__ part_q, float* __restrict__ part_k,
                 float* __restrict__ part_v) {
  using T = RowTile<W, RPT>;
  extern __shared__ float4 smem4[];
  const int A = S::attn(d);
  float4* accs = smem4;  // 3 * A * NT slots
  float* smem = reinterpret_cast<float*>(smem4 + 3 * A * T::NT);
  float* bufs = smem;
  float* xch = smem + A * T::BUF;
  float* red = xch + 2 * T::BUF;
  Ctx<T> c;
  zero_slots<T>(c, accs, 3 * A);
  int phase = 0;
  const int hp = S::head_pairs(d);
  const float inv_hw = 1.0f / (float)d.head_width;
  const RopeLane rope(c.cp, hp);
  const int ntiles = (d.rows + T::TR - 1) / T::TR;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float2 n1[RPT], dn[RPT];
    float inv1[RPT];
    int pos[RPT];
    prefetch_next_tile<W, T::TR>(c.tid, tile, d.rows, x, dq, dk, dv, dxm);
    tile_positions<T>(c, tile, d.sequence, pos);
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      n1[k] = ld2<T>(x, tile * T::TR + c.row(k), d.rows, W, c.cp);
      dn[k] = make_float2(0.f, 0.f);
    }
    rmsnorm_rows<T>(c, n1, inv1, red, phase, W);
    // Unrolled over the three stacks: each copy has its pointers, QK-Norm
    // and RoPE branches fixed at compile time (80 registers, no spills).
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const float4* wg = reinterpret_cast<const float4*>(m == 0 ? wq : (m == 1 ? wk : wv));
      // The stack's output gradient (an L2 hit after the prefetch) is
      // requested before the forward recompute, which hides its latency;
      // loading one stack's rows at a time keeps the register budget.
      const float* gsrc = m == 0 ? dq : (m == 1 ? dk : dv);
      // The inverse RoPE's angles (Q and K, heads within a warp) are
      // requested with the rows.
      const bool early_rope = !S::WIDE && rope.hp > 1 && m < 2;
      float2 a[RPT], gm[RPT];
      float4 ang[RPT];
#pragma unroll
      for (int k = 0; k < RPT; ++k) {
        a[k] = n1[k];
        gm[k] = ld2<T>(gsrc, tile * T::TR + c.row(k), d.rows, W, c.cp);
        ang[k] = early_rope ? rope.angles(pos[k], rope_cs) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      __syncthreads();  // the previous mesh backward may still read bufs
      KeptInputs<T, S::A, S::CONN> kept;
      mesh_forward_kept<W, T, S::A, S::CONN>(c, d, a, wg, A, bufs, kept);
#pragma unroll
      for (int k = 0; k < RPT; ++k) {
        float2 gg = gm[k];
        if (m < 2) {
          // QK-Norm then RoPE in forward; backward: inverse RoPE, then the
          // per-head RMSNorm adjoint.
          float2 qn = a[k];
          float ih = head_rmsnorm<S::WIDE, T>(c, qn, hp, inv_hw, k, red, phase);
          gg = early_rope ? rope.rotate(gg, shfl_xor2(gg, rope.half), ang[k], true)
                          : rope_any<S::WIDE, T>(c, rope, gg, k, pos[k], rope_cs, true, xch);
          float dot = head_sum_any<S::WIDE, T>(c, gg.x * qn.x + gg.y * qn.y, hp, k, red, phase) * inv_hw;
          gg = make_float2(ih * (gg.x - qn.x * dot), ih * (gg.y - qn.y * dot));
        }
        gm[k] = gg;
      }
      mesh_backward_kept<W, T, S::A, S::CONN>(c, d, gm, wg, A, bufs, xch, accs + m * A * T::NT, kept);
#pragma unroll
      for (int k = 0; k < RPT; ++k) dn[k] = dn[k] + gm[k];
    }
    float2 gx[RPT];
#pragma unroll
    for (int k = 0; k < RPT; ++k) gx[k] = ld2<T>(dxm, tile * T::TR + c.row(k), d.rows, W, c.cp);
    rmsnorm_rows_backward<T>(c, n1, inv1, dn, red, phase, W);
#pragma unroll
    for (int k = 0; k < RPT; ++k) {
      const int r = tile * T::TR + c.row(k);
      st2(dx_out, r, d.rows, W, c.cp, gx[k] + dn[k]);
    }
  }
  __syncthreads();
  flush_partials<T>(c, accs, A, part_q);
  flush_partials<T>(c, accs + A * T::NT, A, part_k);
  flush_partials<T>(c, accs + 2 * A * T::NT, A, part_v);
}

// ---------------------------------------------------------------- host glue
template <int W, int RPT>
struct BlockKernels {
  using T = RowTile<W, RPT>;
  static size_t smem_forward() { return (size_t)(2 * T::BUF + 2 * T::TR * T::WPR) * sizeof(float); }
  static size_t smem_post_backward(int A, int F) {
    int dmax = A > F ? A : F;
    return (size_t)(A + F) * T::NT * sizeof(float4) + (size_t)((dmax + 2) * T::BUF + 2 * T::TR * T::WPR) * sizeof(float);
  }
  static size_t smem_qkv_backward(int A) {
    return (size_t)3 * A * T::NT * sizeof(float4) + (size_t)((A + 2) * T::BUF + 2 * T::TR * T::WPR) * sizeof(float);
  }
};

}  // namespace mb
