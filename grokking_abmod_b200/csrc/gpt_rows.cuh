// Row-tile engine for the Mesh GPT block kernels.
//
// A CTA owns a tile of TR token rows of width W.  Thread (rl, cp) owns the
// channel pair (2cp, 2cp+1) of rows rl, rl+RL, ... (RPT rows), keeps those
// values in registers, and exchanges neighbour channels through shared memory
// once per mesh layer.  Per-edge weight gradients accumulate per thread (no
// atomics) and are written as per-(CTA, row-lane) partials that a separate
// kernel reduces in a fixed order, so every result is bitwise reproducible.
//
// Shared-memory row buffers hold the even channels of a row in its first
// W/2 floats and the odd channels in the second W/2 (see Planes), so each
// thread's pair and every neighbour read of any stride are unit-stride,
// bank-conflict-free accesses.
#pragma once

#include "common.cuh"

namespace mb {

template <int W, int RPT_>
struct RowTile {
  static_assert(W % 64 == 0 && W >= 64 && W <= 1024, "width must be a multiple of 64 in 64..1024");
  static constexpr int PAIRS = W / 2;
  static constexpr int RL = PAIRS >= 256 ? 1 : 256 / PAIRS;  // row lanes
  static constexpr int NT = PAIRS * RL;                        // threads per CTA
  static constexpr int RPT = RPT_;                             // rows per thread
  static constexpr int TR = RL * RPT;                          // rows per tile
  static constexpr int WPR = PAIRS / 32;                       // warps per row
  static constexpr int BUF = TR * W;                           // floats per tile buffer
};

// Parameters every block kernel needs.
struct Dims {
  int rows;          // token rows N (a multiple of sequence)
  int sequence;      // T
  int heads;         // H
  int head_width;    // W / H
  int vocab;         // V
  int attn_depth;    // A
  int ffn_depth;     // F
  int connectivity;  // 0 = neighbor (stride 1), 1 = butterfly
  int log2w;         // floor(log2 W)
};

__device__ __forceinline__ int mesh_stride(const Dims& d, int layer) {
  // src/gpt/config.rs:117-122
  return d.connectivity == 0 ? 1 : (1 << (layer % d.log2w));
}

// Mesh-stack shape fixed at compile time: attention and FFN depths (0 = read
// from Dims at run time) and connectivity (-1 = read from Dims).  With a
// fixed shape the layer loops unroll, so every stride, shared-memory offset
// and weight address is a constant instead of per-layer integer work.
// WIDE_: heads of 128 channels or more (hp > 32 pairs), whose per-head
// sums and RoPE partners cross warps (head_sum_any, rope_any); the common
// shapes compile without that path.  HP_: channel pairs per head fixed at
// compile time (0 = head_width / 2 read at run time), so the per-head
// shuffle sums and head indexing need no run-time dispatch.
template <int A_, int F_, int CONN_, bool WIDE_ = false, int HP_ = 0>
struct MeshShape {
  static constexpr int A = A_, F = F_, CONN = CONN_, HP = HP_;
  static constexpr bool WIDE = WIDE_;
  __device__ static __forceinline__ int attn(const Dims& d) { return A > 0 ? A : d.attn_depth; }
  __device__ static __forceinline__ int ffn(const Dims& d) { return F > 0 ? F : d.ffn_depth; }
  __device__ static __forceinline__ int head_pairs(const Dims& d) { return HP > 0 ? HP : d.head_width / 2; }
};
using RuntimeShape = MeshShape<0, 0, -1>;
using RuntimeShapeWide = MeshShape<0, 0, -1, true>;

// floor(log2 W), the butterfly period (Dims::log2w).
template <int W>
__host__ __device__ constexpr int floor_log2() {
  int r = 0;
  while ((2 << r) <= W) ++r;
  return r;
}

template <int W, int CONN>
__device__ __forceinline__ int layer_stride(const Dims& d, int layer) {
  if constexpr (CONN == 0) {
    return 1;
  } else if constexpr (CONN == 1) {
    return 1 << (layer % floor_log2<W>());
  } else {
    return mesh_stride(d, layer);
  }
}

// body(l) for l = 0 .. n-1 (or n-1 .. 0 with `reverse`): unrolled when the
// count N is a compile-time constant, a rolled loop otherwise.
template <int N, bool reverse, class F>
__device__ __forceinline__ void layer_loop(int n, F&& body) {
  if constexpr (N > 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) body(reverse ? N - 1 - i : i);
  } else {
#pragma unroll 1
    for (int i = 0; i < n; ++i) body(reverse ? n - 1 - i : i);
  }
}

template <class T>
struct Ctx {
  int tid, rl, cp, lane, warp;
  // Plane indices of the stride-1 neighbours, fixed per thread: the even
  // channel of pair cp + 1 and the odd channel of pair cp - 1 (both mod P).
  int nxt, prv;
  __device__ Ctx() {
    tid = threadIdx.x;
    rl = tid / T::PAIRS;
    cp = tid % T::PAIRS;
    lane = tid & 31;
    warp = tid >> 5;
    nxt = cp + 1 == T::PAIRS ? 0 : cp + 1;
    prv = T::PAIRS + (cp == 0 ? T::PAIRS - 1 : cp - 1);
  }
  __device__ __forceinline__ int row(int k) const { return k * T::RL + rl; }
};

// One shared row of W channels as an even plane (row[cp] = x[2cp]) and an
// odd plane (row[P + cp] = x[2cp + 1]).
template <int W>
struct Planes {
  static constexpr int P = W / 2;
  __device__ static __forceinline__ void put(float* row, int cp, float2 v) {
    row[cp] = v.x;
    row[P + cp] = v.y;
  }
  __device__ static __forceinline__ float2 get(const float* row, int cp) { return make_float2(row[cp], row[P + cp]); }
  // Channels (2cp + s, 2cp + 1 + s) mod W for an even shift |s| <= W / 2.
  __device__ static __forceinline__ float2 shifted_even(const float* row, int cp, int s) {
    int h = cp + s / 2;
    h = h >= P ? h - P : (h < 0 ? h + P : h);
    return get(row, h);
  }
};

// Full-row sums (heads = 1) of one value per owned row.  `red` holds
// 2 * TR * WPR floats; `phase` alternates the halves so back-to-back
// reductions need one barrier each.
template <class T>
__device__ __forceinline__ void row_sums(const Ctx<T>& c, float (&v)[T::RPT], float* red, int& phase) {
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) v[k] = group_sum<32>(v[k]);
  if constexpr (T::WPR > 1) {
    float* r = red + phase * T::TR * T::WPR;
    phase ^= 1;
    const int wir = c.cp >> 5;  // warp index within the row
    if (c.lane == 0) {
#pragma unroll
      for (int k = 0; k < T::RPT; ++k) r[c.row(k) * T::WPR + wir] = v[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < T::RPT; ++k) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < T::WPR; ++j) s += r[c.row(k) * T::WPR + j];
      v[k] = s;
    }
  }
}

// 1 / sqrt(mean + eps) of a sum of squares over `count` values, with
// inv_count = 1 / count (src/gpt/gpu.rs:65-94).  rsqrtf is the hardware
// reciprocal square root (a couple of ulp), well inside the tolerances.
__device__ __forceinline__ float rms_scale(float sum_sq, float inv_count) {
  return rsqrtf(sum_sq * inv_count + kRmsEpsilon);
}

// Per-head sums over hp = head_width/2 consecutive lanes (hp a power of two <= 32).
__device__ __forceinline__ float head_sum(float v, int hp) {
  switch (hp) {
    case 32: return group_sum<32>(v);
    case 16: return group_sum<16>(v);
    case 8: return group_sum<8>(v);
    case 4: return group_sum<4>(v);
    case 2: return group_sum<2>(v);
    default: return v;
  }
}

// Per-head sums for any head width: up to 64 channels a head lies within a
// warp (shuffles); wider heads (hp > 32 pairs) span hp / 32 warps, whose
// warp sums meet in `red` (2 x TR x WPR floats, halves alternating with
// `phase` as in row_sums) behind one barrier.  Row k of the thread's rows;
// every thread of the CTA calls it at the same point.
template <bool WIDE, class T>
__device__ __forceinline__ float head_sum_any(const Ctx<T>& c, float v, int hp, int k, float* red, int& phase) {
  if constexpr (!WIDE) {
    return head_sum(v, hp);
  } else {
    if (hp <= 32) return head_sum(v, hp);
    v = group_sum<32>(v);
    float* r = red + phase * T::TR * T::WPR;
    phase ^= 1;
    const int wir = c.cp >> 5, row = c.row(k);
    if (c.lane == 0) r[row * T::WPR + wir] = v;
    __syncthreads();
    const int g = hp >> 5, first = (wir / g) * g;
    float s = 0.f;
    for (int j = 0; j < g; ++j) s += r[row * T::WPR + first + j];
    return s;
  }
}

// One forward mesh layer over the owned rows: y = f(x[c] w0 + x[c+s] w1).
// `buf` is a tile buffer the layer input is published into; the caller
// guarantees no thread still reads it from an earlier phase.  With `keep`
// the whole input is published (a backward pass reads it later); otherwise
// a stride-1 layer publishes only the even plane its neighbours read.
template <int W, class T>
__device__ __forceinline__ void mesh_layer_forward(const Ctx<T>& c, float2 (&a)[T::RPT], float4 w, int stride,
                                                   bool activated, float* buf, bool keep) {
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) {
    if (keep || stride != 1) {
      Planes<W>::put(buf + c.row(k) * W, c.cp, a[k]);
    } else {
      buf[c.row(k) * W + c.cp] = a[k].x;
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) {
    const float* srow = buf + c.row(k) * W;
    const float2 nb = stride == 1 ? make_float2(a[k].y, srow[c.nxt])
                                  : Planes<W>::shifted_even(srow, c.cp, stride);
    const float2 z = fma2(nb, make_float2(w.y, w.w), mul2(a[k], make_float2(w.x, w.z)));
    a[k] = activated ? elu2(z) : z;
  }
}

// Edge-gradient slots hold (self c0, self c1, neighbour c0, neighbour c1) of
// a channel pair so the packed updates pair up; parameters are stored per
// channel as (self, neighbour) (src/gpt/config.rs:440-444).
__device__ __forceinline__ float4 slot_to_params(float4 g) { return make_float4(g.x, g.z, g.y, g.w); }

// Forward through a whole mesh stack.  With `keep`, layer l's input stays in
// bufs[l] for a later backward pass; otherwise two buffers alternate.
// DEPTH and CONN fix the depth and connectivity at compile time (see
// MeshShape); `depth` is used when DEPTH is 0.
template <int W, class T, int DEPTH, int CONN>
__device__ __forceinline__ void mesh_forward(const Ctx<T>& c, const Dims& d, float2 (&a)[T::RPT],
                                             const float4* wg, int depth, float* bufs, bool keep) {
  // Each layer's weights are requested one layer ahead: with the row
  // buffers filling shared memory, L1 holds little and they come from L2.
  if constexpr (DEPTH > 0) depth = DEPTH;
  float4 w = __ldg(wg + c.cp);
  layer_loop<DEPTH, false>(depth, [&](int l) {
    const float4 wn = l + 1 < depth ? __ldg(wg + (l + 1) * T::PAIRS + c.cp) : w;
    float* buf = bufs + (keep ? l : (l & 1)) * T::BUF;
    mesh_layer_forward<W, T>(c, a, w, layer_stride<W, CONN>(d, l), l + 1 != depth, buf, keep);
    w = wn;
  });
}

// Backward through a mesh stack whose layer inputs sit in bufs[0..depth-1]
// (written by mesh_forward with keep = true).  dy enters as the gradient of
// the stack output and leaves as the gradient of its input.  Edge gradients
// add into the thread's private accumulator slots acc[l * NT + tid].
template <int W, class T, int DEPTH, int CONN>
__device__ __forceinline__ void mesh_backward(const Ctx<T>& c, const Dims& d, float2 (&dy)[T::RPT],
                                              const float4* wg, int depth, const float* bufs, float* xch,
                                              float4* acc) {
  if constexpr (DEPTH > 0) depth = DEPTH;
  float4 wnext = __ldg(wg + (depth - 1) * T::PAIRS + c.cp);
  layer_loop<DEPTH, true>(depth, [&](int l) {
    const int s = layer_stride<W, CONN>(d, l);
    const float4 w = wnext;
    if (l > 0) wnext = __ldg(wg + (l - 1) * T::PAIRS + c.cp);  // one layer ahead
    const float2 w0 = make_float2(w.x, w.z), w1 = make_float2(w.y, w.w);
    const float* xin = bufs + l * T::BUF;
    const float* yout = bufs + (l + 1) * T::BUF;  // valid when l + 1 < depth
    float* ex = xch + (l & 1) * T::BUF;
    // The rows' edge-gradient terms accumulate straight onto the thread's slot.
    float4& slot = acc[l * T::NT + c.tid];
    const float4 sv = slot;
    float2 gs = make_float2(sv.x, sv.y), gn = make_float2(sv.z, sv.w);
#pragma unroll
    for (int k = 0; k < T::RPT; ++k) {
      const int r = c.row(k);
      float2 dz = dy[k];
      if (l + 1 != depth) dz = mul2(dz, elu_slope2(Planes<W>::get(yout + r * W, c.cp)));
      const float2 x = Planes<W>::get(xin + r * W, c.cp);
      const float2 nb = s == 1 ? make_float2(x.y, xin[r * W + c.nxt])
                               : Planes<W>::shifted_even(xin + r * W, c.cp, s);
      gs = fma2(dz, x, gs);
      gn = fma2(dz, nb, gn);
      dy[k] = dz;
      // Channel c's neighbour term dz*w1 flows back to channel c + s.
      const float2 back = mul2(dz, w1);
      if (s == 1) {
        ex[r * W + Planes<W>::P + c.cp] = back.y;
      } else {
        Planes<W>::put(ex + r * W, c.cp, back);
      }
    }
    slot = make_float4(gs.x, gs.y, gn.x, gn.y);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < T::RPT; ++k) {
      const float* erow = ex + c.row(k) * W;
      const float2 t = s == 1 ? make_float2(erow[c.prv], dy[k].x * w.y)
                              : Planes<W>::shifted_even(erow, c.cp, -s);
      dy[k] = fma2(dy[k], w0, t);
    }
  });
}

// Layer inputs of a mesh stack kept for its backward pass.  With the shape
// compiled in and stride-1 (neighbor) layers, each thread keeps its own
// channel pairs in registers and only the even plane, which the neighbours
// read, goes to shared memory: the backward then reads one shared value per
// row and layer instead of five.  Other shapes keep whole layer inputs in
// shared memory (mesh_forward with keep = true).
template <class T, int DEPTH, int CONN>
struct KeptInputs {
  static constexpr bool kRegs = DEPTH > 0 && CONN == 0;
  float2 x[kRegs ? DEPTH : 1][T::RPT];
};

template <int W, class T, int DEPTH, int CONN>
__device__ __forceinline__ void mesh_forward_kept(const Ctx<T>& c, const Dims& d, float2 (&a)[T::RPT],
                                                  const float4* wg, int depth, float* bufs,
                                                  KeptInputs<T, DEPTH, CONN>& kept) {
  if constexpr (KeptInputs<T, DEPTH, CONN>::kRegs) {
    float4 w = __ldg(wg + c.cp);
    layer_loop<DEPTH, false>(DEPTH, [&](int l) {
      const float4 wn = l + 1 < DEPTH ? __ldg(wg + (l + 1) * T::PAIRS + c.cp) : w;
#pragma unroll
      for (int k = 0; k < T::RPT; ++k) kept.x[l][k] = a[k];
      mesh_layer_forward<W, T>(c, a, w, 1, l + 1 != DEPTH, bufs + l * T::BUF, false);
      w = wn;
    });
  } else {
    mesh_forward<W, T, DEPTH, CONN>(c, d, a, wg, depth, bufs, true);
  }
}

// mesh_backward over inputs kept by mesh_forward_kept.
template <int W, class T, int DEPTH, int CONN>
__device__ __forceinline__ void mesh_backward_kept(const Ctx<T>& c, const Dims& d, float2 (&dy)[T::RPT],
                                                   const float4* wg, int depth, const float* bufs, float* xch,
                                                   float4* acc, const KeptInputs<T, DEPTH, CONN>& kept) {
  if constexpr (KeptInputs<T, DEPTH, CONN>::kRegs) {
    float4 wnext = __ldg(wg + (DEPTH - 1) * T::PAIRS + c.cp);
    layer_loop<DEPTH, true>(DEPTH, [&](int l) {
      const float4 w = wnext;
      if (l > 0) wnext = __ldg(wg + (l - 1) * T::PAIRS + c.cp);  // one layer ahead
      const float2 w0 = make_float2(w.x, w.z), w1 = make_float2(w.y, w.w);
      const float* xin = bufs + l * T::BUF;  // even plane of layer l's input
      float* ex = xch + (l & 1) * T::BUF;
      // The rows' edge-gradient terms accumulate straight onto the thread's slot.
      float4& slot = acc[l * T::NT + c.tid];
      const float4 sv = slot;
      float2 gs = make_float2(sv.x, sv.y), gn = make_float2(sv.z, sv.w);
#pragma unroll
      for (int k = 0; k < T::RPT; ++k) {
        const int r = c.row(k);
        float2 dz = dy[k];
        if (l + 1 != DEPTH) dz = mul2(dz, elu_slope2(kept.x[l + 1 < DEPTH ? l + 1 : l][k]));
        const float2 x = kept.x[l][k];
        const float2 nb = make_float2(x.y, xin[r * W + c.nxt]);
        gs = fma2(dz, x, gs);
        gn = fma2(dz, nb, gn);
        dy[k] = dz;
        // Channel c's neighbour term dz*w1 flows back to channel c + 1.
        ex[r * W + Planes<W>::P + c.cp] = dz.y * w1.y;
      }
      slot = make_float4(gs.x, gs.y, gn.x, gn.y);
      __syncthreads();
#pragma unroll
      for (int k = 0; k < T::RPT; ++k) {
        const float2 t = make_float2(ex[c.row(k) * W + c.prv], dy[k].x * w.y);
        dy[k] = fma2(dy[k], w0, t);
      }
    });
  } else {
    mesh_backward<W, T, DEPTH, CONN>(c, d, dy, wg, depth, bufs, xch, acc);
  }
}

// RMSNorm over the full row: returns normalized values and 1/rms per row.
template <class T>
__device__ __forceinline__ void rmsnorm_rows(const Ctx<T>& c, float2 (&x)[T::RPT], float (&inv)[T::RPT], float* red,
                                             int& phase, int width) {
  float s[T::RPT];
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) s[k] = x[k].x * x[k].x + x[k].y * x[k].y;
  row_sums<T>(c, s, red, phase);
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) {
    inv[k] = rms_scale(s[k], 1.0f / (float)width);
    x[k] = x[k] * inv[k];
  }
}

// RMSNorm backward over the full row: g <- inv * (g - n * mean(g * n)).
template <class T>
__device__ __forceinline__ void rmsnorm_rows_backward(const Ctx<T>& c, const float2 (&n)[T::RPT],
                                                      const float (&inv)[T::RPT], float2 (&g)[T::RPT], float* red,
                                                      int& phase, int width) {
  float s[T::RPT];
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) s[k] = g[k].x * n[k].x + g[k].y * n[k].y;
  row_sums<T>(c, s, red, phase);
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) {
    float m = s[k] / (float)width;
    g[k] = make_float2(inv[k] * (g[k].x - n[k].x * m), inv[k] * (g[k].y - n[k].y * m));
  }
}

// Slice RoPE (src/gpt/gpu.rs:175-208) for one thread's channel pair: the
// split-half partner sits hp/2 lanes away within the head.  The lane
// constants are fixed per thread; `apply` rotates one row's pair.
struct RopeLane {
  int hp, half, i0;
  float sign;  // -1 on the first half of the head (x0 cos - x1 sin)
  __device__ RopeLane(int cp, int hp_) : hp(hp_) {
    const int j = cp % hp;
    half = hp / 2;
    const bool left = j < half;
    i0 = left ? 2 * j : 2 * j - hp;
    sign = left ? -1.0f : 1.0f;
  }
  // cs: table [T][hd/2] of (cos, sin); `inverse` rotates by -angle.
  __device__ __forceinline__ float2 apply(float2 v, int pos, const float2* cs, bool inverse) const {
    if (hp == 1) {
      const float2 t = __ldg(cs + pos);
      const float sn = inverse ? -t.y : t.y;
      return make_float2(v.x * t.x - v.y * sn, v.y * t.x + v.x * sn);
    }
    return combine(v, shfl_xor2(v, half), pos, cs, inverse);
  }
  // (cos, sin) of the pair's two frequencies at position pos, one 16-byte
  // load (i0 and hp are even; hp >= 2), so a caller can request it early.
  __device__ __forceinline__ float4 angles(int pos, const float2* cs) const {
    return __ldg(reinterpret_cast<const float4*>(cs + pos * hp + i0));
  }
  // The rotation given the partner pair p and the pair's angles t (hp >= 2).
  __device__ __forceinline__ float2 rotate(float2 v, float2 p, float4 t, bool inverse) const {
    const float sg = inverse ? -sign : sign;
    return fma2(v, make_float2(t.x, t.z), mul2(p * sg, make_float2(t.y, t.w)));
  }
  __device__ __forceinline__ float2 combine(float2 v, float2 p, int pos, const float2* cs, bool inverse) const {
    return rotate(v, p, angles(pos, cs), inverse);
  }
};

// RoPE of row k's pair for any head width: in heads of 128 channels or more
// the split-half partner sits in another warp, exchanged through `xs`
// (TR x W floats that nothing else uses across the three barriers).  Every
// thread of the CTA calls it at the same point.
template <bool WIDE, class T>
__device__ __forceinline__ float2 rope_any(const Ctx<T>& c, const RopeLane& rope, float2 v, int k, int pos,
                                           const float2* cs, bool inverse, float* xs) {
  if (!WIDE || rope.hp == 1 || rope.half < 32) return rope.apply(v, pos, cs, inverse);
  float2* x2 = reinterpret_cast<float2*>(xs);
  __syncthreads();
  x2[c.row(k) * T::PAIRS + c.cp] = v;
  __syncthreads();
  const float2 p = x2[c.row(k) * T::PAIRS + (c.cp ^ rope.half)];
  __syncthreads();
  return rope.combine(v, p, pos, cs, inverse);
}

// Asks L2 to fetch rows [r0, r0 + n) of a [rows][W] FP32 tensor (one bulk
// prefetch, no registers or shared memory), so that a tile's row loads a few
// microseconds later hit L2 instead of waiting on HBM.  Skipped past the last
// row and for a base that is not 16-byte aligned (the instruction's rule).
template <int W>
__device__ __forceinline__ void prefetch_rows(const float* p, int r0, int n, int rows) {
  if (p == nullptr || r0 >= rows) return;
  n = n < rows - r0 ? n : rows - r0;
  const float* a = p + (size_t)r0 * W;
  if ((reinterpret_cast<uintptr_t>(a) & 15) != 0) return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"((uint32_t)(n * W * 4)) : "memory");
}

// Lanes 0.. of warp 0 each prefetch one of up to five row tensors for the
// CTA's next tile (tile + gridDim.x).
template <int W, int TR>
__device__ __forceinline__ void prefetch_next_tile(int tid, int tile, int rows, const float* p0, const float* p1,
                                                   const float* p2 = nullptr, const float* p3 = nullptr,
                                                   const float* p4 = nullptr) {
  if (tid >= 5) return;
  const float* p = tid == 0 ? p0 : (tid == 1 ? p1 : (tid == 2 ? p2 : (tid == 3 ? p3 : p4)));
  prefetch_rows<W>(p, (tile + (int)gridDim.x) * TR, TR, rows);
}

// Position within its sequence of each owned row of a tile.
template <class T>
__device__ __forceinline__ void tile_positions(const Ctx<T>& c, int tile, int sequence, int (&pos)[T::RPT]) {
  const int base = (tile * T::TR) % sequence;
#pragma unroll
  for (int k = 0; k < T::RPT; ++k) {
    int p = base + c.row(k);
    while (p >= sequence) p -= sequence;
    pos[k] = p;
  }
}

}  // namespace mb
