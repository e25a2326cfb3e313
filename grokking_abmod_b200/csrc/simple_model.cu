// grok-simple executor (host C++) and its kernels: mesh-mlp,
// tied-rotary-residual-dense-mlp, shared-neighbor-mesh-mlp, mlp, bilinear,
// residual-mlp, the residual mesh family (residual-mesh-mlp,
// tied-concat-residual-mesh-mlp, tied-rotary-residual-mesh-mlp) and
// tied-concat-mesh-mlp.
//
// Replaces GpuSimpleModel (src/simple/gpu.rs:1757-2073) and its op-by-op
// plans (forward_with / backward_with, :2140-2700).  One training step is a
// fixed launch sequence captured once per batch size into a CUDA graph; the
// per-step values (minibatch offset, learning rates, AdamW corrections) sit
// in a small device struct refreshed by one host->device copy before each
// launch.
//
// Data flow, B200-first:
//  * Operands are one-hot, so the first layer of every architecture is a
//    gather of embedding rows by operand class (exact: the reference's dense
//    product adds exact zeros, src/simple/dense_tiled.rs:88-159).
//  * Row-local work runs one warp per row with the row in shared memory: the
//    mesh stack of mesh-mlp (:240-339 of gpu.rs), the 64-layer pre-RMSNorm
//    two-parent core of the shared-Neighbor model (:341-443, :505-630),
//    RMSNorm and residual sums.  Backward kernels walk the layers in lockstep
//    across the CTA's warps and reduce the per-row weight contributions in a
//    fixed warp order into one partial per CTA; a second pass sums the CTA
//    partials in order.  No atomics: results are bitwise reproducible.
//  * Every dense contraction (readouts, their input and weight gradients, the
//    residual dense projections, mlp's hidden layers) is a tcgen05 3xTF32
//    GEMM (gemm_tc.cu), with split-K over batch rows for weight gradients.
//    Embedding-row gradients of one-hot inputs are ordered per-class sums.
//  * The shared-Neighbor readout (the transposed Neighbor chain,
//    src/simple/reference.rs:257-268) equals h . E^T with E[k] the chain
//    applied to class k's one-hot row (the reference's own identity,
//    src/simple/mod.rs:1299-1335).  The chain therefore runs once per step on
//    the `modulus` class rows instead of once per batch row, the readout and
//    its gradients become GEMMs, and the chain's weight gradient is the chain
//    backward of dE over those class rows.
//  * Embedding gradients (operand gathers) are per-class ordered sums over
//    the batch rows that use the class (one CTA per class).

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "gemm_tc.h"
#include "simple.h"

namespace mb {
namespace simple {

#define SIMPLE_CUDA(call)                                                                           \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess)                                                                          \
      throw Error(MB_ERR_CUDA, std::string(#call) + " failed: " + cudaGetErrorString(e_));          \
  } while (0)

constexpr float kEps = 1e-5f;         // RMSNORM_EPSILON, src/gpt/mod.rs:39
constexpr int kFwdWarps = 8;          // forward row kernels: warps (= rows) per CTA
constexpr int kBwdWarps = 16;         // backward row kernels: warps per CTA ...
constexpr int kBwdRows = 2;           // ... each walking this many rows per layer

// (c + s) mod W and (c - s) mod W for 0 <= c, s < W: a compare and a
// subtract instead of an integer division in the per-element loops.
__device__ __forceinline__ int wrap_up(int c, int s, int W) { return c + s >= W ? c + s - W : c + s; }
__device__ __forceinline__ int wrap_down(int c, int s, int W) { return c < s ? c - s + W : c - s; }
constexpr int kMaxJ = kMaxKernelWidth / 32;  // row values per lane at the widest row
constexpr int kSplitK = 256;          // batch rows per weight-gradient GEMM chunk
constexpr unsigned kFull = 0xffffffffu;

// Turns every kernel-to-kernel edge of a captured step graph into a
// programmatic edge from the upstream kernel's launch-completion port: the
// downstream grid is scheduled once every block of the upstream grid has
// started, instead of after the upstream grid has completed and the launch
// has gone through, and its threads begin with wait_prior_grids, which
// returns once the upstream grid has completed and its writes are visible.
// Every kernel that a step graph holds (this file's and the GEMM's) starts
// with that wait, so each kernel still sees all of its predecessors' writes
// (the waits chain) and no kernel writes what a predecessor still reads.
// A step of a few hundred microseconds spends much of its time in the
// launch gaps between its 15 to 40 kernels; this overlaps them.
static cudaError_t programmatic_edges(cudaGraph_t g) {
  size_t n = 0;
  cudaError_t e = cudaGraphGetEdges_v2(g, nullptr, nullptr, nullptr, &n);
  if (e != cudaSuccess || n == 0) return e;
  std::vector<cudaGraphNode_t> from(n), to(n);
  std::vector<cudaGraphEdgeData> data(n);
  e = cudaGraphGetEdges_v2(g, from.data(), to.data(), data.data(), &n);
  for (size_t i = 0; e == cudaSuccess && i < n; ++i) {
    cudaGraphNodeType a, b;
    if ((e = cudaGraphNodeGetType(from[i], &a)) != cudaSuccess || (e = cudaGraphNodeGetType(to[i], &b)) != cudaSuccess)
      break;
    if (a != cudaGraphNodeTypeKernel || b != cudaGraphNodeTypeKernel || data[i].type != cudaGraphDependencyTypeDefault)
      continue;
    cudaGraphEdgeData pe;
    std::memset(&pe, 0, sizeof(pe));
    pe.from_port = cudaGraphKernelNodePortProgrammatic;
    pe.type = cudaGraphDependencyTypeProgrammatic;
    e = cudaGraphRemoveDependencies_v2(g, &from[i], &to[i], &data[i], 1);
    if (e == cudaSuccess) e = cudaGraphAddDependencies_v2(g, &from[i], &to[i], &pe, 1);
  }
  return e;
}

// Values that change from step to step, read by the captured kernels: the
// minibatch (table columns and index list), learning rates and corrections.
// The step graph therefore serves every table and batch list of its size.
struct StepScalars {
  const uint32_t *idx, *ta, *tb, *tt;
  uint32_t offset;
  float lr_dense, lr_mesh, weight_decay, beta1, beta2, epsilon, correction1, correction2;
};

// Device status flags: [0] a tensor-core wait gave up, [1] nonfinite logits.
enum { kFlagTc = 0, kFlagNonfinite = 1, kFlags = 2 };

// kLinear: the identity, for residual sums whose branch ends without an
// activation (residual-mlp); it is not a model activation.
constexpr int kLinear = 2;
template <int ACT>
__device__ __forceinline__ float act_f(float x) {
  return ACT == kRelu ? fmaxf(x, 0.f) : (ACT == kSquare ? x * x : x);
}
template <int ACT>
__device__ __forceinline__ float act_g(float x) {
  return ACT == kRelu ? (x > 0.f ? 1.f : 0.f) : (ACT == kSquare ? 2.f * x : 1.f);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Rotate90 roles: channel c of operand b's embedding is b[c^1], negated for
// even c (src/simple/reference.rs:341-351).
__device__ __forceinline__ float rotated(const float* e, int c) { return (c & 1) ? e[c - 1] : -e[c + 1]; }

// ------------------------------------------------------------ batch gather
__global__ void gather_batch(int n, const StepScalars* __restrict__ sc, const uint32_t* __restrict__ idx,
                             const uint32_t* __restrict__ ta, const uint32_t* __restrict__ tb,
                             const uint32_t* __restrict__ tt, uint32_t* __restrict__ a, uint32_t* __restrict__ b,
                             uint32_t* __restrict__ y) {
  wait_prior_grids();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  if (sc != nullptr) {
    idx = sc->idx + sc->offset;
    ta = sc->ta;
    tb = sc->tb;
    tt = sc->tt;
  }
  const uint32_t i = idx[r];
  a[r] = ta[i];
  b[r] = tb[i];
  y[r] = tt[i];
}

// ------------------------------------------------------------- mesh-mlp
// h0 = W0[a] + W0[m + b] (or h0_in, the tied-concat projection, when given);
// per mesh layer h' = act(h)[c] w0 + act(h)[c+s] w1; act = act(h_L) feeds the
// readout GEMM.  h[l] (l = 0..L) is kept for the backward.  Layer l's weights
// start at mesh + l * lstride (lstride 0: tied mesh layers).
template <int ACT, int J>
__global__ void __launch_bounds__(kFwdWarps * 32)
    mlp_forward(int n, int W, int m, int L, int p, int lstride, const int* __restrict__ strides,
                const uint32_t* __restrict__ a,
                const uint32_t* __restrict__ b, const float* __restrict__ w0, const float* __restrict__ h0_in,
                const float* __restrict__ mesh, float* __restrict__ h, float* __restrict__ act) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  float* row = sm + warp * W;
  const size_t nw = (size_t)n * W;
  for (int c = lane; c < W; c += 32) {
    const float v = h0_in != nullptr ? h0_in[(size_t)r * W + c] : w0[(size_t)a[r] * W + c] + w0[(size_t)(m + b[r]) * W + c];
    h[(size_t)r * W + c] = v;
    row[c] = act_f<ACT>(v);
  }
  for (int l = 0; l < L; ++l) {
    __syncwarp();
    const int s = strides[l];
    const float* w = mesh + (size_t)l * lstride;
    float v[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) {
        float y = row[c] * w[c * p];
        if (p == 2) y = fmaf(row[wrap_up(c, s, W)], w[c * p + 1], y);
        v[j] = y;
      }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) {
        h[(l + 1) * nw + (size_t)r * W + c] = v[j];
        row[c] = act_f<ACT>(v[j]);
      }
    }
  }
  __syncwarp();
  for (int c = lane; c < W; c += 32) act[(size_t)r * W + c] = row[c];
}

// dact = dlogits R^T in, dh0 out; per-CTA mesh weight partials
// [gridDim.x][L][p*W].
template <int ACT, int J>
__global__ void __launch_bounds__(kBwdWarps * 32)
    mlp_backward(int n, int W, int L, int p, int lstride, const int* __restrict__ strides, const float* __restrict__ mesh,
                 const float* __restrict__ h, const float* __restrict__ dact, float* __restrict__ dh0,
                 float* __restrict__ partials) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pw = p * W;
  float* arow = sm + warp * 2 * W;  // act(h_l) of the current row
  float* drow = arow + W;           // dh of the current row
  float* contrib = sm + kBwdWarps * 2 * W;
  const size_t nw = (size_t)n * W;
  float dh[kBwdRows][J];
#pragma unroll
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      dh[i][j] = (r < n && c < W) ? dact[(size_t)r * W + c] * act_g<ACT>(h[L * nw + (size_t)r * W + c]) : 0.f;
    }
  }
  for (int l = L - 1; l >= 0; --l) {
    const int s = strides[l];
    const float* w = mesh + (size_t)l * lstride;
    float* mine = contrib + warp * pw;
    // This warp's weight contributions over its rows, summed in registers in
    // row order and written once per layer.
    float g0[J], g1[J];
#pragma unroll
    for (int j = 0; j < J; ++j) g0[j] = g1[j] = 0.f;
#pragma unroll
    for (int i = 0; i < kBwdRows; ++i) {
      const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
      const bool active = r < n;
      float hl[J];
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) {
          hl[j] = active ? h[l * nw + (size_t)r * W + c] : 0.f;
          arow[c] = act_f<ACT>(hl[j]);
          drow[c] = dh[i][j];
        }
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) {
          const float d = drow[c];
          g0[j] += d * arow[c];
          float da = d * w[c * p];
          if (p == 2) {
            g1[j] += d * arow[wrap_up(c, s, W)];
            const int q = wrap_down(c, s, W);
            da = fmaf(drow[q], w[q * p + 1], da);
          }
          dh[i][j] = da * act_g<ACT>(hl[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) {
        mine[c * p] = g0[j];
        if (p == 2) mine[c * p + 1] = g1[j];
      }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < pw; t += blockDim.x) {
      float sum = 0.f;
      for (int q = 0; q < kBwdWarps; ++q) sum += contrib[q * pw + t];
      partials[((size_t)blockIdx.x * L + l) * pw + t] = sum;
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
    if (r >= n) continue;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) dh0[(size_t)r * W + c] = dh[i][j];
    }
  }
}

// Tied mesh layers: out[t] = sum over layers l = L-1 .. 0 of the in-order
// CTA sums of partials[cta][l][t] (the reference adds each lower layer's
// gradient to the last one's, src/simple/gpu.rs:2771-2792).
__global__ void reduce_layer_partials(const float* __restrict__ partials, int ctas, int L, int count,
                                      float* __restrict__ out) {
  wait_prior_grids();
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < count; t += gridDim.x * blockDim.x) {
    float total = 0.f;
    for (int l = L - 1; l >= 0; --l) {
      float s = 0.f;
      for (int q = 0; q < ctas; ++q) s += partials[((size_t)q * L + l) * count + t];
      total += s;
    }
    out[t] = total;
  }
}

// out[t] = sum over CTAs (in order) of partials[cta][t].
__global__ void reduce_cta_partials(const float* __restrict__ partials, int ctas, size_t count,
                                    float* __restrict__ out) {
  wait_prior_grids();
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < count; t += (size_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < ctas; ++q) s += partials[(size_t)q * count + t];
    out[t] = s;
  }
}

// ----------------------------------------------------- RMSNorm row helpers
// y = x / sqrt(mean(x^2) + eps) over the warp's row; returns the inverse.
template <int J>
__device__ __forceinline__ float row_inverse_rms(const float (&x)[J], int W, int lane) {
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j)
    if (lane + 32 * j < W) ss = fmaf(x[j], x[j], ss);
  ss = warp_sum(ss);
  return 1.0f / sqrtf(ss / (float)W + kEps);
}

// Rotary operand embedding h0 = E[a] + rot(E[b]) and n0 = RMSNorm(h0)
// (tied-rotary-residual-dense-mlp; also the shared-Neighbor core input).
template <int J>
__global__ void __launch_bounds__(kFwdWarps * 32)
    rotary_embed(int n, int W, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                 const float* __restrict__ E, float* __restrict__ h0, float* __restrict__ n0,
                 float* __restrict__ inv0) {
  wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  const float* ea = E + (size_t)a[r] * W;
  const float* eb = E + (size_t)b[r] * W;
  float v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < W ? ea[c] + rotated(eb, c) : 0.f;
  }
  const float inv = row_inverse_rms(v, W, lane);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < W) {
      h0[(size_t)r * W + c] = v[j];
      if (n0 != nullptr) n0[(size_t)r * W + c] = v[j] * inv;
    }
  }
  if (inv0 != nullptr && lane == 0) inv0[r] = inv;
}

// h' = h + act(z); n' = RMSNorm(h') (a dense residual block's epilogue).
template <int ACT, int J>
__global__ void __launch_bounds__(kFwdWarps * 32)
    residual_norm(int n, int W, const float* __restrict__ h, const float* __restrict__ z, float* __restrict__ hn,
                  float* __restrict__ nn, float* __restrict__ inv_out) {
  wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  float v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < W ? h[(size_t)r * W + c] + act_f<ACT>(z[(size_t)r * W + c]) : 0.f;
  }
  const float inv = row_inverse_rms(v, W, lane);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < W) {
      hn[(size_t)r * W + c] = v[j];
      nn[(size_t)r * W + c] = v[j] * inv;
    }
  }
  if (lane == 0) inv_out[r] = inv;
}

// residual-mlp input (src/simple/reference.rs:418-419): h0 = x W0 with x
// one-hot at a and m + b, i.e. W0[a] + W0[m + b], and n0 = RMSNorm(h0).
template <int J>
__global__ void __launch_bounds__(kFwdWarps * 32)
    concat_embed(int n, int W, int m, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                 const float* __restrict__ w0, float* __restrict__ h0, float* __restrict__ n0,
                 float* __restrict__ inv0) {
  wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  const float* ra = w0 + (size_t)a[r] * W;
  const float* rb = w0 + (size_t)(m + b[r]) * W;
  float v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    v[j] = c < W ? ra[c] + rb[c] : 0.f;
  }
  const float inv = row_inverse_rms(v, W, lane);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < W) {
      h0[(size_t)r * W + c] = v[j];
      if (n0 != nullptr) n0[(size_t)r * W + c] = v[j] * inv;
    }
  }
  if (inv0 != nullptr && lane == 0) inv0[r] = inv;
}

// dx = add + inv (dy - y <dy, y> / W) with y the normalised row.
template <int J>
__global__ void __launch_bounds__(kFwdWarps * 32)
    rms_backward(int n, int W, const float* __restrict__ y, const float* __restrict__ inv,
                 const float* __restrict__ dy, const float* add, float* dx) {
  wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  float yv[J], dv[J], dot = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    yv[j] = c < W ? y[(size_t)r * W + c] : 0.f;
    dv[j] = c < W ? dy[(size_t)r * W + c] : 0.f;
    dot = fmaf(dv[j], yv[j], dot);
  }
  dot = warp_sum(dot) / (float)W;
  const float iv = inv[r];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < W) {
      const float g = iv * (dv[j] - yv[j] * dot);
      dx[(size_t)r * W + c] = add != nullptr ? add[(size_t)r * W + c] + g : g;
    }
  }
}

// dz = dh * act'(z)
template <int ACT>
__global__ void activation_gradient(size_t count, const float* __restrict__ dh, const float* __restrict__ z,
                                    float* __restrict__ dz) {
  wait_prior_grids();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
    dz[i] = dh[i] * act_g<ACT>(z[i]);
}

// ---------------------------------------------------- shared-Neighbor
// The shared linear Neighbor chain over the class rows.  The rows are
// independent through the chain, so CTA b owns rows [b RG, b RG + RG) (RG =
// 1024 / W row groups) and thread (rg, c) channel c of row b RG + rg; the
// row moves between two shared-memory buffers, one barrier per layer:
//   states[0][k] = e_k
//   states[l+1][k][c] = states[l][k][c] w0[c] + states[l][k][c+1] w1[c]
// states[ed] is the embedding E of the operands and of the readout.
constexpr int kChainThreads = 1024;
__global__ void __launch_bounds__(kChainThreads)
    chain_forward(int m, int W, int ed, const float* __restrict__ chain, float* __restrict__ states) {
  wait_prior_grids();
  __shared__ float buf[2][kChainThreads];
  const int c = threadIdx.x % W, rg = threadIdx.x / W, RG = kChainThreads / W;
  const int k = blockIdx.x * RG + rg;
  const bool active = rg < RG && k < m;
  const int cn = c + 1 == W ? 0 : c + 1;
  const size_t mw = (size_t)m * W;
  if (active) {
    const float e = c == k ? 1.f : 0.f;
    buf[0][rg * W + c] = e;
    states[(size_t)k * W + c] = e;
  }
  __syncthreads();
  for (int l = 0; l < ed; ++l) {
    const float w0 = chain[(size_t)l * 2 * W + 2 * c], w1 = chain[(size_t)l * 2 * W + 2 * c + 1];
    const float* in = buf[l & 1];
    float* out = buf[(l + 1) & 1];
    if (active) {
      const float v = fmaf(in[rg * W + cn], w1, in[rg * W + c] * w0);
      out[rg * W + c] = v;
      states[(l + 1) * mw + (size_t)k * W + c] = v;
    }
    __syncthreads();
  }
}

// Chain backward over the class rows (same layout): dv = dE; for l = ed-1
// .. 0 the chain weights' gradient sums dv[k][c] v_l[k][c] and dv[k][c]
// v_l[k][c+1] over the CTA's rows (in row order) into partials[cta][l][2W],
// which reduce_cta_partials sums over the CTAs in order, and dv <- dv[c] w0[c]
// + dv[c-1] w1[c-1].
__global__ void __launch_bounds__(kChainThreads)
    chain_backward(int m, int W, int ed, const float* __restrict__ chain, const float* __restrict__ states,
                   const float* __restrict__ dE, float* __restrict__ partials) {
  wait_prior_grids();
  __shared__ float buf[2][kChainThreads];
  __shared__ float part[2][kChainThreads];
  const int c = threadIdx.x % W, rg = threadIdx.x / W, RG = kChainThreads / W;
  const int k = blockIdx.x * RG + rg;
  const bool active = rg < RG && k < m;
  const int cp = c == 0 ? W - 1 : c - 1, cn = c + 1 == W ? 0 : c + 1;
  const size_t mw = (size_t)m * W;
  if (active) buf[0][rg * W + c] = dE[(size_t)k * W + c];
  __syncthreads();
  for (int l = ed - 1; l >= 0; --l) {
    const float w0 = chain[(size_t)l * 2 * W + 2 * c], w1p = chain[(size_t)l * 2 * W + 2 * cp + 1];
    const float* dv = buf[(ed - 1 - l) & 1];
    float* out = buf[(ed - l) & 1];
    float g0 = 0.f, g1 = 0.f;
    if (active) {
      const float* v = states + l * mw + (size_t)k * W;
      const float d = dv[rg * W + c];
      g0 = d * v[c];
      g1 = d * v[cn];
      if (l > 0) out[rg * W + c] = fmaf(dv[rg * W + cp], w1p, d * w0);
    }
    part[0][threadIdx.x] = g0;
    part[1][threadIdx.x] = g1;
    __syncthreads();
    if (threadIdx.x < W) {
      float s0 = 0.f, s1 = 0.f;
      for (int q = 0; q < RG; ++q) {
        s0 += part[0][q * W + threadIdx.x];
        s1 += part[1][q * W + threadIdx.x];
      }
      float* out_g = partials + ((size_t)blockIdx.x * ed + l) * 2 * W;
      out_g[2 * threadIdx.x] = s0;
      out_g[2 * threadIdx.x + 1] = s1;
    }
    __syncthreads();
  }
}

// The core's weights, staged in shared memory when they fit (depth x 3W).
constexpr int kCoreSmemFloats = 24576;  // 96 KiB
constexpr int kSmemFloats = 57344;      // 224 KiB: the dynamic shared memory a CTA may use
__device__ __forceinline__ const float* stage_core(const float* __restrict__ core, int n_floats, float* sm) {
  if (n_floats > kCoreSmemFloats) return core;
  for (int i = threadIdx.x; i < n_floats; i += blockDim.x) sm[i] = core[i];
  __syncthreads();
  return sm;
}

// The pre-RMSNorm residual two-parent core: h <- h + act(n[c] w0 + n[c+s] w1
// + bias), n = RMSNorm(h); hs[l] keeps each layer's input, hf = RMSNorm(h).
template <int ACT, int J>
__global__ void __launch_bounds__(kFwdWarps * 32)
    shared_forward(int n, int W, int depth, const int* __restrict__ strides, const uint32_t* __restrict__ a,
                   const uint32_t* __restrict__ b, const float* __restrict__ E, const float* __restrict__ core,
                   float* __restrict__ hs, float* __restrict__ hf, float* __restrict__ invf) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  const float* wts = stage_core(core, depth * 3 * W, sm);
  if (r >= n) return;
  float* row = sm + (depth * 3 * W <= kCoreSmemFloats ? depth * 3 * W : 0) + warp * W;
  const float* ea = E + (size_t)a[r] * W;
  const float* eb = E + (size_t)b[r] * W;
  const size_t nw = (size_t)n * W;
  float h[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    h[j] = c < W ? ea[c] + rotated(eb, c) : 0.f;
  }
  for (int l = 0; l < depth; ++l) {
    const float inv = row_inverse_rms<J>(h, W, lane);
    __syncwarp();
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) {
        hs[l * nw + (size_t)r * W + c] = h[j];
        row[c] = h[j] * inv;
      }
    }
    __syncwarp();
    const int s = strides[l];
    const float* w = wts + (size_t)l * 3 * W;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) {
        const float z = fmaf(row[wrap_up(c, s, W)], w[3 * c + 1], row[c] * w[3 * c]) + w[3 * c + 2];
        h[j] += act_f<ACT>(z);
      }
    }
  }
  const float inv = row_inverse_rms<J>(h, W, lane);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < W) hf[(size_t)r * W + c] = h[j] * inv;
  }
  if (lane == 0) invf[r] = inv;
}

// Backward of the core: dhf (gradient of the final RMSNorm output) in, dh0
// out; per-CTA weight partials [gridDim.x][depth][3W] (w0, w1, bias per unit).
// The next layer's saved inputs are loaded while the current layer computes.
template <int ACT, int J>
__global__ void __launch_bounds__(kBwdWarps * 32)
    shared_backward(int n, int W, int depth, const int* __restrict__ strides, const float* __restrict__ core,
                    const float* __restrict__ hs, const float* __restrict__ hf, const float* __restrict__ invf,
                    const float* __restrict__ dhf, float* __restrict__ dh0, float* __restrict__ partials) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pw = 3 * W;
  const float* wts = stage_core(core, depth * pw, sm);
  float* base = sm + (depth * pw <= kCoreSmemFloats ? depth * pw : 0);
  float* nrow = base + warp * 2 * W;
  float* zrow = nrow + W;  // dz
  float* contrib = base + kBwdWarps * 2 * W;
  const size_t nw = (size_t)n * W;
  float dh[kBwdRows][J];
#pragma unroll
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
    const bool active = r < n;
    float yv[J], dv[J], dot = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      yv[j] = (active && c < W) ? hf[(size_t)r * W + c] : 0.f;
      dv[j] = (active && c < W) ? dhf[(size_t)r * W + c] : 0.f;
      dot = fmaf(dv[j], yv[j], dot);
    }
    dot = warp_sum(dot) / (float)W;
    const float iv = active ? invf[r] : 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) dh[i][j] = iv * (dv[j] - yv[j] * dot);
  }
  float xn[kBwdRows][J];  // saved input of the layer about to be processed
  auto load_inputs = [&](int l) {
#pragma unroll
    for (int i = 0; i < kBwdRows; ++i) {
      const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        xn[i][j] = (r < n && c < W && l >= 0) ? hs[l * nw + (size_t)r * W + c] : 0.f;
      }
    }
  };
  load_inputs(depth - 1);
  for (int l = depth - 1; l >= 0; --l) {
    const int s = strides[l];
    const float* w = wts + (size_t)l * pw;
    float* mine = contrib + warp * pw;
    // Weight contributions (w0, w1, bias) over this warp's rows, summed in
    // registers in row order and written once per layer.
    float g0[J], g1[J], g2[J];
#pragma unroll
    for (int j = 0; j < J; ++j) g0[j] = g1[j] = g2[j] = 0.f;
    float xc[kBwdRows][J];
#pragma unroll
    for (int i = 0; i < kBwdRows; ++i)
#pragma unroll
      for (int j = 0; j < J; ++j) xc[i][j] = xn[i][j];
    load_inputs(l - 1);
#pragma unroll
    for (int i = 0; i < kBwdRows; ++i) {
      const float inv = row_inverse_rms<J>(xc[i], W, lane);
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) nrow[c] = xc[i][j] * inv;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) {
          const float z = fmaf(nrow[wrap_up(c, s, W)], w[3 * c + 1], nrow[c] * w[3 * c]) + w[3 * c + 2];
          zrow[c] = dh[i][j] * act_g<ACT>(z);
        }
      }
      __syncwarp();
      float dn[J], dot = 0.f;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        dn[j] = 0.f;
        if (c < W) {
          const float dz = zrow[c];
          g0[j] += dz * nrow[c];
          g1[j] += dz * nrow[wrap_up(c, s, W)];
          g2[j] += dz;
          const int q = wrap_down(c, s, W);
          dn[j] = fmaf(zrow[q], w[3 * q + 1], dz * w[3 * c]);
          dot = fmaf(dn[j], nrow[c], dot);
        }
      }
      dot = warp_sum(dot) / (float)W;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) dh[i][j] += inv * (dn[j] - nrow[c] * dot);
      }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) {
        mine[3 * c] = g0[j];
        mine[3 * c + 1] = g1[j];
        mine[3 * c + 2] = g2[j];
      }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < pw; t += blockDim.x) {
      float sum = 0.f;
      for (int q = 0; q < kBwdWarps; ++q) sum += contrib[q * pw + t];
      partials[((size_t)blockIdx.x * depth + l) * pw + t] = sum;
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
    if (r >= n) continue;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) dh0[(size_t)r * W + c] = dh[i][j];
    }
  }
}

// ------------------------------------------------------- residual mesh
// residual-mesh-mlp, tied-concat-residual-mesh-mlp and
// tied-rotary-residual-mesh-mlp blocks (src/simple/reference.rs:337-407):
// per block n = RMSNorm(h); the branch runs md mesh layers
//   z_l[c] = x_l[c] w0 + x_l[c+s] w1   (w1 only with two parents)
// with x_0 = n and x_l = act(z_{l-1}), ends in act(z) with the output
// activation, else z, and h += branch.  The mesh weights of all depth * md
// layers are staged in shared memory when `staged` is nonzero.  Kept for the
// backward: ns[b] / invs[b] (each block's normalised input and 1/rms),
// zs[b * md + l] (every pre-activation), hf / invf (the final RMSNorm).
template <int ACT, int J, int P>
__global__ void __launch_bounds__(kFwdWarps * 32)
    resmesh_forward(int n, int W, int depth, int md, int moa, int staged, const int* __restrict__ strides,
                    const float* __restrict__ mesh, const float* __restrict__ h0, float* __restrict__ ns,
                    float* __restrict__ invs, float* __restrict__ zs, float* __restrict__ hf,
                    float* __restrict__ invf) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  const float* wts = mesh;
  if (staged) {
    for (int i = threadIdx.x; i < staged; i += blockDim.x) sm[i] = mesh[i];
    __syncthreads();
    wts = sm;
  }
  if (r >= n) return;
  float* row = sm + staged + warp * W;
  const size_t nw = (size_t)n * W;
  float h[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    h[j] = c < W ? h0[(size_t)r * W + c] : 0.f;
  }
  for (int blk = 0; blk < depth; ++blk) {
    const float inv = row_inverse_rms<J>(h, W, lane);
    float x[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      x[j] = h[j] * inv;
      if (c < W) ns[blk * nw + (size_t)r * W + c] = x[j];
    }
    if (lane == 0) invs[(size_t)blk * n + r] = inv;
    for (int l = 0; l < md; ++l) {
      const int layer = blk * md + l;
      const int s = strides[layer];
      const float* w = wts + (size_t)layer * P * W;
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) row[c] = x[j];
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) {
          float z = x[j] * w[P * c];
          if (P == 2) z = fmaf(row[wrap_up(c, s, W)], w[P * c + 1], z);
          zs[layer * nw + (size_t)r * W + c] = z;
          x[j] = (l + 1 < md || moa) ? act_f<ACT>(z) : z;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) h[j] += x[j];
  }
  const float inv = row_inverse_rms<J>(h, W, lane);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < W) hf[(size_t)r * W + c] = h[j] * inv;
  }
  if (lane == 0) invf[r] = inv;
}

// Backward of the residual mesh blocks: dhf (gradient of the final RMSNorm
// output) in, dh0 out; per-CTA weight partials [gridDim.x][depth * md][P W]
// in parameter order.  Each warp walks its kBwdRows rows through every
// layer; the layer's weight contributions are summed per warp in registers
// in row order, then over the warps in order.
template <int ACT, int J, int P>
__global__ void __launch_bounds__(kBwdWarps * 32)
    resmesh_backward(int n, int W, int depth, int md, int moa, int staged, const int* __restrict__ strides,
                     const float* __restrict__ mesh, const float* __restrict__ ns, const float* __restrict__ invs,
                     const float* __restrict__ zs, const float* __restrict__ hf, const float* __restrict__ invf,
                     const float* __restrict__ dhf, float* __restrict__ dh0, float* __restrict__ partials) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pw = P * W;
  const float* wts = mesh;
  if (staged) {
    for (int i = threadIdx.x; i < staged; i += blockDim.x) sm[i] = mesh[i];
    __syncthreads();
    wts = sm;
  }
  float* xrow = sm + staged + warp * 2 * W;  // the layer input x_l of the current row
  float* zrow = xrow + W;                    // dz of the current row
  float* contrib = sm + staged + kBwdWarps * 2 * W;
  const size_t nw = (size_t)n * W;
  const int layers = depth * md;
  float dh[kBwdRows][J], dz[kBwdRows][J];
#pragma unroll
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
    const bool active = r < n;
    float yv[J], dv[J], dot = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      yv[j] = (active && c < W) ? hf[(size_t)r * W + c] : 0.f;
      dv[j] = (active && c < W) ? dhf[(size_t)r * W + c] : 0.f;
      dot = fmaf(dv[j], yv[j], dot);
    }
    dot = warp_sum(dot) / (float)W;
    const float iv = active ? invf[r] : 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) dh[i][j] = iv * (dv[j] - yv[j] * dot);
  }
  for (int blk = depth - 1; blk >= 0; --blk) {
    // The branch output's gradient is dh (through the output activation).
#pragma unroll
    for (int i = 0; i < kBwdRows; ++i) {
      const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        dz[i][j] = dh[i][j];
        if (moa && r < n && c < W) dz[i][j] *= act_g<ACT>(zs[(blk * md + md - 1) * nw + (size_t)r * W + c]);
      }
    }
    for (int l = md - 1; l >= 0; --l) {
      const int layer = blk * md + l;
      const int s = strides[layer];
      const float* w = wts + (size_t)layer * pw;
      float* mine = contrib + warp * pw;
      float g0[J], g1[J];
#pragma unroll
      for (int j = 0; j < J; ++j) g0[j] = g1[j] = 0.f;
#pragma unroll
      for (int i = 0; i < kBwdRows; ++i) {
        const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
        const bool active = r < n;
        float zp[J];  // z_{l-1}: the layer input is act(z_{l-1}) (n for l = 0)
        __syncwarp();
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const int c = lane + 32 * j;
          if (c < W) {
            float x;
            if (l > 0) {
              zp[j] = active ? zs[(layer - 1) * nw + (size_t)r * W + c] : 0.f;
              x = act_f<ACT>(zp[j]);
            } else {
              zp[j] = 0.f;
              x = active ? ns[blk * nw + (size_t)r * W + c] : 0.f;
            }
            xrow[c] = x;
            zrow[c] = dz[i][j];
          }
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const int c = lane + 32 * j;
          if (c < W) {
            const float d = zrow[c];
            g0[j] += d * xrow[c];
            float dx = d * w[P * c];
            if (P == 2) {
              g1[j] += d * xrow[wrap_up(c, s, W)];
              const int q = wrap_down(c, s, W);
              dx = fmaf(zrow[q], w[P * q + 1], dx);
            }
            dz[i][j] = l > 0 ? dx * act_g<ACT>(zp[j]) : dx;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        if (c < W) {
          mine[P * c] = g0[j];
          if (P == 2) mine[P * c + 1] = g1[j];
        }
      }
      __syncthreads();
      for (int t = threadIdx.x; t < pw; t += blockDim.x) {
        float sum = 0.f;
        for (int q = 0; q < kBwdWarps; ++q) sum += contrib[q * pw + t];
        partials[((size_t)blockIdx.x * layers + layer) * pw + t] = sum;
      }
      __syncthreads();
    }
    // dz now holds dn: dh += inv (dn - n <dn, n> / W)
#pragma unroll
    for (int i = 0; i < kBwdRows; ++i) {
      const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
      const bool active = r < n;
      float nv[J], dot = 0.f;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = lane + 32 * j;
        nv[j] = (active && c < W) ? ns[blk * nw + (size_t)r * W + c] : 0.f;
        dot = fmaf(dz[i][j], nv[j], dot);
      }
      dot = warp_sum(dot) / (float)W;
      const float iv = active ? invs[(size_t)blk * n + r] : 0.f;
#pragma unroll
      for (int j = 0; j < J; ++j) dh[i][j] += iv * (dz[i][j] - nv[j] * dot);
    }
  }
#pragma unroll
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = (blockIdx.x * kBwdWarps + warp) * kBwdRows + i;
    if (r >= n) continue;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (c < W) dh0[(size_t)r * W + c] = dh[i][j];
    }
  }
}

// Tied concatenation (src/simple/reference.rs:303-306, :355-359): the row
// [E a | E b] of each batch row, [n][2W].
__global__ void concat_rows(int n, int W, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                            const float* __restrict__ E, float* __restrict__ cat) {
  wait_prior_grids();
  const size_t total = (size_t)n * 2 * W;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / (2 * W);
    const int c = (int)(i % (2 * W));
    cat[i] = c < W ? E[(size_t)a[r] * W + c] : E[(size_t)b[r] * W + (c - W)];
  }
}

// Non-one-hot encodings: the first dense layer's output for every residue,
// out[k][c] = sum_f table[k mod m][f] Wx[f][c] with Wx the a half (k < m) or
// the b half (k >= m) of the layer (or the a and b embeddings of bilinear).
// One-hot gathers then read these 2m rows exactly as they read the layer's
// own rows for one-hot operands: x W0 = T[a] W0a + T[b] W0b.
__global__ void encoded_embedding(int m, int F, int W, const float* __restrict__ table, const float* __restrict__ wa,
                                  const float* __restrict__ wb, float* __restrict__ out) {
  wait_prior_grids();
  const int total = 2 * m * W;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int k = i / W, c = i % W;
    const float* x = table + (size_t)(k < m ? k : k - m) * F;
    const float* w = k < m ? wa : wb;
    float s = 0.f;
    for (int f = 0; f < F; ++f) s = fmaf(x[f], w[(size_t)f * W + c], s);
    out[i] = s;
  }
}

// Its gradient: ga[f][c] = sum over residues k (in order) of table[k][f]
// dE[k][c], gb[f][c] the same over dE[m + k][c].
__global__ void encoded_embedding_gradient(int m, int F, int W, const float* __restrict__ table,
                                           const float* __restrict__ dE, float* __restrict__ ga,
                                           float* __restrict__ gb) {
  wait_prior_grids();
  const int total = 2 * F * W;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int half = i / (F * W), rem = i % (F * W), f = rem / W, c = rem % W;
    const float* d = dE + (size_t)half * m * W;
    float s = 0.f;
    for (int k = 0; k < m; ++k) s = fmaf(table[(size_t)k * F + f], d[(size_t)k * W + c], s);
    (half == 0 ? ga : gb)[(size_t)f * W + c] = s;
  }
}

// ------------------------------------------------------------- full mesh
// full-mesh-mlp (src/simple/reference.rs:271-290): every layer's unit o
// computes x[p0] w0 + x[p1] w1 + bias with p0 = o * in / out and p1 = (p0 +
// stride) mod in; layer 0 reads the binary operand bits, later layers the
// activated outputs of the layer before.  FmLayer describes one layer: its
// shape, parameter offset (3 floats per unit) and pre-activation offset
// (floats per row of the workspace's zs, laid out [layer][row][outputs]).
struct FmLayer {
  int inputs, outputs, stride, param, z;
};
constexpr int kFmMax = 256;  // widest layer input or output of the full mesh kernels

__device__ __forceinline__ int fm_first(int o, const FmLayer& L) { return (int)((long long)o * L.inputs / L.outputs); }

// One warp per row; two row buffers per warp alternate as layer inputs.
template <int ACT>
__global__ void __launch_bounds__(kFwdWarps * 32)
    fullmesh_forward(int n, int F, int nl, const FmLayer* __restrict__ layers, const float* __restrict__ table,
                     const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, const float* __restrict__ w,
                     float* __restrict__ zs, float* __restrict__ logits) {
  wait_prior_grids();
  __shared__ float bufs[kFwdWarps][2][kFmMax];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  for (int i = lane; i < 2 * F; i += 32)
    bufs[warp][0][i] = i < F ? table[(size_t)a[r] * F + i] : table[(size_t)b[r] * F + i - F];
  __syncwarp();
  for (int l = 0; l < nl; ++l) {
    const FmLayer L = layers[l];
    const float* x = bufs[warp][l & 1];
    float* y = bufs[warp][(l + 1) & 1];
    const bool last = l + 1 == nl;
    float* z = last ? logits + (size_t)r * L.outputs : zs + (size_t)n * L.z + (size_t)r * L.outputs;
    for (int o = lane; o < L.outputs; o += 32) {
      const int p0 = fm_first(o, L);
      int p1 = p0 + L.stride;
      if (p1 >= L.inputs) p1 -= L.inputs;
      const float* u = w + L.param + 3 * o;
      const float v = fmaf(x[p1], u[1], x[p0] * u[0]) + u[2];
      z[o] = v;
      if (!last) y[o] = act_f<ACT>(v);
    }
    __syncwarp();
  }
}

// Backward: dlogits in; per-CTA weight partials [gridDim.x][P] in parameter
// order.  Each warp walks kBwdRows rows per layer: the layer's input is
// rebuilt (bits or act(z)), its output gradient dz sits in shared memory,
// unit o's contributions (dz x[p0], dz x[p1], dz) are summed per warp in
// registers in row order, and the input gradient of input i gathers the
// units whose first or second parent is i — contiguous output ranges, since
// p0(o) = o * in / out is monotone — in output order (no atomics).
template <int ACT, int J>
__global__ void __launch_bounds__(kBwdWarps * 32)
    fullmesh_backward(int n, int F, int nl, const FmLayer* __restrict__ layers, const float* __restrict__ table,
                      const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, const float* __restrict__ w,
                      const float* __restrict__ zs, const float* __restrict__ dlog, int P,
                      float* __restrict__ partials) {
  wait_prior_grids();
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* xrow = sm + warp * (kBwdRows + 1) * kFmMax;  // the layer input of the current row
  float* drow = xrow + kFmMax;                        // kBwdRows output gradients
  float* contrib = sm + kBwdWarps * (kBwdRows + 1) * kFmMax;
  const int row0 = (blockIdx.x * kBwdWarps + warp) * kBwdRows;
  const FmLayer top = layers[nl - 1];
  for (int i = 0; i < kBwdRows; ++i) {
    const int r = row0 + i;
    for (int o = lane; o < top.outputs; o += 32) drow[i * kFmMax + o] = r < n ? dlog[(size_t)r * top.outputs + o] : 0.f;
  }
  __syncwarp();
  for (int l = nl - 1; l >= 0; --l) {
    const FmLayer L = layers[l];
    float g0[J], g1[J], g2[J];
#pragma unroll
    for (int j = 0; j < J; ++j) g0[j] = g1[j] = g2[j] = 0.f;
    for (int i = 0; i < kBwdRows; ++i) {
      const int r = row0 + i;
      const bool active = r < n;
      float* d = drow + i * kFmMax;
      __syncwarp();
      for (int k = lane; k < L.inputs; k += 32) {
        float x = 0.f;
        if (active) {
          if (l == 0)
            x = k < F ? table[(size_t)a[r] * F + k] : table[(size_t)b[r] * F + k - F];
          else
            x = act_f<ACT>(zs[(size_t)n * layers[l - 1].z + (size_t)r * L.inputs + k]);
        }
        xrow[k] = x;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int o = lane + 32 * j;
        if (o < L.outputs) {
          const int p0 = fm_first(o, L);
          int p1 = p0 + L.stride;
          if (p1 >= L.inputs) p1 -= L.inputs;
          const float dz = d[o];
          g0[j] += dz * xrow[p0];
          g1[j] += dz * xrow[p1];
          g2[j] += dz;
        }
      }
      if (l > 0) {
        // dx[k] over the units whose first parent is k, then those whose
        // second parent is k (first parent (k - stride) mod in).
        float dx[kFmMax / 32];
#pragma unroll
        for (int q = 0; q < kFmMax / 32; ++q) {
          const int k = lane + 32 * q;
          dx[q] = 0.f;
          if (k < L.inputs) {
            float s = 0.f;
            for (int pass = 0; pass < 2; ++pass) {
              int first = k - (pass ? L.stride : 0);
              if (first < 0) first += L.inputs;
              // units o with o * in / out == first: o in [ceil(first out / in), ceil((first + 1) out / in))
              const int lo = (int)(((long long)first * L.outputs + L.inputs - 1) / L.inputs);
              const int hi = (int)(((long long)(first + 1) * L.outputs + L.inputs - 1) / L.inputs);
              for (int o = lo; o < hi && o < L.outputs; ++o) s = fmaf(d[o], w[L.param + 3 * o + pass], s);
            }
            const float zp = active ? zs[(size_t)n * layers[l - 1].z + (size_t)r * L.inputs + k] : 0.f;
            dx[q] = s * act_g<ACT>(zp);
          }
        }
        __syncwarp();
#pragma unroll
        for (int q = 0; q < kFmMax / 32; ++q) {
          const int k = lane + 32 * q;
          if (k < L.inputs) d[k] = dx[q];
        }
      }
    }
    float* mine = contrib + warp * 3 * kFmMax;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int o = lane + 32 * j;
      if (o < L.outputs) {
        mine[3 * o] = g0[j];
        mine[3 * o + 1] = g1[j];
        mine[3 * o + 2] = g2[j];
      }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < 3 * L.outputs; t += blockDim.x) {
      float sum = 0.f;
      for (int q = 0; q < kBwdWarps; ++q) sum += contrib[q * 3 * kFmMax + t];
      partials[(size_t)blockIdx.x * P + L.param + t] = sum;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------- mlp, bilinear
// mlp input layer on one-hot rows (src/simple/reference.rs:292-299): x W0
// with x one-hot at a and at m + b is W0[a] + W0[m + b]; z keeps the
// pre-activation for the backward pass and act = act(z) feeds layer 1.
template <int ACT>
__global__ void mlp_input(int n, int W, int m, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                          const float* __restrict__ w0, float* __restrict__ z, float* __restrict__ act) {
  wait_prior_grids();
  const size_t count = (size_t)n * W;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / W, c = i % W;
    const float v = w0[(size_t)a[r] * W + c] + w0[(size_t)(m + b[r]) * W + c];
    z[i] = v;
    act[i] = act_f<ACT>(v);
  }
}

template <int ACT>
__global__ void activate(size_t count, const float* __restrict__ z, float* __restrict__ act) {
  wait_prior_grids();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
    act[i] = act_f<ACT>(z[i]);
}

// bilinear (src/simple/reference.rs:434-444): left = E_a[a], right = E_b[b]
// (one-hot rows), p = left * right elementwise.
__global__ void bilinear_input(int n, int W, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                               const float* __restrict__ ea, const float* __restrict__ eb, float* __restrict__ p) {
  wait_prior_grids();
  const size_t count = (size_t)n * W;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / W, c = i % W;
    p[i] = ea[(size_t)a[r] * W + c] * eb[(size_t)b[r] * W + c];
  }
}

// dleft = dp * right, dright = dp * left (the embeddings gathered again).
__global__ void bilinear_gradient(int n, int W, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                                  const float* __restrict__ ea, const float* __restrict__ eb,
                                  const float* __restrict__ dp, float* __restrict__ dleft,
                                  float* __restrict__ dright) {
  wait_prior_grids();
  const size_t count = (size_t)n * W;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / W, c = i % W;
    dleft[i] = dp[i] * eb[(size_t)b[r] * W + c];
    dright[i] = dp[i] * ea[(size_t)a[r] * W + c];
  }
}

// ------------------------------------------------------------ embedding
// Per class k (one CTA each): the ordered sum over batch rows of the
// operand-embedding gradients that use row k of the embedding.
//  mode 0 (mesh-mlp, 2m rows of W0): k < m takes rows with a == k,
//         k >= m rows with b == k - m, both as dh0[r][c].
//  mode 1 (rotary): rows with a == k add dh0[r][c]; rows with b == k add
//         the transposed rotation of dh0[r] (dh0[r][c^1], negated for odd c).
//  mode 2 / 3 (bilinear, m rows of one operand's embedding): rows with
//         a == k (mode 2) or b == k (mode 3) add dh0[r][c].
//  mode 4 (tied concatenation, dh0 rows of 2W): rows with a == k add
//         dh0[r][c], rows with b == k add dh0[r][W + c].
// `extra` ([rows][W], may be null) is added (the readout's share of dE).
// The block of class k first gathers every matching row (in row order) into
// a shared list, scanning 512 rows per round, and only then sums the rows'
// gradients, 16 loads in flight per thread: the additions per column keep
// row order, so the result does not depend on the launch shape.  A list
// that could overflow is summed and emptied on the way.
constexpr int kClassThreads = 512;
constexpr int kClassList = 4096;  // matching rows held before they are summed
__global__ void __launch_bounds__(kClassThreads)
    class_gradient(int n, int W, int m, int mode, const uint32_t* __restrict__ a, const uint32_t* __restrict__ b,
                   const float* __restrict__ dh0, const float* __restrict__ extra, float* __restrict__ out) {
  wait_prior_grids();
  __shared__ int list[kClassList];
  __shared__ uint8_t kinds[kClassList];
  __shared__ int warp_count[kClassThreads / 32];
  __shared__ int total;
  const int k = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kPer = (kMaxKernelWidth + kClassThreads - 1) / kClassThreads;
  float acc[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) acc[j] = 0.f;
  if (tid == 0) total = 0;
  __syncthreads();
  const int stride = mode == 4 ? 2 * W : W;
  // Sums list[0, cnt) into acc in list order, kBatch rows' loads at a time.
  auto sum_list = [&](int cnt) {
    constexpr int kBatch = 16;
    for (int e0 = 0; e0 < cnt; e0 += kBatch) {
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int c = tid + kClassThreads * j;
        if (c >= W) continue;
        const int c2 = mode == 4 ? W + c : (c ^ 1);
        float v1[kBatch], v2[kBatch];
        int kd[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          kd[i] = e0 + i < cnt ? kinds[e0 + i] : 0;
          const float* g = dh0 + (size_t)(e0 + i < cnt ? list[e0 + i] : 0) * stride;
          v1[i] = (kd[i] & 1) ? g[c] : 0.f;
          v2[i] = (kd[i] & 2) ? g[c2] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
          if (kd[i] & 1) acc[j] += v1[i];
          if (kd[i] & 2) acc[j] += (mode == 4 || !(c & 1)) ? v2[i] : -v2[i];
        }
      }
    }
  };
  for (int r0 = 0; r0 < n; r0 += kClassThreads) {
    const int r = r0 + tid;
    int kind = 0;
    if (r < n) {
      if (mode == 0) {
        kind = (k < m) ? (a[r] == (uint32_t)k ? 1 : 0) : (b[r] == (uint32_t)(k - m) ? 1 : 0);
      } else if (mode == 2 || mode == 3) {
        kind = (mode == 2 ? a[r] : b[r]) == (uint32_t)k ? 1 : 0;
      } else {  // modes 1 and 4
        kind = (a[r] == (uint32_t)k ? 1 : 0) | (b[r] == (uint32_t)k ? 2 : 0);
      }
    }
    const unsigned ballot = __ballot_sync(kFull, kind != 0);
    if (lane == 0) warp_count[warp] = __popc(ballot);
    __syncthreads();
    if (tid == 0) {
      int s = total;
      for (int q = 0; q < kClassThreads / 32; ++q) {
        const int c = warp_count[q];
        warp_count[q] = s;
        s += c;
      }
      total = s;
    }
    __syncthreads();
    if (kind != 0) {
      const int pos = warp_count[warp] + __popc(ballot & ((1u << lane) - 1u));
      list[pos] = r;
      kinds[pos] = (uint8_t)kind;
    }
    __syncthreads();
    if (total > kClassList - kClassThreads) {  // room for one more round only
      sum_list(total);
      __syncthreads();
      if (tid == 0) total = 0;
      __syncthreads();
    }
  }
  sum_list(total);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int c = tid + kClassThreads * j;
    if (c < W) out[(size_t)k * W + c] = acc[j] + (extra != nullptr ? extra[(size_t)k * W + c] : 0.f);
  }
}

// ------------------------------------------------------- loss and update
// dlogits = (softmax - onehot) / rows (src/simple/gpu.rs:664-739); flags
// nonfinite logits.
__global__ void __launch_bounds__(kFwdWarps * 32)
    cross_entropy_gradient(int n, int m, const float* __restrict__ logits, const uint32_t* __restrict__ y,
                           float* __restrict__ dlog, int* __restrict__ flags) {
  wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  const float* x = logits + (size_t)r * m;
  float mx = -INFINITY;
  bool finite = true;
  for (int k = lane; k < m; k += 32) {
    finite &= isfinite(x[k]);
    mx = fmaxf(mx, x[k]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
  float s = 0.f;
  for (int k = lane; k < m; k += 32) s += expf(x[k] - mx);
  s = warp_sum(s);
  if (!__all_sync(kFull, finite) && lane == 0) atomicExch(flags + kFlagNonfinite, 1);
  const float scale = 1.0f / (float)n;
  const uint32_t t = y[r];
  for (int k = lane; k < m; k += 32) {
    const float p = expf(x[k] - mx) / s;
    dlog[(size_t)r * m + k] = (p - (k == (int)t ? 1.f : 0.f)) * scale;
  }
}

// First maximum per row; nonfinite rows get 0xFFFFFFFF
// (src/simple/gpu.rs:748-772).
__global__ void __launch_bounds__(kFwdWarps * 32)
    predictions(int n, int m, const float* __restrict__ logits, uint32_t* __restrict__ out) {
  wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kFwdWarps + warp;
  if (r >= n) return;
  const float* x = logits + (size_t)r * m;
  float best = -INFINITY;
  int arg = m;
  bool finite = true;
  for (int k = lane; k < m; k += 32) {
    finite &= isfinite(x[k]);
    if (x[k] > best || arg == m) {
      if (arg == m || x[k] > best) {
        best = x[k];
        arg = k;
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ob = __shfl_xor_sync(kFull, best, o);
    const int oa = __shfl_xor_sync(kFull, arg, o);
    if (ob > best || (ob == best && oa < arg)) {
      best = ob;
      arg = oa;
    }
  }
  finite = __all_sync(kFull, finite);
  if (lane == 0) out[r] = finite ? (uint32_t)arg : 0xFFFFFFFFu;
}

// simple_adam (src/simple/gpu.rs:787-812) over the flat parameters; groups
// from index `mesh_start` on train at lr_mesh.
// With `channel` (one-layer mlp, decay_factors != 2) the decay of the input
// layer's weight i (< n_in, channel i % W) and of the readout's weight i
// (channel (i - n_in) / m) is channel[c] instead of the uniform decay
// (simple_adam_channels, src/simple/gpu.rs:846-881).
__global__ void adamw(size_t count, size_t mesh_start, const StepScalars* __restrict__ sc,
                      const float* __restrict__ grad, float* __restrict__ w, float* __restrict__ m1,
                      float* __restrict__ m2, const float* __restrict__ channel, int W, int m, size_t n_in) {
  wait_prior_grids();
  const float b1 = sc->beta1, b2 = sc->beta2, eps = sc->epsilon;
  const float c1 = sc->correction1, c2 = sc->correction2;
  const float ob1 = __fsub_rn(1.0f, b1), ob2 = __fsub_rn(1.0f, b2);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const float wd = channel == nullptr ? sc->weight_decay : channel[i < n_in ? i % W : (i - n_in) / m];
    const float lr = i < mesh_start ? sc->lr_dense : sc->lr_mesh;
    const float g = grad[i];
    const float mm = __fadd_rn(__fmul_rn(b1, m1[i]), __fmul_rn(ob1, g));
    const float vv = __fadd_rn(__fmul_rn(b2, m2[i]), __fmul_rn(__fmul_rn(ob2, g), g));
    m1[i] = mm;
    m2[i] = vv;
    const float mh = __fdiv_rn(mm, c1), vh = __fdiv_rn(vv, c2);
    const float upd = __fadd_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), __fmul_rn(wd, w[i]));
    w[i] = __fsub_rn(w[i], __fmul_rn(lr, upd));
  }
}

// Channel decay of a one-layer mlp (simple_channel_decay, src/simple/gpu.rs:
// 814-844): out[c] = min(wd max(s_c, FLT_MIN)^exponent, 1 / lr) with
// s_c = (sum_i E[i][c]^2 + sum_k R[c][k]^2) / 2 over the weights before
// the step (E input-major [inputs][W], R [W][m]).
__global__ void channel_decay(int inputs, int W, int m, float exponent, const StepScalars* __restrict__ sc,
                              const float* __restrict__ E, const float* __restrict__ R, float* __restrict__ out) {
  wait_prior_grids();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= W) return;
  float squares = 0.f;
  for (int i = 0; i < inputs; ++i) {
    const float x = E[(size_t)i * W + c];
    squares = __fadd_rn(squares, __fmul_rn(x, x));
  }
  for (int k = 0; k < m; ++k) {
    const float x = R[(size_t)c * m + k];
    squares = __fadd_rn(squares, __fmul_rn(x, x));
  }
  const float scale = powf(fmaxf(0.5f * squares, 1.17549435e-38f), exponent);
  out[c] = fminf(sc->weight_decay * scale, 1.0f / sc->lr_dense);
}

// ================================================================ executor
class DeviceBuffers {
 public:
  ~DeviceBuffers() {
    for (void* p : ptrs_) cudaFree(p);
  }
  template <class T>
  T* alloc(size_t n) {
    void* p = nullptr;
    SIMPLE_CUDA(cudaMalloc(&p, n == 0 ? 16 : n * sizeof(T)));
    ptrs_.push_back(p);
    return static_cast<T*>(p);
  }

 private:
  std::vector<void*> ptrs_;
};

struct Workspace {
  int n = 0;
  DeviceBuffers mem;
  uint32_t *a = nullptr, *b = nullptr, *y = nullptr;
  float *logits = nullptr, *dlog = nullptr;
  float *h = nullptr, *act = nullptr, *dact = nullptr, *dh0 = nullptr, *part = nullptr;  // mesh-mlp
  float *hs = nullptr, *ns = nullptr, *invs = nullptr, *zs = nullptr, *dh = nullptr, *dz = nullptr, *dn = nullptr,
        *dhf = nullptr, *dEread = nullptr, *gemm_part = nullptr;
  float *hf = nullptr, *invf = nullptr, *states = nullptr, *dEemb = nullptr,
        *dv = nullptr;  // shared-Neighbor (dv: the chain's per-CTA weight partials)
  float *es = nullptr, *as = nullptr, *dex = nullptr, *dax = nullptr;  // residual-mlp expansion
  float *cat = nullptr, *dcat = nullptr;  // tied concatenation [E a | E b] and its gradient
  int bwd_ctas = 0;
  cudaGraphExec_t step_graph = nullptr;
  uint32_t step_launches = 0;
  ~Workspace() {
    if (step_graph) cudaGraphExecDestroy(step_graph);
  }
};

}  // namespace simple
}  // namespace mb

struct mb_simple_table {
  const void* owner;
  size_t rows;
  mb::simple::DeviceBuffers mem;
  uint32_t *a, *b, *t, *identity;
};

namespace mb {
namespace simple {
// Device index buffers kept by a model for its uploaded batches.  A batch
// set takes a buffer from the pool and gives it back when destroyed, so the
// per-epoch upload of the reference's training loop (one per step at full
// batch) allocates nothing once the pool holds a buffer of that size.  Each
// buffer has a page-locked staging copy: the caller's indices are copied
// there on the host and then to the device asynchronously (a copy from
// pageable memory may wait for the stream, which would serialise the host
// with every queued step); an event recorded after that copy guards the
// staging buffer's next reuse.  The pool outlives the model while batch sets
// still hold buffers.  Device buffers are only written by copies on the
// model's stream, in order after every step that read them before.
struct IndexBuffer {
  uint32_t* dev = nullptr;
  uint32_t* host = nullptr;
  size_t capacity = 0;
  cudaEvent_t copied = nullptr;
};

class IndexPool {
 public:
  explicit IndexPool(int device) : device_(device) {}
  ~IndexPool() {
    cudaSetDevice(device_);
    for (auto& kv : free_) release(kv.second);
  }
  IndexBuffer take(size_t count) {
    {
      std::lock_guard<std::mutex> lock(mu_);
      auto it = free_.lower_bound(count);
      if (it != free_.end() && it->first <= 2 * count + 4096) {
        IndexBuffer b = it->second;
        free_.erase(it);
        return b;
      }
    }
    IndexBuffer b;
    b.capacity = count;
    SIMPLE_CUDA(cudaMalloc(&b.dev, count * sizeof(uint32_t)));
    cudaError_t e = cudaHostAlloc(&b.host, count * sizeof(uint32_t), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b.copied, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      release(b);
      throw Error(MB_ERR_CUDA, std::string("index staging buffer: ") + cudaGetErrorString(e));
    }
    return b;
  }
  void give(const IndexBuffer& b) {
    std::lock_guard<std::mutex> lock(mu_);
    free_.emplace(b.capacity, b);
    while (free_.size() > 8) {  // keep a few: the largest go first
      auto last = std::prev(free_.end());
      cudaSetDevice(device_);
      release(last->second);
      free_.erase(last);
    }
  }

 private:
  static void release(const IndexBuffer& b) {
    if (b.copied) {
      cudaEventSynchronize(b.copied);
      cudaEventDestroy(b.copied);
    }
    if (b.host) cudaFreeHost(b.host);
    if (b.dev) cudaFree(b.dev);
  }
  int device_;
  std::mutex mu_;
  std::multimap<size_t, IndexBuffer> free_;
};
}  // namespace simple
}  // namespace mb

struct mb_simple_batches {
  const void* owner;
  size_t count, table_rows;
  std::shared_ptr<mb::simple::IndexPool> pool;
  mb::simple::IndexBuffer buf;
  uint32_t* idx = nullptr;
  ~mb_simple_batches() {
    if (idx != nullptr) pool->give(buf);
  }
};

namespace mb {
namespace simple {

class SimpleModel {
 public:
  SimpleModel(int device, const mb_simple_config& c, uint64_t seed) : c_(c), device_(device) {
    validate_kernel_shapes(c);
    int count = 0;
    SIMPLE_CUDA(cudaGetDeviceCount(&count));
    require(device >= 0 && device < count, "CUDA device index out of range");
    SIMPLE_CUDA(cudaSetDevice(device));
    SIMPLE_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    index_pool_ = std::make_shared<IndexPool>(device);
    gemm_prepare();
    groups_ = groups(c);
    size_t off = 0;
    for (size_t g : groups_) {
      offsets_.push_back(off);
      off += g;
    }
    P_ = off;
    mesh_start_ = 0;
    for (size_t i = 0; i < dense_layers(c).size(); ++i) mesh_start_ += groups_[i];
    w_ = mem_.alloc<float>(P_);
    m1_ = mem_.alloc<float>(P_);
    m2_ = mem_.alloc<float>(P_);
    grad_ = mem_.alloc<float>(P_);
    flags_ = mem_.alloc<int>(kFlags);
    scalars_ = mem_.alloc<StepScalars>(1);
    SIMPLE_CUDA(cudaHostAlloc((void**)&host_scalars_, kScalarSlots * sizeof(StepScalars), cudaHostAllocDefault));
    for (int i = 0; i < kScalarSlots; ++i)
      SIMPLE_CUDA(cudaEventCreateWithFlags(&scalar_copied_[i], cudaEventDisableTiming));
    SIMPLE_CUDA(cudaMemsetAsync(flags_, 0, kFlags * sizeof(int), stream_));
    SIMPLE_CUDA(cudaMemsetAsync(grad_, 0, P_ * sizeof(float), stream_));
    // Strides per mesh layer (mesh stacks) or per core layer (shared-Neighbor).
    const bool per_mesh = c.architecture == kMeshMlp || c.architecture == kTiedConcatMesh || residual_mesh(c);
    const int nstr = per_mesh ? std::max(1, mesh_layers(c)) : std::max(1, (int)c.depth);
    std::vector<int> st(nstr);
    for (int l = 0; l < nstr; ++l) st[l] = stride(c, l);
    strides_ = mem_.alloc<int>(nstr);
    SIMPLE_CUDA(cudaMemcpy(strides_, st.data(), nstr * sizeof(int), cudaMemcpyHostToDevice));
    if (c.encoding != kOneHot) {
      // Encoded operands: the residues' rows through the first layer are
      // formed per step (encoded_embedding) and gathered like one-hot rows.
      const std::vector<float> t = encoding_table(c);
      const size_t mw = (size_t)c.modulus * c.width;
      enc_table_ = mem_.alloc<float>(t.size());
      enc_rows_ = mem_.alloc<float>(2 * mw);
      enc_grad_ = mem_.alloc<float>(2 * mw);
      SIMPLE_CUDA(cudaMemcpy(enc_table_, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    if (c.decay_factors != 2) chan_decay_ = mem_.alloc<float>(c.width);
    if (c.architecture == kFullMesh) {
      std::vector<FmLayer> fl;
      int param = 0, z = 0;
      for (const auto& l : two_parent_layers(c)) {
        fl.push_back({(int)l.inputs, (int)l.outputs, (int)l.stride, param, z});
        param += 3 * (int)l.outputs;
        z += (int)l.outputs;
      }
      fm_z_ = z - (int)c.modulus;  // the readout writes the logits
      fm_layers_ = mem_.alloc<FmLayer>(fl.size());
      SIMPLE_CUDA(cudaMemcpy(fm_layers_, fl.data(), fl.size() * sizeof(FmLayer), cudaMemcpyHostToDevice));
    }
    set_parameters(initial_parameters(c, seed).data(), P_);
    set_attributes();
  }
  ~SimpleModel() {
    workspaces_.clear();
    if (stream_) cudaStreamSynchronize(stream_);
    for (cudaEvent_t e : scalar_copied_)
      if (e) cudaEventDestroy(e);
    if (host_scalars_) cudaFreeHost(host_scalars_);
    if (stream_) cudaStreamDestroy(stream_);
  }

  const mb_simple_config& config() const { return c_; }
  size_t count() const { return P_; }
  cudaStream_t stream() const { return stream_; }

  void set_parameters(const float* v, size_t n) {
    require(n == P_, "parameter count does not match the model");
    for (size_t i = 0; i < n; ++i) require(std::isfinite(v[i]), "parameters must be finite", MB_ERR_NONFINITE);
    SIMPLE_CUDA(cudaSetDevice(device_));
    SIMPLE_CUDA(cudaMemcpyAsync(w_, v, P_ * sizeof(float), cudaMemcpyHostToDevice, stream_));
    SIMPLE_CUDA(cudaMemsetAsync(m1_, 0, P_ * sizeof(float), stream_));
    SIMPLE_CUDA(cudaMemsetAsync(m2_, 0, P_ * sizeof(float), stream_));
    SIMPLE_CUDA(cudaStreamSynchronize(stream_));
    beta1_power_ = 1.0f;
    beta2_power_ = 1.0f;
  }

  void get_parameters(float* out, size_t n) {
    require(n == P_, "parameter count does not match the model");
    SIMPLE_CUDA(cudaSetDevice(device_));
    SIMPLE_CUDA(cudaMemcpyAsync(out, w_, P_ * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    SIMPLE_CUDA(cudaStreamSynchronize(stream_));
    for (size_t i = 0; i < n; ++i) require(std::isfinite(out[i]), "nonfinite parameters", MB_ERR_NONFINITE);
  }

  mb_simple_table* upload_table(const float* features, const uint32_t* targets, size_t rows) {
    require(rows >= 1 && rows <= kMaxRows, "tables need 1..=131072 rows");
    std::vector<uint32_t> a, b;
    decode_operands(c_, features, targets, rows, a, b);
    std::vector<uint32_t> ident(rows);
    for (size_t i = 0; i < rows; ++i) ident[i] = (uint32_t)i;
    SIMPLE_CUDA(cudaSetDevice(device_));
    auto t = std::make_unique<mb_simple_table>();
    t->owner = this;
    t->rows = rows;
    t->a = t->mem.alloc<uint32_t>(rows);
    t->b = t->mem.alloc<uint32_t>(rows);
    t->t = t->mem.alloc<uint32_t>(rows);
    t->identity = t->mem.alloc<uint32_t>(rows);
    SIMPLE_CUDA(cudaMemcpy(t->a, a.data(), rows * 4, cudaMemcpyHostToDevice));
    SIMPLE_CUDA(cudaMemcpy(t->b, b.data(), rows * 4, cudaMemcpyHostToDevice));
    SIMPLE_CUDA(cudaMemcpy(t->t, targets, rows * 4, cudaMemcpyHostToDevice));
    SIMPLE_CUDA(cudaMemcpy(t->identity, ident.data(), rows * 4, cudaMemcpyHostToDevice));
    return t.release();
  }

  mb_simple_batches* upload_batches(const mb_simple_table* table, const uint32_t* idx, size_t count) {
    check_table(table);
    require(count >= 1 && count <= kMaxRows, "batches need 1..=131072 indices");
    for (size_t i = 0; i < count; ++i) require(idx[i] < table->rows, "batch index is outside the table");
    SIMPLE_CUDA(cudaSetDevice(device_));
    auto bt = std::make_unique<mb_simple_batches>();
    bt->owner = this;
    bt->count = count;
    bt->table_rows = table->rows;
    bt->pool = index_pool_;
    bt->buf = index_pool_->take(count);
    bt->idx = bt->buf.dev;
    // The staging copy's previous transfer has completed; the device copy is
    // ordered on the model's stream after every step that read a recycled
    // buffer, and the caller's indices may be reused as soon as this returns.
    SIMPLE_CUDA(cudaEventSynchronize(bt->buf.copied));
    std::memcpy(bt->buf.host, idx, count * 4);
    SIMPLE_CUDA(cudaMemcpyAsync(bt->idx, bt->buf.host, count * 4, cudaMemcpyHostToDevice, stream_));
    SIMPLE_CUDA(cudaEventRecord(bt->buf.copied, stream_));
    return bt.release();
  }

  void train_step(const mb_simple_table* table, const mb_simple_batches* batches, size_t offset, size_t rows,
                  const mb_adamw& o) {
    check_table(table);
    check_batches(table, batches, offset, rows);
    mb::validate_optimizer(o);
    SIMPLE_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace((int)rows);
    // AdamW corrections from f32 host powers (src/simple/gpu.rs:2044-2047).
    beta1_power_ *= o.beta1;
    beta2_power_ *= o.beta2;
    StepScalars s{};
    s.idx = batches->idx;
    s.ta = table->a;
    s.tb = table->b;
    s.tt = table->t;
    s.offset = (uint32_t)offset;
    s.lr_dense = o.learning_rate;
    s.lr_mesh = o.learning_rate * (float)c_.mesh_learning_rate_multiplier;
    s.weight_decay = o.weight_decay;
    s.beta1 = o.beta1;
    s.beta2 = o.beta2;
    s.epsilon = o.epsilon;
    s.correction1 = 1.0f - beta1_power_;
    s.correction2 = 1.0f - beta2_power_;
    // Through a ring of page-locked slots, so the copy does not wait for the
    // stream; a slot is rewritten once its copy of kScalarSlots steps ago is done.
    const int slot = (int)(scalar_step_++ % kScalarSlots);
    SIMPLE_CUDA(cudaEventSynchronize(scalar_copied_[slot]));
    host_scalars_[slot] = s;
    SIMPLE_CUDA(cudaMemcpyAsync(scalars_, host_scalars_ + slot, sizeof(s), cudaMemcpyHostToDevice, stream_));
    SIMPLE_CUDA(cudaEventRecord(scalar_copied_[slot], stream_));
    if (ws.step_graph == nullptr) {
      cudaGraph_t g = nullptr;
      SIMPLE_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
      launches_ = 0;
      try {
        enqueue_gather(ws, table, batches->idx, true);
        enqueue_forward(ws);
        enqueue_loss(ws);
        enqueue_backward(ws);
        enqueue_update();
      } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      SIMPLE_CUDA(cudaStreamEndCapture(stream_, &g));
      cudaError_t e = programmatic_edges(g);
      if (e == cudaSuccess) e = cudaGraphInstantiate(&ws.step_graph, g, 0);
      cudaGraphDestroy(g);
      SIMPLE_CUDA(e);
      ws.step_launches = launches_;
    }
    last_launches_ = ws.step_launches;
    SIMPLE_CUDA(cudaGraphLaunch(ws.step_graph, stream_));
  }

  void evaluate(const mb_simple_table* table, float* logits, uint32_t* preds) {
    check_table(table);
    SIMPLE_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace((int)table->rows);
    enqueue_gather(ws, table, table->identity, false);
    enqueue_forward(ws);
    const int n = ws.n, m = (int)c_.modulus;
    predictions<<<(n + kFwdWarps - 1) / kFwdWarps, kFwdWarps * 32, 0, stream_>>>(n, m, ws.logits, ws.a); ++launches_;
    SIMPLE_CUDA(cudaGetLastError());
    std::vector<uint32_t> p(n);
    SIMPLE_CUDA(cudaMemcpyAsync(p.data(), ws.a, n * 4, cudaMemcpyDeviceToHost, stream_));
    if (logits != nullptr)
      SIMPLE_CUDA(cudaMemcpyAsync(logits, ws.logits, (size_t)n * m * 4, cudaMemcpyDeviceToHost, stream_));
    SIMPLE_CUDA(cudaStreamSynchronize(stream_));
    check_tc();
    for (uint32_t v : p) require(v != 0xFFFFFFFFu, "logits must contain only finite values", MB_ERR_NONFINITE);
    if (preds != nullptr) std::memcpy(preds, p.data(), n * 4);
  }

  double loss_and_gradient(const mb_simple_table* table, const uint32_t* idx, size_t count, float* grad,
                           size_t ngrad) {
    require(ngrad == P_, "gradient length must equal the parameter count");
    std::unique_ptr<mb_simple_batches> bt(upload_batches(table, idx, count));
    Workspace& ws = workspace((int)count);
    enqueue_gather(ws, table, bt->idx, false);
    enqueue_forward(ws);
    enqueue_loss(ws);
    enqueue_backward(ws);
    const int m = (int)c_.modulus;
    std::vector<float> lg((size_t)count * m);
    std::vector<uint32_t> tg(table->rows);
    SIMPLE_CUDA(cudaMemcpyAsync(lg.data(), ws.logits, lg.size() * 4, cudaMemcpyDeviceToHost, stream_));
    SIMPLE_CUDA(cudaMemcpyAsync(grad, grad_, P_ * 4, cudaMemcpyDeviceToHost, stream_));
    SIMPLE_CUDA(cudaMemcpyAsync(tg.data(), table->t, table->rows * 4, cudaMemcpyDeviceToHost, stream_));
    SIMPLE_CUDA(cudaStreamSynchronize(stream_));
    check_tc();
    // The mean answer cross-entropy from the f32 logits in f64, row order
    // (src/simple/gpu.rs:2005-2019).
    double loss = 0.0;
    for (size_t r = 0; r < count; ++r) {
      const float* x = lg.data() + r * m;
      double mx = -INFINITY;
      for (int k = 0; k < m; ++k) {
        require(std::isfinite(x[k]), "logits must contain only finite values", MB_ERR_NONFINITE);
        mx = std::max(mx, (double)x[k]);
      }
      double s = 0.0;
      for (int k = 0; k < m; ++k) s += std::exp((double)x[k] - mx);
      loss += std::log(s) + mx - (double)x[tg[idx[r]]];
    }
    for (size_t i = 0; i < P_; ++i) require(std::isfinite(grad[i]), "nonfinite gradients", MB_ERR_NONFINITE);
    return loss / (double)count;
  }

  void check() {
    SIMPLE_CUDA(cudaSetDevice(device_));
    SIMPLE_CUDA(cudaStreamSynchronize(stream_));
    check_tc();
    int f[kFlags];
    SIMPLE_CUDA(cudaMemcpy(f, flags_, sizeof(f), cudaMemcpyDeviceToHost));
    if (f[kFlagNonfinite]) {
      SIMPLE_CUDA(cudaMemset(flags_, 0, sizeof(f)));
      throw Error(MB_ERR_NONFINITE, "nonfinite logits during training");
    }
  }

  // Kernels launched by the latest training step (0 before the first).
  uint32_t step_launches() const { return last_launches_; }

 private:
  // Row values per lane (J) of the templated row kernels for this width.
  template <class F>
  static void with_j(int W, F&& f) {
    if (W <= 128)
      f(std::integral_constant<int, 4>{});
    else if (W <= 256)
      f(std::integral_constant<int, 8>{});
    else if (W <= 384)
      f(std::integral_constant<int, 12>{});
    else
      f(std::integral_constant<int, 16>{});
  }
  int core_smem_floats() const {
    const int f = (int)c_.depth * 3 * (int)c_.width;
    return c_.architecture == kSharedNeighbor && f <= kCoreSmemFloats ? f : 0;
  }
  int fwd_smem() const { return (core_smem_floats() + kFwdWarps * (int)c_.width) * 4; }
  // CTAs of the chain kernels: kChainThreads / W class rows each.
  int chain_ctas() const {
    const int RG = kChainThreads / (int)c_.width;
    return ((int)c_.modulus + RG - 1) / RG;
  }
  int bwd_smem() const { return (core_smem_floats() + kBwdWarps * 5 * (int)c_.width) * 4; }
  // Residual mesh kernels: all mesh weights staged in shared memory when
  // they fit beside the backward's per-warp rows and contributions.
  int resmesh_staged() const {
    if (!residual_mesh(c_)) return 0;
    const int f = mesh_layers(c_) * parents(c_) * (int)c_.width;
    const int rows = kBwdWarps * (2 + parents(c_)) * (int)c_.width;
    return f <= kCoreSmemFloats && f + rows <= kSmemFloats ? f : 0;
  }
  int resmesh_fwd_smem() const { return (resmesh_staged() + kFwdWarps * (int)c_.width) * 4; }
  static int fullmesh_bwd_smem() { return (kBwdWarps * (kBwdRows + 1) * kFmMax + kBwdWarps * 3 * kFmMax) * 4; }
  int resmesh_bwd_smem() const {
    return (resmesh_staged() + kBwdWarps * (2 + parents(c_)) * (int)c_.width) * 4;
  }

  template <int ACT>
  void set_attributes_impl() {
    const int fs = fwd_smem(), bs = bwd_smem();
    with_j(j_width(), [&](auto jc) {
      constexpr int J = decltype(jc)::value;
      SIMPLE_CUDA(cudaFuncSetAttribute(&mlp_forward<ACT, J>, cudaFuncAttributeMaxDynamicSharedMemorySize, fs));
      SIMPLE_CUDA(cudaFuncSetAttribute(&mlp_backward<ACT, J>, cudaFuncAttributeMaxDynamicSharedMemorySize, bs));
      SIMPLE_CUDA(cudaFuncSetAttribute(&shared_forward<ACT, J>, cudaFuncAttributeMaxDynamicSharedMemorySize, fs));
      SIMPLE_CUDA(cudaFuncSetAttribute(&shared_backward<ACT, J>, cudaFuncAttributeMaxDynamicSharedMemorySize, bs));
      if (c_.architecture == kFullMesh)
        SIMPLE_CUDA(cudaFuncSetAttribute(&fullmesh_backward<ACT, J>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         fullmesh_bwd_smem()));
      if (residual_mesh(c_)) {
        const int rf = resmesh_fwd_smem(), rb = resmesh_bwd_smem();
        SIMPLE_CUDA(cudaFuncSetAttribute(&resmesh_forward<ACT, J, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, rf));
        SIMPLE_CUDA(cudaFuncSetAttribute(&resmesh_forward<ACT, J, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, rf));
        SIMPLE_CUDA(cudaFuncSetAttribute(&resmesh_backward<ACT, J, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, rb));
        SIMPLE_CUDA(cudaFuncSetAttribute(&resmesh_backward<ACT, J, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, rb));
      }
    });
  }
  void set_attributes() {
    if (c_.activation == kRelu)
      set_attributes_impl<kRelu>();
    else
      set_attributes_impl<kSquare>();
  }

  void check_table(const mb_simple_table* t) const {
    need(t, "table");
    require(t->owner == this, "the table belongs to another model");
  }
  void check_batches(const mb_simple_table* t, const mb_simple_batches* b, size_t offset, size_t rows) const {
    need(b, "batches");
    require(b->owner == this, "the batches belong to another model");
    require(b->table_rows == t->rows, "batch indices belong to a table with another row count");
    require(rows >= 1 && rows <= kMaxRows && offset <= b->count && rows <= b->count - offset,
            "minibatch is outside the uploaded indices");
  }
  void check_tc() {
    int f = 0;
    SIMPLE_CUDA(cudaMemcpy(&f, flags_ + kFlagTc, sizeof(int), cudaMemcpyDeviceToHost));
    if (f) {
      SIMPLE_CUDA(cudaMemset(flags_ + kFlagTc, 0, sizeof(int)));
      throw Error(MB_ERR_CUDA, "a tensor-core wait gave up (bounded mbarrier wait)");
    }
  }

  Workspace& workspace(int n) {
    for (auto& w : workspaces_)
      if (w->n == n) return *w;
    if (workspaces_.size() == 3) workspaces_.erase(workspaces_.begin());
    auto w = std::make_unique<Workspace>();
    w->n = n;
    const size_t W = c_.width, m = c_.modulus, N = (size_t)n;
    const size_t nw = N * W;
    auto& M = w->mem;
    w->a = M.alloc<uint32_t>(N);
    w->b = M.alloc<uint32_t>(N);
    w->y = M.alloc<uint32_t>(N);
    w->logits = M.alloc<float>(N * m);
    w->dlog = M.alloc<float>(N * m);
    w->dh0 = M.alloc<float>(nw);
    w->dhf = M.alloc<float>(nw);
    const int ctas = (int)((N + kBwdWarps * kBwdRows - 1) / (kBwdWarps * kBwdRows));
    w->bwd_ctas = ctas;
    size_t part = 0;
    if (tied_concat(c_)) {
      w->cat = M.alloc<float>(2 * nw);
      w->dcat = M.alloc<float>(2 * nw);
      w->dEread = M.alloc<float>(m * W);
      part = std::max(gemm_partial_floats((int)(2 * W), (int)W, n, kSplitK),
                      gemm_partial_floats((int)m, (int)W, n, kSplitK));
    }
    if (c_.architecture == kFullMesh) {
      w->zs = M.alloc<float>((size_t)fm_z_ * N);
      w->part = M.alloc<float>((size_t)ctas * P_);
    } else if (c_.architecture == kMeshMlp || c_.architecture == kTiedConcatMesh) {
      const int L = mesh_layers(c_);
      w->h = M.alloc<float>((L + 1) * nw);
      w->act = M.alloc<float>(nw);
      w->dact = w->dhf;
      w->part = M.alloc<float>((size_t)ctas * std::max(L, 1) * parents(c_) * W);
      part = std::max(part, gemm_partial_floats((int)W, (int)m, n, kSplitK));
    } else if (residual_mesh(c_)) {
      // h0, per block ns / invs, every mesh pre-activation zs, hf / invf
      const size_t d = c_.depth, L = (size_t)mesh_layers(c_);
      w->h = M.alloc<float>(nw);
      w->ns = M.alloc<float>(d * nw);
      w->invs = M.alloc<float>(d * N);
      w->zs = M.alloc<float>(L * nw);
      w->hf = M.alloc<float>(nw);
      w->invf = M.alloc<float>(N);
      w->part = M.alloc<float>((size_t)ctas * L * parents(c_) * W);
      if (w->dEread == nullptr) w->dEread = M.alloc<float>(m * W);
      part = std::max({part, gemm_partial_floats((int)W, (int)m, n, kSplitK),
                       gemm_partial_floats((int)m, (int)W, n, kSplitK)});
    } else if (c_.architecture == kMlp) {
      // zs: pre-activations of layers 0..depth-1, hs: their activations
      const size_t d = c_.depth;
      w->zs = M.alloc<float>(d * nw);
      w->hs = M.alloc<float>(d * nw);
      w->dh = M.alloc<float>(nw);
      w->dz = M.alloc<float>(nw);
      part = std::max(gemm_partial_floats((int)W, (int)m, n, kSplitK), gemm_partial_floats((int)W, (int)W, n, kSplitK));
    } else if (c_.architecture == kResidualMlp) {
      // per block l: hs/ns/invs the residual stream and its RMSNorm, es the
      // expanded pre-activation, as its activation, zs the branch output
      const size_t d = c_.depth, H = (size_t)W * c_.expansion, nh = N * H;
      w->hs = M.alloc<float>((d + 1) * nw);
      w->ns = M.alloc<float>((d + 1) * nw);
      w->invs = M.alloc<float>((d + 1) * N);
      w->es = M.alloc<float>(d * nh);
      w->as = M.alloc<float>(d * nh);
      w->zs = M.alloc<float>(d * nw);
      w->dh = M.alloc<float>(nw);
      w->dn = M.alloc<float>(nw);
      w->dex = M.alloc<float>(nh);
      w->dax = M.alloc<float>(nh);
      part = std::max({gemm_partial_floats((int)H, (int)W, n, kSplitK), gemm_partial_floats((int)W, (int)H, n, kSplitK),
                       gemm_partial_floats((int)W, (int)m, n, kSplitK)});
    } else if (c_.architecture == kBilinear) {
      w->hs = M.alloc<float>(nw);  // p = left * right
      w->dn = M.alloc<float>(nw);  // dp
      w->dh = M.alloc<float>(nw);  // dleft
      w->dz = M.alloc<float>(nw);  // dright
      part = gemm_partial_floats((int)W, (int)m, n, kSplitK);
    } else if (c_.architecture == kRotaryDense) {
      const size_t d = c_.depth;
      w->hs = M.alloc<float>((d + 1) * nw);
      w->ns = M.alloc<float>((d + 1) * nw);
      w->invs = M.alloc<float>((d + 1) * N);
      w->zs = M.alloc<float>(d * nw);
      w->dh = M.alloc<float>(nw);
      w->dz = M.alloc<float>(nw);
      w->dn = M.alloc<float>(nw);
      w->dEread = M.alloc<float>(m * W);
      part = std::max(gemm_partial_floats((int)m, (int)W, n, kSplitK), gemm_partial_floats((int)W, (int)W, n, kSplitK));
    } else {
      const size_t d = c_.depth, ed = c_.embedding_mesh_depth;
      w->hs = M.alloc<float>(d * nw);
      w->hf = M.alloc<float>(nw);
      w->invf = M.alloc<float>(N);
      w->part = M.alloc<float>((size_t)ctas * d * 3 * W);
      w->states = M.alloc<float>((ed + 1) * m * W);
      w->dEemb = M.alloc<float>(m * W);
      w->dEread = M.alloc<float>(m * W);
      w->dv = M.alloc<float>((size_t)chain_ctas() * ed * 2 * W);  // chain weight partials
      part = gemm_partial_floats((int)m, (int)W, n, kSplitK);
    }
    w->gemm_part = M.alloc<float>(std::max<size_t>(part, 1));
    workspaces_.push_back(std::move(w));
    return *workspaces_.back();
  }

  void gemm(const GemmOperand& A, const GemmOperand& B, float* C, int ldc, int Mr, int Nc, int K, float* partial,
            int k_chunk = 0) {
    launch_gemm(A, B, C, ldc, Mr, Nc, K, k_chunk, partial, flags_ + kFlagTc, stream_);
    launches_ += (uint32_t)gemm_launches(K, k_chunk);
  }

  void enqueue_gather(Workspace& ws, const mb_simple_table* t, const uint32_t* idx, bool step) {
    const int n = ws.n;
    gather_batch<<<(n + 255) / 256, 256, 0, stream_>>>(n, step ? scalars_ : nullptr, idx, t->a, t->b, t->t, ws.a,
                                                        ws.b, ws.y); ++launches_;
    SIMPLE_CUDA(cudaGetLastError());
  }

  // The first layer's rows per operand residue, [2m][W] (a rows, then b
  // rows): the layer's own weights for one-hot operands, else the encoded
  // embeddings formed here from the current weights.
  const float* operand_rows() {
    if (enc_rows_ == nullptr) return w_ + offsets_[0];
    const int m = (int)c_.modulus, W = (int)c_.width, F = (int)operand_features(c_);
    const float* wa = w_ + offsets_[0];
    const float* wb = c_.architecture == kBilinear ? w_ + offsets_[1] : wa + (size_t)F * W;
    encoded_embedding<<<(2 * m * W + 255) / 256, 256, 0, stream_>>>(m, F, W, enc_table_, wa, wb, enc_rows_);
    ++launches_;
    return enc_rows_;
  }
  // Where the per-residue row gradients go: the first layer's gradient for
  // one-hot operands, else a scratch that operand_rows_gradient maps back.
  float* operand_rows_grad() { return enc_grad_ != nullptr ? enc_grad_ : grad_ + offsets_[0]; }
  void operand_rows_gradient() {
    if (enc_grad_ == nullptr) return;
    const int m = (int)c_.modulus, W = (int)c_.width, F = (int)operand_features(c_);
    float* ga = grad_ + offsets_[0];
    float* gb = c_.architecture == kBilinear ? grad_ + offsets_[1] : ga + (size_t)F * W;
    encoded_embedding_gradient<<<(2 * F * W + 255) / 256, 256, 0, stream_>>>(m, F, W, enc_table_, enc_grad_, ga, gb);
    ++launches_;
  }

  // Floats between consecutive mesh layers' weights (0: tied mesh layers).
  int mesh_lstride() const { return c_.tied_mesh ? 0 : parents(c_) * (int)c_.width; }

  // Mesh weight gradients from per-CTA partials [ctas][L][pw]: per layer, or
  // summed over the layers into the one stored layer when they are tied.
  void reduce_mesh_partials(Workspace& ws, int L, int pw, float* out) {
    if (c_.tied_mesh) {
      reduce_layer_partials<<<(pw + 255) / 256, 256, 0, stream_>>>(ws.part, ws.bwd_ctas, L, pw, out);
    } else {
      const size_t cnt = (size_t)L * pw;
      reduce_cta_partials<<<(int)std::min<size_t>((cnt + 255) / 256, 1184), 256, 0, stream_>>>(
          ws.part, ws.bwd_ctas, cnt, out);
    }
    ++launches_;
  }

  // h0 = [E a | E b] . Pj (Pj [2W][W]); ws.cat keeps the concatenation.
  void enqueue_concat(Workspace& ws, const float* E, const float* Pj, float* h0) {
    const int n = ws.n, W = (int)c_.width;
    const size_t total = (size_t)n * 2 * W;
    concat_rows<<<(int)std::min<size_t>((total + 255) / 256, 1184), 256, 0, stream_>>>(n, W, ws.a, ws.b, E,
                                                                                      ws.cat); ++launches_;
    gemm({ws.cat, 2 * W, false}, {Pj, W, true}, h0, W, n, W, 2 * W, nullptr);
  }

  // Gradients of the tied concatenation from dh0: dPj = cat^T dh0, dcat =
  // dh0 Pj^T, and dE = the per-class sums of dcat's halves plus `extra`.
  void enqueue_concat_backward(Workspace& ws, const float* dh0, const float* extra) {
    const int n = ws.n, W = (int)c_.width, m = (int)c_.modulus;
    const float* Pj = w_ + offsets_[1];
    gemm({ws.cat, 2 * W, true}, {dh0, W, true}, grad_ + offsets_[1], W, 2 * W, W, n, ws.gemm_part, kSplitK);
    gemm({dh0, W, false}, {Pj, W, false}, ws.dcat, 2 * W, n, 2 * W, W, nullptr);
    class_gradient<<<m, kClassThreads, 0, stream_>>>(n, W, m, 4, ws.a, ws.b, ws.dcat, extra, grad_ + offsets_[0]); ++launches_;
  }

  // Row values per lane of the templated kernels: the width, or for the full
  // mesh the widest layer (its readout may be wider than the hidden layers).
  int j_width() const {
    return c_.architecture == kFullMesh ? (int)std::max(c_.width, c_.modulus) : (int)c_.width;
  }

  template <int ACT>
  void forward_impl(Workspace& ws) {
    with_j(j_width(), [&](auto jc) { forward_j<ACT, decltype(jc)::value>(ws); });
  }

  template <int ACT, int J>
  void forward_j(Workspace& ws) {
    const int n = ws.n, W = (int)c_.width, m = (int)c_.modulus;
    const size_t nw = (size_t)n * W;
    const int fgrid = (n + kFwdWarps - 1) / kFwdWarps;
    const float* w = w_;
    if (c_.architecture == kFullMesh) {
      fullmesh_forward<ACT><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, (int)operand_features(c_),
                                                                   mesh_layers(c_), fm_layers_, enc_table_, ws.a,
                                                                   ws.b, w, ws.zs, ws.logits); ++launches_;
    } else if (c_.architecture == kMeshMlp) {
      const int L = mesh_layers(c_), p = parents(c_);
      const float* R = w + offsets_[1];
      mlp_forward<ACT, J><<<fgrid, kFwdWarps * 32, fwd_smem(), stream_>>>(
          n, W, m, L, p, mesh_lstride(), strides_, ws.a, ws.b, operand_rows(), nullptr,
          w + (L > 0 ? offsets_[2] : 0), ws.h, ws.act); ++launches_;
      // logits = act . R  (R [W][m]: B element (j, c) at R[c * m + j])
      gemm({ws.act, W, false}, {R, m, true}, ws.logits, m, n, m, W, nullptr);
    } else if (c_.architecture == kTiedConcatMesh) {
      // src/simple/reference.rs:300-335: h0 = [E a | E b] Pj, the mesh stack
      // of mesh-mlp, logits = act(h_L) E^T
      const int L = mesh_layers(c_), p = parents(c_);
      const float* E = w + offsets_[0];
      enqueue_concat(ws, E, w + offsets_[1], ws.h);
      mlp_forward<ACT, J><<<fgrid, kFwdWarps * 32, fwd_smem(), stream_>>>(
          n, W, m, L, p, mesh_lstride(), strides_, ws.a, ws.b, nullptr, ws.h, w + (L > 0 ? offsets_[2] : 0), ws.h,
          ws.act); ++launches_;
      gemm({ws.act, W, false}, {E, W, false}, ws.logits, m, n, m, W, nullptr);
    } else if (residual_mesh(c_)) {
      // src/simple/reference.rs:337-407
      const float* E = w + offsets_[0];
      if (c_.architecture == kResidualMesh) {
        concat_embed<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, m, ws.a, ws.b, operand_rows(), ws.h, nullptr,
                                                              nullptr); ++launches_;
      } else if (c_.architecture == kTiedRotaryResidualMesh) {
        rotary_embed<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.a, ws.b, E, ws.h, nullptr, nullptr); ++launches_;
      } else {
        enqueue_concat(ws, E, w + offsets_[1], ws.h);
      }
      const float* mesh = w + offsets_[dense_layers(c_).size()];
      const int d = (int)c_.depth, md = (int)c_.mesh_depth, moa = (int)c_.mesh_output_activation;
      const int st = resmesh_staged();
      if (parents(c_) == 2)
        resmesh_forward<ACT, J, 2><<<fgrid, kFwdWarps * 32, resmesh_fwd_smem(), stream_>>>(
            n, W, d, md, moa, st, strides_, mesh, ws.h, ws.ns, ws.invs, ws.zs, ws.hf, ws.invf);
      else
        resmesh_forward<ACT, J, 1><<<fgrid, kFwdWarps * 32, resmesh_fwd_smem(), stream_>>>(
            n, W, d, md, moa, st, strides_, mesh, ws.h, ws.ns, ws.invs, ws.zs, ws.hf, ws.invf);
      ++launches_;
      if (c_.architecture == kResidualMesh)  // logits = hf . R  (R [W][m])
        gemm({ws.hf, W, false}, {w + offsets_[1], m, true}, ws.logits, m, n, m, W, nullptr);
      else  // logits = hf . E^T
        gemm({ws.hf, W, false}, {E, W, false}, ws.logits, m, n, m, W, nullptr);
    } else if (c_.architecture == kMlp) {
      const int d = (int)c_.depth;
      const int eg = (int)std::min<size_t>((nw + 255) / 256, 1184);
      mlp_input<ACT><<<eg, 256, 0, stream_>>>(n, W, m, ws.a, ws.b, operand_rows(), ws.zs, ws.hs); ++launches_;
      for (int l = 1; l < d; ++l) {
        // z_l = act_{l-1} . W_l  (W_l [in][out]: B element (out, in) at W_l[in * W + out])
        gemm({ws.hs + (l - 1) * nw, W, false}, {w + offsets_[l], W, true}, ws.zs + l * nw, W, n, W, W, nullptr);
        activate<ACT><<<eg, 256, 0, stream_>>>(nw, ws.zs + l * nw, ws.hs + l * nw); ++launches_;
      }
      // logits = act_{d-1} . R  (R [W][m])
      gemm({ws.hs + (d - 1) * nw, W, false}, {w + offsets_[d], m, true}, ws.logits, m, n, m, W, nullptr);
    } else if (c_.architecture == kResidualMlp) {
      // src/simple/reference.rs:418-433
      const int d = (int)c_.depth, H = W * (int)c_.expansion;
      const size_t nh = (size_t)n * H;
      const int hg = (int)std::min<size_t>((nh + 255) / 256, 1184);
      concat_embed<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, m, ws.a, ws.b, operand_rows(), ws.hs, ws.ns,
                                                            ws.invs); ++launches_;
      for (int l = 0; l < d; ++l) {
        const float* U = w + offsets_[1 + 2 * l];  // [W][H]
        const float* D = w + offsets_[2 + 2 * l];  // [H][W]
        gemm({ws.ns + l * nw, W, false}, {U, H, true}, ws.es + l * nh, H, n, H, W, nullptr);
        activate<ACT><<<hg, 256, 0, stream_>>>(nh, ws.es + l * nh, ws.as + l * nh); ++launches_;
        gemm({ws.as + l * nh, H, false}, {D, W, true}, ws.zs + l * nw, W, n, W, H, nullptr);
        residual_norm<kLinear, J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.hs + l * nw, ws.zs + l * nw,
                                                                     ws.hs + (l + 1) * nw, ws.ns + (l + 1) * nw,
                                                                     ws.invs + (l + 1) * n); ++launches_;
      }
      gemm({ws.ns + d * nw, W, false}, {w + offsets_[1 + 2 * d], m, true}, ws.logits, m, n, m, W, nullptr);
    } else if (c_.architecture == kBilinear) {
      const int eg = (int)std::min<size_t>((nw + 255) / 256, 1184);
      const float* rows = operand_rows();
      const float* eb = enc_rows_ != nullptr ? rows + (size_t)m * W : w + offsets_[1];
      bilinear_input<<<eg, 256, 0, stream_>>>(n, W, ws.a, ws.b, rows, eb, ws.hs); ++launches_;
      gemm({ws.hs, W, false}, {w + offsets_[2], m, true}, ws.logits, m, n, m, W, nullptr);
    } else if (c_.architecture == kRotaryDense) {
      const float* E = w + offsets_[0];
      rotary_embed<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.a, ws.b, E, ws.hs, ws.ns, ws.invs); ++launches_;
      for (uint32_t l = 0; l < c_.depth; ++l) {
        const float* D = w + offsets_[1 + l];
        // z = n_l . D  (D [in][out]: B element (out, in) at D[in * W + out])
        gemm({ws.ns + l * nw, W, false}, {D, W, true}, ws.zs + l * nw, W, n, W, W, nullptr);
        residual_norm<ACT, J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.hs + l * nw, ws.zs + l * nw,
                                                                  ws.hs + (l + 1) * nw, ws.ns + (l + 1) * nw,
                                                                  ws.invs + (l + 1) * n); ++launches_;
      }
      // logits = hf . E^T
      gemm({ws.ns + c_.depth * nw, W, false}, {E, W, false}, ws.logits, m, n, m, W, nullptr);
    } else {
      const int ed = (int)c_.embedding_mesh_depth;
      const float* chain = w;
      const float* core = w + offsets_[ed];
      chain_forward<<<chain_ctas(), kChainThreads, 0, stream_>>>(m, W, ed, chain, ws.states); ++launches_;
      const float* E = ws.states + (size_t)ed * m * W;
      shared_forward<ACT, J><<<fgrid, kFwdWarps * 32, fwd_smem(), stream_>>>(
          n, W, (int)c_.depth, strides_, ws.a, ws.b, E, core, ws.hs, ws.hf, ws.invf); ++launches_;
      gemm({ws.hf, W, false}, {E, W, false}, ws.logits, m, n, m, W, nullptr);
    }
    SIMPLE_CUDA(cudaGetLastError());
  }

  void enqueue_forward(Workspace& ws) {
    if (c_.activation == kRelu)
      forward_impl<kRelu>(ws);
    else
      forward_impl<kSquare>(ws);
  }

  void enqueue_loss(Workspace& ws) {
    const int n = ws.n, m = (int)c_.modulus;
    cross_entropy_gradient<<<(n + kFwdWarps - 1) / kFwdWarps, kFwdWarps * 32, 0, stream_>>>(n, m, ws.logits, ws.y,
                                                                                            ws.dlog, flags_); ++launches_;
    SIMPLE_CUDA(cudaGetLastError());
  }

  template <int ACT>
  void backward_impl(Workspace& ws) {
    with_j(j_width(), [&](auto jc) { backward_j<ACT, decltype(jc)::value>(ws); });
  }

  template <int ACT, int J>
  void backward_j(Workspace& ws) {
    const int n = ws.n, W = (int)c_.width, m = (int)c_.modulus;
    const size_t nw = (size_t)n * W;
    const int fgrid = (n + kFwdWarps - 1) / kFwdWarps;
    const int bsm = bwd_smem();
    float* g = grad_;
    const float* w = w_;
    if (c_.architecture == kFullMesh) {
      fullmesh_backward<ACT, J><<<ws.bwd_ctas, kBwdWarps * 32, fullmesh_bwd_smem(), stream_>>>(
          n, (int)operand_features(c_), mesh_layers(c_), fm_layers_, enc_table_, ws.a, ws.b, w, ws.zs, ws.dlog,
          (int)P_, ws.part); ++launches_;
      reduce_cta_partials<<<(int)std::min<size_t>((P_ + 255) / 256, 1184), 256, 0, stream_>>>(ws.part, ws.bwd_ctas, P_,
                                                                                              g); ++launches_;
    } else if (c_.architecture == kMeshMlp) {
      const int L = mesh_layers(c_), p = parents(c_);
      const float* R = w + offsets_[1];
      // dR = act^T . dlog  (split-K over rows)
      gemm({ws.act, W, true}, {ws.dlog, m, true}, g + offsets_[1], m, W, m, n, ws.gemm_part, kSplitK);
      // dact = dlog . R^T  (B element (c, j) at R[c * m + j])
      gemm({ws.dlog, m, false}, {R, m, false}, ws.dact, W, n, W, m, nullptr);
      if (L > 0) {
        mlp_backward<ACT, J><<<ws.bwd_ctas, kBwdWarps * 32, bsm, stream_>>>(n, W, L, p, mesh_lstride(), strides_,
                                                                            w + offsets_[2], ws.h, ws.dact, ws.dh0,
                                                                            ws.part); ++launches_;
        reduce_mesh_partials(ws, L, p * W, g + offsets_[2]);
      } else {
        activation_gradient<ACT><<<(int)std::min<size_t>((nw + 255) / 256, 1184), 256, 0, stream_>>>(
            nw, ws.dact, ws.h, ws.dh0); ++launches_;
      }
      class_gradient<<<2 * m, kClassThreads, 0, stream_>>>(n, W, m, 0, ws.a, ws.b, ws.dh0, nullptr,
                                                           operand_rows_grad()); ++launches_;
      operand_rows_gradient();
    } else if (c_.architecture == kTiedConcatMesh) {
      const int L = mesh_layers(c_), p = parents(c_);
      const float* E = w + offsets_[0];
      // dE (readout share) = dlog^T . act ; dact = dlog . E
      gemm({ws.dlog, m, true}, {ws.act, W, true}, ws.dEread, W, m, W, n, ws.gemm_part, kSplitK);
      gemm({ws.dlog, m, false}, {E, W, true}, ws.dact, W, n, W, m, nullptr);
      if (L > 0) {
        mlp_backward<ACT, J><<<ws.bwd_ctas, kBwdWarps * 32, bsm, stream_>>>(n, W, L, p, mesh_lstride(), strides_,
                                                                            w + offsets_[2], ws.h, ws.dact, ws.dh0,
                                                                            ws.part); ++launches_;
        reduce_mesh_partials(ws, L, p * W, g + offsets_[2]);
      } else {
        activation_gradient<ACT><<<(int)std::min<size_t>((nw + 255) / 256, 1184), 256, 0, stream_>>>(
            nw, ws.dact, ws.h, ws.dh0); ++launches_;
      }
      enqueue_concat_backward(ws, ws.dh0, ws.dEread);
    } else if (residual_mesh(c_)) {
      const float* E = w + offsets_[0];
      const bool tied = c_.architecture != kResidualMesh;
      if (tied) {
        // dE (readout share) = dlog^T . hf ; dhf = dlog . E
        gemm({ws.dlog, m, true}, {ws.hf, W, true}, ws.dEread, W, m, W, n, ws.gemm_part, kSplitK);
        gemm({ws.dlog, m, false}, {E, W, true}, ws.dhf, W, n, W, m, nullptr);
      } else {
        const float* R = w + offsets_[1];
        // dR = hf^T . dlog ; dhf = dlog . R^T
        gemm({ws.hf, W, true}, {ws.dlog, m, true}, g + offsets_[1], m, W, m, n, ws.gemm_part, kSplitK);
        gemm({ws.dlog, m, false}, {R, m, false}, ws.dhf, W, n, W, m, nullptr);
      }
      const size_t mesh_off = offsets_[dense_layers(c_).size()];
      const int d = (int)c_.depth, md = (int)c_.mesh_depth, moa = (int)c_.mesh_output_activation;
      const int st = resmesh_staged(), p = parents(c_);
      if (p == 2)
        resmesh_backward<ACT, J, 2><<<ws.bwd_ctas, kBwdWarps * 32, resmesh_bwd_smem(), stream_>>>(
            n, W, d, md, moa, st, strides_, w + mesh_off, ws.ns, ws.invs, ws.zs, ws.hf, ws.invf, ws.dhf, ws.dh0,
            ws.part);
      else
        resmesh_backward<ACT, J, 1><<<ws.bwd_ctas, kBwdWarps * 32, resmesh_bwd_smem(), stream_>>>(
            n, W, d, md, moa, st, strides_, w + mesh_off, ws.ns, ws.invs, ws.zs, ws.hf, ws.invf, ws.dhf, ws.dh0,
            ws.part);
      ++launches_;
      const size_t cnt = (size_t)mesh_layers(c_) * p * W;
      reduce_cta_partials<<<(int)std::min<size_t>((cnt + 255) / 256, 1184), 256, 0, stream_>>>(
          ws.part, ws.bwd_ctas, cnt, g + mesh_off); ++launches_;
      if (c_.architecture == kResidualMesh) {
        class_gradient<<<2 * m, kClassThreads, 0, stream_>>>(n, W, m, 0, ws.a, ws.b, ws.dh0, nullptr,
                                                             operand_rows_grad()); ++launches_;
        operand_rows_gradient();
      } else if (c_.architecture == kTiedRotaryResidualMesh) {
        class_gradient<<<m, kClassThreads, 0, stream_>>>(n, W, m, 1, ws.a, ws.b, ws.dh0, ws.dEread,
                                                         g + offsets_[0]); ++launches_;
      } else {
        enqueue_concat_backward(ws, ws.dh0, ws.dEread);
      }
    } else if (c_.architecture == kMlp) {
      const int d = (int)c_.depth;
      const int eg = (int)std::min<size_t>((nw + 255) / 256, 1184);
      const float* R = w + offsets_[d];
      // dR = act_{d-1}^T . dlog ; da = dlog . R^T
      gemm({ws.hs + (d - 1) * nw, W, true}, {ws.dlog, m, true}, g + offsets_[d], m, W, m, n, ws.gemm_part, kSplitK);
      gemm({ws.dlog, m, false}, {R, m, false}, ws.dh, W, n, W, m, nullptr);
      for (int l = d - 1; l >= 1; --l) {
        activation_gradient<ACT><<<eg, 256, 0, stream_>>>(nw, ws.dh, ws.zs + l * nw, ws.dz); ++launches_;
        // dW_l = act_{l-1}^T . dz ; da = dz . W_l^T
        gemm({ws.hs + (l - 1) * nw, W, true}, {ws.dz, W, true}, g + offsets_[l], W, W, W, n, ws.gemm_part, kSplitK);
        gemm({ws.dz, W, false}, {w + offsets_[l], W, false}, ws.dh, W, n, W, W, nullptr);
      }
      activation_gradient<ACT><<<eg, 256, 0, stream_>>>(nw, ws.dh, ws.zs, ws.dh0); ++launches_;
      class_gradient<<<2 * m, kClassThreads, 0, stream_>>>(n, W, m, 0, ws.a, ws.b, ws.dh0, nullptr,
                                                           operand_rows_grad()); ++launches_;
      operand_rows_gradient();
    } else if (c_.architecture == kResidualMlp) {
      const int d = (int)c_.depth, H = W * (int)c_.expansion;
      const size_t nh = (size_t)n * H;
      const int hg = (int)std::min<size_t>((nh + 255) / 256, 1184);
      const float* R = w + offsets_[1 + 2 * d];
      // dR = n_d^T . dlog ; dn_d = dlog . R^T ; dh = RMSNorm adjoint
      gemm({ws.ns + d * nw, W, true}, {ws.dlog, m, true}, g + offsets_[1 + 2 * d], m, W, m, n, ws.gemm_part,
           kSplitK);
      gemm({ws.dlog, m, false}, {R, m, false}, ws.dn, W, n, W, m, nullptr);
      rms_backward<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.ns + d * nw, ws.invs + d * n, ws.dn, nullptr,
                                                           ws.dh); ++launches_;
      for (int l = d - 1; l >= 0; --l) {
        const float* U = w + offsets_[1 + 2 * l];
        const float* D = w + offsets_[2 + 2 * l];
        // the branch output's gradient is dh: dD = a^T dh, da = dh D^T
        gemm({ws.as + l * nh, H, true}, {ws.dh, W, true}, g + offsets_[2 + 2 * l], W, H, W, n, ws.gemm_part,
             kSplitK);
        gemm({ws.dh, W, false}, {D, W, false}, ws.dax, H, n, H, W, nullptr);
        activation_gradient<ACT><<<hg, 256, 0, stream_>>>(nh, ws.dax, ws.es + l * nh, ws.dex); ++launches_;
        // dU = n_l^T de, dn = de U^T, dh += RMSNorm adjoint of dn
        gemm({ws.ns + l * nw, W, true}, {ws.dex, H, true}, g + offsets_[1 + 2 * l], H, W, H, n, ws.gemm_part,
             kSplitK);
        gemm({ws.dex, H, false}, {U, H, false}, ws.dn, W, n, W, H, nullptr);
        rms_backward<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.ns + l * nw, ws.invs + l * n, ws.dn, ws.dh,
                                                             ws.dh); ++launches_;
      }
      class_gradient<<<2 * m, kClassThreads, 0, stream_>>>(n, W, m, 0, ws.a, ws.b, ws.dh, nullptr,
                                                           operand_rows_grad()); ++launches_;
      operand_rows_gradient();
    } else if (c_.architecture == kBilinear) {
      const int eg = (int)std::min<size_t>((nw + 255) / 256, 1184);
      const float* R = w + offsets_[2];
      // dR = p^T . dlog ; dp = dlog . R^T
      gemm({ws.hs, W, true}, {ws.dlog, m, true}, g + offsets_[2], m, W, m, n, ws.gemm_part, kSplitK);
      gemm({ws.dlog, m, false}, {R, m, false}, ws.dn, W, n, W, m, nullptr);
      const float* ea = enc_rows_ != nullptr ? enc_rows_ : w + offsets_[0];
      const float* eb = enc_rows_ != nullptr ? enc_rows_ + (size_t)m * W : w + offsets_[1];
      bilinear_gradient<<<eg, 256, 0, stream_>>>(n, W, ws.a, ws.b, ea, eb, ws.dn, ws.dh,
                                                 ws.dz); ++launches_;
      float* ga = operand_rows_grad();
      float* gb = enc_grad_ != nullptr ? enc_grad_ + (size_t)m * W : g + offsets_[1];
      class_gradient<<<m, kClassThreads, 0, stream_>>>(n, W, m, 2, ws.a, ws.b, ws.dh, nullptr, ga); ++launches_;
      class_gradient<<<m, kClassThreads, 0, stream_>>>(n, W, m, 3, ws.a, ws.b, ws.dz, nullptr, gb); ++launches_;
      operand_rows_gradient();
    } else if (c_.architecture == kRotaryDense) {
      const float* E = w + offsets_[0];
      const int d = (int)c_.depth;
      const float* hf = ws.ns + d * nw;
      // dE (readout share) = dlog^T . hf ; dhf = dlog . E
      gemm({ws.dlog, m, true}, {hf, W, true}, ws.dEread, W, m, W, n, ws.gemm_part, kSplitK);
      gemm({ws.dlog, m, false}, {E, W, true}, ws.dhf, W, n, W, m, nullptr);
      rms_backward<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, hf, ws.invs + d * n, ws.dhf, nullptr, ws.dh); ++launches_;
      for (int l = d - 1; l >= 0; --l) {
        const float* D = w + offsets_[1 + l];
        activation_gradient<ACT><<<(int)std::min<size_t>((nw + 255) / 256, 1184), 256, 0, stream_>>>(
            nw, ws.dh, ws.zs + l * nw, ws.dz); ++launches_;
        // dD = n_l^T . dz ; dn = dz . D^T
        gemm({ws.ns + l * nw, W, true}, {ws.dz, W, true}, g + offsets_[1 + l], W, W, W, n, ws.gemm_part, kSplitK);
        gemm({ws.dz, W, false}, {D, W, false}, ws.dn, W, n, W, W, nullptr);
        rms_backward<J><<<fgrid, kFwdWarps * 32, 0, stream_>>>(n, W, ws.ns + l * nw, ws.invs + l * n, ws.dn, ws.dh,
                                                             ws.dh); ++launches_;
      }
      class_gradient<<<m, kClassThreads, 0, stream_>>>(n, W, m, 1, ws.a, ws.b, ws.dh, ws.dEread, g + offsets_[0]); ++launches_;
    } else {
      const int ed = (int)c_.embedding_mesh_depth, d = (int)c_.depth;
      const float* E = ws.states + (size_t)ed * m * W;
      gemm({ws.dlog, m, true}, {ws.hf, W, true}, ws.dEread, W, m, W, n, ws.gemm_part, kSplitK);
      gemm({ws.dlog, m, false}, {E, W, true}, ws.dhf, W, n, W, m, nullptr);
      shared_backward<ACT, J><<<ws.bwd_ctas, kBwdWarps * 32, bsm, stream_>>>(
          n, W, d, strides_, w + offsets_[ed], ws.hs, ws.hf, ws.invf, ws.dhf, ws.dh0, ws.part); ++launches_;
      const size_t cnt = (size_t)d * 3 * W;
      reduce_cta_partials<<<(int)std::min<size_t>((cnt + 255) / 256, 1184), 256, 0, stream_>>>(
          ws.part, ws.bwd_ctas, cnt, g + offsets_[ed]); ++launches_;
      class_gradient<<<m, kClassThreads, 0, stream_>>>(n, W, m, 1, ws.a, ws.b, ws.dh0, ws.dEread, ws.dEemb); ++launches_;
      chain_backward<<<chain_ctas(), kChainThreads, 0, stream_>>>(m, W, ed, w, ws.states, ws.dEemb, ws.dv);
      ++launches_;
      const size_t ccnt = (size_t)ed * 2 * W;
      reduce_cta_partials<<<(int)std::min<size_t>((ccnt + 255) / 256, 1184), 256, 0, stream_>>>(
          ws.dv, chain_ctas(), ccnt, g); ++launches_;
    }
    SIMPLE_CUDA(cudaGetLastError());
  }

  void enqueue_backward(Workspace& ws) {
    if (c_.activation == kRelu)
      backward_impl<kRelu>(ws);
    else
      backward_impl<kSquare>(ws);
  }

  void enqueue_update() {
    const int W = (int)c_.width, m = (int)c_.modulus;
    const size_t n_in = groups_[0];
    if (chan_decay_ != nullptr) {
      const float exponent = (float)(2.0 / (double)c_.decay_factors - 1.0);
      channel_decay<<<(W + 127) / 128, 128, 0, stream_>>>((int)(n_in / W), W, m, exponent, scalars_, w_,
                                                          w_ + offsets_[1], chan_decay_); ++launches_;
    }
    adamw<<<(int)std::min<size_t>((P_ + 255) / 256, 1184), 256, 0, stream_>>>(P_, mesh_start_, scalars_, grad_, w_,
                                                                               m1_, m2_, chan_decay_, W, m, n_in);
    ++launches_;
    SIMPLE_CUDA(cudaGetLastError());
  }

  mb_simple_config c_;
  int device_;
  cudaStream_t stream_ = nullptr;
  DeviceBuffers mem_;
  std::vector<size_t> groups_, offsets_;
  size_t P_ = 0, mesh_start_ = 0;
  float *w_, *m1_, *m2_, *grad_;
  int* flags_;
  int* strides_;
  float *enc_table_ = nullptr, *enc_rows_ = nullptr, *enc_grad_ = nullptr;  // non-one-hot encodings
  float* chan_decay_ = nullptr;  // per-channel decay (decay_factors != 2)
  FmLayer* fm_layers_ = nullptr;  // full mesh layer descriptors
  int fm_z_ = 0;                  // full mesh pre-activation floats per row (all but the readout)
  StepScalars* scalars_;
  static constexpr int kScalarSlots = 16;
  StepScalars* host_scalars_ = nullptr;  // page-locked [kScalarSlots]
  cudaEvent_t scalar_copied_[kScalarSlots] = {};
  uint64_t scalar_step_ = 0;
  float beta1_power_ = 1.0f, beta2_power_ = 1.0f;
  std::vector<std::unique_ptr<Workspace>> workspaces_;
  std::shared_ptr<IndexPool> index_pool_;
  uint32_t launches_ = 0, last_launches_ = 0;
};

}  // namespace simple
}  // namespace mb

struct mb_simple {
  std::unique_ptr<mb::simple::SimpleModel> model;
};

// ------------------------------------------------------------------- C ABI
using mb::guarded;
using mb::need;
using mb::require;

extern "C" {

int mb_simple_validate(const mb_simple_config* config) {
  return guarded([&] {
    need(config, "config");
    mb::simple::validate(*config);
  });
}

int mb_simple_parameter_count(const mb_simple_config* config, size_t* count) {
  return guarded([&] {
    need(config, "config");
    need(count, "count");
    mb::simple::validate(*config);
    *count = mb::simple::parameter_count(*config);
  });
}

int mb_simple_groups(const mb_simple_config* config, uint32_t* groups, size_t* n_groups) {
  return guarded([&] {
    need(config, "config");
    need(n_groups, "n_groups");
    mb::simple::validate(*config);
    const auto g = mb::simple::groups(*config);
    if (groups != nullptr) {
      require(*n_groups >= g.size(), "groups buffer is too small");
      for (size_t i = 0; i < g.size(); ++i) groups[i] = (uint32_t)g[i];
    }
    *n_groups = g.size();
  });
}

int mb_simple_initial_parameters(const mb_simple_config* config, uint64_t seed, float* out, size_t count) {
  return guarded([&] {
    need(config, "config");
    need(out, "out");
    const auto p = mb::simple::initial_parameters(*config, seed);
    require(count == p.size(), "parameter count does not match the model");
    std::memcpy(out, p.data(), p.size() * sizeof(float));
  });
}

int mb_simple_encode(const mb_simple_config* config, const uint32_t* equations, size_t n, float* features,
                     uint32_t* targets) {
  return guarded([&] {
    need(config, "config");
    need(equations, "equations");
    need(features, "features");
    need(targets, "targets");
    mb::simple::validate(*config);
    const uint32_t m = config->modulus, f = mb::simple::operand_features(*config);
    for (size_t r = 0; r < n; ++r)
      for (int j = 0; j < 3; ++j)
        require(equations[3 * r + j] < m, "equation residue is outside the model's modulus");
    const std::vector<float> table = mb::simple::encoding_table(*config);
    for (size_t r = 0; r < n; ++r) {
      std::memcpy(features + r * 2 * f, table.data() + (size_t)equations[3 * r] * f, f * sizeof(float));
      std::memcpy(features + r * 2 * f + f, table.data() + (size_t)equations[3 * r + 1] * f, f * sizeof(float));
      targets[r] = equations[3 * r + 2];
    }
  });
}

int mb_simple_create(int device, const mb_simple_config* config, uint64_t seed, mb_simple** out) {
  return guarded([&] {
    need(config, "config");
    need(out, "out");
    *out = nullptr;
    auto h = std::make_unique<mb_simple>();
    h->model = std::make_unique<mb::simple::SimpleModel>(device, *config, seed);
    *out = h.release();
  });
}

int mb_simple_destroy(mb_simple* model) {
  return guarded([&] { delete model; });
}

int mb_simple_get_parameters(mb_simple* model, float* out, size_t count) {
  return guarded([&] {
    need(model, "model");
    need(out, "out");
    model->model->get_parameters(out, count);
  });
}

int mb_simple_set_parameters(mb_simple* model, const float* values, size_t count) {
  return guarded([&] {
    need(model, "model");
    need(values, "values");
    model->model->set_parameters(values, count);
  });
}

int mb_simple_upload_table(mb_simple* model, const float* features, const uint32_t* targets, size_t rows,
                           mb_simple_table** out) {
  return guarded([&] {
    need(model, "model");
    need(features, "features");
    need(targets, "targets");
    need(out, "out");
    *out = model->model->upload_table(features, targets, rows);
  });
}

int mb_simple_table_destroy(mb_simple_table* table) {
  return guarded([&] { delete table; });
}

int mb_simple_upload_batches(mb_simple* model, const mb_simple_table* table, const uint32_t* indices, size_t count,
                             mb_simple_batches** out) {
  return guarded([&] {
    need(model, "model");
    need(indices, "indices");
    need(out, "out");
    *out = model->model->upload_batches(table, indices, count);
  });
}

int mb_host_alloc(size_t bytes, void** out) {
  return guarded([&] {
    need(out, "out");
    *out = nullptr;
    mb::require(bytes >= 1, "a host buffer needs at least one byte");
    cudaError_t e = cudaHostAlloc(out, bytes, cudaHostAllocDefault);
    if (e != cudaSuccess) throw mb::Error(MB_ERR_CUDA, std::string("cudaHostAlloc failed: ") + cudaGetErrorString(e));
  });
}

int mb_host_free(void* p) {
  return guarded([&] {
    cudaError_t e = p != nullptr ? cudaFreeHost(p) : cudaSuccess;
    if (e != cudaSuccess) throw mb::Error(MB_ERR_CUDA, std::string("cudaFreeHost failed: ") + cudaGetErrorString(e));
  });
}

int mb_simple_batches_destroy(mb_simple_batches* batches) {
  return guarded([&] { delete batches; });
}

int mb_simple_train_step(mb_simple* model, const mb_simple_table* table, const mb_simple_batches* batches,
                         size_t offset, size_t rows, const mb_adamw* options) {
  return guarded([&] {
    need(model, "model");
    need(options, "options");
    model->model->train_step(table, batches, offset, rows, *options);
  });
}

int mb_simple_evaluate(mb_simple* model, const mb_simple_table* table, float* logits, uint32_t* predictions) {
  return guarded([&] {
    need(model, "model");
    model->model->evaluate(table, logits, predictions);
  });
}

int mb_simple_loss_and_gradient(mb_simple* model, const mb_simple_table* table, const uint32_t* indices,
                                size_t count, double* loss, float* gradient, size_t n_gradient) {
  return guarded([&] {
    need(model, "model");
    need(indices, "indices");
    need(loss, "loss");
    need(gradient, "gradient");
    *loss = model->model->loss_and_gradient(table, indices, count, gradient, n_gradient);
  });
}

int mb_simple_stream(mb_simple* model, void** stream) {
  return guarded([&] {
    need(model, "model");
    need(stream, "stream");
    *stream = (void*)model->model->stream();
  });
}

int mb_simple_check(mb_simple* model) {
  return guarded([&] {
    need(model, "model");
    model->model->check();
  });
}

int mb_simple_step_launches(mb_simple* model, uint32_t* launches) {
  return guarded([&] {
    need(model, "model");
    need(launches, "launches");
    *launches = model->model->step_launches();
  });
}

}  // extern "C"
