// Tied embedding mesh, vocabulary head, cross-entropy, gradient reduction and
// AdamW for Mesh GPT on sm_100a.  The embedding gradient itself
// (gpt_embedding_gradient_partials / _reduce, src/gpt/gpu.rs:1159-1218) is
// one split-K tensor-core GEMM over the head's dlogits and the token
// indicator written here (see the gradient pass of gpt_model.cu).
//
// Reference kernels restated: gpt_embed / gpt_embedding_transpose / gpt_head /
// gpt_cross_entropy / gpt_head_backward (src/gpt/gpu.rs:41-56, :904-1021),
// the embedding mesh forward/backward over the vocabulary (:2094-2156,
// :2564-2605), gpt_mesh_gradient_reduce (:1126-1149) and gpt_adam (:1369-1391).

#include "common.cuh"

namespace mb {

// ---- embedding mesh over the vocabulary: one CTA per token row, one thread
// per channel.  acts: [A+1][V][W] (acts[0] = fixed codes).  Also writes the
// transposed final layer Et [W][V] for coalesced head reads.
__global__ void embedding_forward(int W, int V, int depth, int connectivity, int log2w,
                                  const float* __restrict__ weights, float* __restrict__ acts,
                                  float* __restrict__ et) {
  extern __shared__ float row[];
  const int t = blockIdx.x, ch = threadIdx.x;
  float x = acts[(size_t)t * W + ch];
  for (int l = 0; l < depth; ++l) {
    row[ch] = x;
    __syncthreads();
    const int s = connectivity == 0 ? 1 : (1 << (l % log2w));
    const float* w = weights + (size_t)l * 2 * W + 2 * ch;
    float z = x * w[0] + row[(ch + s) % W] * w[1];
    x = l + 1 != depth ? elu(z) : z;
    acts[((size_t)(l + 1) * V + t) * W + ch] = x;
    __syncthreads();
  }
  et[(size_t)ch * V + t] = x;
}

// Backward through the embedding mesh for one token row per CTA; writes the
// per-row edge-gradient partial [V][depth][W][2] (reduced by reduce_partials).
__global__ void embedding_backward(int W, int V, int depth, int connectivity, int log2w,
                                   const float* __restrict__ weights, const float* __restrict__ acts,
                                   const float* __restrict__ dE, float* __restrict__ partial) {
  extern __shared__ float row[];
  const int t = blockIdx.x, ch = threadIdx.x;
  float g = dE[(size_t)t * W + ch];
  for (int l = depth - 1; l >= 0; --l) {
    const int s = connectivity == 0 ? 1 : (1 << (l % log2w));
    const float* w = weights + (size_t)l * 2 * W;
    const float* xin = acts + ((size_t)l * V + t) * W;
    if (l + 1 != depth) g *= elu_slope(acts[((size_t)(l + 1) * V + t) * W + ch]);
    const int nb = (ch + s) % W;
    float* out = partial + ((size_t)t * depth + l) * 2 * W + 2 * ch;
    out[0] = g * xin[ch];
    out[1] = g * xin[nb];
    row[ch] = g * w[2 * ch + 1];
    __syncthreads();
    const int prev = (ch - s + W) % W;
    g = g * w[2 * ch] + row[prev];
    __syncthreads();
  }
}

// ---- the head as row kernels around two tensor-core GEMMs (gemm_tc.cu):
// head_norm (final RMSNorm), logits = nf E^T, head_loss (cross-entropy and
// dlogits), dn = dlogits E, head_norm_backward (the RMSNorm adjoint -> dx).
// One warp per row.
constexpr int kHeadWarps = 8;

__global__ void __launch_bounds__(kHeadWarps * 32)
    head_norm(int rows, int W, const float* __restrict__ x, float* __restrict__ nf, float* __restrict__ inv_out) {
  const int lane = threadIdx.x & 31, r = blockIdx.x * kHeadWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* xr = x + (size_t)r * W;
  float s = 0.f;
  for (int ch = lane * 4; ch < W; ch += 128) {
    const float4 v = *reinterpret_cast<const float4*>(xr + ch);
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  s = group_sum<32>(s);
  const float iv = 1.0f / sqrtf(s / (float)W + kRmsEpsilon);
  if (lane == 0) inv_out[r] = iv;
  for (int ch = lane * 4; ch < W; ch += 128) {
    const float4 v = *reinterpret_cast<const float4*>(xr + ch);
    *reinterpret_cast<float4*>(nf + (size_t)r * W + ch) = make_float4(v.x * iv, v.y * iv, v.z * iv, v.w * iv);
  }
}

// Cross-entropy per row (src/gpt/gpu.rs:955-994): loss_rows and
// dlogits = (softmax - onehot) / supervised; ignored rows get zeros.  Also
// writes the row's input-token indicator (1 at tokens[r], else 0), the
// second half of the embedding-gradient contraction's left operand.
__global__ void __launch_bounds__(kHeadWarps * 32)
    head_loss(int rows, int V, const float* __restrict__ logits, const uint32_t* __restrict__ targets,
              const float* __restrict__ supervised, const uint32_t* __restrict__ tokens,
              float* __restrict__ loss_rows, float* __restrict__ dlogits, float* __restrict__ indicator) {
  const int lane = threadIdx.x & 31, r = blockIdx.x * kHeadWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* l = logits + (size_t)r * V;
  float* d = dlogits + (size_t)r * V;
  const uint32_t tok = tokens[r];
  for (int t = lane; t < V; t += 32) indicator[(size_t)r * V + t] = (uint32_t)t == tok ? 1.f : 0.f;
  const uint32_t tg = targets[r];
  if (tg == kIgnoreTarget) {
    for (int t = lane; t < V; t += 32) d[t] = 0.f;
    if (lane == 0) loss_rows[r] = 0.f;
    return;
  }
  const float sup = *supervised;
  float m = -INFINITY;
  for (int t = lane; t < V; t += 32) m = fmaxf(m, l[t]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.f;
  for (int t = lane; t < V; t += 32) s += expf(l[t] - m);
  s = group_sum<32>(s);
  if (lane == 0) loss_rows[r] = logf(s) + m - l[tg < (uint32_t)V ? tg : 0];
  for (int t = lane; t < V; t += 32) {
    const float p = expf(l[t] - m) / s;
    d[t] = (p - (t == (int)tg ? 1.0f : 0.0f)) / sup;
  }
}

// dx = inv (dn - n mean(dn n)), the RMSNorm adjoint of the final norm.
__global__ void __launch_bounds__(kHeadWarps * 32)
    head_norm_backward(int rows, int W, const float* __restrict__ nf, const float* __restrict__ inv,
                       const float* __restrict__ dn, float* __restrict__ dx) {
  const int lane = threadIdx.x & 31, r = blockIdx.x * kHeadWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* nr = nf + (size_t)r * W;
  const float* gr = dn + (size_t)r * W;
  float s = 0.f;
  for (int ch = lane * 4; ch < W; ch += 128) {
    const float4 n = *reinterpret_cast<const float4*>(nr + ch), g = *reinterpret_cast<const float4*>(gr + ch);
    s += g.x * n.x + g.y * n.y + g.z * n.z + g.w * n.w;
  }
  s = group_sum<32>(s) / (float)W;
  const float iv = inv[r];
  for (int ch = lane * 4; ch < W; ch += 128) {
    const float4 n = *reinterpret_cast<const float4*>(nr + ch), g = *reinterpret_cast<const float4*>(gr + ch);
    *reinterpret_cast<float4*>(dx + (size_t)r * W + ch) =
        make_float4(iv * (g.x - n.x * s), iv * (g.y - n.y * s), iv * (g.z - n.z * s), iv * (g.w - n.w * s));
  }
}

// ---- deterministic reduction of per-slot partials: out[p] = sum_s part[s][p]
// in slot order.  One job per parameter group (or the embedding adjoint).
struct ReduceJob {
  const float* partial;  // [slots][size]
  float* out;            // [size]
  int slots;
  int size;
};

// A thread sums four consecutive parameters (one float4 per slot), with the
// loads of eight slots in flight before they are added in slot order.
__global__ void reduce_partials(const ReduceJob* __restrict__ jobs, int njobs) {
  const ReduceJob job = jobs[blockIdx.y];
  const bool vec = (job.size & 3) == 0 && (reinterpret_cast<uintptr_t>(job.partial) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(job.out) & 15) == 0;
  if (!vec) {
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < job.size; p += gridDim.x * blockDim.x) {
      float s = 0.f;
      for (int k = 0; k < job.slots; ++k) s += job.partial[(size_t)k * job.size + p];
      job.out[p] = s;
    }
    return;
  }
  const int n4 = job.size >> 2;
  const float4* part = reinterpret_cast<const float4*>(job.partial);
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n4; p += gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    int k = 0;
    for (; k + 8 <= job.slots; k += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = part[(size_t)(k + j) * n4 + p];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s.x += v[j].x;
        s.y += v[j].y;
        s.z += v[j].z;
        s.w += v[j].w;
      }
    }
    for (; k < job.slots; ++k) {
      const float4 v = part[(size_t)k * n4 + p];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    reinterpret_cast<float4*>(job.out)[p] = s;
  }
}

// ---- AdamW (src/gpt/gpu.rs:1369-1391) over the flat parameter buffer.  The
// bias-correction powers accumulate in f32 on the device exactly as the
// reference host accumulates them (src/gpt/gpu.rs:1980-1981).
struct OptimizerState {
  float learning_rate, weight_decay, beta1, beta2, epsilon;
  float beta1_power, beta2_power;
  int step;
};

// Sets this step's hyperparameters and advances the bias-correction powers
// (beta_power *= beta in f32, once per update).  A step whose batch the
// device rejected (step_flags != 0) changes nothing: neither the powers nor,
// in adamw, the weights and moments.
__global__ void optimizer_set(OptimizerState* st, OptimizerState h, const int* __restrict__ step_flags) {
  if (*step_flags != 0) return;
  st->learning_rate = h.learning_rate;
  st->weight_decay = h.weight_decay;
  st->beta1 = h.beta1;
  st->beta2 = h.beta2;
  st->epsilon = h.epsilon;
  st->beta1_power = __fmul_rn(st->beta1_power, h.beta1);
  st->beta2_power = __fmul_rn(st->beta2_power, h.beta2);
  st->step += 1;
}

// One parameter's AdamW update with bias corrections c1 = 1 - beta1^t and
// c2 = 1 - beta2^t: unfused f32 arithmetic, term by term as
// src/bin/mesh-gpt.rs:459-466.
__device__ __forceinline__ void adamw_element(float g, float& w, float& m, float& v, float lr, float wd, float b1,
                                              float b2, float eps, float c1, float c2) {
  const float mi = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(__fsub_rn(1.0f, b1), g));
  const float vi = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, b2), g), g));
  m = mi;
  v = vi;
  const float mh = __fdiv_rn(mi, c1);
  const float vh = __fdiv_rn(vi, c2);
  const float step = __fadd_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), __fmul_rn(wd, w));
  w = __fsub_rn(w, __fmul_rn(lr, step));
}

__global__ void adamw(int n, const OptimizerState* __restrict__ st, const float* __restrict__ grad,
                      float* __restrict__ w, float* __restrict__ m, float* __restrict__ v,
                      const int* __restrict__ step_flags) {
  if (*step_flags != 0) return;
  const float lr = st->learning_rate, wd = st->weight_decay, b1 = st->beta1, b2 = st->beta2, eps = st->epsilon;
  const float c1 = __fsub_rn(1.0f, st->beta1_power), c2 = __fsub_rn(1.0f, st->beta2_power);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float wi = w[i], mi = m[i], vi = v[i];
    adamw_element(grad[i], wi, mi, vi, lr, wd, b1, b2, eps, c1, c2);
    w[i] = wi;
    m[i] = mi;
    v[i] = vi;
  }
}

// ---- batch validation and supervised count (src/gpt/config.rs:230-253), on
// the device so device-resident batches need no host round trip.  flags bit 0:
// token outside the vocabulary; bit 1: target outside the vocabulary; bit 2: no
// supervised target.  stats[4] = (supervised count, bad token, bad target, 0)
// as floats, so that data-parallel ranks can sum them in one all-reduce; the
// count is what the cross-entropy divides by.  step_flags holds this step's
// flags (read by the optimizer), flags accumulates them until the host
// reads them.
//   dp == 0: the count and flags are final (a count of 0 becomes 1, flag 4).
//   dp != 0: stats holds this rank's raw values; finish_supervised turns
//            their sum over ranks into the final count and flags.
__global__ void count_supervised(int rows, int V, const uint32_t* __restrict__ tokens,
                                 const uint32_t* __restrict__ targets, float* __restrict__ stats,
                                 int* __restrict__ step_flags, int* __restrict__ flags, int dp) {
  __shared__ int s_count[32];
  __shared__ int s_flags[32];
  int cnt = 0, fl = 0;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const uint32_t t = tokens[i], y = targets[i];
    if (t >= (uint32_t)V) fl |= 1;
    if (y != kIgnoreTarget) {
      if (y >= (uint32_t)V) fl |= 2;
      ++cnt;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    fl |= __shfl_xor_sync(0xffffffffu, fl, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_count[threadIdx.x >> 5] = cnt;
    s_flags[threadIdx.x >> 5] = fl;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0, f = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      c += s_count[w];
      f |= s_flags[w];
    }
    if (dp) {
      stats[0] = (float)c;
      stats[1] = (float)(f & 1);
      stats[2] = (float)((f >> 1) & 1);
      stats[3] = 0.f;
      return;
    }
    if (c == 0) f |= 4;
    stats[0] = (float)(c > 0 ? c : 1);
    *step_flags = f;
    *flags |= f;
  }
}

// The data-parallel end of count_supervised: stats now holds the sums over
// ranks (counts stay exact in f32 up to 2^24 rows), so every rank divides by
// the global supervised count and takes the same flags.
__global__ void finish_supervised(float* __restrict__ stats, int* __restrict__ step_flags, int* __restrict__ flags) {
  const int f = (stats[1] > 0.f ? 1 : 0) | (stats[2] > 0.f ? 2 : 0) | (stats[0] == 0.f ? 4 : 0);
  if (stats[0] == 0.f) stats[0] = 1.f;
  *step_flags = f;
  *flags |= f;
}

// ---- mean cross-entropy: f64 sum of the f32 per-row losses in a fixed
// order (the reference sums on the host in f64, src/gpt/gpu.rs:2310-2312).
__global__ void loss_reduce(int rows, const float* __restrict__ loss_rows, const float* __restrict__ supervised,
                            double* __restrict__ loss) {
  __shared__ double s[1024];
  double acc = 0.0;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) acc += (double)loss_rows[i];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int o = blockDim.x / 2; o >= 1; o >>= 1) {
    if ((int)threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = s[0] / (double)(*supervised);
}

}  // namespace mb
