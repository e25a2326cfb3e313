// Per-op entry points of the Mesh GPT operators: device pointers, the
// caller's cudaStream_t, host-side validation before any launch.  They are
// the op-level boundary of the reference's kernels
//   gpt_rmsnorm_statistics / gpt_rmsnorm_apply  src/gpt/gpu.rs:65-94, :1035-1077
//   gpt_rope                                    :175-208
//   gpt_flash_forward / _delta / _query_gradient / _key_value_gradient /
//   _unpack                                     :381-779
//   exclusive_terms / gpt_exclusive / gpt_exclusive_backward   :781-897
//   gpt_head / gpt_cross_entropy / gpt_head_backward           :927-1021
//   gpt_adam                                    :1369-1391
// for callers that compose the model themselves and for per-op parity tests.
// The training step does not use these launches: it runs the same arithmetic
// fused into the block, attention and head kernels.  Attention and the head
// run the model's own tensor-core kernels; the norm, RoPE, XSA and delta
// launches here are plain row kernels (one warp per row and head, bound by
// HBM like their reference counterparts).
//
// This file is part of the gpt_model.cu translation unit (it launches the
// kernels defined there).

namespace mb {
namespace ops {

#define OP_CUDA(call) MB_CUDA(call)

constexpr int kOpWarps = 8;
constexpr int kOpThreads = kOpWarps * 32;

// One warp per (row, head) unit u = row * heads + head; lanes stride over
// the head's hd channels.
struct Unit {
  int lane;
  size_t u, row;
  int head;
  __device__ Unit(int heads) {
    lane = threadIdx.x & 31;
    u = (size_t)blockIdx.x * kOpWarps + (threadIdx.x >> 5);
    row = u / heads;
    head = (int)(u % heads);
  }
};

// y = x / rms(x) per (row, head) with eps 1e-5; inv [rows][heads] = 1/rms
// (may be null).  In place (y == x) is allowed.
__global__ void __launch_bounds__(kOpThreads)
    rmsnorm_forward_op(size_t units, int W, int H, const float* x, float* y, float* inv) {
  const Unit t(H);
  if (t.u >= units) return;
  const int hd = W / H;
  const float* xr = x + t.row * W + (size_t)t.head * hd;
  float s = 0.f;
  for (int c = t.lane; c < hd; c += 32) s += xr[c] * xr[c];
  const float iv = rms_scale(group_sum<32>(s), 1.0f / (float)hd);
  if (inv != nullptr && t.lane == 0) inv[t.u] = iv;
  float* yr = y + t.row * W + (size_t)t.head * hd;
  for (int c = t.lane; c < hd; c += 32) yr[c] = xr[c] * iv;
}

// dx = inv (dy - n mean(dy n)), n = x inv, with the statistics recomputed
// from the input x as the reference's backward does.
__global__ void __launch_bounds__(kOpThreads)
    rmsnorm_backward_op(size_t units, int W, int H, const float* __restrict__ x, const float* __restrict__ dy,
                        float* __restrict__ dx) {
  const Unit t(H);
  if (t.u >= units) return;
  const int hd = W / H;
  const size_t base = t.row * W + (size_t)t.head * hd;
  float s = 0.f;
  for (int c = t.lane; c < hd; c += 32) s += x[base + c] * x[base + c];
  const float iv = rms_scale(group_sum<32>(s), 1.0f / (float)hd);
  float dot = 0.f;
  for (int c = t.lane; c < hd; c += 32) dot += dy[base + c] * (x[base + c] * iv);
  const float mean = group_sum<32>(dot) / (float)hd;
  for (int c = t.lane; c < hd; c += 32) dx[base + c] = iv * (dy[base + c] - (x[base + c] * iv) * mean);
}

// Slice RoPE: per head the channel pairs (i, i + hd/2) rotate by
// angle = pos / 10000^(i / (hd/2)), pos = row mod sequence; `inverse`
// rotates by -angle (the backward).  Angles are evaluated in f64 and rounded
// to f32, as the model's table is.  One thread per (row, head, pair).
__global__ void rope_op(size_t pairs, int W, int H, int T, int inverse, const float* __restrict__ x, float* y) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= pairs) return;
  const int hd = W / H, half = hd / 2;
  const int i = (int)(idx % half);
  const size_t rh = idx / half;
  const int h = (int)(rh % H);
  const size_t row = rh / H;
  const int pos = (int)(row % (size_t)T);
  const double ang = (double)pos / pow(10000.0, (double)i / (double)half);
  const float c = (float)cos(ang);
  const float s = inverse ? -(float)sin(ang) : (float)sin(ang);
  const size_t base = row * W + (size_t)h * hd + i;
  const float a = x[base], b = x[base + half];
  y[base] = a * c - b * s;
  y[base + half] = b * c + a * s;
}

// XSA forward: z = y - (y.u)u, u = v / max(|v|, 1e-12) per head.
__global__ void __launch_bounds__(kOpThreads)
    xsa_forward_op(size_t units, int W, int H, const float* __restrict__ y, const float* __restrict__ v,
                   float* __restrict__ z) {
  const Unit t(H);
  if (t.u >= units) return;
  const int hd = W / H;
  const size_t base = t.row * W + (size_t)t.head * hd;
  float sq = 0.f;
  for (int c = t.lane; c < hd; c += 32) sq += v[base + c] * v[base + c];
  const float iv = xsa_scale(group_sum<32>(sq));
  float proj = 0.f;
  for (int c = t.lane; c < hd; c += 32) proj += y[base + c] * (v[base + c] * iv);
  proj = group_sum<32>(proj);
  for (int c = t.lane; c < hd; c += 32) z[base + c] = y[base + c] - proj * (v[base + c] * iv);
}

// XSA backward from dz: dy = dz - (dz.u)u and dv through u and the norm,
// whose gradient is taken only above the 1e-12 floor.
__global__ void __launch_bounds__(kOpThreads)
    xsa_backward_op(size_t units, int W, int H, const float* __restrict__ y, const float* __restrict__ v,
                    const float* __restrict__ dz, float* __restrict__ dy, float* __restrict__ dv) {
  const Unit t(H);
  if (t.u >= units) return;
  const int hd = W / H;
  const size_t base = t.row * W + (size_t)t.head * hd;
  float sq = 0.f;
  for (int c = t.lane; c < hd; c += 32) sq += v[base + c] * v[base + c];
  sq = group_sum<32>(sq);
  const float iv = xsa_scale(sq);
  const bool above = sq >= kXsaEpsilon * kXsaEpsilon;
  float proj = 0.f, gp = 0.f;
  for (int c = t.lane; c < hd; c += 32) {
    const float u = v[base + c] * iv;
    proj += y[base + c] * u;
    gp += dz[base + c] * u;
  }
  proj = group_sum<32>(proj);
  gp = group_sum<32>(gp);
  for (int c = t.lane; c < hd; c += 32) {
    const float u = v[base + c] * iv, g = dz[base + c];
    float d = -gp * y[base + c] - proj * g;
    if (above) d += 2.0f * proj * gp * u;
    dy[base + c] = g - gp * u;
    dv[base + c] = d * iv;
  }
}

// delta[h][row] = sum over the head's channels of dO * O (gpt_flash_delta).
__global__ void __launch_bounds__(kOpThreads)
    attention_delta_op(size_t units, size_t rows, int W, int H, const float* __restrict__ o,
                       const float* __restrict__ dout, float* __restrict__ delta) {
  const Unit t(H);
  if (t.u >= units) return;
  const int hd = W / H;
  const size_t base = t.row * W + (size_t)t.head * hd;
  float s = 0.f;
  for (int c = t.lane; c < hd; c += 32) s += dout[base + c] * o[base + c];
  s = group_sum<32>(s);
  if (t.lane == 0) delta[(size_t)t.head * rows + t.row] = s;
}

// Supervised count of the head's targets (stats[0], at least 1) and their
// validation: status |= 2 for a target outside the vocabulary, 4 when no
// row is supervised.
__global__ void count_targets_op(int rows, int V, const uint32_t* __restrict__ targets, float* __restrict__ stats,
                                 int* __restrict__ status) {
  __shared__ int s_count[32], s_bad[32];
  int cnt = 0, bad = 0;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const uint32_t y = targets[i];
    if (y != kIgnoreTarget) {
      bad |= y >= (uint32_t)V;
      ++cnt;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_count[threadIdx.x >> 5] = cnt;
    s_bad[threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0, b = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      c += s_count[w];
      b |= s_bad[w];
    }
    stats[0] = (float)(c > 0 ? c : 1);
    const int f = (b ? 2 : 0) | (c == 0 ? 4 : 0);
    if (f) atomicOr(status, f);
  }
}

// AdamW over a flat buffer with this step's bias corrections.
__global__ void adamw_op(size_t n, float lr, float wd, float b1, float b2, float eps, float c1, float c2,
                         const float* __restrict__ grad, float* __restrict__ w, float* __restrict__ m,
                         float* __restrict__ v) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float wi = w[i], mi = m[i], vi = v[i];
    adamw_element(grad[i], wi, mi, vi, lr, wd, b1, b2, eps, c1, c2);
    w[i] = wi;
    m[i] = mi;
    v[i] = vi;
  }
}

// ---------------------------------------------------------------- host side
inline void aligned16(const void* p, const char* what) {
  require((reinterpret_cast<uintptr_t>(p) & 15) == 0, std::string(what) + " must be 16-byte aligned");
}

struct RowHeads {
  size_t rows;
  int W, H, hd;
  size_t units() const { return rows * (size_t)H; }
  unsigned blocks() const { return (unsigned)((units() + kOpWarps - 1) / kOpWarps); }
};

inline RowHeads row_heads(size_t rows, uint32_t width, uint32_t heads) {
  require(rows >= 1 && rows <= 131072, "rows must be in 1..131072");
  require(width >= 2 && width <= 4096, "width must be in 2..4096");
  require(heads >= 1 && heads <= 64 && width % heads == 0, "heads must be in 1..64 and divide width");
  return RowHeads{rows, (int)width, (int)heads, (int)(width / heads)};
}

// Device scratch taken with cudaMallocAsync on the call's stream and
// released on it after the call's launches.
class StreamScratch {
 public:
  explicit StreamScratch(cudaStream_t s) : st_(s) {}
  ~StreamScratch() {
    if (p_ != nullptr) cudaFreeAsync(p_, st_);
  }
  template <class T>
  T* take(size_t n) {
    const size_t bytes = ((n * sizeof(T) + 255) / 256) * 256;
    const size_t off = used_;
    used_ += bytes;
    return reinterpret_cast<T*>(off);  // an offset until commit(); resolve it with at()
  }
  // Allocates everything taken so far in one piece; returns its base.
  char* commit() {
    OP_CUDA(cudaMallocAsync(&p_, std::max<size_t>(used_, 256), st_));
    return static_cast<char*>(p_);
  }

 private:
  cudaStream_t st_;
  void* p_ = nullptr;
  size_t used_ = 0;
};

template <class T>
T* at(char* base, T* offset) {
  return reinterpret_cast<T*>(base + reinterpret_cast<uintptr_t>(offset));
}

struct AttentionShape {
  size_t rows;
  int T, W, H, hd;
};

inline AttentionShape attention_shape(size_t rows, uint32_t sequence, uint32_t width, uint32_t heads) {
  const RowHeads rh = row_heads(rows, width, heads);
  require(sequence >= 1 && sequence <= 4096 && rows % sequence == 0,
          "rows must hold whole sequences of 1..4096 tokens");
  require(width % 4 == 0, "width must be a multiple of 4");
  require(rh.hd == 32 || rh.hd == 64 || rh.hd == 128 || rh.hd <= 16,
          "attention supports head widths 2..16, 32, 64 and 128", MB_ERR_UNSUPPORTED);
  return AttentionShape{rows, (int)sequence, rh.W, rh.H, rh.hd};
}

}  // namespace ops
}  // namespace mb

extern "C" {

using namespace mb::ops;

int mb_op_rmsnorm_forward(const float* x, float* y, float* inv, size_t rows, uint32_t width, uint32_t heads,
                          void* stream) {
  return mb::guarded([&] {
    mb::need(x, "x");
    mb::need(y, "y");
    const RowHeads rh = row_heads(rows, width, heads);
    rmsnorm_forward_op<<<rh.blocks(), kOpThreads, 0, (cudaStream_t)stream>>>(rh.units(), rh.W, rh.H, x, y, inv);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_rmsnorm_backward(const float* x, const float* dy, float* dx, size_t rows, uint32_t width, uint32_t heads,
                           void* stream) {
  return mb::guarded([&] {
    mb::need(x, "x");
    mb::need(dy, "dy");
    mb::need(dx, "dx");
    const RowHeads rh = row_heads(rows, width, heads);
    rmsnorm_backward_op<<<rh.blocks(), kOpThreads, 0, (cudaStream_t)stream>>>(rh.units(), rh.W, rh.H, x, dy, dx);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_rope(const float* x, float* y, size_t rows, uint32_t sequence, uint32_t width, uint32_t heads,
               int inverse, void* stream) {
  return mb::guarded([&] {
    mb::need(x, "x");
    mb::need(y, "y");
    const RowHeads rh = row_heads(rows, width, heads);
    mb::require(rh.hd % 2 == 0, "slice RoPE requires an even number of channels per head");
    mb::require(sequence >= 1 && sequence <= 4096 && rows % sequence == 0,
                "rows must hold whole sequences of 1..4096 tokens");
    const size_t pairs = rh.units() * (size_t)(rh.hd / 2);
    rope_op<<<(unsigned)((pairs + 255) / 256), 256, 0, (cudaStream_t)stream>>>(pairs, rh.W, rh.H, (int)sequence,
                                                                               inverse != 0, x, y);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_xsa_forward(const float* y, const float* v, float* z, size_t rows, uint32_t width, uint32_t heads,
                      void* stream) {
  return mb::guarded([&] {
    mb::need(y, "y");
    mb::need(v, "v");
    mb::need(z, "z");
    const RowHeads rh = row_heads(rows, width, heads);
    xsa_forward_op<<<rh.blocks(), kOpThreads, 0, (cudaStream_t)stream>>>(rh.units(), rh.W, rh.H, y, v, z);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_xsa_backward(const float* y, const float* v, const float* dz, float* dy, float* dv, size_t rows,
                       uint32_t width, uint32_t heads, void* stream) {
  return mb::guarded([&] {
    mb::need(y, "y");
    mb::need(v, "v");
    mb::need(dz, "dz");
    mb::need(dy, "dy");
    mb::need(dv, "dv");
    const RowHeads rh = row_heads(rows, width, heads);
    xsa_backward_op<<<rh.blocks(), kOpThreads, 0, (cudaStream_t)stream>>>(rh.units(), rh.W, rh.H, y, v, dz, dy,
                                                                           dv);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_attn_forward(const float* q, const float* k, const float* v, float* o, float* lse, size_t rows,
                       uint32_t sequence, uint32_t width, uint32_t heads, int* d_status, void* stream) {
  return mb::guarded([&] {
    for (const void* p : {(const void*)q, (const void*)k, (const void*)v, (const void*)o, (const void*)lse})
      mb::need(p, "attention operand");
    mb::need(d_status, "status");
    const AttentionShape a = attention_shape(rows, sequence, width, heads);
    for (const void* p : {(const void*)q, (const void*)k, (const void*)v, (const void*)o}) aligned16(p, "Q, K, V, O");
    cudaStream_t st = (cudaStream_t)stream;
    auto att = mb::make_attention_ops(a.hd, d_status);
    StreamScratch scratch(st);
    float* fmt = scratch.take<float>(att->scratch_floats((int)rows, a.H, 1));
    char* base = scratch.commit();
    att->scratch = at(base, fmt);
    att->layer = 0;
    att->forward(st, (int)rows, a.W, a.T, a.H, a.hd, q, k, v, o, lse);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_attn_backward(const float* q, const float* k, const float* v, const float* o, const float* dout,
                        const float* lse, float* dq, float* dk, float* dv, size_t rows, uint32_t sequence,
                        uint32_t width, uint32_t heads, int* d_status, void* stream) {
  return mb::guarded([&] {
    for (const void* p : {(const void*)q, (const void*)k, (const void*)v, (const void*)o, (const void*)dout,
                          (const void*)lse, (const void*)dq, (const void*)dk, (const void*)dv})
      mb::need(p, "attention operand");
    mb::need(d_status, "status");
    const AttentionShape a = attention_shape(rows, sequence, width, heads);
    for (const void* p : {(const void*)q, (const void*)k, (const void*)v, (const void*)o, (const void*)dout,
                          (const void*)dq, (const void*)dk, (const void*)dv})
      aligned16(p, "attention operands");
    cudaStream_t st = (cudaStream_t)stream;
    auto att = mb::make_attention_ops(a.hd, d_status);
    StreamScratch scratch(st);
    float* fmt = scratch.take<float>(att->scratch_floats((int)rows, a.H, 1));
    float* delta = scratch.take<float>(rows * (size_t)a.H);
    char* base = scratch.commit();
    att->scratch = at(base, fmt);
    att->layer = 0;
    delta = at(base, delta);
    const size_t units = rows * (size_t)a.H;
    attention_delta_op<<<(unsigned)((units + kOpWarps - 1) / kOpWarps), kOpThreads, 0, st>>>(units, rows, a.W, a.H,
                                                                                            o, dout, delta);
    att->prepare_keys(st, (int)rows, a.W, a.H, k, v);
    att->backward_dkdv(st, (int)rows, a.W, a.T, a.H, a.hd, q, k, v, dout, lse, delta, nullptr, dk, dv);
    att->backward_dq(st, (int)rows, a.W, a.T, a.H, a.hd, q, k, v, dout, lse, delta, dq);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_head_ce(const float* h, const float* embeddings, const uint32_t* targets, size_t rows, uint32_t width,
                  uint32_t vocab, float* logits, double* loss, float* dh, float* dembeddings, int* d_status,
                  void* stream) {
  return mb::guarded([&] {
    mb::need(h, "h");
    mb::need(embeddings, "embeddings");
    mb::need(targets, "targets");
    mb::need(logits, "logits");
    mb::need(loss, "loss");
    mb::need(d_status, "status");
    mb::require(rows >= 1 && rows <= 131072, "rows must be in 1..131072");
    mb::require(width >= 4 && width <= 4096 && width % 4 == 0, "width must be a multiple of 4 in 4..4096");
    mb::require(vocab >= 2 && vocab <= 65536, "vocab must be in 2..65536");
    aligned16(h, "h");
    if (dh != nullptr) aligned16(dh, "dh");
    const int R = (int)rows, W = (int)width, V = (int)vocab;
    cudaStream_t st = (cudaStream_t)stream;
    mb::gemm_prepare();
    // split-K chunk of the embedding gradient: about two CTAs per SM over
    // the V x W output tiles, as the model's embedding gradient does
    int dev = 0, sms = 1;
    OP_CUDA(cudaGetDevice(&dev));
    OP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int tiles = ((V + 127) / 128) * ((W + 63) / 64);
    const int kc = std::max(256, ((R + std::max(1, sms / tiles) - 1) / std::max(1, sms / tiles) + 31) / 32 * 32);
    StreamScratch scratch(st);
    float* nf = scratch.take<float>((size_t)R * W);
    float* inv = scratch.take<float>(R);
    float* dlog = scratch.take<float>((size_t)R * V);
    float* indicator = scratch.take<float>((size_t)R * V);
    float* dn = scratch.take<float>((size_t)R * W);
    float* loss_rows = scratch.take<float>(R);
    float* stats = scratch.take<float>(4);
    float* partial = scratch.take<float>(std::max<size_t>(1, mb::gemm_partial_floats(V, W, R, kc)));
    char* base = scratch.commit();
    nf = at(base, nf);
    inv = at(base, inv);
    dlog = at(base, dlog);
    indicator = at(base, indicator);
    dn = at(base, dn);
    loss_rows = at(base, loss_rows);
    stats = at(base, stats);
    partial = at(base, partial);
    const int hgrid = (R + mb::kHeadWarps - 1) / mb::kHeadWarps;
    count_targets_op<<<1, 1024, 0, st>>>(R, V, targets, stats, d_status);
    mb::head_norm<<<hgrid, mb::kHeadWarps * 32, 0, st>>>(R, W, h, nf, inv);
    mb::launch_gemm({nf, W, false}, {embeddings, W, false}, logits, V, R, V, W, 0, nullptr, d_status, st);
    // the targets stand in for the input tokens: the indicator half of the
    // model's embedding-gradient operand is not used here
    mb::head_loss<<<hgrid, mb::kHeadWarps * 32, 0, st>>>(R, V, logits, targets, stats, targets, loss_rows, dlog,
                                                         indicator);
    mb::loss_reduce<<<1, 1024, 0, st>>>(R, loss_rows, stats, loss);
    if (dh != nullptr) {
      mb::launch_gemm({dlog, V, false}, {embeddings, W, true}, dn, W, R, W, V, 0, nullptr, d_status, st);
      mb::head_norm_backward<<<hgrid, mb::kHeadWarps * 32, 0, st>>>(R, W, nf, inv, dn, dh);
    }
    if (dembeddings != nullptr)
      mb::launch_gemm({dlog, V, true}, {nf, W, true}, dembeddings, W, V, W, R, kc, partial, d_status, st);
    OP_CUDA(cudaGetLastError());
  });
}

int mb_op_adamw(float* weights, float* m, float* v, const float* gradient, size_t count, const mb_adamw* options,
                uint32_t step, void* stream) {
  return mb::guarded([&] {
    mb::need(weights, "weights");
    mb::need(m, "m");
    mb::need(v, "v");
    mb::need(gradient, "gradient");
    mb::need(options, "options");
    mb::validate_optimizer(*options);
    mb::require(count >= 1, "count must be positive");
    mb::require(step >= 1, "step counts updates from 1");
    // beta^t accumulated in f32, one multiplication per update, as the
    // reference's host does (src/gpt/gpu.rs:1980-1981)
    float b1p = 1.0f, b2p = 1.0f;
    for (uint32_t t = 0; t < step; ++t) {
      b1p *= options->beta1;
      b2p *= options->beta2;
    }
    const float c1 = 1.0f - b1p, c2 = 1.0f - b2p;
    int dev = 0, sms = 1;
    OP_CUDA(cudaGetDevice(&dev));
    OP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const unsigned blocks = (unsigned)std::min<size_t>((count + 255) / 256, (size_t)sms * 8);
    adamw_op<<<blocks, 256, 0, (cudaStream_t)stream>>>(count, options->learning_rate, options->weight_decay,
                                                        options->beta1, options->beta2, options->epsilon, c1, c2,
                                                        gradient, weights, m, v);
    OP_CUDA(cudaGetLastError());
  });
}

}  // extern "C"
