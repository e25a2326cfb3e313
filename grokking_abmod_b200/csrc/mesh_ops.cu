// Op-level entry points for one two-parent mesh stack (device pointers and
// the caller's stream), the per-op boundary of the reference's gpt_mesh
// forward/backward and per-edge gradient kernels (src/gpt/gpu.rs:103-146,
// :1087-1149, host loop :2370-2444).
//
// A stack is `depth` layers over rows x width: y = f(x[c] w0[c] + x[c+s] w1[c])
// with ELU (alpha 1) on every layer but the last, s the layer's connectivity
// stride.  Backward recomputes the stack from its input, produces dx and the
// f32 edge gradients dweights [depth][width][2], reduced deterministically
// from per-(CTA, row lane) partials held in scratch memory.

#include <cstring>
#include <mutex>
#include <string>

#include "gpt_rows.cuh"
#include "host.h"

namespace mb {

#define OPS_CUDA(call)                                                                              \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess)                                                                          \
      throw Error(MB_ERR_CUDA, std::string(#call) + " failed: " + cudaGetErrorString(e_));          \
  } while (0)

constexpr int kOpRpt = 4;

template <int W>
__global__ void __launch_bounds__(RowTile<W, kOpRpt>::NT)
    mesh_stack_forward(Dims d, const float* __restrict__ x, const float* __restrict__ weights,
                       float* __restrict__ y) {
  using T = RowTile<W, kOpRpt>;
  extern __shared__ float4 smem4[];
  float* bufs = reinterpret_cast<float*>(smem4);
  Ctx<T> c;
  const int ntiles = (d.rows + T::TR - 1) / T::TR;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float2 a[kOpRpt];
#pragma unroll
    for (int k = 0; k < kOpRpt; ++k) {
      const int r = tile * T::TR + c.row(k);
      a[k] = r < d.rows ? __ldg(reinterpret_cast<const float2*>(x + (size_t)r * W) + c.cp) : make_float2(0.f, 0.f);
    }
    mesh_forward<W, T, 0, -1>(c, d, a, reinterpret_cast<const float4*>(weights), d.attn_depth, bufs, false);
#pragma unroll
    for (int k = 0; k < kOpRpt; ++k) {
      const int r = tile * T::TR + c.row(k);
      if (r < d.rows) reinterpret_cast<float2*>(y + (size_t)r * W)[c.cp] = a[k];
    }
    __syncthreads();
  }
}

// partial: [gridDim.x * RL][depth][W][2]
template <int W>
__global__ void __launch_bounds__(RowTile<W, kOpRpt>::NT)
    mesh_stack_backward(Dims d, const float* __restrict__ x, const float* __restrict__ dy,
                        const float* __restrict__ weights, float* __restrict__ dx, float* __restrict__ partial) {
  using T = RowTile<W, kOpRpt>;
  extern __shared__ float4 smem4[];
  const int depth = d.attn_depth;
  float4* acc = smem4;
  float* bufs = reinterpret_cast<float*>(smem4 + depth * T::NT);
  float* xch = bufs + depth * T::BUF;
  Ctx<T> c;
  for (int l = 0; l < depth; ++l) acc[l * T::NT + c.tid] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* wg = reinterpret_cast<const float4*>(weights);
  const int ntiles = (d.rows + T::TR - 1) / T::TR;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    float2 a[kOpRpt], g[kOpRpt];
#pragma unroll
    for (int k = 0; k < kOpRpt; ++k) {
      const int r = tile * T::TR + c.row(k);
      const bool in = r < d.rows;
      a[k] = in ? __ldg(reinterpret_cast<const float2*>(x + (size_t)r * W) + c.cp) : make_float2(0.f, 0.f);
      g[k] = in ? __ldg(reinterpret_cast<const float2*>(dy + (size_t)r * W) + c.cp) : make_float2(0.f, 0.f);
    }
    mesh_forward<W, T, 0, -1>(c, d, a, wg, depth, bufs, true);
    mesh_backward<W, T, 0, -1>(c, d, g, wg, depth, bufs, xch, acc);
#pragma unroll
    for (int k = 0; k < kOpRpt; ++k) {
      const int r = tile * T::TR + c.row(k);
      if (r < d.rows) reinterpret_cast<float2*>(dx + (size_t)r * W)[c.cp] = g[k];
    }
    __syncthreads();
  }
  const int slot = blockIdx.x * T::RL + c.rl;
  float4* out = reinterpret_cast<float4*>(partial) + (size_t)slot * depth * T::PAIRS;
  for (int l = 0; l < depth; ++l) out[l * T::PAIRS + c.cp] = slot_to_params(acc[l * T::NT + c.tid]);
}

// out[p] = sum over slots of partial[slot][p], in slot order.
__global__ void reduce_slots(const float* __restrict__ partial, int slots, int size, float* __restrict__ out) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < size; p += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < slots; ++k) s += partial[(size_t)k * size + p];
    out[p] = s;
  }
}

namespace {

struct MeshOpShape {
  int W, depth, rows;
  Dims d;
  int nt, rl, tile_rows;
  size_t smem_fwd, smem_bwd;
  void* fwd;
  void* bwd;
  int occ_bwd = 1;
  int sms = 1;
};

template <int W>
void fill_shape(MeshOpShape& s) {
  using T = RowTile<W, kOpRpt>;
  s.nt = T::NT;
  s.rl = T::RL;
  s.tile_rows = T::TR;
  s.smem_fwd = (size_t)2 * T::BUF * sizeof(float);
  s.smem_bwd = (size_t)s.depth * T::NT * sizeof(float4) + (size_t)(s.depth + 2) * T::BUF * sizeof(float);
  s.fwd = (void*)&mesh_stack_forward<W>;
  s.bwd = (void*)&mesh_stack_backward<W>;
}

MeshOpShape mesh_shape(size_t rows, uint32_t width, uint32_t depth, uint32_t connectivity) {
  require(rows >= 1 && rows <= 131072, "rows must be in 1..131072");
  require(depth >= 1 && depth <= 16, "mesh depth must be in 1..16");
  require(connectivity <= 1, "connectivity must be 0 (neighbor) or 1 (butterfly)");
  MeshOpShape s{};
  s.W = (int)width;
  s.depth = (int)depth;
  s.rows = (int)rows;
  switch (width) {
    case 64: fill_shape<64>(s); break;
    case 128: fill_shape<128>(s); break;
    case 256: fill_shape<256>(s); break;
    case 384: fill_shape<384>(s); break;
    case 512: fill_shape<512>(s); break;
    default: throw Error(MB_ERR_UNSUPPORTED, "mesh ops support widths 64, 128, 256, 384 and 512");
  }
  s.d = Dims{};
  s.d.rows = (int)rows;
  s.d.sequence = 1;
  s.d.heads = 1;
  s.d.head_width = 2;
  s.d.vocab = 2;
  s.d.attn_depth = (int)depth;
  s.d.ffn_depth = (int)depth;
  s.d.connectivity = (int)connectivity;
  s.d.log2w = 31 - __builtin_clz(width);
  int dev = 0;
  OPS_CUDA(cudaGetDevice(&dev));
  OPS_CUDA(cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev));
  OPS_CUDA(cudaFuncSetAttribute(s.fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s.smem_fwd));
  OPS_CUDA(cudaFuncSetAttribute(s.bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s.smem_bwd));
  OPS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&s.occ_bwd, s.bwd, s.nt, s.smem_bwd));
  require(s.occ_bwd > 0, "mesh backward does not fit on this device", MB_ERR_UNSUPPORTED);
  return s;
}

int grid_for(const MeshOpShape& s, int per_sm) {
  const int tiles = (s.rows + s.tile_rows - 1) / s.tile_rows;
  return std::max(1, std::min(tiles, s.sms * per_sm));
}

// Launches the backward kernel on `grid` CTAs with `partial` holding
// grid * RL slots, then reduces the slots into dweights.
void launch_mesh_backward(const MeshOpShape& s, int grid, const float* x, const float* dy, const float* weights,
                          float* dx, float* dweights, float* partial, cudaStream_t st) {
  Dims d = s.d;
  void* args[] = {&d, (void*)&x, (void*)&dy, (void*)&weights, &dx, &partial};
  OPS_CUDA(cudaLaunchKernel(s.bwd, dim3(grid), dim3(s.nt), args, s.smem_bwd, st));
  const int size = s.depth * 2 * s.W;
  reduce_slots<<<(size + 255) / 256, 256, 0, st>>>(partial, grid * s.rl, size, dweights);
  OPS_CUDA(cudaGetLastError());
}

// ---- allocation-free mesh backward
//
// mb_op_mesh_backward_noalloc keeps its gradient partials in this file-scope
// device array instead of memory from cudaMalloc/cudaMallocAsync.  Every GPU
// that loads the library holds the array (4 MiB) until the process exits.
// Host code must not pass `g_noalloc_partials` itself to a kernel: on the host
// that name is only a stand-in symbol, not a device address.  The address is
// looked up once per device with cudaGetSymbolAddress (noalloc_scratch).
constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB of f32
static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_address[256] = {};

// Device address of g_noalloc_partials on the current device; the first call
// on a device looks it up (with that device current) and caches it.
float* noalloc_scratch() {
  int dev = 0;
  OPS_CUDA(cudaGetDevice(&dev));
  require(dev >= 0 && dev < 256, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_address[dev] == nullptr) {
    void* p = nullptr;
    OPS_CUDA(cudaGetSymbolAddress(&p, g_noalloc_partials));
    g_noalloc_address[dev] = static_cast<float*>(p);
  }
  return g_noalloc_address[dev];
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" {

int mb_op_mesh_forward(const float* x, float* y, size_t rows, uint32_t width, uint32_t depth, uint32_t connectivity,
                       const float* weights, void* stream) {
  return guarded([&] {
    need(x, "x");
    need(y, "y");
    need(weights, "weights");
    MeshOpShape s = mesh_shape(rows, width, depth, connectivity);
    Dims d = s.d;
    const int grid = grid_for(s, 4);
    void* args[] = {&d, (void*)&x, (void*)&weights, &y};
    OPS_CUDA(cudaLaunchKernel(s.fwd, dim3(grid), dim3(s.nt), args, s.smem_fwd, (cudaStream_t)stream));
  });
}

int mb_op_mesh_backward(const float* x, const float* dy, float* dx, float* dweights, size_t rows, uint32_t width,
                        uint32_t depth, uint32_t connectivity, const float* weights, void* stream) {
  return guarded([&] {
    need(x, "x");
    need(dy, "dy");
    need(dx, "dx");
    need(dweights, "dweights");
    need(weights, "weights");
    MeshOpShape s = mesh_shape(rows, width, depth, connectivity);
    cudaStream_t st = (cudaStream_t)stream;
    const int grid = grid_for(s, s.occ_bwd);
    float* partial = nullptr;
    const size_t bytes = (size_t)grid * s.rl * s.depth * 2 * s.W * sizeof(float);
    OPS_CUDA(cudaMallocAsync((void**)&partial, bytes, st));
    try {
      launch_mesh_backward(s, grid, x, dy, weights, dx, dweights, partial, st);
    } catch (...) {
      cudaFreeAsync(partial, st);
      throw;
    }
    OPS_CUDA(cudaFreeAsync(partial, st));
  });
}

}  // extern "C"

extern "C" int mb_op_mesh_backward_noalloc(const float* x, const float* dy, float* dx, float* dweights, size_t rows,
                                           uint32_t width, uint32_t depth, uint32_t connectivity,
                                           const float* weights, void* stream) {
  return guarded([&] {
    need(x, "x");
    need(dy, "dy");
    need(dx, "dx");
    need(dweights, "dweights");
    need(weights, "weights");
    MeshOpShape s = mesh_shape(rows, width, depth, connectivity);
    // One CTA needs row_lanes partial slots of depth*2*width floats; the grid
    // is capped so that all its slots fit the static scratch.
    const size_t per_cta = (size_t)s.rl * s.depth * 2 * s.W;
    require(per_cta <= kNoAllocScratchFloats,
            "mesh stack too large for the allocation-free scratch (row_lanes * depth * 2 * width must be <= "
            "1048576 floats)");
    const int cap = (int)(kNoAllocScratchFloats / per_cta);
    const int grid = std::min(grid_for(s, s.occ_bwd), cap);
    launch_mesh_backward(s, grid, x, dy, weights, dx, dweights, noalloc_scratch(), (cudaStream_t)stream);
  });
}
