// Mesh GPT executor (host C++) and its C ABI.
//
// Replaces SpecializedMeshGpt (src/gpt/gpu.rs:1701-2092) and its op-by-op
// plan (src/gpt/gpu.rs:1395-1547, :2158-2607): instead of ~500 small launches
// and a host sync per step, one training step is a fixed sequence of
// 7*layers+10 fused kernels on one stream, captured once per batch shape as a
// CUDA graph; the loss stays on the device until the caller reads it.
//
// Device layout (HBM, all FP32 unless noted):
//   weights / adam_m / adam_v / gradient : flat [P] in the reference's layout
//       order (embedding mesh, then per block Q, K, V, O, FFN meshes; each
//       group layer-major with (self, neighbour) pairs) - SoA instead of the
//       reference's AoS [w, m, v] so AdamW streams 4 coalesced arrays.
//   embedding acts [A+1][V][W] and its transpose Et [W][V]
//   per workspace (one per (rows, sequence) shape, up to 3 retained):
//       x[L+1], per block Q, K, V, O, x_mid [N][W], lse2 [H][N];
//       backward scratch dx, dO, dV(XSA), dx_mid, dQ, dK, dV [N][W],
//       delta [H][N], head scratch nf [N][W], dlogits [N][V]; per-CTA
//       gradient partials [slots][group size] per parameter group.

#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>

#include "gemm_tc.h"
#include "host.h"

#include "gpt_attention.cu"
#include "gpt_blocks.cu"
#include "gpt_attention_f16.cu"
#include "gpt_head.cu"

namespace mb {

#define MB_CUDA(call)                                                                               \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess)                                                                          \
      throw Error(MB_ERR_CUDA, std::string(#call) + " failed: " + cudaGetErrorString(e_));          \
  } while (0)

// ------------------------------------------------------------------ memory
class DeviceArena {
 public:
  ~DeviceArena() {
    for (void* p : ptrs_) cudaFree(p);
  }
  template <class T>
  T* alloc(size_t n) {
    void* p = nullptr;
    const size_t bytes = n == 0 ? 16 : n * sizeof(T);
    MB_CUDA(cudaMalloc(&p, bytes));
    ptrs_.push_back(p);
    bytes_ += bytes;
    return static_cast<T*>(p);
  }
  size_t bytes() const { return bytes_; }

 private:
  std::vector<void*> ptrs_;
  size_t bytes_ = 0;
};

// ------------------------------------------------- width-specialised blocks
struct BlockOps {
  virtual ~BlockOps() = default;
  int row_lanes = 1, tile_rows = 1, tile_rows_post = 1, tile_rows_bwd = 1;
  int occ_qf = 1, occ_pf = 1, occ_pb = 1, occ_qb = 1;
  size_t smem_f = 0, smem_pf = 0, smem_pb = 0, smem_qb = 0;
  virtual void qkv_forward(cudaStream_t s, int grid, const Dims& d, const float* x, const uint32_t* tokens,
                           const float* emb, float* x_out, const float* wq, const float* wk, const float* wv,
                           const float2* rope, float* q, float* k, float* v) = 0;
  virtual void post_forward(cudaStream_t s, int grid, const Dims& d, const float* o, const float* v,
                            const float* x, const float* wo, const float* wf, float* xm, float* xn) = 0;
  virtual void post_backward(cudaStream_t s, int grid, const Dims& d, const float* dxn, const float* xm,
                             const float* o, const float* v, const float* wo, const float* wf, float* dO,
                             float* dvx, float* dxm, float* delta, float* part_o, float* part_f) = 0;
  virtual void qkv_backward(cudaStream_t s, int grid, const Dims& d, const float* dq, const float* dk,
                            const float* dv, const float* x, const float* dxm, const float* wq, const float* wk,
                            const float* wv, const float2* rope, float* dx, float* pq, float* pk, float* pv) = 0;
};

// Rows per thread of the block kernels, from measured sweeps: qkv_forward
// runs fastest with 4, post_forward with 2, the backward kernels with 2.
constexpr int kRptForward = 4;
constexpr int kRptPostForward = 2;
constexpr int kRptBackward = 2;

template <int W, class S>
struct BlockOpsW final : BlockOps {
  using TF = RowTile<W, kRptForward>;
  using TP = RowTile<W, kRptPostForward>;
  using TB = RowTile<W, kRptBackward>;
  explicit BlockOpsW(int A, int F) {
    row_lanes = TB::RL;
    tile_rows = TF::TR;
    tile_rows_post = TP::TR;
    tile_rows_bwd = TB::TR;
    smem_f = BlockKernels<W, kRptForward>::smem_forward();
    smem_pf = BlockKernels<W, kRptPostForward>::smem_forward();
    smem_pb = BlockKernels<W, kRptBackward>::smem_post_backward(A, F);
    smem_qb = BlockKernels<W, kRptBackward>::smem_qkv_backward(A);
    MB_CUDA(cudaFuncSetAttribute(qkv_forward_k(), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_f));
    MB_CUDA(cudaFuncSetAttribute(post_forward_k(), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_pf));
    MB_CUDA(cudaFuncSetAttribute(post_backward_k(), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_pb));
    MB_CUDA(cudaFuncSetAttribute(qkv_backward_k(), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_qb));
    MB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_qf, qkv_forward_k(), TF::NT, smem_f));
    MB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_pf, post_forward_k(), TP::NT, smem_pf));
    MB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_pb, post_backward_k(), TB::NT, smem_pb));
    MB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_qb, qkv_backward_k(), TB::NT, smem_qb));
    require(occ_qf > 0 && occ_pf > 0 && occ_pb > 0 && occ_qb > 0,
            "fused block kernels do not fit on this device for these mesh depths", MB_ERR_UNSUPPORTED);
  }
  static auto qkv_forward_k() { return &mb::qkv_forward<W, kRptForward, S>; }
  static auto post_forward_k() { return &mb::post_forward<W, kRptPostForward, S>; }
  static auto post_backward_k() { return &mb::post_backward<W, kRptBackward, S>; }
  static auto qkv_backward_k() { return &mb::qkv_backward<W, kRptBackward, S>; }
  void qkv_forward(cudaStream_t s, int grid, const Dims& d, const float* x, const uint32_t* tokens,
                   const float* emb, float* x_out, const float* wq, const float* wk, const float* wv,
                   const float2* rope, float* q, float* k, float* v) override {
    qkv_forward_k()<<<grid, TF::NT, smem_f, s>>>(d, x, tokens, emb, x_out, wq, wk, wv, rope, q, k, v);
  }
  void post_forward(cudaStream_t s, int grid, const Dims& d, const float* o, const float* v, const float* x,
                    const float* wo, const float* wf, float* xm, float* xn) override {
    post_forward_k()<<<grid, TP::NT, smem_pf, s>>>(d, o, v, x, wo, wf, xm, xn);
  }
  void post_backward(cudaStream_t s, int grid, const Dims& d, const float* dxn, const float* xm, const float* o,
                     const float* v, const float* wo, const float* wf, float* dO, float* dvx, float* dxm,
                     float* delta, float* part_o, float* part_f) override {
    post_backward_k()<<<grid, TB::NT, smem_pb, s>>>(d, dxn, xm, o, v, wo, wf, dO, dvx, dxm, delta,
                                                                     part_o, part_f);
  }
  void qkv_backward(cudaStream_t s, int grid, const Dims& d, const float* dq, const float* dk, const float* dv,
                    const float* x, const float* dxm, const float* wq, const float* wk, const float* wv,
                    const float2* rope, float* dx, float* pq, float* pk, float* pv) override {
    qkv_backward_k()<<<grid, TB::NT, smem_qb, s>>>(d, dq, dk, dv, x, dxm, wq, wk, wv, rope, dx, pq,
                                                                    pk, pv);
  }
};

// The reference's default mesh depths (attention 4, FFN 6; src/gpt/config.rs:46-47)
// get kernels with the shape compiled in (and, for 64-channel heads, the
// head width too); other depths run the same kernels
// with the shape read at run time, and heads of 128 channels or more (hd,
// from width 128 up) the variant whose head sums and RoPE partners cross warps.
template <int W>
std::unique_ptr<BlockOps> make_block_ops_w(int A, int F, int conn, int hd) {
  if constexpr (W >= 128) {
    if (hd > 64) return std::make_unique<BlockOpsW<W, RuntimeShapeWide>>(A, F);
  }
  if (A == 4 && F == 6 && hd == 64) {
    if (conn == 0) return std::make_unique<BlockOpsW<W, MeshShape<4, 6, 0, false, 32>>>(A, F);
    if (conn == 1) return std::make_unique<BlockOpsW<W, MeshShape<4, 6, 1, false, 32>>>(A, F);
  }
  if (A == 4 && F == 6 && conn == 0) return std::make_unique<BlockOpsW<W, MeshShape<4, 6, 0>>>(A, F);
  if (A == 4 && F == 6 && conn == 1) return std::make_unique<BlockOpsW<W, MeshShape<4, 6, 1>>>(A, F);
  return std::make_unique<BlockOpsW<W, RuntimeShape>>(A, F);
}

std::unique_ptr<BlockOps> make_block_ops(int W, int A, int F, int conn, int hd) {
  switch (W) {
    case 64: return make_block_ops_w<64>(A, F, conn, hd);
    case 128: return make_block_ops_w<128>(A, F, conn, hd);
    case 256: return make_block_ops_w<256>(A, F, conn, hd);
    case 384: return make_block_ops_w<384>(A, F, conn, hd);
    case 512: return make_block_ops_w<512>(A, F, conn, hd);
  }
  throw Error(MB_ERR_UNSUPPORTED, "unsupported width");
}

// ------------------------------------------------- head-width attention ops
struct AttentionOps {
  virtual ~AttentionOps() = default;
  // Device scratch (floats) the kernels need for `rows` token rows of a
  // `layers`-block model; the model allocates it per workspace and sets
  // `scratch` (and `layer`, the block being enqueued) before enqueueing.
  virtual size_t scratch_floats(int rows, int H, int layers) const { return 0; }
  // Kernel launches of one forward / one backward (dK/dV + dQ) call.
  virtual int forward_launches() const { return 1; }
  virtual int backward_launches() const { return 2; }
  float* scratch = nullptr;
  int layer = 0;
  // Lays out the key operand tiles that forward and dQ read (tensor-core
  // kernels only); forward does it itself.
  virtual void prepare_keys(cudaStream_t s, int rows, int W, int H, const float* k, const float* v) {}
  virtual void forward(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
                       const float* v, float* o, float* lse) = 0;
  virtual void backward_dkdv(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q,
                             const float* k, const float* v, const float* dout, const float* lse,
                             const float* delta, const float* dv_add, float* dk, float* dv) = 0;  // dv_add may be dv
  virtual void backward_dq(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
                           const float* v, const float* dout, const float* lse, const float* delta,
                           float* dq) = 0;
};

template <int HD>
struct AttentionOpsD final : AttentionOps {
  using K = AttentionKernels<HD>;
  AttentionOpsD() {
    MB_CUDA(cudaFuncSetAttribute(&attention_forward<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)K::smem_forward()));
    MB_CUDA(cudaFuncSetAttribute(&attention_backward_dq<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)K::smem_dq()));
    MB_CUDA(cudaFuncSetAttribute(&attention_backward_dkdv<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)K::smem_dkdv()));
  }
  void forward(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
               const float* v, float* o, float* lse) override {
    dim3 grid((rows + 63) / 64, H);
    attention_forward<HD><<<grid, 256, K::smem_forward(), s>>>(rows, W, T, hd, 1.0f / sqrtf((float)hd), q, k, v, o,
                                                                lse);
  }
  void backward_dkdv(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
                     const float* v, const float* dout, const float* lse, const float* delta, const float* dv_add,
                     float* dk, float* dv) override {
    dim3 grid((rows + 63) / 64, H);
    attention_backward_dkdv<HD><<<grid, 256, K::smem_dkdv(), s>>>(rows, W, T, hd, 1.0f / sqrtf((float)hd), q, k, v,
                                                                   dout, lse, delta, dv_add, dk, dv);
  }
  void backward_dq(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
                   const float* v, const float* dout, const float* lse, const float* delta, float* dq) override {
    dim3 grid((rows + 63) / 64, H);
    attention_backward_dq<HD><<<grid, 256, K::smem_dq(), s>>>(rows, W, T, hd, 1.0f / sqrtf((float)hd), q, k, v, dout,
                                                               lse, delta, dq);
  }
};

// Tensor-core (tcgen05, 3xF16) attention for head widths 32 and 64.
template <int HD>
struct AttentionOpsTc final : AttentionOps {
  int* err;
  int sms = 148;  // CTAs of the persistent dK/dV kernel: one per SM
  explicit AttentionOpsTc(int* e) : err(e) {
    int dev = 0;
    MB_CUDA(cudaGetDevice(&dev));
    MB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    MB_CUDA(cudaFuncSetAttribute(&attention_forward_f16<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)F16Att<HD>::smem_forward));
    MB_CUDA(cudaFuncSetAttribute(&attention_backward_dq_f16<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)F16Dq<HD>::smem));
    MB_CUDA(cudaFuncSetAttribute(&attention_backward_dkdv_f16<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)F16Kv<HD>::smem));
  }
  // per block: the FP16 key tiles the forward and dQ read
  static size_t key_floats(int rows, int H) {
    return (size_t)H * ((rows + kTcK - 1) / kTcK) * F16Fmt<HD>::KTILE_BYTES / sizeof(float);
  }
  static size_t query_floats(int rows, int H) {
    return (size_t)H * ((rows + kTcQ - 1) / kTcQ) * F16Q<HD>::QTILE_BYTES / sizeof(float);
  }
  // One query-tile set (rebuilt per backward block) and one key-tile set per
  // block: the forward formats every key part once and dQ reuses them.
  size_t scratch_floats(int rows, int H, int layers) const override {
    return query_floats(rows, H) + (size_t)layers * key_floats(rows, H);
  }
  int forward_launches() const override { return 2; }   // key format + forward
  int backward_launches() const override { return 3; }  // query format + dK/dV, dQ
  uint8_t* qfmt16() const { return reinterpret_cast<uint8_t*>(scratch); }
  uint8_t* kfmt16(int rows, int H) const {
    return reinterpret_cast<uint8_t*>(scratch + query_floats(rows, H) + (size_t)layer * key_floats(rows, H));
  }
  void prepare_keys(cudaStream_t s, int rows, int W, int H, const float* k, const float* v) override {
    attention_format_keys_f16<HD><<<dim3((rows + kTcK - 1) / kTcK, H), kFmtThreads, 0, s>>>(
        rows, W, k, v, kfmt16(rows, H));
  }
  void forward(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
               const float* v, float* o, float* lse) override {
    prepare_keys(s, rows, W, H, k, v);
    CUtensorMap mq, mo;
    require(encode_rows_map(&mq, q, rows, W, kTcRows) && encode_rows_map(&mo, o, rows, W, kTcRows),
            "attention forward: TMA maps need 16-byte aligned tensors", MB_ERR_UNSUPPORTED);
    const int items = ((rows + kTcRows - 1) / kTcRows) * H;
    attention_forward_f16<HD><<<std::min(items, sms), kFwdThreads, F16Att<HD>::smem_forward, s>>>(
        rows, T, H, 1.0f / sqrtf((float)hd), mq, kfmt16(rows, H), mo, lse, err);
  }
  void backward_dkdv(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
                     const float* v, const float* dout, const float* lse, const float* delta, const float* dv_add,
                     float* dk, float* dv) override {
    attention_format_queries_f16<HD><<<dim3((rows + kTcQ - 1) / kTcQ, H), kFmtThreads, 0, s>>>(rows, W, q, dout, lse,
                                                                                           delta, qfmt16());
    // TMA maps over the [rows][W] K, V, dK and dV tensors, 128 x 32 boxes.
    CUtensorMap mk, mv, mdk, mdv;
    require(encode_rows_map(&mk, k, rows, W, kTcRows) && encode_rows_map(&mv, v, rows, W, kTcRows) &&
                encode_rows_map(&mdk, dk, rows, W, kTcRows) && encode_rows_map(&mdv, dv, rows, W, kTcRows),
            "attention backward: TMA maps need 16-byte aligned tensors", MB_ERR_UNSUPPORTED);
    // dV is added onto the XSA term: in place when dv_add is dv, else onto a copy.
    if (dv_add != nullptr && dv_add != dv)
      MB_CUDA(cudaMemcpyAsync(dv, dv_add, (size_t)rows * W * sizeof(float), cudaMemcpyDeviceToDevice, s));
    const int items = ((rows + kTcRows - 1) / kTcRows) * H;
    attention_backward_dkdv_f16<HD><<<std::min(items, sms), kKvThreadsP, F16Kv<HD>::smem, s>>>(
        rows, T, H, 1.0f / sqrtf((float)hd), mk, mv, qfmt16(), mdk, mdv, dv_add != nullptr ? 1 : 0, err);
  }
  void backward_dq(cudaStream_t s, int rows, int W, int T, int H, int hd, const float* q, const float* k,
                   const float* v, const float* dout, const float* lse, const float* delta, float* dq) override {
    (void)k;
    (void)v;  // read through the key tiles of the forward's format pass
    CUtensorMap mq, mo, mdq;
    require(encode_rows_map(&mq, q, rows, W, kTcRows) && encode_rows_map(&mo, dout, rows, W, kTcRows) &&
                encode_rows_map(&mdq, dq, rows, W, kTcRows),
            "attention backward: TMA maps need 16-byte aligned tensors", MB_ERR_UNSUPPORTED);
    const int items = ((rows + kTcRows - 1) / kTcRows) * H;
    attention_backward_dq_f16<HD><<<std::min(items, sms), kKvThreadsP, F16Dq<HD>::smem, s>>>(
        rows, T, H, 1.0f / sqrtf((float)hd), mq, mo, kfmt16(rows, H), lse, delta, mdq, err);
  }
};

std::unique_ptr<AttentionOps> make_attention_ops(int hd, int* err) {
  if (hd == 64) return std::make_unique<AttentionOpsTc<64>>(err);
  if (hd == 32) return std::make_unique<AttentionOpsTc<32>>(err);
  if (hd <= 16) return std::make_unique<AttentionOpsD<16>>();
  if (hd <= 32) return std::make_unique<AttentionOpsD<32>>();
  if (hd <= 64) return std::make_unique<AttentionOpsD<64>>();
  if (hd <= 128) return std::make_unique<AttentionOpsD<128>>();
  throw Error(MB_ERR_UNSUPPORTED, "unsupported head width");
}

// ------------------------------------------------------------------- NCCL
struct NcclApi {
  void* handle = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // Reuses the NCCL already loaded by the process (e.g. torch's) when present.
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    api.handle = h;
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
    api.comm_abort = (decltype(api.comm_abort))dlsym(h, "ncclCommAbort");
    api.comm_count = (decltype(api.comm_count))dlsym(h, "ncclCommCount");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
  });
  require(api.handle != nullptr && api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy,
          "libnccl.so.2 could not be loaded", MB_ERR_NCCL);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess)
    throw Error(MB_ERR_NCCL, std::string(what) + " failed: " + (nccl().error_string ? nccl().error_string(r) : "?"));
}

// ---------------------------------------------------------------- workspace
struct Workspace {
  int rows = 0, seq = 0;
  DeviceArena mem;
  std::vector<float*> x;  // L + 1
  std::vector<float*> q, k, v, o, xm, lse;
  // nf and g are one allocation ([2][rows][W]), as are dlog and indicator
  // ([2][rows][V]): the embedding gradient contracts both halves in one GEMM.
  float *nf, *dlog, *indicator, *logits, *loss_rows, *g, *dO, *dvx, *dxm, *delta, *dq, *dk, *emb_partial, *dE;
  float *head_inv, *head_dn;  // final RMSNorm's 1/rms per row and the head's dn = dlogits E
  float* emb_mesh_partial;
  float* att_scratch;
  float2* rope;
  uint32_t *tokens, *targets;
  float* stats;     // [4]: supervised count (the loss divisor), bad-token and bad-target indicators
  int* step_flags;  // this step's batch flags (the optimizer skips a flagged step)
  int* flags;       // flags accumulated until mb_gpt_check reads them
  double* loss;
  std::vector<float*> part;  // per parameter group
  ReduceJob* d_jobs;  // group reductions
  int njobs = 0, max_job = 0, emb_k_chunk = 0;
  int grid_qf = 1, grid_pf = 1, grid_pb = 1, grid_qb = 1;
  cudaGraphExec_t graph = nullptr;
  bool graph_dp = false;  // captured for data parallelism (the batch count runs outside the graph)
  // Kernel boundary events captured into the graph when timing is enabled:
  // marks[i] precedes launch i, marks.back() follows the last one.
  std::vector<cudaEvent_t> marks;
  std::vector<std::string> mark_names;
  ~Workspace() {
    if (graph) cudaGraphExecDestroy(graph);
    for (cudaEvent_t e : marks) cudaEventDestroy(e);
  }
};

// --------------------------------------------------------------------- model
class GptModel {
 public:
  // shared: a stream the caller owns (a context's), used instead of the
  // model's own.
  GptModel(int device, const mb_gpt_config& cfg, uint64_t seed, cudaStream_t shared = nullptr)
      : cfg_(cfg), device_(device) {
    validate_kernel_shapes(cfg);
    layout_ = make_layout(cfg);
    int count = 0;
    MB_CUDA(cudaGetDeviceCount(&count));
    require(device >= 0 && device < count, "CUDA device index out of range");
    MB_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    MB_CUDA(cudaGetDeviceProperties(&prop, device));
    require(prop.major >= 10, "this library is built for sm_100a (B200)", MB_ERR_UNSUPPORTED);
    sms_ = prop.multiProcessorCount;
    if (shared != nullptr) {
      stream_ = shared;
    } else {
      MB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
      owns_stream_ = true;
    }
    blocks_ = make_block_ops(cfg.width, cfg.attention_mesh_depth, cfg.ffn_mesh_depth, (int)cfg.connectivity,
                             (int)(cfg.width / cfg.heads));
    tc_err_ = mem_.alloc<int>(1);
    MB_CUDA(cudaMemset(tc_err_, 0, sizeof(int)));
    attention_ = make_attention_ops(cfg.width / cfg.heads, tc_err_);
    gemm_prepare();
    const size_t P = layout_.count();
    w_ = mem_.alloc<float>(P);
    m_ = mem_.alloc<float>(P);
    v_ = mem_.alloc<float>(P);
    grad_ = mem_.alloc<float>(P);
    const size_t VW = (size_t)cfg.vocab_size * cfg.width;
    emb_acts_ = mem_.alloc<float>(VW * (cfg.attention_mesh_depth + 1));
    et_ = mem_.alloc<float>(VW);
    opt_ = mem_.alloc<OptimizerState>(1);
    std::vector<float> codes = token_codes(cfg);
    MB_CUDA(cudaMemcpy(emb_acts_, codes.data(), VW * sizeof(float), cudaMemcpyHostToDevice));
    set_parameters(initial_parameters(cfg, seed));
  }

  ~GptModel() {
    workspaces_.clear();
    for (cudaEvent_t e : opt_marks_) cudaEventDestroy(e);
    detach_nccl();
    if (stream_ && owns_stream_) cudaStreamDestroy(stream_);
  }

  const mb_gpt_config& config() const { return cfg_; }
  size_t count() const { return layout_.count(); }
  cudaStream_t stream() const { return stream_; }

  void set_parameters(const std::vector<float>& values) { set_parameters(values.data(), values.size()); }
  void set_parameters(const float* values, size_t n) {
    require(n == count(), "parameter count does not match GPT configuration");
    for (size_t i = 0; i < n; ++i) require(std::isfinite(values[i]), "parameters must contain only finite values",
                                           MB_ERR_NONFINITE);
    MB_CUDA(cudaSetDevice(device_));
    MB_CUDA(cudaMemcpyAsync(w_, values, n * sizeof(float), cudaMemcpyHostToDevice, stream_));
    MB_CUDA(cudaMemsetAsync(m_, 0, n * sizeof(float), stream_));
    MB_CUDA(cudaMemsetAsync(v_, 0, n * sizeof(float), stream_));
    OptimizerState st{0.f, 0.f, 0.9f, 0.999f, 1e-8f, 1.0f, 1.0f, 0};
    MB_CUDA(cudaMemcpyAsync(opt_, &st, sizeof(st), cudaMemcpyHostToDevice, stream_));
    MB_CUDA(cudaStreamSynchronize(stream_));
  }

  void get_parameters(float* out, size_t n) {
    require(n == count(), "parameter count does not match GPT configuration");
    MB_CUDA(cudaSetDevice(device_));
    MB_CUDA(cudaMemcpyAsync(out, w_, n * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    MB_CUDA(cudaStreamSynchronize(stream_));
    for (size_t i = 0; i < n; ++i) require(std::isfinite(out[i]), "parameters must contain only finite values",
                                           MB_ERR_NONFINITE);
  }

  // ---- host-batch entry points (validate on the host like the reference)
  double train_step(const uint32_t* in, const uint32_t* tgt, size_t rows, size_t seq, const mb_adamw* opt) {
    validate_optimizer(*opt);
    validate_batch(cfg_, in, tgt, rows, seq, data_parallel());
    MB_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(rows, seq);
    MB_CUDA(cudaMemcpyAsync(ws.tokens, in, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    MB_CUDA(cudaMemcpyAsync(ws.targets, tgt, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    gradient_pass(ws);
    update(ws, opt);
    return read_loss(ws);
  }

  double loss_and_gradient(const uint32_t* in, const uint32_t* tgt, size_t rows, size_t seq, float* grad,
                           size_t n) {
    require(n == count(), "gradient length does not match GPT configuration");
    validate_batch(cfg_, in, tgt, rows, seq, data_parallel());
    MB_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(rows, seq);
    MB_CUDA(cudaMemcpyAsync(ws.tokens, in, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    MB_CUDA(cudaMemcpyAsync(ws.targets, tgt, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    gradient_pass(ws);
    const double loss = read_loss(ws);
    MB_CUDA(cudaMemcpyAsync(grad, grad_, n * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    MB_CUDA(cudaStreamSynchronize(stream_));
    for (size_t i = 0; i < n; ++i) require(std::isfinite(grad[i]), "gradients must contain only finite values",
                                           MB_ERR_NONFINITE);
    return loss;
  }

  double cross_entropy(const uint32_t* in, const uint32_t* tgt, size_t rows, size_t seq) {
    validate_batch(cfg_, in, tgt, rows, seq);
    MB_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(rows, seq);
    MB_CUDA(cudaMemcpyAsync(ws.tokens, in, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    MB_CUDA(cudaMemcpyAsync(ws.targets, tgt, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    enqueue_forward(ws, true, true);
    launch_loss(ws);
    return read_loss(ws);
  }

  void logits(const uint32_t* in, size_t rows, size_t seq, float* out, bool hidden) {
    validate_batch(cfg_, in, nullptr, rows, seq);
    MB_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(rows, seq);
    MB_CUDA(cudaMemcpyAsync(ws.tokens, in, rows * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    enqueue_forward(ws, false, false);
    const size_t n = rows * (hidden ? cfg_.width : cfg_.vocab_size);
    MB_CUDA(cudaMemcpyAsync(out, hidden ? ws.x[cfg_.layers] : ws.logits, n * sizeof(float), cudaMemcpyDeviceToHost,
                            stream_));
    MB_CUDA(cudaStreamSynchronize(stream_));
    for (size_t i = 0; i < n; ++i) require(std::isfinite(out[i]), "logits must contain only finite values",
                                           MB_ERR_NONFINITE);
  }

  void token_embeddings(float* out, size_t n) {
    const size_t VW = (size_t)cfg_.vocab_size * cfg_.width;
    require(n == VW, "token embedding buffer must hold vocab * width floats");
    MB_CUDA(cudaSetDevice(device_));
    if (!table()) launch_embedding_forward();
    MB_CUDA(cudaMemcpyAsync(out, final_embedding(), VW * sizeof(float), cudaMemcpyDeviceToHost, stream_));
    MB_CUDA(cudaStreamSynchronize(stream_));
  }

  // ---- device-batch entry point (no host synchronisation)
  void train_step_device(const uint32_t* d_in, const uint32_t* d_tgt, size_t rows, size_t seq, const mb_adamw* opt,
                         double* d_loss) {
    validate_optimizer(*opt);
    require(seq >= 1 && seq <= cfg_.context && rows >= 1 && rows % seq == 0 && rows <= 131072,
            "tokens must form a nonempty batch of equal sequences within context and 131072 rows");
    MB_CUDA(cudaSetDevice(device_));
    Workspace& ws = workspace(rows, seq);
    MB_CUDA(cudaMemcpyAsync(ws.tokens, d_in, rows * sizeof(uint32_t), cudaMemcpyDeviceToDevice, stream_));
    MB_CUDA(cudaMemcpyAsync(ws.targets, d_tgt, rows * sizeof(uint32_t), cudaMemcpyDeviceToDevice, stream_));
    gradient_pass(ws);
    update(ws, opt);
    if (d_loss != nullptr)
      MB_CUDA(cudaMemcpyAsync(d_loss, ws.loss, sizeof(double), cudaMemcpyDeviceToDevice, stream_));
    last_ = &ws;
  }

  void check() {
    MB_CUDA(cudaSetDevice(device_));
    MB_CUDA(cudaStreamSynchronize(stream_));
    int tc_err = 0;
    MB_CUDA(cudaMemcpy(&tc_err, tc_err_, sizeof(int), cudaMemcpyDeviceToHost));
    if (tc_err) {
      MB_CUDA(cudaMemset(tc_err_, 0, sizeof(int)));
      throw Error(MB_ERR_CUDA, "a tensor-core completion wait timed out; the last step's results are invalid");
    }
    for (auto& w : workspaces_) {
      int flags = 0;
      MB_CUDA(cudaMemcpy(&flags, w->flags, sizeof(int), cudaMemcpyDeviceToHost));
      if (flags) {
        MB_CUDA(cudaMemset(w->flags, 0, sizeof(int)));
        if (flags & 1) throw Error(MB_ERR_INVALID, "token ID is outside the vocabulary");
        if (flags & 2) throw Error(MB_ERR_INVALID, "target ID is outside the vocabulary");
        if (flags & 4) throw Error(MB_ERR_INVALID, "batch must contain at least one supervised target");
      }
    }
  }

  // src/gpt/gpu.rs:1779-1791: how many batch-shape workspaces stay cached
  // (1..3); lowering it frees the oldest ones at once.
  void set_workspace_capacity(size_t capacity) {
    require(capacity >= 1 && capacity <= 3, "workspace capacity must be in 1..3");
    capacity_ = capacity;
    if (workspaces_.size() > capacity_) MB_CUDA(cudaStreamSynchronize(stream_));
    while (workspaces_.size() > capacity_) {
      if (last_ == workspaces_.front().get()) last_ = nullptr;
      workspaces_.pop_front();
    }
  }
  size_t workspace_capacity() const { return capacity_; }

  void set_timing(bool on) {
    if (on == timing_) return;
    timing_ = on;
    for (auto& w : workspaces_) {  // recapture with or without boundary events
      if (w->graph) cudaGraphExecDestroy(w->graph);
      w->graph = nullptr;
    }
  }

  // Per-launch durations (ms) of the most recent training step: the graph's
  // kernels followed by the optimizer kernels.
  std::vector<std::pair<std::string, float>> kernel_times() {
    MB_CUDA(cudaStreamSynchronize(stream_));
    std::vector<std::pair<std::string, float>> out;
    require(timing_ && last_ != nullptr && last_->marks.size() > 1, "no timed step has run");
    for (size_t i = 0; i + 1 < last_->marks.size(); ++i) {
      float ms = 0.f;
      MB_CUDA(cudaEventElapsedTime(&ms, last_->marks[i], last_->marks[i + 1]));
      out.emplace_back(last_->mark_names[i], ms);
    }
    for (size_t i = 0; i + 1 < opt_marks_.size(); ++i) {
      float ms = 0.f;
      MB_CUDA(cudaEventElapsedTime(&ms, opt_marks_[i], opt_marks_[i + 1]));
      out.emplace_back(opt_names_[i], ms);
    }
    return out;
  }

  size_t allocated_bytes() const {
    size_t b = mem_.bytes();
    for (auto& w : workspaces_) b += w->mem.bytes();
    return b;
  }

  // K chunk of the embedding-gradient GEMM (K = 2 rows): one CTA per SM
  // (the GEMM's shared-memory pipeline fills an SM) over its V x W output
  // tiles, chunks a multiple of 32 and at least 256.
  int embedding_k_chunk(int rows) const {
    const int K = 2 * rows;
    const int tiles = ((cfg_.vocab_size + 127) / 128) * ((cfg_.width + 63) / 64);
    const int chunks = std::max(1, sms_ / tiles);
    const int kc = ((K + chunks - 1) / chunks + 31) / 32 * 32;
    return std::max(256, kc);
  }

  size_t step_launches(int rows) const {
    // count + embedding fwd + per block (qkv, attention, post) forward + head
    // (norm, GEMM, loss, GEMM, norm adjoint) + loss + per block (post,
    // attention, qkv) backward + embedding-gradient GEMM (+ its chunk sum) +
    // group reduce + embedding bwd + optimizer advance + AdamW
    // (a table embedding has no embedding mesh forward or backward)
    const size_t L = cfg_.layers, mesh = table() ? 0 : 1;
    // data parallelism adds finish_supervised to the count (NCCL calls are not counted)
    return 1 + (data_parallel() ? 1 : 0) + mesh + L * (2 + attention_->forward_launches()) + 5 + 1 + L * (2 + attention_->backward_launches()) +
           gemm_launches(2 * rows, embedding_k_chunk(rows)) + 1 + mesh + mesh + 2;
  }

  // ---- data parallelism
  void attach_nccl(const uint8_t* id, int rank, int world) {
    require(world >= 1 && rank >= 0 && rank < world, "invalid rank / world size");
    detach_nccl();
    MB_CUDA(cudaSetDevice(device_));
    ncclUniqueId uid;
    static_assert(sizeof(uid) == MB_NCCL_ID_BYTES, "NCCL unique id size");
    std::memcpy(&uid, id, sizeof(uid));
    nccl_check(nccl().comm_init_rank(&comm_, world, uid, rank), "ncclCommInitRank");
    owns_comm_ = true;
    world_ = world;
  }
  // A communicator the caller created (and keeps ownership of) for this
  // model's device; world is its size, checked against NCCL's own count.
  void attach_nccl_comm(ncclComm_t comm, int world) {
    require(comm != nullptr && world >= 1, "communicator must not be null and world size must be positive");
    detach_nccl();
    MB_CUDA(cudaSetDevice(device_));
    if (nccl().comm_count != nullptr) {
      int n = 0;
      nccl_check(nccl().comm_count(comm, &n), "ncclCommCount");
      require(n == world, "world size does not match the communicator");
    }
    comm_ = comm;
    owns_comm_ = false;
    world_ = world;
  }
  void detach_nccl() {
    if (comm_ != nullptr) {
      cudaStreamSynchronize(stream_);
      if (owns_comm_) nccl().comm_destroy(comm_);
      comm_ = nullptr;
    }
    owns_comm_ = false;
    world_ = 1;
  }
  bool data_parallel() const { return comm_ != nullptr && world_ > 1; }

 private:
  Workspace& workspace(size_t rows, size_t seq) {
    for (size_t i = 0; i < workspaces_.size(); ++i) {
      if (workspaces_[i]->rows == (int)rows && workspaces_[i]->seq == (int)seq) {
        auto w = std::move(workspaces_[i]);
        workspaces_.erase(workspaces_.begin() + i);
        workspaces_.push_back(std::move(w));
        return *workspaces_.back();
      }
    }
    if (workspaces_.size() >= capacity_) {
      MB_CUDA(cudaStreamSynchronize(stream_));
      if (last_ == workspaces_.front().get()) last_ = nullptr;
      workspaces_.pop_front();
    }
    workspaces_.push_back(build_workspace((int)rows, (int)seq));
    return *workspaces_.back();
  }

  Dims dims(const Workspace& ws) const {
    Dims d;
    d.rows = ws.rows;
    d.sequence = ws.seq;
    d.heads = cfg_.heads;
    d.head_width = cfg_.width / cfg_.heads;
    d.vocab = cfg_.vocab_size;
    d.attn_depth = cfg_.attention_mesh_depth;
    d.ffn_depth = cfg_.ffn_mesh_depth;
    d.connectivity = cfg_.connectivity;
    d.log2w = 31 - __builtin_clz(cfg_.width);
    return d;
  }

  std::unique_ptr<Workspace> build_workspace(int rows, int seq) {
    auto ws = std::make_unique<Workspace>();
    ws->rows = rows;
    ws->seq = seq;
    const int L = cfg_.layers, H = cfg_.heads, W = cfg_.width, V = cfg_.vocab_size;
    const size_t NW = (size_t)rows * W;
    DeviceArena& a = ws->mem;
    for (int b = 0; b <= L; ++b) ws->x.push_back(a.alloc<float>(NW));
    for (int b = 0; b < L; ++b) {
      ws->q.push_back(a.alloc<float>(NW));
      ws->k.push_back(a.alloc<float>(NW));
      ws->v.push_back(a.alloc<float>(NW));
      ws->o.push_back(a.alloc<float>(NW));
      ws->xm.push_back(a.alloc<float>(NW));
      ws->lse.push_back(a.alloc<float>((size_t)H * rows));
    }
    ws->nf = a.alloc<float>(2 * NW);
    ws->g = ws->nf + NW;
    ws->dlog = a.alloc<float>((size_t)2 * rows * V);
    ws->indicator = ws->dlog + (size_t)rows * V;
    ws->logits = a.alloc<float>((size_t)rows * V);
    ws->head_inv = a.alloc<float>(rows);
    ws->head_dn = a.alloc<float>((size_t)rows * W);
    ws->loss_rows = a.alloc<float>(rows);
    ws->dO = a.alloc<float>(NW);
    ws->dvx = a.alloc<float>(NW);
    ws->dxm = a.alloc<float>(NW);
    ws->delta = a.alloc<float>((size_t)H * rows);
    ws->dq = a.alloc<float>(NW);
    ws->dk = a.alloc<float>(NW);
    ws->emb_k_chunk = embedding_k_chunk(rows);
    ws->emb_partial = a.alloc<float>(std::max<size_t>(1, gemm_partial_floats(V, W, 2 * rows, ws->emb_k_chunk)));
    ws->dE = a.alloc<float>((size_t)V * W);
    ws->att_scratch = a.alloc<float>(attention_->scratch_floats(rows, H, cfg_.layers));
    if (!table()) ws->emb_mesh_partial = a.alloc<float>((size_t)V * layout_.groups[layout_.embedding].size);
    ws->tokens = a.alloc<uint32_t>(rows);
    ws->targets = a.alloc<uint32_t>(rows);
    ws->stats = a.alloc<float>(4);
    ws->step_flags = a.alloc<int>(1);
    ws->flags = a.alloc<int>(1);
    ws->loss = a.alloc<double>(1);
    MB_CUDA(cudaMemset(ws->flags, 0, sizeof(int)));
    MB_CUDA(cudaMemset(ws->step_flags, 0, sizeof(int)));
    // RoPE table [seq][hd/2] of (cos, sin), angle = pos / 10000^(i / (hd/2)),
    // evaluated in f64 (src/gpt/gpu.rs:175-208 evaluates it in f32).
    const int half = W / H / 2;
    std::vector<float2> cs((size_t)seq * half);
    for (int p = 0; p < seq; ++p)
      for (int i = 0; i < half; ++i) {
        const double ang = (double)p / std::pow(10000.0, (double)i / half);
        cs[(size_t)p * half + i] = make_float2((float)std::cos(ang), (float)std::sin(ang));
      }
    ws->rope = a.alloc<float2>(cs.size());
    MB_CUDA(cudaMemcpy(ws->rope, cs.data(), cs.size() * sizeof(float2), cudaMemcpyHostToDevice));
    // Persistent grids: every SM busy, at most one tile per CTA.
    auto grid = [&](int tile_rows, int occ) {
      const int tiles = (rows + tile_rows - 1) / tile_rows;
      return std::max(1, std::min(tiles, sms_ * occ));
    };
    ws->grid_qf = grid(blocks_->tile_rows, blocks_->occ_qf);
    ws->grid_pf = grid(blocks_->tile_rows_post, blocks_->occ_pf);
    ws->grid_pb = grid(blocks_->tile_rows_bwd, blocks_->occ_pb);
    ws->grid_qb = grid(blocks_->tile_rows_bwd, blocks_->occ_qb);
    const int slots_pb = ws->grid_pb * blocks_->row_lanes;
    const int slots_qb = ws->grid_qb * blocks_->row_lanes;
    std::vector<ReduceJob> jobs;
    ws->part.assign(layout_.groups.size(), nullptr);
    for (size_t gi = 0; gi < layout_.groups.size(); ++gi) {
      const Group& g = layout_.groups[gi];
      int slots;
      if ((int)gi == layout_.embedding && table()) {
        continue;  // the embedding reduction writes the table's gradient directly
      } else if ((int)gi == layout_.embedding) {
        ws->part[gi] = ws->emb_mesh_partial;
        slots = V;
      } else {
        const int within = (int)((gi - 1) % 5);  // q, k, v, o, ffn
        slots = within < 3 ? slots_qb : slots_pb;
        ws->part[gi] = a.alloc<float>((size_t)slots * g.size);
      }
      jobs.push_back(ReduceJob{ws->part[gi], grad_ + g.offset, slots, (int)g.size});
      ws->max_job = std::max(ws->max_job, (int)g.size);
    }
    ws->njobs = (int)jobs.size();
    ws->d_jobs = a.alloc<ReduceJob>(jobs.size());
    MB_CUDA(cudaMemcpy(ws->d_jobs, jobs.data(), jobs.size() * sizeof(ReduceJob), cudaMemcpyHostToDevice));
    return ws;
  }

  const float* group(int gi) const { return w_ + layout_.groups[gi].offset; }

  void launch_embedding_forward() {
    const int W = cfg_.width, V = cfg_.vocab_size;
    embedding_forward<<<V, W, W * sizeof(float), stream_>>>(W, V, cfg_.attention_mesh_depth, cfg_.connectivity,
                                                            31 - __builtin_clz(W), group(layout_.embedding),
                                                            emb_acts_, et_);
  }

  // A table embedding is the parameter group itself; a mesh embedding is the
  // last layer of the embedding mesh over the token codes.
  bool table() const { return cfg_.embedding == 1; }
  const float* final_embedding() const {
    if (table()) return group(layout_.embedding);
    return emb_acts_ + (size_t)cfg_.vocab_size * cfg_.width * cfg_.attention_mesh_depth;
  }

  // with_targets: the head also computes the cross-entropy and its adjoint;
  // count: the batch's supervised count is taken here (single-rank graphs and
  // the rank-local evaluation), else count_and_exchange has taken it.
  void enqueue_forward(Workspace& ws, bool with_targets, bool count) {
    const Dims d = dims(ws);
    attention_->scratch = ws.att_scratch;
    const int L = cfg_.layers, W = cfg_.width, V = cfg_.vocab_size, H = cfg_.heads;
    if (with_targets && count) {
      mark("count_supervised");
      count_supervised<<<1, 1024, 0, stream_>>>(ws.rows, V, ws.tokens, ws.targets, ws.stats, ws.step_flags,
                                                ws.flags, 0);
    }
    mark("embedding_forward");
    if (!table()) launch_embedding_forward();
    for (int b = 0; b < L; ++b) {
      const BlockGroups& bg = layout_.blocks[b];
      mark("qkv_forward");
      blocks_->qkv_forward(stream_, ws.grid_qf, d, ws.x[b], b == 0 ? ws.tokens : nullptr, final_embedding(),
                           b == 0 ? ws.x[0] : nullptr, group(bg.query), group(bg.key), group(bg.value), ws.rope,
                           ws.q[b], ws.k[b], ws.v[b]);
      mark("attention_forward");
      attention_->layer = b;
      attention_->forward(stream_, ws.rows, W, ws.seq, H, W / H, ws.q[b], ws.k[b], ws.v[b], ws.o[b], ws.lse[b]);
      mark("post_forward");
      blocks_->post_forward(stream_, ws.grid_pf, d, ws.o[b], ws.v[b], ws.x[b], group(bg.projection), group(bg.ffn),
                            ws.xm[b], ws.x[b + 1]);
    }
    // Head: final RMSNorm, logits = nf E^T on the tensor cores; in training
    // also the cross-entropy, dn = dlogits E and the RMSNorm adjoint into g.
    mark("head_forward_backward");
    const int hgrid = (ws.rows + kHeadWarps - 1) / kHeadWarps;
    const float* E = final_embedding();
    head_norm<<<hgrid, kHeadWarps * 32, 0, stream_>>>(ws.rows, W, ws.x[L], ws.nf, ws.head_inv);
    launch_gemm({ws.nf, W, false}, {E, W, false}, ws.logits, V, ws.rows, V, W, 0, nullptr, tc_err_, stream_);
    if (with_targets) {
      head_loss<<<hgrid, kHeadWarps * 32, 0, stream_>>>(ws.rows, V, ws.logits, ws.targets, ws.stats,
                                                          ws.tokens, ws.loss_rows, ws.dlog, ws.indicator);
      launch_gemm({ws.dlog, V, false}, {E, W, true}, ws.head_dn, W, ws.rows, W, V, 0, nullptr, tc_err_, stream_);
      head_norm_backward<<<hgrid, kHeadWarps * 32, 0, stream_>>>(ws.rows, W, ws.nf, ws.head_inv, ws.head_dn, ws.g);
    }
    MB_CUDA(cudaGetLastError());
  }

  void launch_loss(Workspace& ws) {
    mark("loss_reduce");
    loss_reduce<<<1, 1024, 0, stream_>>>(ws.rows, ws.loss_rows, ws.stats, ws.loss);
  }

  void enqueue_backward(Workspace& ws) {
    const Dims d = dims(ws);
    attention_->scratch = ws.att_scratch;
    const int L = cfg_.layers, W = cfg_.width, V = cfg_.vocab_size, H = cfg_.heads;
    for (int b = L - 1; b >= 0; --b) {
      const BlockGroups& bg = layout_.blocks[b];
      mark("post_backward");
      blocks_->post_backward(stream_, ws.grid_pb, d, ws.g, ws.xm[b], ws.o[b], ws.v[b], group(bg.projection),
                             group(bg.ffn), ws.dO, ws.dvx, ws.dxm, ws.delta, ws.part[bg.projection],
                             ws.part[bg.ffn]);
      mark("attention_backward_dkdv");
      attention_->layer = b;
      attention_->backward_dkdv(stream_, ws.rows, W, ws.seq, H, W / H, ws.q[b], ws.k[b], ws.v[b], ws.dO, ws.lse[b],
                                ws.delta, ws.dvx, ws.dk, ws.dvx);  // dV added into the XSA term in place
      mark("attention_backward_dq");
      attention_->backward_dq(stream_, ws.rows, W, ws.seq, H, W / H, ws.q[b], ws.k[b], ws.v[b], ws.dO, ws.lse[b],
                              ws.delta, ws.dq);
      mark("qkv_backward");
      blocks_->qkv_backward(stream_, ws.grid_qb, d, ws.dq, ws.dk, ws.dvx, ws.x[b], ws.dxm, group(bg.query),
                            group(bg.key), group(bg.value), ws.rope, ws.g, ws.part[bg.query], ws.part[bg.key],
                            ws.part[bg.value]);
    }
    // Tied embedding: head and input-lookup contributions in one contraction
    // over K = 2 rows, dE[t][c] = sum_r dlogits[r][t] nf[r][c]
    // + sum_r [tok_r == t] dx0[r][c], split over K chunks summed in order.
    mark("embedding_gradient");
    launch_gemm({ws.dlog, V, true}, {ws.nf, W, true},
                table() ? grad_ + layout_.groups[layout_.embedding].offset : ws.dE, W, V, W, 2 * ws.rows,
                ws.emb_k_chunk, ws.emb_partial, tc_err_, stream_);
    mark("embedding_backward");
    if (!table())
      embedding_backward<<<V, W, W * sizeof(float), stream_>>>(W, V, cfg_.attention_mesh_depth, cfg_.connectivity,
                                                               31 - __builtin_clz(W), group(layout_.embedding),
                                                               emb_acts_, ws.dE, ws.emb_mesh_partial);
    mark("reduce_partials");
    reduce_partials<<<dim3(std::max(1, (ws.max_job / 4 + 255) / 256), ws.njobs), 256, 0, stream_>>>(ws.d_jobs,
                                                                                               ws.njobs);
    mark("end");
    MB_CUDA(cudaGetLastError());
  }

  // One gradient evaluation.  Single rank: the captured graph (count,
  // forward, loss, backward).  Data parallel (the reference's loss is the mean
  // over the supervised rows of the whole batch, src/gpt/gpu.rs:2296-2313):
  // every rank's supervised count and flags are summed first, so each rank
  // divides its cross-entropy adjoint by the global count; the graph then
  // yields this rank's share of the gradient and of the loss, and one sum
  // over ranks of each gives the global mean loss and its exact gradient for
  // any split of the supervised targets.
  void gradient_pass(Workspace& ws) {
    const bool dp = data_parallel();
    if (dp) {
      count_supervised<<<1, 1024, 0, stream_>>>(ws.rows, cfg_.vocab_size, ws.tokens, ws.targets, ws.stats,
                                                ws.step_flags, ws.flags, 1);
      MB_CUDA(cudaGetLastError());
      nccl_check(nccl().all_reduce(ws.stats, ws.stats, 4, ncclFloat32, ncclSum, comm_, stream_), "ncclAllReduce");
      finish_supervised<<<1, 1, 0, stream_>>>(ws.stats, ws.step_flags, ws.flags);
      MB_CUDA(cudaGetLastError());
    }
    run_gradient_graph(ws, dp);
    if (dp) {
      nccl_check(nccl().all_reduce(grad_, grad_, count(), ncclFloat32, ncclSum, comm_, stream_), "ncclAllReduce");
      nccl_check(nccl().all_reduce(ws.loss, ws.loss, 1, ncclFloat64, ncclSum, comm_, stream_), "ncclAllReduce");
    }
  }

  void run_gradient_graph(Workspace& ws, bool dp) {
    if (ws.graph != nullptr && ws.graph_dp != dp) {
      cudaGraphExecDestroy(ws.graph);
      ws.graph = nullptr;
    }
    if (ws.graph == nullptr) {
      ws.graph_dp = dp;
      cudaGraph_t g = nullptr;
      for (cudaEvent_t e : ws.marks) cudaEventDestroy(e);
      ws.marks.clear();
      ws.mark_names.clear();
      MB_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
      capturing_ = &ws;
      try {
        enqueue_forward(ws, true, !dp);
        launch_loss(ws);
        enqueue_backward(ws);
      } catch (...) {
        capturing_ = nullptr;
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      capturing_ = nullptr;
      MB_CUDA(cudaStreamEndCapture(stream_, &g));
      cudaError_t e = cudaGraphInstantiate(&ws.graph, g, 0);
      cudaGraphDestroy(g);
      MB_CUDA(e);
    }
    MB_CUDA(cudaGraphLaunch(ws.graph, stream_));
    last_ = &ws;
  }

  void update(Workspace& ws, const mb_adamw* opt) {
    const size_t P = count();
    auto omark = [&](size_t i, const char* name) {
      if (!timing_) return;
      if (opt_marks_.size() <= i) {
        cudaEvent_t e;
        MB_CUDA(cudaEventCreate(&e));
        opt_marks_.push_back(e);
        opt_names_.push_back(name);
      }
      MB_CUDA(cudaEventRecord(opt_marks_[i], stream_));
    };
    OptimizerState st{opt->learning_rate, opt->weight_decay, opt->beta1, opt->beta2, opt->epsilon, 0.f, 0.f, 0};
    omark(0, "optimizer_set");
    optimizer_set<<<1, 1, 0, stream_>>>(opt_, st, ws.step_flags);
    const int threads = 256;
    const int blocks = std::min((int)((P + threads - 1) / threads), sms_ * 8);
    omark(1, "adamw");
    adamw<<<blocks, threads, 0, stream_>>>((int)P, opt_, grad_, w_, m_, v_, ws.step_flags);
    omark(2, "end");
    MB_CUDA(cudaGetLastError());
  }

  // The step's loss; with data parallelism also the step's flags, since
  // only the device sees whether the ranks' batches together hold a
  // supervised target (a step that holds none updated nothing).
  double read_loss(Workspace& ws) {
    double loss = 0.0;
    int flags = 0;
    MB_CUDA(cudaMemcpyAsync(&loss, ws.loss, sizeof(double), cudaMemcpyDeviceToHost, stream_));
    if (ws.graph_dp) MB_CUDA(cudaMemcpyAsync(&flags, ws.step_flags, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    MB_CUDA(cudaStreamSynchronize(stream_));
    if (flags != 0) {
      MB_CUDA(cudaMemset(ws.flags, 0, sizeof(int)));
      require(!(flags & 4), "batch must contain at least one supervised target over all ranks");
      require(false, "a rank's batch holds a token or target outside the vocabulary");
    }
    require(std::isfinite(loss), "cross-entropy must contain only finite values", MB_ERR_NONFINITE);
    return loss;
  }

  mb_gpt_config cfg_;
  int device_ = 0, sms_ = 1;
  Layout layout_;
  cudaStream_t stream_ = nullptr;
  bool owns_stream_ = false;
  DeviceArena mem_;
  std::unique_ptr<BlockOps> blocks_;
  std::unique_ptr<AttentionOps> attention_;
  float *w_ = nullptr, *m_ = nullptr, *v_ = nullptr, *grad_ = nullptr, *emb_acts_ = nullptr, *et_ = nullptr;
  OptimizerState* opt_ = nullptr;
  int* tc_err_ = nullptr;
  std::deque<std::unique_ptr<Workspace>> workspaces_;
  size_t capacity_ = 1;  // the reference's default (src/gpt/gpu.rs:1767)
  Workspace* last_ = nullptr;
  ncclComm_t comm_ = nullptr;
  bool owns_comm_ = false;
  int world_ = 1;
  bool timing_ = false;
  Workspace* capturing_ = nullptr;
  std::vector<cudaEvent_t> opt_marks_;
  std::vector<std::string> opt_names_;

  // Records a boundary event before the next launch (timing mode, inside
  // graph capture only).
  void mark(const char* name) {
    if (!timing_ || capturing_ == nullptr) return;
    Workspace& ws = *capturing_;
    cudaEvent_t e;
    MB_CUDA(cudaEventCreate(&e));
    ws.marks.push_back(e);
    ws.mark_names.push_back(name);
    MB_CUDA(cudaEventRecordWithFlags(e, stream_, cudaEventRecordExternal));
  }
};

}  // namespace mb

// ================================================================== C ABI
using mb::Error;

struct mb_gpt {
  std::unique_ptr<mb::GptModel> model;
};

// A device and one stream that models created in it share
// (mb_ctx_create; src/gpt/gpu.rs:1718-1736 takes an Arc<CudaContext>).
struct mb_ctx {
  int device;
  cudaStream_t stream;
};

namespace {
thread_local std::string g_error;
thread_local int g_code = MB_OK;

using mb::guarded;
using mb::need;

mb::GptModel& model_of(mb_gpt* m) {
  mb::require(m != nullptr && m->model != nullptr, "model handle is null");
  return *m->model;
}
}  // namespace

namespace mb {
void set_last_error(int code, const char* message) {
  g_code = code;
  g_error = message;
}
}  // namespace mb

extern "C" {

int mb_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    std::strncpy(buf, g_error.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return g_code;
}

int mb_version(int* major, int* minor) {
  return guarded([&] {
    need(major, "major");
    need(minor, "minor");
    *major = 0;
    *minor = 1;
  });
}

int mb_device_count(int* count) {
  return guarded([&] {
    need(count, "count");
    MB_CUDA(cudaGetDeviceCount(count));
  });
}

int mb_gpt_validate(const mb_gpt_config* c) {
  return guarded([&] {
    need(c, "config");
    mb::validate_kernel_shapes(*c);
  });
}

int mb_gpt_parameter_count(const mb_gpt_config* c, size_t* count) {
  return guarded([&] {
    need(c, "config");
    need(count, "count");
    *count = mb::make_layout(*c).count();
  });
}

int mb_gpt_initial_parameters(const mb_gpt_config* c, uint64_t seed, float* out, size_t count) {
  return guarded([&] {
    need(c, "config");
    need(out, "out");
    std::vector<float> p = mb::initial_parameters(*c, seed);
    mb::require(count == p.size(), "parameter count does not match GPT configuration");
    std::memcpy(out, p.data(), p.size() * sizeof(float));
  });
}

int mb_gpt_token_codes(const mb_gpt_config* c, float* out, size_t count) {
  return guarded([&] {
    need(c, "config");
    need(out, "out");
    std::vector<float> codes = mb::token_codes(*c);
    mb::require(count == codes.size(), "token code buffer must hold vocab * width floats");
    std::memcpy(out, codes.data(), codes.size() * sizeof(float));
  });
}

int mb_gpt_create(int device, const mb_gpt_config* c, uint64_t seed, mb_gpt** out) {
  return guarded([&] {
    need(c, "config");
    need(out, "model");
    *out = nullptr;
    auto h = std::make_unique<mb_gpt>();
    h->model = std::make_unique<mb::GptModel>(device, *c, seed);
    *out = h.release();
  });
}

int mb_ctx_create(int device, mb_ctx** out) {
  return guarded([&] {
    need(out, "context");
    *out = nullptr;
    int count = 0;
    MB_CUDA(cudaGetDeviceCount(&count));
    mb::require(device >= 0 && device < count, "CUDA device index out of range");
    MB_CUDA(cudaSetDevice(device));
    auto c = std::make_unique<mb_ctx>();
    c->device = device;
    MB_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    *out = c.release();
  });
}

int mb_ctx_destroy(mb_ctx* ctx) {
  return guarded([&] {
    if (ctx == nullptr) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
  });
}

int mb_ctx_stream(mb_ctx* ctx, void** stream) {
  return guarded([&] {
    need(ctx, "context");
    need(stream, "stream");
    *stream = (void*)ctx->stream;
  });
}

int mb_gpt_create_in(mb_ctx* ctx, const mb_gpt_config* c, uint64_t seed, mb_gpt** out) {
  return guarded([&] {
    need(ctx, "context");
    need(c, "config");
    need(out, "model");
    *out = nullptr;
    auto h = std::make_unique<mb_gpt>();
    h->model = std::make_unique<mb::GptModel>(ctx->device, *c, seed, ctx->stream);
    *out = h.release();
  });
}

int mb_gpt_destroy(mb_gpt* m) {
  return guarded([&] { delete m; });
}

int mb_gpt_get_config(const mb_gpt* m, mb_gpt_config* c) {
  return guarded([&] {
    need(m, "model");
    need(c, "config");
    *c = m->model->config();
  });
}

int mb_gpt_get_parameters(mb_gpt* m, float* out, size_t count) {
  return guarded([&] {
    need(out, "out");
    model_of(m).get_parameters(out, count);
  });
}

int mb_gpt_set_parameters(mb_gpt* m, const float* values, size_t count) {
  return guarded([&] {
    need(values, "values");
    model_of(m).set_parameters(values, count);
  });
}

int mb_gpt_logits(mb_gpt* m, const uint32_t* tokens, size_t rows, size_t sequence, float* out) {
  return guarded([&] {
    need(out, "out");
    model_of(m).logits(tokens, rows, sequence, out, false);
  });
}

int mb_gpt_hidden_states(mb_gpt* m, const uint32_t* tokens, size_t rows, size_t sequence, float* out) {
  return guarded([&] {
    need(out, "out");
    model_of(m).logits(tokens, rows, sequence, out, true);
  });
}

int mb_gpt_token_embeddings(mb_gpt* m, float* out, size_t count) {
  return guarded([&] {
    need(out, "out");
    model_of(m).token_embeddings(out, count);
  });
}

int mb_gpt_cross_entropy(mb_gpt* m, const uint32_t* in, const uint32_t* tgt, size_t rows, size_t sequence,
                         double* loss) {
  return guarded([&] {
    need(loss, "loss");
    need(tgt, "targets");
    *loss = model_of(m).cross_entropy(in, tgt, rows, sequence);
  });
}

int mb_gpt_loss_and_gradient(mb_gpt* m, const uint32_t* in, const uint32_t* tgt, size_t rows, size_t sequence,
                             double* loss, float* gradient, size_t count) {
  return guarded([&] {
    need(loss, "loss");
    need(gradient, "gradient");
    need(tgt, "targets");
    *loss = model_of(m).loss_and_gradient(in, tgt, rows, sequence, gradient, count);
  });
}

int mb_gpt_train_step(mb_gpt* m, const uint32_t* in, const uint32_t* tgt, size_t rows, size_t sequence,
                      const mb_adamw* opt, double* loss) {
  return guarded([&] {
    need(opt, "optimizer");
    need(tgt, "targets");
    const double l = model_of(m).train_step(in, tgt, rows, sequence, opt);
    if (loss != nullptr) *loss = l;
  });
}

int mb_gpt_train_step_device(mb_gpt* m, const uint32_t* d_in, const uint32_t* d_tgt, size_t rows, size_t sequence,
                             const mb_adamw* opt, double* d_loss) {
  return guarded([&] {
    need(opt, "optimizer");
    need(d_in, "inputs");
    need(d_tgt, "targets");
    model_of(m).train_step_device(d_in, d_tgt, rows, sequence, opt, d_loss);
  });
}

int mb_gpt_check(mb_gpt* m) {
  return guarded([&] { model_of(m).check(); });
}

int mb_gpt_stream(mb_gpt* m, void** stream) {
  return guarded([&] {
    need(stream, "stream");
    *stream = (void*)model_of(m).stream();
  });
}

int mb_gpt_allocated_device_bytes(mb_gpt* m, size_t* bytes) {
  return guarded([&] {
    need(bytes, "bytes");
    *bytes = model_of(m).allocated_bytes();
  });
}

int mb_gpt_step_launches(mb_gpt* m, size_t rows, size_t sequence, size_t* launches) {
  return guarded([&] {
    need(launches, "launches");
    (void)sequence;
    mb::require(rows >= 1 && rows <= (size_t)INT32_MAX / 2, "rows out of range");
    *launches = model_of(m).step_launches((int)rows);
  });
}

int mb_gpt_set_workspace_capacity(mb_gpt* m, size_t capacity) {
  return guarded([&] { model_of(m).set_workspace_capacity(capacity); });
}

int mb_gpt_workspace_capacity(mb_gpt* m, size_t* capacity) {
  return guarded([&] {
    need(capacity, "capacity");
    *capacity = model_of(m).workspace_capacity();
  });
}

int mb_gpt_set_timing(mb_gpt* m, int enable) {
  return guarded([&] { model_of(m).set_timing(enable != 0); });
}

int mb_gpt_kernel_times(mb_gpt* m, char* names, size_t names_len, float* ms, size_t* count) {
  return guarded([&] {
    need(count, "count");
    auto t = model_of(m).kernel_times();
    std::string joined;
    for (size_t i = 0; i < t.size(); ++i) {
      if (i) joined += ',';
      joined += t[i].first;
      if (ms != nullptr && i < *count) ms[i] = t[i].second;
    }
    if (names != nullptr && names_len > 0) {
      std::strncpy(names, joined.c_str(), names_len - 1);
      names[names_len - 1] = '\0';
    }
    *count = t.size();
  });
}

int mb_nccl_unique_id(uint8_t id[MB_NCCL_ID_BYTES]) {
  return guarded([&] {
    need(id, "id");
    ncclUniqueId uid;
    mb::nccl_check(mb::nccl().get_unique_id(&uid), "ncclGetUniqueId");
    std::memcpy(id, &uid, sizeof(uid));
  });
}

int mb_gpt_attach_nccl(mb_gpt* m, const uint8_t id[MB_NCCL_ID_BYTES], int rank, int world_size) {
  return guarded([&] {
    need(id, "id");
    model_of(m).attach_nccl(id, rank, world_size);
  });
}

int mb_gpt_attach_nccl_comm(mb_gpt* m, void* comm, int world_size) {
  return guarded([&] { model_of(m).attach_nccl_comm(static_cast<ncclComm_t>(comm), world_size); });
}

int mb_gpt_detach_nccl(mb_gpt* m) {
  return guarded([&] { model_of(m).detach_nccl(); });
}

int mb_random_units(uint64_t seed, float* out, size_t count) {
  return guarded([&] {
    need(out, "out");
    mb::Random r(seed);
    for (size_t i = 0; i < count; ++i) out[i] = r.unit();
  });
}

int mb_equation_dataset(uint32_t modulus, uint32_t operation, double fraction, uint64_t seed,
                        uint32_t* residue_tokens, uint32_t* train, size_t* n_train, uint32_t* valid,
                        size_t* n_valid) {
  return guarded([&] {
    need(n_train, "n_train");
    need(n_valid, "n_valid");
    std::vector<uint32_t> res;
    std::vector<mb::Equation> tr, va;
    mb::equation_dataset(modulus, operation, fraction, seed, res, tr, va);
    if (residue_tokens != nullptr) std::memcpy(residue_tokens, res.data(), res.size() * sizeof(uint32_t));
    if (train != nullptr) {
      mb::require(*n_train >= tr.size(), "train buffer too small");
      std::memcpy(train, tr.data(), tr.size() * sizeof(mb::Equation));
    }
    if (valid != nullptr) {
      mb::require(*n_valid >= va.size(), "validation buffer too small");
      std::memcpy(valid, va.data(), va.size() * sizeof(mb::Equation));
    }
    *n_train = tr.size();
    *n_valid = va.size();
  });
}

int mb_equation_sampler(size_t examples, uint64_t seed, size_t batch, size_t steps, uint32_t* indices,
                        uint32_t* sizes) {
  return guarded([&] {
    need(indices, "indices");
    need(sizes, "sizes");
    mb::require(examples >= 1 && examples <= 65536, "sampler needs 1..65536 training equations");
    mb::require(batch >= 1 && batch <= examples && batch <= 131072 / 4, "invalid equation minibatch size");
    std::vector<uint32_t> idx(examples);
    for (size_t i = 0; i < examples; ++i) idx[i] = (uint32_t)i;
    mb::Random r(seed ^ 0x6261746368657303ull);
    mb::shuffle(idx, r);
    size_t pos = 0, out = 0;
    for (size_t s = 0; s < steps; ++s) {
      if (pos == examples) {
        mb::shuffle(idx, r);
        pos = 0;
      }
      const size_t end = std::min(examples, pos + batch);
      sizes[s] = (uint32_t)(end - pos);
      for (size_t i = pos; i < end; ++i) indices[out++] = idx[i];
      pos = end;
    }
  });
}

int mb_zipf_batch(uint64_t base_seed, uint32_t rank, uint64_t step, size_t sequences, size_t context,
                  uint32_t vocab, double exponent, uint32_t* inputs, uint32_t* targets) {
  return guarded([&] {
    need(inputs, "inputs");
    need(targets, "targets");
    mb::zipf_batch(base_seed, rank, step, sequences, context, vocab, exponent, inputs, targets);
  });
}

}  // extern "C"

#include "gpt_ops.cu"
