/*
 * meshb200.h - C ABI of the B200-native (sm_100a) Mesh GPT training hot path.
 *
 * This library replaces, behind plain C types, the model-level API that the
 * reference's Rust host code calls (fxeqxmulfx/grokking_abmod):
 *   SpecializedMeshGpt::{new, parameters, set_parameters, logits,
 *   loss_and_gradient, train_batch_with_optimizer, token_embeddings,
 *   hidden_states}                         src/gpt/gpu.rs:1718-2092
 * plus the seeded data and initialisation helpers it depends on
 * (src/mesh.rs:256-288, src/gpt/config.rs:144-591, src/gpt/grokking.rs:128-306).
 *
 * Conventions (mirroring the reference's error model, src/lib.rs:11):
 *   - Every entry point returns an int status: 0 = success, < 0 = error.  The
 *     message of the calling thread's last error is available through
 *     mb_last_error().  Nothing aborts, traps or frees caller memory.
 *   - Host pointers ("host") and device pointers ("device") are marked.
 *   - Validation (shapes, token ranges, finite values, configuration limits)
 *     happens on the host before any launch, as the reference's launch
 *     contracts do (src/gpt/config.rs:210-253).
 *   - A model is single-threaded: one CUDA device, one stream, like the
 *     reference's CudaContext + default stream (src/gpt/gpu.rs:1735-1736).
 */
#ifndef MESHB200_H
#define MESHB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MB_OK 0
#define MB_ERR_INVALID (-1)    /* invalid argument, configuration or batch */
#define MB_ERR_CUDA (-2)       /* CUDA runtime failure */
#define MB_ERR_NONFINITE (-3)  /* nonfinite loss, logits, gradients or parameters */
#define MB_ERR_NCCL (-4)       /* collective failure or timeout */
#define MB_ERR_UNSUPPORTED (-5) /* valid for the reference, outside this build's kernel shapes */

#define MB_IGNORE_TARGET 0xFFFFFFFFu /* src/gpt/mod.rs:26 */

/* GptConfig (src/gpt/config.rs:22-56); connectivity 0 = neighbor, 1 = butterfly;
 * embedding 0 = mesh (fixed token codes through the embedding mesh), 1 = table
 * (a learned [vocab][width] table, initialised as the tabulated mesh
 * embedding; src/gpt/config.rs:60-67,416-433).  The default geometry (parity
 * codes, token order, no normalisation) is the only embedding geometry on
 * this path. */
typedef struct mb_gpt_config {
  uint32_t vocab_size;
  uint32_t context;
  uint32_t width;
  uint32_t heads;
  uint32_t layers;
  uint32_t attention_mesh_depth;
  uint32_t ffn_mesh_depth;
  uint32_t connectivity;
  uint32_t embedding;
} mb_gpt_config;

/* AdamWOptions (src/gpt/config.rs:258-295). */
typedef struct mb_adamw {
  float learning_rate;
  float weight_decay;
  float beta1;
  float beta2;
  float epsilon;
} mb_adamw;

typedef struct mb_gpt mb_gpt; /* opaque model handle */
typedef struct mb_ctx mb_ctx; /* a device and the stream its models share */

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to len) and returns its status code. */
int mb_last_error(char* buf, size_t len);

/* Library / device queries. */
int mb_version(int* major, int* minor);
int mb_device_count(int* count);

/* ---- configuration and seeded initialisation (host only, no GPU) ---- */
/* GptConfig::validate (src/gpt/config.rs:144-172) and the kernel-shape limits
 * of this build (MB_ERR_UNSUPPORTED). */
int mb_gpt_validate(const mb_gpt_config* config);
/* Layout::count (src/gpt/config.rs:358-414). */
int mb_gpt_parameter_count(const mb_gpt_config* config, size_t* count);
/* Layout::initialize (src/gpt/config.rs:416-459); out: host, count floats. */
int mb_gpt_initial_parameters(const mb_gpt_config* config, uint64_t seed, float* out, size_t count);
/* token_codes (src/gpt/config.rs:552-591); out: host, vocab*width floats. */
int mb_gpt_token_codes(const mb_gpt_config* config, float* out, size_t count);

/* ---- context: the Arc<CudaContext> + default stream a SpecializedMeshGpt
 * is built on (src/gpt/gpu.rs:1718-1736).  mb_ctx_create selects the device
 * and creates one non-blocking stream; models made with mb_gpt_create_in
 * enqueue all their work on it.  Destroy those models before the context. */
int mb_ctx_create(int device, mb_ctx** ctx);
int mb_ctx_destroy(mb_ctx* ctx);
int mb_ctx_stream(mb_ctx* ctx, void** stream);

/* ---- model (SpecializedMeshGpt, src/gpt/gpu.rs:1701-2092) ---- */
/* SpecializedMeshGpt::new (:1718-1806) on its own device and stream. */
int mb_gpt_create(int device, const mb_gpt_config* config, uint64_t seed, mb_gpt** model);
/* The same on a context's device and stream. */
int mb_gpt_create_in(mb_ctx* ctx, const mb_gpt_config* config, uint64_t seed, mb_gpt** model);
int mb_gpt_destroy(mb_gpt* model);
int mb_gpt_get_config(const mb_gpt* model, mb_gpt_config* config);
/* parameters() (:1846-1853); out: host. */
int mb_gpt_get_parameters(mb_gpt* model, float* out, size_t count);
/* set_parameters() (:1856-1872): sets weights and resets AdamW moments/steps. */
int mb_gpt_set_parameters(mb_gpt* model, const float* values, size_t count);
/* logits() (:1875-1887); tokens: host [rows]; out: host [rows][vocab]. */
int mb_gpt_logits(mb_gpt* model, const uint32_t* tokens, size_t rows, size_t sequence, float* out);
/* hidden_states() (:2070-2092): residual stream before the final RMSNorm;
 * out: host [rows][width]. */
int mb_gpt_hidden_states(mb_gpt* model, const uint32_t* tokens, size_t rows, size_t sequence, float* out);
/* token_embeddings() (:2056-2067); out: host [vocab][width]. */
int mb_gpt_token_embeddings(mb_gpt* model, float* out, size_t count);
/* cross_entropy() (:1915-1929): mean supervised cross-entropy. */
int mb_gpt_cross_entropy(mb_gpt* model, const uint32_t* inputs, const uint32_t* targets, size_t rows,
                         size_t sequence, double* loss);
/* loss_and_gradient() (:1932-1946); gradient: host [parameter_count]. */
int mb_gpt_loss_and_gradient(mb_gpt* model, const uint32_t* inputs, const uint32_t* targets, size_t rows,
                             size_t sequence, double* loss, float* gradient, size_t count);
/* train_batch_with_optimizer() (:1971-2004): one AdamW step on host batches,
 * returning the mean cross-entropy before the update. */
int mb_gpt_train_step(mb_gpt* model, const uint32_t* inputs, const uint32_t* targets, size_t rows,
                      size_t sequence, const mb_adamw* optimizer, double* loss);
/* The same step on device-resident batches, enqueued on the model's stream
 * without a host synchronisation (captured as a CUDA graph per batch shape).
 * d_loss: device double written when the step completes; may be NULL.  Bad
 * tokens/targets are reported by mb_gpt_check() after the step. */
int mb_gpt_train_step_device(mb_gpt* model, const uint32_t* d_inputs, const uint32_t* d_targets, size_t rows,
                             size_t sequence, const mb_adamw* optimizer, double* d_loss);
/* Waits for the model's stream and reports device-side batch errors. */
int mb_gpt_check(mb_gpt* model);
/* The model's CUDA stream (cudaStream_t) for callers that order work on it. */
int mb_gpt_stream(mb_gpt* model, void** stream);
/* Device bytes owned by the model (allocated_device_bytes(), :1808-1844). */
int mb_gpt_allocated_device_bytes(mb_gpt* model, size_t* bytes);
/* Batch-shape workspaces kept cached (src/gpt/gpu.rs:1779-1791
 * set_workspace_capacity / workspace_capacity): each distinct
 * (rows, sequence) gets a workspace with its own captured step graph; at
 * most `capacity` (1..3, MB_ERR_INVALID otherwise; default 1 as in the
 * reference) are kept, the least recently used dropped first.  Lowering the
 * capacity frees the excess at once (after the model's stream drains). */
int mb_gpt_set_workspace_capacity(mb_gpt* model, size_t capacity);
int mb_gpt_workspace_capacity(mb_gpt* model, size_t* capacity);

/* Number of kernel launches one training step enqueues (diagnostics). */
int mb_gpt_step_launches(mb_gpt* model, size_t rows, size_t sequence, size_t* launches);

/* Kernel timing (diagnostics, no reference counterpart): with enable != 0
 * the step graphs are recaptured with CUDA events between launches.
 * mb_gpt_kernel_times writes the comma-separated launch names and per-launch
 * milliseconds of the most recent training step (*count in: capacity of ms,
 * out: number of launches). */
int mb_gpt_set_timing(mb_gpt* model, int enable);
int mb_gpt_kernel_times(mb_gpt* model, char* names, size_t names_len, float* ms, size_t* count);

/* ---- data parallelism (no reference counterpart: the reference is single
 * GPU).  Every rank holds the full model and passes its own share of the
 * batch.  The loss is the reference's mean over the supervised rows of the
 * whole batch (src/gpt/gpu.rs:2296-2313): each training step and each
 * loss_and_gradient first sums the ranks' supervised counts over NCCL,
 * divides the cross-entropy adjoint by that global count, then sums the flat
 * FP32 gradient and the loss over the ranks.  Loss and gradient are
 * therefore exact for any split of the supervised targets (a rank's share
 * may hold none), every rank returns the global loss, and AdamW keeps the
 * ranks identical.  logits, hidden_states and cross_entropy stay local to
 * the rank.  Every rank must make the same sequence of these calls. ---- */
#define MB_NCCL_ID_BYTES 128
int mb_nccl_unique_id(uint8_t id[MB_NCCL_ID_BYTES]);
/* Creates the model's own communicator from NCCL's 128-byte unique id. */
int mb_gpt_attach_nccl(mb_gpt* model, const uint8_t id[MB_NCCL_ID_BYTES], int rank, int world_size);
/* Uses a communicator the caller created on this model's device (an
 * ncclComm_t passed as void*); the caller keeps ownership and destroys it
 * after mb_gpt_detach_nccl or mb_gpt_destroy. */
int mb_gpt_attach_nccl_comm(mb_gpt* model, void* comm, int world_size);
int mb_gpt_detach_nccl(mb_gpt* model);

/* ---- per-op entry points: device pointers, the caller's cudaStream_t (NULL =
 * legacy default stream), no host synchronisation.  One two-parent mesh stack
 * of `depth` layers over rows x width (ELU, alpha 1, on every layer but the
 * last; layer l reads channels c and (c + stride_l) mod width); weights
 * [depth][width][2] = (self, neighbour) per channel. ---- */
/* Forward of a stack: gpt_mesh<W,0> layer by layer (src/gpt/gpu.rs:103-146,
 * host loop :2206-2232). */
int mb_op_mesh_forward(const float* x, float* y, size_t rows, uint32_t width, uint32_t depth,
                       uint32_t connectivity, const float* weights, void* stream);
/* Backward of a stack from its input x and output gradient dy: dx and the
 * edge gradients dweights [depth][width][2] (gpt_mesh<W,1>,
 * gpt_mesh_gradient and gpt_mesh_gradient_reduce, src/gpt/gpu.rs:103-146,
 * :1087-1149, host loop :2371-2444).  The stack is recomputed from x.  The
 * per-CTA gradient partials live in scratch memory taken with
 * cudaMallocAsync on `stream` and released on it. */
int mb_op_mesh_backward(const float* x, const float* dy, float* dx, float* dweights, size_t rows,
                        uint32_t width, uint32_t depth, uint32_t connectivity, const float* weights,
                        void* stream);

/* C[m][n] = op(A) . op(B) in FP32 on the tcgen05 tensor cores with the
 * 3xTF32 split (hi.hi + hi.lo + lo.hi), the dense contraction of the
 * reference's FP32 blocked_product GEMMs (src/simple/dense_tiled.rs:161-232).
 * layout is a set of bit flags: 1 = B stored [k][n] (C = A B; otherwise B is
 * [n][k] and C = A B^T); 4 = A stored [k][m] (otherwise [m][k]); 2 is
 * accepted and changes nothing (A always goes through tensor memory, the
 * A-from-TMEM MMA form) but may not be combined with 4.  Valid layouts:
 * 0-5.  All row-major FP32 device arrays.  d_status (device int) is set to
 * 1 if a tensor-core completion wait gave up. */
int mb_op_gemm_tf32x3(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k, uint32_t layout,
                      int* d_status, void* stream);

/* Test hook of the tensor-core waits (no counterpart in the reference): the
 * GEMM of mb_op_gemm_tf32x3 (layout 0) with K block `lost_block` never handed
 * to the MMA warp and every wait bounded by `wait_rounds` rounds of four
 * polls (1..2^22; product launches use 2^22).  Each CTA gives up, waits for
 * its copies in flight, skips its epilogue, frees its tensor memory and sets
 * *d_status to 1; the context stays usable.  Returns MB_OK once launched. */
int mb_test_gemm_lost_arrival(const float* a, const float* b, float* c, uint32_t m, uint32_t n, uint32_t k,
                              uint32_t lost_block, uint32_t wait_rounds, int* d_status, void* stream);

/* ---- per-op entry points of the Mesh GPT operators (device pointers, the
 * caller's stream, validation on the host before any launch).  The training
 * step runs the same arithmetic fused into its own kernels; these serve
 * callers that compose the model themselves and per-op tests.  rows x width
 * row-major FP32 arrays; heads divides width (head width hd = width/heads);
 * head h owns channels [h*hd, (h+1)*hd) of each row. */
/* Parameter-free RMSNorm per (row, head), eps 1e-5: y = x / rms(x); inv
 * [rows][heads] receives 1/rms (may be NULL); heads = 1 is the full-row norm
 * (gpt_rmsnorm_statistics + gpt_rmsnorm_apply, src/gpt/gpu.rs:65-94,
 * :1035-1077).  y may equal x. */
int mb_op_rmsnorm_forward(const float* x, float* y, float* inv, size_t rows, uint32_t width, uint32_t heads,
                          void* stream);
/* Its backward from the input x: dx = inv (dy - n mean(dy n)), n = x inv
 * (statistics recomputed from x, as the reference's backward does). */
int mb_op_rmsnorm_backward(const float* x, const float* dy, float* dx, size_t rows, uint32_t width,
                           uint32_t heads, void* stream);
/* Slice RoPE (gpt_rope, src/gpt/gpu.rs:175-208): per head, channels i and
 * i + hd/2 rotate by pos / 10000^(i/(hd/2)), pos = row mod sequence; inverse
 * != 0 rotates back (the backward).  hd even; y may equal x. */
int mb_op_rope(const float* x, float* y, size_t rows, uint32_t sequence, uint32_t width, uint32_t heads,
               int inverse, void* stream);
/* Causal softmax(Q K^T / sqrt(hd)) V per head over sequences of `sequence`
 * rows (diagonal included), the FA2 forward of src/gpt/gpu.rs:381-498,
 * :752-779.  lse: device [heads][rows], each row's base-2 log-sum-exp of
 * its scaled scores times log2(e).  Head widths 32 and 64 run on the tcgen05
 * tensor cores (3xF16: scaled FP16 hi/lo parts, three MMAs per product),
 * 2..16 and 128 on FP32 SIMT; others MB_ERR_UNSUPPORTED.
 * Q, K, V, O 16-byte aligned, width a multiple of 4.  Scratch for the
 * formatted key tiles comes from cudaMallocAsync on `stream`.  d_status
 * (device int) is set to 1 if a tensor-core wait gave up. */
int mb_op_attn_forward(const float* q, const float* k, const float* v, float* o, float* lse, size_t rows,
                       uint32_t sequence, uint32_t width, uint32_t heads, int* d_status, void* stream);
/* Its backward from dO, O and the forward's lse: dQ, dK, dV
 * (gpt_flash_delta, gpt_flash_query_gradient, gpt_flash_key_value_gradient,
 * src/gpt/gpu.rs:500-750).  Same shapes, limits and status as the forward. */
int mb_op_attn_backward(const float* q, const float* k, const float* v, const float* o, const float* dout,
                        const float* lse, float* dq, float* dk, float* dv, size_t rows, uint32_t sequence,
                        uint32_t width, uint32_t heads, int* d_status, void* stream);
/* Exclusive self-attention (exclusive_terms, gpt_exclusive,
 * src/gpt/gpu.rs:781-853): z = y - (y.u)u per head, u = v / max(|v|, 1e-12). */
int mb_op_xsa_forward(const float* y, const float* v, float* z, size_t rows, uint32_t width, uint32_t heads,
                      void* stream);
/* Its backward (gpt_exclusive_backward, :861-897): dy and dv from dz; the
 * norm's gradient is taken only above the 1e-12 floor. */
int mb_op_xsa_backward(const float* y, const float* v, const float* dz, float* dy, float* dv, size_t rows,
                       uint32_t width, uint32_t heads, void* stream);
/* The tied head and cross-entropy (gpt_head, gpt_cross_entropy,
 * gpt_head_backward, src/gpt/gpu.rs:927-1021): logits = RMSNorm(h) E^T
 * ([rows][vocab], E = embeddings [vocab][width]); *loss (device double) =
 * mean cross-entropy over the rows whose target is not MB_IGNORE_TARGET;
 * dh (may be NULL) = its gradient with respect to h; dembeddings (may be
 * NULL) = the head's contribution to dE, [vocab][width].  targets: device
 * [rows].  d_status (device int) becomes nonzero on failure: 1 a tensor-core
 * wait gave up, 2 a target outside the vocabulary, 4 no supervised row.
 * h and dh 16-byte aligned, width a multiple of 4.  Scratch from
 * cudaMallocAsync on `stream`. */
int mb_op_head_ce(const float* h, const float* embeddings, const uint32_t* targets, size_t rows, uint32_t width,
                  uint32_t vocab, float* logits, double* loss, float* dh, float* dembeddings, int* d_status,
                  void* stream);
/* AdamW with decoupled decay over a flat buffer (gpt_adam,
 * src/gpt/gpu.rs:1369-1391): the update number `step` (>= 1) gives the bias
 * corrections 1 - beta^step with beta^step accumulated in f32 one factor per
 * update, as the reference's host does (:1980-1981).  Updates weights, m and
 * v in place. */
int mb_op_adamw(float* weights, float* m, float* v, const float* gradient, size_t count, const mb_adamw* options,
                uint32_t step, void* stream);

/* The same mesh stack backward without any allocation (no reference
 * counterpart: the reference always allocates its workspace).  For callers
 * that must not allocate device memory per call - a service that fixes its
 * device memory at start-up, or a host whose own caching allocator must see
 * every allocation - this variant keeps its gradient partials in a 4 MiB
 * static device array that every GPU loading the library holds until exit.
 * Limit: row_lanes * depth * 2 * width <= 1048576 floats per CTA (always true
 * for the supported widths and depths <= 16); larger requests return
 * MB_ERR_INVALID, and the CTA count is capped so all partials fit.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls share the array: every partial a call reads is written by the
 * same call first, so nothing needs clearing, but calls that overlap on the
 * GPU (other streams, other threads) race on it and must be serialised.
 * The looked-up address is kept for the life of the process: after a
 * cudaDeviceReset of a device, do not call this entry point on it again. */
int mb_op_mesh_backward_noalloc(const float* x, const float* dy, float* dx, float* dweights, size_t rows,
                                uint32_t width, uint32_t depth, uint32_t connectivity, const float* weights,
                                void* stream);

/* ---- checkpoints (src/gpt/checkpoint.rs:25-196) --------------------------
 * MSHGPT07 (default architecture) / MSHGPT08 (table embedding or butterfly
 * connectivity) files:
 * magic, config as LE u32, the tokenizer's characters as u32 code points,
 * the parameters as LE f32, no trailing bytes.  Write from host arrays
 * (parameters from mb_gpt_get_parameters); read with NULL arrays to query
 * *n_characters / *n_parameters, then again with buffers.  Load into a model
 * with mb_gpt_create + mb_gpt_set_parameters (which resets AdamW, as
 * Checkpoint::load's callers do).  MSHGPT09 geometry ablations return
 * MB_ERR_UNSUPPORTED. */
int mb_gpt_checkpoint_write(const char* path, const mb_gpt_config* config, const uint32_t* characters,
                            size_t n_characters, const float* parameters, size_t n_parameters);
int mb_gpt_checkpoint_read(const char* path, mb_gpt_config* config, uint32_t* characters, size_t* n_characters,
                           float* parameters, size_t* n_parameters);

/* ---- seeded data (src/mesh.rs:256-288, src/gpt/grokking.rs:128-306) ---- */
/* SplitMix64 Random::unit() draws (f32). */
int mb_random_units(uint64_t seed, float* out, size_t count);
/* EquationDataset::new: operation 0=add 1=mul 2=sub 3=div 4=mixed
 * 5=square-sum 6=quadratic 7=quadratic-linear 8=cubic-product 9=cubic-mixed.
 * Writes the residue permutation (modulus u32) and the split as
 * (a, b, answer) triples; sizes are returned through *n_train / *n_valid
 * (call with NULL arrays to query them). */
int mb_equation_dataset(uint32_t modulus, uint32_t operation, double train_fraction, uint64_t seed,
                        uint32_t* residue_tokens, uint32_t* train, size_t* n_train, uint32_t* valid,
                        size_t* n_valid);
/* EquationSampler (src/gpt/grokking.rs:274-306): writes the index sequence
 * of `steps` successive sample(batch) calls; sizes[i] = rows of call i. */
int mb_equation_sampler(size_t examples, uint64_t seed, size_t batch, size_t steps, uint32_t* indices,
                        uint32_t* sizes);
/* Zipf(s) token streams of the benchmark: `sequences` streams of context+1
 * tokens from Random(base_seed + 1000003*rank + step); inputs and targets are
 * host [sequences*context]. */
int mb_zipf_batch(uint64_t base_seed, uint32_t rank, uint64_t step, size_t sequences, size_t context,
                  uint32_t vocab, double exponent, uint32_t* inputs, uint32_t* targets);

/* ---- grok-simple models (src/simple/mod.rs, src/simple/gpu.rs) ----------
 * Replaces GpuSimpleModel::{new, parameters, set_parameters, upload_table,
 * upload_batches, logits, evaluate, loss_and_gradient, train_batch}
 * (src/simple/gpu.rs:1757-2073) for the eleven architectures of SimpleConfig
 * (src/simple/mod.rs:500-558).  Operand encodings (src/simple/mod.rs:348-414):
 * one-hot for every architecture but the full mesh; binary, scalar and
 * discrete-log for mlp, mesh-mlp, bilinear, residual-mlp and
 * residual-mesh-mlp; binary for full-mesh-mlp.
 *   architecture 0 = mesh-mlp, 1 = tied-rotary-residual-dense-mlp,
 *                2 = shared-neighbor-mesh-mlp, 3 = mlp, 4 = bilinear,
 *                5 = residual-mlp, 6 = residual-mesh-mlp,
 *                7 = tied-concat-residual-mesh-mlp,
 *                8 = tied-rotary-residual-mesh-mlp, 9 = tied-concat-mesh-mlp,
 *                10 = full-mesh-mlp (binary operands, widths and moduli <= 256)
 *   expansion    residual-mlp's hidden width / width (reference default 4)
 *   mesh_depth   mesh layers per residual mesh branch (reference default 4)
 *   mesh_output_activation  1: activate a residual mesh branch's output
 *   tied_mesh    1: mesh-mlp / tied-concat-mesh-mlp store one mesh layer that
 *                every mesh layer uses (its gradient sums over the layers)
 *   decay_factors  n != 2 (one-layer mlp only): AdamW decays hidden channel
 *                c's input column and readout row at min(wd s_c^(2/n-1), 1/lr),
 *                s_c = (|E_c|^2 + |R_c|^2) / 2 (src/simple/gpu.rs:814-881)
 *   activation   0 = relu, 1 = square
 *   connectivity 0 = own, 1 = neighbor, 2 = butterfly
 *   full_mesh_initialization 0 = kaiming, 1 = identity-hidden
 * Fields an architecture does not read are ignored, as in the reference. */
typedef struct mb_simple_config {
  uint32_t architecture;
  uint32_t activation;
  uint32_t modulus;
  uint32_t width;
  uint32_t depth;
  uint32_t connectivity;
  uint32_t embedding_mesh_depth;
  uint32_t full_mesh_initialization;
  uint32_t mesh_learning_rate_multiplier;
  uint32_t expansion;
  uint32_t mesh_depth;             /* mesh layers per residual mesh branch (6-8) */
  uint32_t mesh_output_activation; /* 1: activate a residual mesh branch's output (6-8) */
  uint32_t tied_mesh;              /* 1: every mesh layer uses one stored layer (0, 9) */
  uint32_t encoding;               /* 0 one-hot, 1 binary, 2 scalar, 3 discrete-log */
  uint32_t decay_factors;          /* 2, or more for a one-layer mlp's channel decay */
} mb_simple_config;

typedef struct mb_simple mb_simple;
typedef struct mb_simple_table mb_simple_table;     /* DeviceTable (src/simple/gpu.rs:1868-1893) */
typedef struct mb_simple_batches mb_simple_batches; /* DeviceBatches (:1896-1909) */

/* SimpleConfig::validate (src/simple/mod.rs:561-694). */
int mb_simple_validate(const mb_simple_config* config);
/* SimpleConfig::parameter_count / groups (:871-893); pass groups = NULL to
 * query *n_groups. */
int mb_simple_parameter_count(const mb_simple_config* config, size_t* count);
int mb_simple_groups(const mb_simple_config* config, uint32_t* groups, size_t* n_groups);
/* SimpleConfig::initial_parameters (:938-1036), host out[count]. */
int mb_simple_initial_parameters(const mb_simple_config* config, uint64_t seed, float* out, size_t count);
/* SimpleConfig::encode (:1039-1055): host equations [n][3] (a, b, answer)
 * -> host features [n][2*F] (F = features per operand of the encoding),
 * targets [n]. */
int mb_simple_encode(const mb_simple_config* config, const uint32_t* equations, size_t n, float* features,
                     uint32_t* targets);

/* GpuSimpleModel::new (src/simple/gpu.rs:1758-1806). */
int mb_simple_create(int device, const mb_simple_config* config, uint64_t seed, mb_simple** out);
int mb_simple_destroy(mb_simple* model);
/* parameters (:1819-1826) and set_parameters, which resets AdamW (:1856-1875). */
int mb_simple_get_parameters(mb_simple* model, float* out, size_t count);
int mb_simple_set_parameters(mb_simple* model, const float* values, size_t count);
/* upload_table (:1878-1906): host features [rows][2*modulus] (one-hot
 * operand blocks) and targets [rows] < modulus. */
int mb_simple_upload_table(mb_simple* model, const float* features, const uint32_t* targets, size_t rows,
                           mb_simple_table** out);
int mb_simple_table_destroy(mb_simple_table* table);
/* upload_batches (:1909-1920): host indices into the table.  The device
 * buffer comes from a pool the model keeps (destroying the batches returns
 * it), and the copy is asynchronous on the model's stream, so a training
 * loop that uploads every epoch allocates nothing after its first upload. */
int mb_simple_upload_batches(mb_simple* model, const mb_simple_table* table, const uint32_t* indices,
                             size_t count, mb_simple_batches** out);
int mb_simple_batches_destroy(mb_simple_batches* batches);
/* train_batch (:2031-2073): one AdamW step on rows indices[offset ..
 * offset + rows) of the batches, f32 host beta powers. */
int mb_simple_train_step(mb_simple* model, const mb_simple_table* table, const mb_simple_batches* batches,
                         size_t offset, size_t rows, const mb_adamw* options);
/* evaluate (:1938-1995): logits [rows][modulus] and first-maximum
 * predictions [rows] of every table row (either output may be NULL);
 * nonfinite logits fail with MB_ERR_NONFINITE. */
int mb_simple_evaluate(mb_simple* model, const mb_simple_table* table, float* logits, uint32_t* predictions);
/* loss_and_gradient (:1998-2029): mean answer cross-entropy (f64, from the
 * f32 logits) and every parameter gradient on the selected table rows. */
int mb_simple_loss_and_gradient(mb_simple* model, const mb_simple_table* table, const uint32_t* indices,
                                size_t count, double* loss, float* gradient, size_t n_gradient);
/* Page-locked host memory (PinnedHostBuffer, src/simple/gpu.rs:1827-1842):
 * logits, predictions and parameters copied into it cross the bus at full
 * speed.  The host mirrors keep such buffers in a pool, as the reference's
 * pinned_parameters / reuse do. */
int mb_host_alloc(size_t bytes, void** ptr);
int mb_host_free(void* ptr);
/* Device stream, pending device errors, and kernels per train step. */
int mb_simple_stream(mb_simple* model, void** stream);
int mb_simple_check(mb_simple* model);
int mb_simple_step_launches(mb_simple* model, uint32_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* MESHB200_H */
