/*
 * spt_moe.h -- C ABI of the B200 (sm_100a) MoE FFN block for Stream-PT.
 *
 * The entry points replace the reference's Go functions in package
 * `forward` (paths relative to the Stream-PT repository root):
 *
 *   spt_forward_moe_batch        forwardMoEBatch   forward/moe_batch.go:78-194
 *   spt_forward_moe              forwardMoE        forward/moe.go:28-64
 *   spt_route_moe_batch          routeMoEBatch     forward/moe_batch.go:221-303
 *   spt_select_moe_batch         selectMoEBatch    forward/moe_batch.go:305-342
 *   spt_dispatch_moe_batch       dispatch lists    forward/moe_batch.go:142-159
 *   spt_mul_moe_batch_expert     mulMoEBatchExpert forward/mxfp4_batch.go:31-95
 *   spt_swiglu                   gptOSSSwiGLU      forward/moe.go:66-70
 *   spt_combine_moe_batch        combine loop      forward/moe_batch.go:163-192
 *   spt_rmsnorm                  normBatch         forward/layer_batch.go:139-195
 *   spt_mul_q80                  MulQ80Into/Argmax forward/q80.go:22-148
 *   spt_mul_q40                  MulQ40Into        forward/q40.go:35-40
 *   spt_mul_q40_batch            MulQ40BatchInto   forward/q40.go:46-101
 *   spt_arena_create             ggufmap.WithExpertRanges + readExpertBias
 *                                (ggufmap/mmap_linux.go:391-555, forward/moe.go:72-92):
 *                                the streamed mmap window becomes an HBM arena
 *                                uploaded once.
 *
 * Conventions: plain pointers and sizes; every function returns an
 * spt_status; the message of the last failure on a context is returned by
 * spt_last_error().  Host-pointer entry points are synchronous (they return
 * after the device work and the copies back have finished), like the Go
 * functions they replace.  `*_device` entry points take device pointers and
 * only enqueue work on the context's stream.  A non-NULL `cancel` flag is
 * polled between stages; a nonzero value returns SPT_ERR_CANCELED
 * (the reference returns ctx.Err()).
 */
#ifndef SPT_MOE_H
#define SPT_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum spt_status {
  SPT_OK = 0,
  SPT_ERR_NULL_ARG = 1,      /* "nil MoE context, reader, configuration or weights" */
  SPT_ERR_DIMENSIONS = 2,    /* "invalid MoE batch dimensions" / overflow / config */
  SPT_ERR_OVERLAP = 3,       /* "MoE input and output overlap" */
  SPT_ERR_ROUTER = 4,        /* "invalid F32 router shape or range" */
  SPT_ERR_EXPERT = 5,        /* "expected MXFP4 expert tensor" / invalid expert range */
  SPT_ERR_BIAS = 6,          /* unsupported bias type / invalid bias shape or range */
  SPT_ERR_FILE_RANGE = 7,    /* tensor range outside the reader's file */
  SPT_ERR_SCRATCH = 8,       /* "MoE batch scratch dimensions mismatch" */
  SPT_ERR_CANCELED = 9,      /* context.Canceled */
  SPT_ERR_CUDA = 10,         /* CUDA runtime failure (message in spt_last_error) */
  SPT_ERR_NCCL = 11,         /* NCCL failure in the expert-parallel path */
  SPT_ERR_TIMEOUT = 12,      /* a bounded device wait gave up */
  SPT_ERR_UNSUPPORTED = 13,  /* shape or option this build does not implement */
  SPT_ERR_NO_DEVICE = 14,    /* no CUDA device / extension unusable */
  SPT_ERR_FORMAT = 15        /* malformed or inconsistent GGUF model files */
} spt_status;

/* ggufindex.Tensor (ggufindex/index.go:15-26): name, GGML type, shape with
 * ne0 fastest, byte range inside the model file.  name == NULL or "" marks an
 * absent optional tensor (an unnamed bias, forward/moe_batch.go:196-201). */
typedef struct spt_tensor {
  const char *name;
  uint32_t type;      /* 0 F32, 1 F16, 2 Q4_0, 8 Q8_0, 30 BF16, 39 MXFP4 */
  uint32_t n_dims;    /* entries of shape[] in use (0..4) */
  uint64_t shape[4];
  uint64_t start, end;
} spt_tensor;

/* ggufmap.Reader stand-in: one contiguous host view of the model file (an
 * mmap of the GGUF shard, or any host buffer). */
typedef struct spt_reader {
  const uint8_t *base;
  uint64_t size;
} spt_reader;

/* The forward.Config fields the MoE block reads (forward/config.go:57-75). */
typedef struct spt_moe_config {
  int64_t hidden_dim;        /* H, 2880 for GPT-OSS-120B */
  int64_t expert_hidden_dim; /* D, 2880 */
  int64_t num_experts;       /* E, 128 */
  int64_t num_experts_used;  /* k, 4 */
} spt_moe_config;

/* The MoE tensors of forward.LayerWeights (forward/layer.go:66-81). */
typedef struct spt_layer_weights {
  spt_tensor ffn_gate_inp, ffn_gate_inp_bias;
  spt_tensor ffn_gate_exps, ffn_gate_exps_bias;
  spt_tensor ffn_up_exps, ffn_up_exps_bias;
  spt_tensor ffn_down_exps, ffn_down_exps_bias;
  /* LayerWeights.PostAttnNorm (blk.N.post_attention_norm.weight, F32, F16 or
   * BF16 [hidden]): the RMSNorm in front of the block (layer_batch.go:102).
   * Optional; only the layer-stack entry points use it. */
  spt_tensor post_attention_norm;
} spt_layer_weights;

typedef struct spt_context spt_context;
typedef struct spt_arena spt_arena;

/* ---- context ---------------------------------------------------------- */

/* Create a context on CUDA device `device` with its own stream. */
spt_status spt_context_create(int device, spt_context **out);
void spt_context_destroy(spt_context *ctx);
/* Message of the last failure on ctx (never NULL). */
const char *spt_last_error(const spt_context *ctx);
const char *spt_status_string(spt_status status);
/* The cudaStream_t all of this context's work is enqueued on. */
void *spt_context_stream(spt_context *ctx);
/* Use an external cudaStream_t (NULL restores the context's own stream). */
spt_status spt_context_set_stream(spt_context *ctx, void *stream);
/* Synchronize the context's stream. */
spt_status spt_context_sync(spt_context *ctx);

/* ---- validation (no device work) ------------------------------------- */

/* Exactly the tensor/config checks of forwardMoEBatch
 * (forward/moe_batch.go:81-130, mxfp4_batch.go:17-27,
 * moe_batch.go:196-219, mmap_linux.go:318-334). */
spt_status spt_validate_moe_layer(spt_context *ctx, const spt_reader *reader,
                                  const spt_moe_config *cfg, const spt_layer_weights *lw);

/* ---- HBM expert arena -------------------------------------------------- */

#define SPT_ARENA_GEMV 1u /* CUDA-core GEMV layout (decode, bit-exact order) */
#define SPT_ARENA_MMA 2u  /* tcgen05 block-scaled GEMM layout (prefill) */

/* Validate and upload n_layers layers (readers[i], layers[i]) once through
 * pinned memory, repacking MXFP4 blocks on the device.  Replaces the
 * ggufmap mmap window, hot-expert cache and lookahead. */
spt_status spt_arena_create(spt_context *ctx, const spt_reader *readers,
                            const spt_moe_config *cfg, const spt_layer_weights *layers,
                            int64_t n_layers, uint32_t flags, spt_arena **out);

/* The same from per-tensor views, for readers that hand out each tensor's
 * bytes separately (ggufmap.Reader.WithTensor, ggufmap/mmap_linux.go:210:
 * a read-only slice valid inside its callback): data->X points at the first
 * byte of tensor layers->X ([start, end) of its file), NULL for an absent
 * optional tensor.  The views need to stay valid only for the duration of
 * the call; the library keeps nothing of them.  expert_end 0: every expert. */
typedef struct spt_layer_data {
  const uint8_t *ffn_gate_inp, *ffn_gate_inp_bias;
  const uint8_t *ffn_gate_exps, *ffn_gate_exps_bias;
  const uint8_t *ffn_up_exps, *ffn_up_exps_bias;
  const uint8_t *ffn_down_exps, *ffn_down_exps_bias;
  const uint8_t *post_attention_norm;
} spt_layer_data;
spt_status spt_arena_create_views(spt_context *ctx, const spt_moe_config *cfg, const spt_layer_weights *layers,
                                  const spt_layer_data *data, int64_t n_layers, uint32_t flags, int64_t expert_begin,
                                  int64_t expert_end, spt_arena **out);

/* Seeded synthetic GPT-OSS-style weights generated on the device
 * (counter-based Philox4x32-10; identical bytes from
 * spt_synth_layer_host).  Not a reference interface: benchmark input. */
typedef struct spt_synth_params {
  uint64_t seed;
  float router_std;   /* N(0, router_std) router weights (0.02) */
  float bias_std;     /* N(0, bias_std) router and expert biases (0.01) */
  uint8_t scale_lo;   /* E8M0 scale bytes uniform in [scale_lo, scale_hi] */
  uint8_t scale_hi;
  uint8_t expert_bias; /* 1: F32 expert biases present; 0: unnamed */
  uint8_t router_bias; /* 1: router bias present */
  float zipf_s;       /* >0: add a Zipf(zipf_s) skew to the router bias */
  float zipf_beta;    /* logit scale of that skew */
} spt_synth_params;

spt_status spt_arena_create_synthetic(spt_context *ctx, const spt_moe_config *cfg,
                                      const spt_synth_params *params, int64_t n_layers,
                                      uint32_t flags, spt_arena **out);
void spt_arena_destroy(spt_arena *arena);
/* Device bytes held by the arena. */
uint64_t spt_arena_bytes(const spt_arena *arena);

/* Host copy of one synthetic layer in GGUF tensor layout (for the CPU
 * oracle and the baseline).  Sizes: router E*H*4, router_bias E*4,
 * gate/up E*D*(H/32)*17, down E*H*(D/32)*17, gate/up bias E*D*4,
 * down bias E*H*4.  Any pointer may be NULL to skip that tensor. */
spt_status spt_synth_layer_host(const spt_moe_config *cfg, const spt_synth_params *params,
                                int64_t layer, uint8_t *router, float *router_bias,
                                uint8_t *gate, uint8_t *up, uint8_t *down, float *gate_bias,
                                float *up_bias, float *down_bias);
/* Seeded N(mean, std) fp32 activations (Box-Muller in double). */
spt_status spt_synth_normal_host(uint64_t seed, uint64_t stream, float mean, float std,
                                 float *out, int64_t n);

/* ---- expert-GEMM path ---------------------------------------------------- */

/* SPT_PATH_EXACT: CUDA-core MXFP4 GEMV reproducing the reference's AVX2
 * arithmetic bit for bit (needs an SPT_ARENA_GEMV arena).
 * SPT_PATH_MMA: tcgen05 block-scaled grouped GEMM on the packed FP4 weights,
 * activations written as block-scaled terms (4 e2m1 terms; 3 e4m3 terms for
 * 128-token tiles with SPT_OPT_PREFILL_FP8), fp32 accumulation; routing
 * stays bit-exact, block outputs agree with the reference to a few 1e-4 of
 * the largest output (needs SPT_ARENA_MMA).
 * SPT_PATH_GEMV16: decode GEMV on the same packed weights: in-register
 * dequantisation to f16, activations as two f16 terms, fp32 sums; block
 * outputs agree with the reference to ~1e-6 (needs SPT_ARENA_MMA with every
 * E8M0 scale byte in [104, 140], K <= 3072).
 * SPT_PATH_AUTO (default): on an SPT_ARENA_MMA arena, the decode GEMV while
 * batch x top-k <= SPT_OPT_GEMV16_SLOTS (and the layer's scales allow it),
 * the tcgen05 GEMM above; else EXACT. */
#define SPT_PATH_AUTO 0
#define SPT_PATH_EXACT 1
#define SPT_PATH_MMA 2
#define SPT_PATH_GEMV16 3
spt_status spt_context_set_path(spt_context *ctx, int path);

/* Per-context tuning and test options.  Values are seeded once, when the
 * context is created, from the environment variable named beside each.
 *   SPT_OPT_TILE_TOKENS   tcgen05 token-tile width 8, 16 or 128; 0 picks it
 *                         from the batch (SPT_MMA_BN)
 *   SPT_OPT_FUSED_SELECT  batches of up to 8 tokens on one device: 1 (default)
 *                         top-k selection and dispatch run in the router's
 *                         last CTA when the router stages its rows in shared
 *                         memory, else selection inside the dispatch kernel;
 *                         2: selection inside the dispatch kernel; 0: each
 *                         its own launch (SPT_FUSED_SELECT); same results
 *   SPT_OPT_L2_PREFETCH   tcgen05 weight tiles prefetched into L2 ahead of
 *                         the ring, 0 off (SPT_MMA_PREFETCH)
 *   SPT_OPT_GEMV16_SLOTS  SPT_PATH_AUTO runs the decode GEMV while
 *                         batch x top-k <= value (default 16;
 *                         SPT_GEMV16_SLOTS)
 *   SPT_OPT_WAIT_LIMIT    every bounded device wait gives up after about
 *                         2^value clock cycles, 10..31 (default 31, about a
 *                         second) and the call returns SPT_ERR_TIMEOUT
 *   SPT_OPT_FAULT_STAGE   test hook, -1 off: the tcgen05 producer of CTA 0
 *                         skips this pipeline stage, so the MMA issuer's wait
 *                         for it runs out (the failure path without a fault);
 *                         1000: the shared-memory router's CTA 0 leaves out
 *                         one row's copy, so its wait runs out
 *   SPT_OPT_HOST_GRAPHS   1 (default): spt_forward_moe_batch / spt_forward_moe
 *                         capture the block's kernels into a CUDA graph on the
 *                         second call with the same arena, layer, batch and
 *                         options, and replay it afterwards (one launch
 *                         instead of five to eight); 0: plain launches
 *                         (SPT_HOST_GRAPHS)
 *   SPT_OPT_PREFILL_FP8   0 (default): 128-token tensor-core tiles take the
 *                         activations as four e2m1 terms (kind::mxf4); 1:
 *                         three e4m3 terms (kind::mxf8f6f4, about ten times
 *                         finer, more time) (SPT_PREFILL_FP8) */
#define SPT_OPT_TILE_TOKENS 1
#define SPT_OPT_FUSED_SELECT 2
#define SPT_OPT_L2_PREFETCH 3
#define SPT_OPT_GEMV16_SLOTS 4
#define SPT_OPT_WAIT_LIMIT 5
#define SPT_OPT_FAULT_STAGE 6
#define SPT_OPT_HOST_GRAPHS 7
#define SPT_OPT_PREFILL_FP8 8
spt_status spt_context_set_option(spt_context *ctx, int option, int64_t value);
int64_t spt_context_get_option(const spt_context *ctx, int option);

/* ---- the block ----------------------------------------------------------- */

/* forwardMoEBatch: x and out are host arrays of x_len / out_len floats,
 * [batch, H] row-major; they must not overlap.  out is fully overwritten. */
spt_status spt_forward_moe_batch(spt_context *ctx, spt_arena *arena, int64_t layer,
                                 const float *x, int64_t x_len, float *out, int64_t out_len,
                                 int64_t batch, const volatile int32_t *cancel);
/* forwardMoE: the batch-1 decode wrapper. */
spt_status spt_forward_moe(spt_context *ctx, spt_arena *arena, int64_t layer, const float *x,
                           int64_t x_len, float *out, int64_t out_len,
                           const volatile int32_t *cancel);
/* Same block on device pointers (16-byte aligned), enqueued on the context
 * stream. */
spt_status spt_forward_moe_batch_device(spt_context *ctx, spt_arena *arena, int64_t layer,
                                        const float *x, float *out, int64_t batch);

/* Allocation-free variant of spt_forward_moe_batch_device (no counterpart in
 * the reference).  For callers that cannot let the library allocate device
 * memory while they run: an engine that reserved all of HBM at load time, or
 * a latency-critical decode loop that must not pay cudaMalloc/cudaFree's
 * device-wide synchronisation.  Runs the exact (bit-identical) path with all
 * intermediates in one static device array of about 2.2 MB, held by every GPU
 * that loads the library.  Limits: batch x top-k <= 64, hidden and expert
 * dimensions <= 4096, experts <= 256 (SPT_ERR_UNSUPPORTED otherwise); needs an
 * SPT_ARENA_GEMV arena.  spt_context_create looks up the array's device
 * address, which loads the library's device code and the array on that
 * device: create the context before reserving the rest of HBM.  All calls share the array: calls that overlap on the
 * GPU race and must be serialised.  The call's routing stays in the array, so
 * spt_last_routing and spt_stage_times refuse after it (until the next
 * allocating forward). */
spt_status spt_forward_moe_batch_device_static(spt_context *ctx, spt_arena *arena, int64_t layer,
                                               const float *x, float *out, int64_t batch);

/* Drop-in one-shot form of forwardMoEBatch: validates every tensor against
 * the reader, uploads the layer, runs it and frees it. */
spt_status spt_forward_moe_batch_reader(spt_context *ctx, const spt_reader *reader,
                                        const spt_moe_config *cfg,
                                        const spt_layer_weights *lw, const float *x,
                                        int64_t x_len, float *out, int64_t out_len,
                                        int64_t batch, const volatile int32_t *cancel);

/* Intermediates of the last single-GPU spt_forward_moe_batch* call (host
 * copies, for parity tests): logits [batch*E], selected index/weight
 * [batch*k], dispatch permutation perm [dispatched] and per-expert counts [E].
 * Refused (SPT_ERR_DIMENSIONS) after an allocation-free or expert-parallel
 * call, whose intermediates live elsewhere.
 * Any pointer may be NULL.  *dispatched receives the dispatched slot count. */
spt_status spt_last_routing(spt_context *ctx, float *logits, int32_t *sel_index,
                            float *sel_weight, int32_t *perm, int32_t *expert_count,
                            int64_t *dispatched);

/* Per-stage device timing of the block.  When enabled, every forward call
 * records CUDA events on the context stream around its stages; spt_stage_times
 * returns the durations (ms) of the last call:
 * [0] router, [1] select, [2] dispatch, [3] activation operand (tcgen05:
 * quantisation into terms; decode GEMV: the f16 split), [4] gate/up +
 * SwiGLU, [5] quantisation of the SwiGLU output (tcgen05 only), [6] down,
 * [7] combine (stage 3 is empty on the exact path, stage 5 on the others).
 * Returns the number of stages written (<= n). */
#define SPT_NUM_STAGES 8
spt_status spt_set_stage_timing(spt_context *ctx, int enable);
int spt_stage_times(spt_context *ctx, float *ms, int n);
/* Number of kernels the last forward call launched. */
int spt_kernels_per_forward(spt_context *ctx);
/* Expert path the last forward call took: SPT_PATH_EXACT, SPT_PATH_MMA or
 * SPT_PATH_GEMV16; *tile_tokens (may be NULL) gets the tcgen05 token-tile
 * width (8, 16 or 128; 0 on the other paths).  Instrumentation, no
 * counterpart in the reference. */
int spt_last_expert_path(spt_context *ctx, int *tile_tokens);

/* ---- stage entry points (host pointers, synchronous) -------------------- */

/* routeMoEBatch: data = E rows x hidden little-endian F32 (any byte
 * alignment, data_len == E*hidden*4); logits[t*E+e]. */
spt_status spt_route_moe_batch(spt_context *ctx, const uint8_t *data, uint64_t data_len,
                               const float *x, int64_t x_len, const float *router_bias,
                               int64_t batch, int64_t hidden, int64_t experts, float *logits,
                               const volatile int32_t *cancel);
/* selectMoEBatch for every token row of logits [batch, E]. */
spt_status spt_select_moe_batch(spt_context *ctx, const float *logits, int64_t batch,
                                int64_t experts, int64_t k, int32_t *index, float *weight);
/* The reference's per-expert dispatch lists as a permutation: slots with
 * weight > 0 or NaN, grouped by expert ascending, each group in
 * descending slot order (the push-front list walk).  expert_offsets has
 * E+1 entries; *dispatched = expert_offsets[E]. */
spt_status spt_dispatch_moe_batch(spt_context *ctx, const int32_t *index, const float *weight,
                                  int64_t batch, int64_t k, int64_t experts, int32_t *perm,
                                  int32_t *expert_offsets, int64_t *dispatched);
/* mulMoEBatchExpert: data = `output` rows of input/32 17-byte MXFP4 blocks;
 * y[y_offsets[j]+r] = dot(row r, x[x_offsets[j] : +input]) + bias[r].
 * bias may be NULL (zeros).  Offsets are bounds-checked against x_len/y_len. */
spt_status spt_mul_moe_batch_expert(spt_context *ctx, const uint8_t *data, uint64_t data_len,
                                    int64_t input, int64_t output, const float *x, int64_t x_len,
                                    const int64_t *x_offsets, int64_t count, const float *bias,
                                    float *y, int64_t y_len, const int64_t *y_offsets,
                                    const volatile int32_t *cancel);
/* act[i] = gptOSSSwiGLU(gate[i], up[i]). */
spt_status spt_swiglu(spt_context *ctx, const float *gate, const float *up, float *act,
                      int64_t n);
/* out[t,:] = sum over ranks r (weight > 0 or NaN) of fma(results[t*k+r,:], w, out). */
spt_status spt_combine_moe_batch(spt_context *ctx, const float *results, const float *weight,
                                 int64_t batch, int64_t k, int64_t hidden, float *out);
/* normBatch RMSNorm with an F32 weight vector, 8 accumulation lanes. */
spt_status spt_rmsnorm(spt_context *ctx, const float *x, const float *weight, int64_t batch,
                       int64_t dim, float eps, float *y);
/* MulQ80Into + MulQ80Argmax (forward/q80.go:22-148): Q8_0 matrix [output
 * rows x input/32 34-byte blocks] in host memory, uploaded for this call;
 * y may be NULL; *argmax gets the lowest row of the largest logit (NaN never
 * wins; 0 when no logit beats -Inf), *best_logit that logit. */
spt_status spt_mul_q80(spt_context *ctx, const uint8_t *data, uint64_t data_len, int64_t input,
                       int64_t output, const float *x, float *y, int64_t *argmax,
                       float *best_logit);
/* The same with the matrix resident in HBM: uploaded once (the reference
 * streams it from the mmap window for every token, q80.go:86-104) and
 * repacked on the device into four-row groups; the caller's bytes are not
 * kept.  Creation needs the packed matrix (the file's size rounded up to
 * whole four-row groups, + 64 bytes) plus a transient device copy of the
 * file's bytes, freed before it returns. */
typedef struct spt_q80_matrix spt_q80_matrix;
spt_status spt_q80_matrix_create(spt_context *ctx, const uint8_t *data, uint64_t data_len,
                                 int64_t input, int64_t output, spt_q80_matrix **out);
void spt_q80_matrix_destroy(spt_q80_matrix *m);
/* Host x [input] / y [output] (y may be NULL), synchronous. */
spt_status spt_mul_q80_matrix(spt_context *ctx, spt_q80_matrix *m, const float *x, float *y,
                              int64_t *argmax, float *best_logit);
/* Device pointers; enqueue only.  y, argmax (one int64) and best_logit (one
 * float) may each be NULL. */
spt_status spt_mul_q80_matrix_device(spt_context *ctx, spt_q80_matrix *m, const float *x, float *y,
                                     int64_t *argmax, float *best_logit);

/* ---- Q4_0 products -----------------------------------------------------------
 * MulQ40Into / MulQ40BatchInto (forward/q40.go:35-101): y[item*output + r] =
 * row r of the Q4_0 tensor (`tensor` in `reader`, GGML type 2, shape
 * [input, output], output rows of input/32 18-byte blocks) dotted with
 * x[item*input ...].  Batch 1 follows the reference's one-input order
 * (quantQ40AVX2, forward/quant_amd64.go:75-90), larger batches its batched
 * order (quantDotQ40Batch, :118-148); both bit for bit.  Checks as q40Shape
 * and MulQ40BatchInto (q40.go:58-71,105-130): SPT_ERR_DIMENSIONS for the
 * type, rank, shape, batch (< 1 or overflowing) and x_len/y_len != batch *
 * input/output; SPT_ERR_FILE_RANGE for the byte range; SPT_ERR_OVERLAP when x
 * and y overlap; SPT_ERR_CANCELED when *cancel is set on entry (the one
 * launch is not interrupted).  This build needs input <= 4,768
 * (SPT_ERR_UNSUPPORTED above; GPT-OSS uses 2,880 and 4,096).  The matrix is
 * uploaded for the call; spt_q40_matrix keeps it resident. */
spt_status spt_mul_q40(spt_context *ctx, const spt_reader *reader, const spt_tensor *tensor, const float *x,
                       int64_t x_len, float *y, int64_t y_len, const volatile int32_t *cancel);
spt_status spt_mul_q40_batch(spt_context *ctx, const spt_reader *reader, const spt_tensor *tensor, const float *x,
                             int64_t x_len, float *y, int64_t y_len, int64_t batch,
                             const volatile int32_t *cancel);
typedef struct spt_q40_matrix spt_q40_matrix;
spt_status spt_q40_matrix_create(spt_context *ctx, const spt_reader *reader, const spt_tensor *tensor,
                                 spt_q40_matrix **out);
void spt_q40_matrix_destroy(spt_q40_matrix *m);
spt_status spt_q40_matrix_shape(const spt_q40_matrix *m, int64_t *input, int64_t *output);
/* Host x [batch*input] / y [batch*output], synchronous. */
spt_status spt_mul_q40_matrix(spt_context *ctx, spt_q40_matrix *m, const float *x, int64_t x_len, float *y,
                              int64_t y_len, int64_t batch, const volatile int32_t *cancel);
/* Device pointers; enqueue only (one kernel launch, no allocation). */
spt_status spt_mul_q40_matrix_device(spt_context *ctx, spt_q40_matrix *m, const float *x, float *y,
                                     int64_t batch);

/* ---- GGUF model files -------------------------------------------------------
 * ggufindex.Open (ggufindex/index.go:55-575): headers, metadata and tensor
 * directories of one model, split files in any order, each file mapped
 * read-only for the life of the handle; the same validation and error
 * messages (SPT_ERR_FORMAT; the text is in spt_last_error(NULL)). */
typedef struct spt_gguf spt_gguf;
spt_status spt_gguf_open(const char *const *paths, int64_t n_paths, spt_gguf **out);
void spt_gguf_close(spt_gguf *g);
int64_t spt_gguf_layer_count(const spt_gguf *g);
/* NewConfig's MoE fields (forward/config.go:56-125): the gpt-oss.* metadata
 * when present and positive, else GPT-OSS-120B's defaults. */
spt_status spt_gguf_config(const spt_gguf *g, spt_moe_config *cfg, float *rms_eps);
/* NewLayerWeights (forward/layer.go:39-86) for one layer: the MoE tensors and
 * post_attention_norm with absolute byte ranges, and the reader of the file
 * that holds them (all of a layer's MoE tensors must lie in one file).
 * Tensor names point into the handle. */
spt_status spt_gguf_layer(const spt_gguf *g, int64_t layer, spt_layer_weights *lw, spt_reader *reader);
/* Any tensor by name (e.g. "output.weight" for the LM head) and its file. */
spt_status spt_gguf_tensor(const spt_gguf *g, const char *name, spt_tensor *t, spt_reader *reader);
/* spt_arena_create_range over layers [first_layer, first_layer + n_layers)
 * of a GGUF model (expert_end 0: every expert). */
spt_status spt_arena_create_gguf(spt_context *ctx, const spt_gguf *g, int64_t first_layer, int64_t n_layers,
                                 uint32_t flags, int64_t expert_begin, int64_t expert_end, spt_arena **out);

/* ---- Layer stack -------------------------------------
 * The MoE half of forwardLayerBatch (forward/layer_batch.go:102-120) over
 * layers [first_layer, first_layer + n_layers): for each layer,
 *   normed = normBatch(post_attention_norm, x, eps)  (8 lanes, layer_batch.go:139-195)
 *   ffn    = the MoE block of `normed`
 *   x     += ffn                                     (addVector, layer.go:305-340)
 * x is the residual stream, updated in place.  `ep` may be NULL; otherwise
 * every layer's block runs expert-parallel (the arena is this rank's shard).
 * Synthetic arenas carry N(1, 0.02) norm weights (spt_synth_norm_host). */
spt_status spt_forward_stack_device(spt_context *ctx, struct spt_ep *ep, spt_arena *arena,
                                    int64_t first_layer, int64_t n_layers, float *x, int64_t batch,
                                    float eps);
spt_status spt_forward_stack(spt_context *ctx, struct spt_ep *ep, spt_arena *arena, int64_t first_layer,
                             int64_t n_layers, float *x, int64_t x_len, int64_t batch, float eps,
                             const volatile int32_t *cancel);
/* Host copy of a synthetic layer's norm weights [dim]. */
spt_status spt_synth_norm_host(const spt_synth_params *params, int64_t layer, int64_t dim, float *out);

/* ---- Expert parallelism ---------------------------------------------------
 * No counterpart in the reference, which runs the block on one host; the
 * build's target asks for experts sharded 128/world per GPU with all-to-all
 * dispatch and combine over NVLink.  Rank r of `world` holds experts
 * [r*E/world, (r+1)*E/world) of every layer (an arena made with
 * spt_arena_create_range or spt_arena_create_synthetic_range over
 * spt_ep_expert_range) plus the whole router, and calls the forward with its
 * own tokens; every rank must call it the same number of times, in the same
 * order.  Results equal the single-GPU block's for those tokens (bit for bit
 * on the exact path).  The exchange uses NCCL point-to-point calls on the
 * context's stream; libnccl.so.2 is opened at run time. */
#define SPT_EP_UNIQUE_ID_BYTES 128
typedef struct spt_ep spt_ep;
/* Experts of rank `rank`: [rank*E/world, (rank+1)*E/world). */
void spt_ep_expert_range(int64_t num_experts, int32_t world, int32_t rank, int64_t *begin,
                         int64_t *end);
/* Rank 0 makes the id and hands it to the other ranks out of band. */
spt_status spt_ep_unique_id(uint8_t id[SPT_EP_UNIQUE_ID_BYTES]);
/* Collective over the `world` ranks (each on its own context and device). */
spt_status spt_ep_create(spt_context *ctx, const uint8_t id[SPT_EP_UNIQUE_ID_BYTES], int32_t rank,
                         int32_t world, spt_ep **out);
void spt_ep_destroy(spt_ep *ep);
/* Fixed-capacity exchange for decode-sized batches: every rank sends every
 * peer a slot of max_tokens_per_rank * top-k rows per call, with the live row
 * count in the same NCCL group, so no count reaches the host and a call never
 * synchronises.  Every rank must set the same value, and calls with more
 * tokens fail with SPT_ERR_DIMENSIONS.  0 (the default) exchanges counts
 * first and sends only live rows (one host synchronisation per call). */
spt_status spt_ep_set_capacity(spt_ep *ep, int64_t max_tokens_per_rank);
/* Transport of the fixed-capacity exchange.  SPT_EP_EXCHANGE_PEER (the
 * default, when every rank has its own GPU): each rank's receive window is
 * mapped into every other rank (CUDA IPC, set up by the first fixed-capacity
 * call, collectively); senders write their live rows straight into the
 * owners' windows over NVLink and publish a sequence number, receivers wait
 * on it on the device (bounded by SPT_OPT_WAIT_LIMIT, SPT_ERR_TIMEOUT at the
 * next synchronisation): no NCCL call and no padding rows per call.  Ranks
 * that share a GPU fall back to SPT_EP_EXCHANGE_NCCL (grouped send/receive of
 * full slots).  Every rank must choose the same transport. */
#define SPT_EP_EXCHANGE_PEER 0
#define SPT_EP_EXCHANGE_NCCL 1
spt_status spt_ep_set_exchange(spt_ep *ep, int32_t exchange);
/* Device pointers (16-byte aligned), this rank's `batch` tokens.  Enqueues on
 * the context's stream; without a capacity it synchronises the stream once,
 * after the per-rank row counts are exchanged. */
spt_status spt_forward_moe_batch_ep_device(spt_context *ctx, spt_ep *ep, spt_arena *arena,
                                           int64_t layer, const float *x, float *out,
                                           int64_t batch);
/* Active experts and dispatched rows of the last dispatch this context ran
 * (on an expert-parallel call: the rows this rank received and how many of
 * its experts they used).  Synchronises the stream.  No counterpart in the
 * reference (instrumentation for the benchmark). */
spt_status spt_last_dispatch(spt_context *ctx, int64_t *active_experts, int64_t *dispatched);
/* Host buffers, synchronous: the expert-parallel spt_forward_moe_batch. */
spt_status spt_forward_moe_batch_ep(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t layer,
                                    const float *x, int64_t x_len, float *out, int64_t out_len,
                                    int64_t batch, const volatile int32_t *cancel);

/* Arenas holding experts [expert_begin, expert_end) only (an expert-parallel
 * shard; the router is always whole).  The single-GPU forward entry points
 * refuse such an arena. */
spt_status spt_arena_create_range(spt_context *ctx, const spt_reader *readers,
                                  const spt_moe_config *cfg, const spt_layer_weights *layers,
                                  int64_t n_layers, uint32_t flags, int64_t expert_begin,
                                  int64_t expert_end, spt_arena **out);
spt_status spt_arena_create_synthetic_range(spt_context *ctx, const spt_moe_config *cfg,
                                            const spt_synth_params *params, int64_t n_layers,
                                            uint32_t flags, int64_t expert_begin,
                                            int64_t expert_end, spt_arena **out);
void spt_arena_expert_range(const spt_arena *arena, int64_t *expert_begin, int64_t *expert_end);

#ifdef __cplusplus
}
#endif
#endif /* SPT_MOE_H */
