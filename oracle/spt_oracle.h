/*
 * spt_oracle.h -- CPU restatement of Stream-PT's MoE FFN hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels and the timed CPU baseline in bench.py.  Nothing in the
 * product (the CUDA library under stream-pt_b200/) links, loads or calls it.
 *
 * Parity pinning: the reference (Go 1.27, GOEXPERIMENT=simd) cannot run in
 * this image (no Go toolchain).  The restatement is pinned by the reference
 * tests' own known answers and independent float64 oracle, re-expressed in
 * tests/test_oracle_pins.py (TestMXFP4Dot, TestMXFP4AllScales,
 * TestSIMDKernelMXFP4DecodeAllEncodings, TestGPTOSSExpertBiasesAndSwiGLU,
 * TestSparseMoEIndependentReference, TestForwardMoEBatchMatchesSequential,
 * TestSIMDKernelGather, TestSIMDKernelRouter, TestMXFP4NibbleReference).
 *
 * All functions use IEEE fp32 round-to-nearest with explicit fmaf where the
 * reference uses a fused multiply-add (archsimd MulAdd) and separate
 * rounding everywhere else (build flag -ffp-contract=off).
 */
#ifndef SPT_ORACLE_H
#define SPT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One selected expert (forward/moe.go:15-18 ExpertSelection). */
typedef struct spo_selection {
  int32_t index;
  float weight;
} spo_selection;

/* Build the E8M0 and scaled-FP4 tables (forward/mxfp4.go:10-28). Idempotent. */
void spo_init(void);

/* E8M0 byte -> float32(2^(b-127)); 255 -> +Inf (forward/mxfp4.go:22). */
float spo_e8m0(uint8_t b);
/* scaledFP4Table[scale][code] (forward/mxfp4.go:24). */
float spo_scaled_fp4(uint8_t scale, uint8_t code);

/* F16 bits -> f32 (forward/q40.go:149-180 float16). */
float spo_f16(uint16_t bits);
/* BF16 bits -> f32 (forward/layer.go:296). */
float spo_bf16(uint16_t bits);
/* Decode `n` values of GGML type 0 (F32), 1 (F16) or 30 (BF16) from raw bytes
 * (forward/layer.go:279-303 readFloatVector).  Returns 0, or -1 on a bad type. */
int spo_decode_float_vector(const uint8_t *data, uint32_t type, int64_t n, float *dst);

/* Decode 17-byte MXFP4 blocks into 32 floats each, exactly as
 * decodeMXFP4Fast (forward/mxfp4_amd64.go:58-72). */
void spo_decode_mxfp4(const uint8_t *row, int64_t nblocks, float *out);

/* MXFP4 row . x in the reference AVX2 order (forward/mxfp4_amd64.go:11-26,
 * forward/quant_amd64.go:112-116): 32 FMA chains, fixed reduction tree.
 * `input` is the number of elements (multiple of 32). */
float spo_dot_mxfp4(const uint8_t *row, const float *x, int64_t input);
/* Same value computed with scalar fmaf lane emulation (independent check of
 * the AVX2-intrinsic version). */
float spo_dot_mxfp4_scalar(const uint8_t *row, const float *x, int64_t input);

/* Router dot of one little-endian F32 row (possibly unaligned bytes) with x:
 * dotF32AVX2 order when hidden%32==0 (forward/vector_amd64.go:28-56),
 * else the portable simd.Float32s order with `spo_portable_lanes` lanes
 * (forward/moe_batch.go:228-302). */
float spo_dot_router(const uint8_t *row, const float *x, int64_t hidden);

/* simd.Float32s width assumed for the portable (non-AVX2) reference paths:
 * router with hidden%32 != 0 and RMSNorm.  Default 8 (AVX2). */
void spo_set_portable_lanes(int lanes);
int spo_get_portable_lanes(void);

/* routeMoEBatch (forward/moe_batch.go:221-303): logits[t*E+e] =
 * dot(router row e, x[t]) + bias[e].  router = E rows x hidden F32 bytes. */
void spo_route(const uint8_t *router, const float *x, const float *bias,
               int64_t batch, int64_t hidden, int64_t experts, float *logits);

/* selectMoEBatch (forward/moe_batch.go:305-342) for one token. */
void spo_select(const float *logits, int64_t experts, int64_t k, spo_selection *sel);

/* gptOSSSwiGLU (forward/moe.go:66-70). */
float spo_swiglu(float gate, float up);

/* mulMoEBatchExpert (forward/mxfp4_batch.go:31-95):
 * y[yoff[j]+r] = dot(row r of data, x[xoff[j] : +input]) + bias[r],
 * r in [0,output), j in [0,count).  bias may be NULL (zeros).  workers <= 0
 * means 1.  Rows are split into contiguous ranges like the reference. */
void spo_mul_moe_batch_expert(const uint8_t *data, int64_t input, int64_t output,
                              const float *x, const int64_t *xoff, int64_t count,
                              const float *bias, float *y, const int64_t *yoff,
                              int workers);

/* Dense inputs for the whole block (already decoded/validated by the caller):
 *  router:      E x H F32 bytes (GGUF ffn_gate_inp, row e = expert e)
 *  router_bias: E floats or NULL
 *  gate/up:     E experts x D rows x (H/32) 17-byte MXFP4 blocks
 *  down:        E experts x H rows x (D/32) blocks
 *  gate_bias/up_bias: E x D floats or NULL; down_bias: E x H floats or NULL */
typedef struct spo_moe_weights {
  int64_t hidden, expert_dim, experts, top_k;
  const uint8_t *router;
  const float *router_bias;
  const uint8_t *gate, *up, *down;
  const float *gate_bias, *up_bias, *down_bias;
} spo_moe_weights;

/* forwardMoEBatch (forward/moe_batch.go:78-194) for `batch` tokens.
 * Optional outputs (may be NULL): logits [batch*E], selections [batch*k],
 * dispatch order `perm` [batch*k] (slots grouped by expert ascending, each
 * expert's slots in the reference's linked-list order = descending slot),
 * `expert_count` [E] (dispatched slots per expert), `act` [batch*k*D]
 * (SwiGLU activations by slot), `results` [batch*k*H] (down+bias by slot).
 * Returns the number of dispatched slots. */
int64_t spo_forward_moe_batch(const spo_moe_weights *w, const float *x, int64_t batch,
                              float *out, int workers, float *logits,
                              spo_selection *selections, int32_t *perm,
                              int32_t *expert_count, float *act, float *results);

/* Independent float64 reference (tests/testdata/forward/moe_sparse_test.go:18-76
 * scalarSparseMoE) for one token: stable-sort top-k on f64 logits (no router
 * bias), f64 softmax, f64 MXFP4 decode, clamped SwiGLU; biases ignored. */
void spo_scalar_sparse_moe_f64(const spo_moe_weights *w, const float *x, float *out);

/* normBatch RMSNorm (forward/layer_batch.go:139-195) with the portable lane
 * count: y = (x*w)*f, f = 1/float32(sqrt(float64(sum/float32(dim)+eps))). */
void spo_rmsnorm(const float *x, const float *weight, int64_t batch, int64_t dim,
                 float eps, float *y);
/* addVector (forward/layer.go:305-340): dst[i] += src[i]. */
void spo_add(float *dst, const float *src, int64_t n);

/* Q8_0 row dot (forward/quant_amd64.go:92-110 order). */
float spo_dot_q80(const uint8_t *row, const float *x, int64_t input);
/* MulQ80Into / MulQ80Argmax (forward/q80.go:22-148): logits for every row,
 * and the argmax with ties to the lowest row. Returns the argmax row. */
int64_t spo_mul_q80(const uint8_t *data, int64_t input, int64_t output, const float *x,
                    float *y, float *best_logit, int workers);

/* Q4_0 row dot, one input (forward/quant_amd64.go:75-90 order). */
float spo_dot_q40(const uint8_t *row, const float *x, int64_t input);
/* The batched order (forward/quant_amd64.go:118-148): y[item*output + row_index]. */
void spo_dot_q40_batch(const uint8_t *row, const float *x, float *y, int64_t input, int64_t output,
                       int64_t row_index, int64_t batch);
/* MulQ40BatchInto (forward/q40.go:46-101): batch 1 takes the one-input order,
 * larger batches the batched one; y is [batch][output]. */
void spo_mul_q40(const uint8_t *data, int64_t input, int64_t output, const float *x, int64_t batch, float *y,
                 int workers);

/* out[i] = fmaf(a[i], b[i], c[i]) (single rounding), for test references. */
void spo_fmaf_vec(const float *a, const float *b, const float *c, float *out, int64_t n);

/* ---- the benchmark's synthetic layer (spt_synth.c) ----------------------
 * Seeded GPT-OSS-style weights with the same bytes as the CUDA library's own
 * generator, so the CPU baseline needs nothing from the library under test. */
typedef struct spo_synth_params {
  uint64_t seed;
  float router_std, bias_std;
  uint8_t scale_lo, scale_hi;
  uint8_t expert_bias, router_bias;
  float zipf_s, zipf_beta;
} spo_synth_params;
/* One layer in GGUF tensor layout (any output may be NULL); MXFP4 tensors
 * are generated on `threads` threads.  Returns 0, or -1 on bad dimensions. */
int spo_synth_layer(const spo_synth_params *p, int64_t hidden, int64_t expert_dim, int64_t experts,
                    int64_t layer, uint8_t *router, float *router_bias, uint8_t *gate, uint8_t *up,
                    uint8_t *down, float *gate_bias, float *up_bias, float *down_bias, int threads);
void spo_synth_router_bias(const spo_synth_params *p, int64_t experts, int64_t layer, float *bias);
/* The MXFP4 blocks of experts ids[0..n_ids) only, written at their places in
 * whole-tensor buffers (gate/up E*D*(H/32)*17 bytes, down E*H*(D/32)*17;
 * any may be NULL); the rest is left untouched.  Returns 0 or -1. */
int spo_synth_experts(const spo_synth_params *p, int64_t hidden, int64_t expert_dim, int64_t experts, int64_t layer,
                      const int32_t *ids, int64_t n_ids, uint8_t *gate, uint8_t *up, uint8_t *down, int threads);
/* n Gaussians N(mean, sd) of tensor tag `tag` (activations: tag = stream). */
void spo_synth_normal(uint64_t seed, uint32_t tag, float mean, float sd, float *out, int64_t n);
/* RMSNorm weights N(1, 0.02) of a synthetic layer. */
void spo_synth_norm(uint64_t seed, int64_t layer, int64_t dim, float *out);

/* 1 if this build's AVX2 kernels are in use, else 0 (scalar fallback). */
int spo_has_avx2(void);

#ifdef __cplusplus
}
#endif
#endif
