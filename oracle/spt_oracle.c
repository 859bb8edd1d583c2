/*
 * spt_oracle.c -- CPU restatement of Stream-PT's MoE FFN path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); the
 * product never links it.  Each function names the reference file:line it
 * restates; paths are relative to the Stream-PT repository root.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, pthreads).  The AVX2
 * functions are compiled with target("avx2,fma") and selected at run time;
 * the scalar versions reproduce the same 8-lane chains with fmaf.
 */
#include "spt_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

/* ---- tables: forward/mxfp4.go:10-28 ------------------------------------ */

static float g_e8m0[256];
static float g_scaled[256][16];
static int g_init = 0;
static int g_avx2 = 0;
static int g_lanes = 8;

/* Run fn(ctx, i) for i in [0,n) on up to `workers` pthreads, contiguous
 * index ranges per worker (the reference's row partition,
 * forward/mxfp4_batch.go:34-51). */
typedef void (*spo_range_fn)(void *ctx, int64_t begin, int64_t end);
typedef struct { spo_range_fn fn; void *ctx; int64_t begin, end; } spo_job;
static void *spo_job_main(void *p) { spo_job *j = (spo_job *)p; j->fn(j->ctx, j->begin, j->end); return NULL; }
static void spo_parallel(int64_t n, int workers, spo_range_fn fn, void *ctx) {
  if (workers > n) workers = (int)n;
  if (workers <= 1) { if (n > 0) fn(ctx, 0, n); return; }
  pthread_t th[256];
  spo_job jobs[256];
  if (workers > 256) workers = 256;
  for (int w = 0; w < workers; w++) {
    jobs[w].fn = fn; jobs[w].ctx = ctx;
    jobs[w].begin = (int64_t)w * n / workers; jobs[w].end = (int64_t)(w + 1) * n / workers;
  }
  int started[256];
  for (int w = 1; w < workers; w++) started[w] = pthread_create(&th[w], NULL, spo_job_main, &jobs[w]) == 0;
  spo_job_main(&jobs[0]);
  for (int w = 1; w < workers; w++) { if (started[w]) pthread_join(th[w], NULL); else spo_job_main(&jobs[w]); }
}

static const float k_fp4[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

void spo_init(void) {
  if (g_init) return;
  for (int i = 0; i < 256; i++) {
    /* float32(math.Ldexp(1.0, i-127)): 2^128 rounds to +Inf. */
    volatile double d = ldexp(1.0, i - 127);
    g_e8m0[i] = (float)d;
    for (int j = 0; j < 16; j++) {
      volatile float s = g_e8m0[i];
      g_scaled[i][j] = s * k_fp4[j];
    }
  }
  __builtin_cpu_init();
  g_avx2 = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  g_init = 1;
}

int spo_has_avx2(void) { spo_init(); return g_avx2; }
void spo_set_portable_lanes(int lanes) { if (lanes > 0 && lanes <= 64) g_lanes = lanes; }
int spo_get_portable_lanes(void) { return g_lanes; }

float spo_e8m0(uint8_t b) { spo_init(); return g_e8m0[b]; }
float spo_scaled_fp4(uint8_t scale, uint8_t code) { spo_init(); return g_scaled[scale][code & 15]; }

static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* forward/q40.go:149-180 */
float spo_f16(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exponent = (bits >> 10) & 0x1f;
  uint32_t mantissa = bits & 0x03ff;
  if (exponent == 0) {
    if (mantissa == 0) return f32_from_bits(sign);
    uint32_t e = 113;
    while ((mantissa & 0x0400) == 0) { mantissa <<= 1; e--; }
    return f32_from_bits(sign | e << 23 | (mantissa & 0x03ff) << 13);
  }
  if (exponent == 31) return f32_from_bits(sign | 0x7f800000u | mantissa << 13);
  return f32_from_bits(sign | (exponent + 112) << 23 | mantissa << 13);
}

/* forward/layer.go:296 */
float spo_bf16(uint16_t bits) { return f32_from_bits((uint32_t)bits << 16); }

/* forward/layer.go:279-303 */
int spo_decode_float_vector(const uint8_t *data, uint32_t type, int64_t n, float *dst) {
  for (int64_t i = 0; i < n; i++) {
    if (type == 0) {
      uint32_t u; memcpy(&u, data + 4 * i, 4); dst[i] = f32_from_bits(u);
    } else if (type == 1) {
      uint16_t h; memcpy(&h, data + 2 * i, 2); dst[i] = spo_f16(h);
    } else if (type == 30) {
      uint16_t h; memcpy(&h, data + 2 * i, 2); dst[i] = spo_bf16(h);
    } else {
      return -1;
    }
  }
  return 0;
}

/* ---- MXFP4 decode: forward/mxfp4_amd64.go:43-72 --------------------------
 * Element i of a block is the low nibble of byte 1+i, element i+16 the high
 * nibble.  Value = scaledFP4Table[scale][code]; the AVX2 path gets negative
 * codes by XOR-ing the sign into the positive level, which is the same
 * number. */
void spo_decode_mxfp4(const uint8_t *row, int64_t nblocks, float *out) {
  spo_init();
  for (int64_t b = 0; b < nblocks; b++) {
    const uint8_t *enc = row + 17 * b;
    const float *lv = g_scaled[enc[0]];
    for (int i = 0; i < 16; i++) {
      uint8_t p = enc[1 + i];
      uint32_t lo = bits_from_f32(lv[p & 7]) ^ ((uint32_t)(p & 8) << 28);
      uint32_t hi = bits_from_f32(lv[(p >> 4) & 7]) ^ ((uint32_t)((p >> 4) & 8) << 28);
      out[32 * b + i] = f32_from_bits(lo);
      out[32 * b + 16 + i] = f32_from_bits(hi);
    }
  }
}

/* quantSumAVX2 (forward/quant_amd64.go:112-116) on an 8-lane vector s:
 * p[i] = s[i]+s[i+4]; ((p0+p1)+(p2+p3)). */
static inline float qsum8_scalar(const float s[8]) {
  float p0 = s[0] + s[4], p1 = s[1] + s[5], p2 = s[2] + s[6], p3 = s[3] + s[7];
  return (p0 + p1) + (p2 + p3);
}

/* 32 chains -> forward/mxfp4_amd64.go:25 a0.Add(a1).Add(a2).Add(a3) then qsum. */
static inline float reduce32_scalar(const float a[32]) {
  float s[8];
  for (int l = 0; l < 8; l++) s[l] = ((a[l] + a[8 + l]) + a[16 + l]) + a[24 + l];
  return qsum8_scalar(s);
}

float spo_dot_mxfp4_scalar(const uint8_t *row, const float *x, int64_t input) {
  spo_init();
  float a[32];
  for (int c = 0; c < 32; c++) a[c] = 0.0f;
  float w[32];
  for (int64_t b = 0; b < input / 32; b++) {
    spo_decode_mxfp4(row + 17 * b, 1, w);
    for (int c = 0; c < 32; c++) a[c] = fmaf(w[c], x[32 * b + c], a[c]);
  }
  return reduce32_scalar(a);
}

__attribute__((target("avx2,fma"))) static inline float qsum_avx(__m256 v) {
  __m128 p = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  p = _mm_hadd_ps(p, p);
  p = _mm_hadd_ps(p, p);
  return _mm_cvtss_f32(p);
}

/* mxfp4BlockAVX2 (forward/mxfp4_amd64.go:43-56). */
__attribute__((target("avx2,fma"))) static inline void block_avx(const uint8_t *enc, __m256 *w0,
                                                                 __m256 *w1, __m256 *w2,
                                                                 __m256 *w3) {
  __m256 levels = _mm256_loadu_ps(g_scaled[enc[0]]);
  __m128i packed = _mm_loadu_si128((const __m128i *)(enc + 1));
  __m256i a = _mm256_cvtepu8_epi32(packed);
  __m256i b = _mm256_cvtepu8_epi32(_mm_srli_si128(packed, 8));
  __m256i ha = _mm256_srli_epi32(a, 4), hb = _mm256_srli_epi32(b, 4);
  __m256i sign = _mm256_set1_epi32(8);
#define SPO_LV(idx)                                                                      \
  _mm256_castsi256_ps(_mm256_xor_si256(                                                  \
      _mm256_castps_si256(_mm256_permutevar8x32_ps(levels, idx)),                        \
      _mm256_slli_epi32(_mm256_and_si256(idx, sign), 28)))
  *w0 = SPO_LV(a);
  *w1 = SPO_LV(b);
  *w2 = SPO_LV(ha);
  *w3 = SPO_LV(hb);
#undef SPO_LV
}

/* dotMXFP4Fast (forward/mxfp4_amd64.go:11-26). */
__attribute__((target("avx2,fma"))) static float dot_mxfp4_avx(const uint8_t *row, const float *x,
                                                               int64_t input) {
  __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
  for (int64_t b = 0; b < input / 32; b++) {
    __m256 w0, w1, w2, w3;
    block_avx(row + 17 * b, &w0, &w1, &w2, &w3);
    const float *in = x + 32 * b;
    a0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(in), a0);
    a1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(in + 8), a1);
    a2 = _mm256_fmadd_ps(w2, _mm256_loadu_ps(in + 16), a2);
    a3 = _mm256_fmadd_ps(w3, _mm256_loadu_ps(in + 24), a3);
  }
  return qsum_avx(_mm256_add_ps(_mm256_add_ps(_mm256_add_ps(a0, a1), a2), a3));
}

/* dotMoEBatchDecodedFast (forward/mxfp4_amd64.go:28-41): same chains over a
 * pre-decoded fp32 row. */
__attribute__((target("avx2,fma"))) static float dot_decoded_avx(const float *w, const float *x,
                                                                 int64_t input) {
  __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
  for (int64_t o = 0; o < input; o += 32) {
    a0 = _mm256_fmadd_ps(_mm256_loadu_ps(w + o), _mm256_loadu_ps(x + o), a0);
    a1 = _mm256_fmadd_ps(_mm256_loadu_ps(w + o + 8), _mm256_loadu_ps(x + o + 8), a1);
    a2 = _mm256_fmadd_ps(_mm256_loadu_ps(w + o + 16), _mm256_loadu_ps(x + o + 16), a2);
    a3 = _mm256_fmadd_ps(_mm256_loadu_ps(w + o + 24), _mm256_loadu_ps(x + o + 24), a3);
  }
  return qsum_avx(_mm256_add_ps(_mm256_add_ps(_mm256_add_ps(a0, a1), a2), a3));
}

static float dot_decoded_scalar(const float *w, const float *x, int64_t input) {
  float a[32];
  for (int c = 0; c < 32; c++) a[c] = 0.0f;
  for (int64_t o = 0; o < input; o += 32)
    for (int c = 0; c < 32; c++) a[c] = fmaf(w[o + c], x[o + c], a[c]);
  return reduce32_scalar(a);
}

float spo_dot_mxfp4(const uint8_t *row, const float *x, int64_t input) {
  spo_init();
  return g_avx2 ? dot_mxfp4_avx(row, x, input) : spo_dot_mxfp4_scalar(row, x, input);
}

static float dot_decoded(const float *w, const float *x, int64_t input) {
  return g_avx2 ? dot_decoded_avx(w, x, input) : dot_decoded_scalar(w, x, input);
}

/* ---- router: forward/vector_amd64.go:11-56, forward/moe_batch.go:228-302 -- */

static inline float load_f32_le(const uint8_t *p) { uint32_t u; memcpy(&u, p, 4); return f32_from_bits(u); }

/* dotF32AVX2 order restated with scalar fmaf lanes: 64 chains c = 8j+l. */
static float dot_router_exact(const uint8_t *row, const float *x, int64_t hidden) {
  float a[64];
  for (int c = 0; c < 64; c++) a[c] = 0.0f;
  int64_t o = 0;
  for (; o + 64 <= hidden; o += 64)
    for (int c = 0; c < 64; c++) a[c] = fmaf(load_f32_le(row + 4 * (o + c)), x[o + c], a[c]);
  for (; o < hidden; o += 32) /* tail of 32 into a0..a3 */
    for (int c = 0; c < 32; c++) a[c] = fmaf(load_f32_le(row + 4 * (o + c)), x[o + c], a[c]);
  float s[8];
  for (int l = 0; l < 8; l++) {
    float sum0 = ((a[l] + a[8 + l]) + a[16 + l]) + a[24 + l];
    float sum1 = ((a[32 + l] + a[40 + l]) + a[48 + l]) + a[56 + l];
    s[l] = sum0 + sum1;
  }
  return qsum8_scalar(s);
}

/* Portable simd.Float32s order: `lanes` chains, zero-padded tail, then a
 * sequential sum of the lanes (forward/moe_batch.go:240-254, 291-300). */
static float dot_router_portable(const uint8_t *row, const float *x, int64_t hidden) {
  int L = g_lanes;
  float acc[64];
  for (int l = 0; l < L; l++) acc[l] = 0.0f;
  for (int64_t o = 0; o < hidden; o += L) {
    for (int l = 0; l < L; l++) {
      float w = 0.0f, v = 0.0f;
      if (o + l < hidden) { w = load_f32_le(row + 4 * (o + l)); v = x[o + l]; }
      acc[l] = fmaf(w, v, acc[l]);
    }
  }
  float sum = 0.0f;
  for (int l = 0; l < L; l++) sum += acc[l];
  return sum;
}

float spo_dot_router(const uint8_t *row, const float *x, int64_t hidden) {
  spo_init();
  if (hidden % 32 == 0) return dot_router_exact(row, x, hidden);
  return dot_router_portable(row, x, hidden);
}

typedef struct { const uint8_t *router; const float *x, *bias; int64_t batch, hidden, experts; float *logits; } route_ctx;
static void route_range(void *p, int64_t begin, int64_t end) {
  route_ctx *c = (route_ctx *)p;
  for (int64_t e = begin; e < end; e++)
    for (int64_t t = 0; t < c->batch; t++)
      c->logits[t * c->experts + e] =
          spo_dot_router(c->router + 4 * c->hidden * e, c->x + c->hidden * t, c->hidden) +
          (c->bias ? c->bias[e] : 0.0f);
}

static int g_route_workers = 1;
void spo_route(const uint8_t *router, const float *x, const float *bias, int64_t batch,
               int64_t hidden, int64_t experts, float *logits) {
  spo_init();
  route_ctx c = {router, x, bias, batch, hidden, experts, logits};
  spo_parallel(experts, g_route_workers, route_range, &c);
}

/* ---- selectMoEBatch: forward/moe_batch.go:305-342 ----------------------- */
void spo_select(const float *logits, int64_t experts, int64_t k, spo_selection *sel) {
  for (int64_t r = 0; r < k; r++) {
    int64_t best = -1;
    float value = -INFINITY;
    for (int64_t e = 0; e < experts; e++) {
      int already = 0;
      for (int64_t p = 0; p < r; p++)
        if (sel[p].index == e) { already = 1; break; }
      if (!already && logits[e] > value) { best = e; value = logits[e]; }
    }
    if (best < 0) { best = r; value = 0.0f; }
    sel[r].index = (int32_t)best;
    sel[r].weight = value;
  }
  float maxl = -INFINITY;
  for (int64_t r = 0; r < k; r++)
    if (sel[r].weight > maxl) maxl = sel[r].weight;
  float sum = 0.0f;
  for (int64_t r = 0; r < k; r++) {
    float d = sel[r].weight - maxl;
    sel[r].weight = (float)exp((double)d);
    sum += sel[r].weight;
  }
  if (sum > 0.0f) {
    float inv = 1.0f / sum;
    for (int64_t r = 0; r < k; r++) sel[r].weight *= inv;
  }
}

/* ---- gptOSSSwiGLU: forward/moe.go:66-70 ---------------------------------
 * Go's min/max propagate NaN; -1.702 is rounded to float32 first. */
static inline float go_min(float a, float b) { return (a != a || b != b) ? NAN : (a < b ? a : b); }
static inline float go_max(float a, float b) { return (a != a || b != b) ? NAN : (a > b ? a : b); }

float spo_swiglu(float gate, float up) {
  gate = go_min(gate, 7.0f);
  up = go_max(-7.0f, go_min(up, 7.0f));
  float t = -1.702f * gate;
  float e = (float)exp((double)t);
  float d = 1.0f + e;
  return gate / d * (up + 1.0f);
}

/* ---- mulMoEBatchExpert: forward/mxfp4_batch.go:31-95 -------------------- */
typedef struct {
  const uint8_t *data; int64_t input; const float *x; const int64_t *xoff; int64_t count;
  const float *bias; float *y; const int64_t *yoff;
} mul_ctx;
static void mul_range(void *p, int64_t begin, int64_t end) {
  mul_ctx *c = (mul_ctx *)p;
  int64_t row_bytes = c->input / 32 * 17;
  float *dec = c->count > 1 ? (float *)malloc(sizeof(float) * (size_t)c->input) : NULL;
  for (int64_t r = begin; r < end; r++) {
    const uint8_t *row = c->data + r * row_bytes;
    float b = c->bias ? c->bias[r] : 0.0f;
    if (c->count == 1) {
      c->y[c->yoff[0] + r] = spo_dot_mxfp4(row, c->x + c->xoff[0], c->input) + b;
    } else {
      spo_decode_mxfp4(row, c->input / 32, dec);
      for (int64_t j = 0; j < c->count; j++)
        c->y[c->yoff[j] + r] = dot_decoded(dec, c->x + c->xoff[j], c->input) + b;
    }
  }
  free(dec);
}

void spo_mul_moe_batch_expert(const uint8_t *data, int64_t input, int64_t output, const float *x,
                              const int64_t *xoff, int64_t count, const float *bias, float *y,
                              const int64_t *yoff, int workers) {
  spo_init();
  mul_ctx c = {data, input, x, xoff, count, bias, y, yoff};
  spo_parallel(output, workers < 1 ? 1 : workers, mul_range, &c);
}

/* ---- forwardMoEBatch: forward/moe_batch.go:78-194, moe_schedule.go:25-127 */
int64_t spo_forward_moe_batch(const spo_moe_weights *w, const float *x, int64_t batch, float *out,
                              int workers, float *logits_out, spo_selection *sel_out,
                              int32_t *perm_out, int32_t *count_out, float *act_out,
                              float *results_out) {
  spo_init();
  const int64_t H = w->hidden, D = w->expert_dim, E = w->experts, K = w->top_k;
  const int64_t S = batch * K;
  float *logits = (float *)malloc(sizeof(float) * (size_t)(batch * E));
  spo_selection *sel = (spo_selection *)malloc(sizeof(spo_selection) * (size_t)S);
  int64_t *heads = (int64_t *)malloc(sizeof(int64_t) * (size_t)E);
  int64_t *next = (int64_t *)malloc(sizeof(int64_t) * (size_t)(S > 0 ? S : 1));
  float *gate = (float *)calloc((size_t)(S * D), sizeof(float));
  float *up = (float *)calloc((size_t)(S * D), sizeof(float));
  float *act = (float *)calloc((size_t)(S * D), sizeof(float));
  float *res = (float *)calloc((size_t)(S * H), sizeof(float));

  g_route_workers = workers < 1 ? 1 : workers;
  spo_route(w->router, x, w->router_bias, batch, H, E, logits);
  g_route_workers = 1;
  for (int64_t e = 0; e < E; e++) heads[e] = -1;
  for (int64_t t = 0; t < batch; t++) {
    spo_select(logits + t * E, E, K, sel + t * K);
    for (int64_t r = 0; r < K; r++) {
      int64_t idx = t * K + r;
      if (sel[idx].weight <= 0.0f) continue; /* NaN is kept */
      next[idx] = heads[sel[idx].index];
      heads[sel[idx].index] = idx;
    }
  }
  int64_t dispatched = 0;
  int64_t xoff[16], yoff[16];
  /* gate and up (moe_schedule.go:31-68), tiles of moeBatchTile=16 slots */
  for (int pass = 0; pass < 3; pass++) {
    for (int64_t e = 0; e < E; e++) {
      int64_t head = heads[e];
      while (head >= 0) {
        int64_t count = 0;
        while (head >= 0 && count < 16) {
          if (pass < 2) { xoff[count] = head / K * H; yoff[count] = head * D; }
          else { xoff[count] = head * D; yoff[count] = head * H; }
          head = next[head];
          count++;
        }
        if (pass == 0)
          spo_mul_moe_batch_expert(w->gate + e * D * (H / 32 * 17), H, D, x, xoff, count,
                                   w->gate_bias ? w->gate_bias + e * D : NULL, gate, yoff, workers);
        else if (pass == 1)
          spo_mul_moe_batch_expert(w->up + e * D * (H / 32 * 17), H, D, x, xoff, count,
                                   w->up_bias ? w->up_bias + e * D : NULL, up, yoff, workers);
        else
          spo_mul_moe_batch_expert(w->down + e * H * (D / 32 * 17), D, H, act, xoff, count,
                                   w->down_bias ? w->down_bias + e * H : NULL, res, yoff, workers);
      }
    }
    if (pass == 1) {
      /* SwiGLU for every dispatched slot (moe_schedule.go:69-80) */
      for (int64_t idx = 0; idx < S; idx++) {
        if (sel[idx].weight <= 0.0f) continue;
        for (int64_t i = idx * D; i < idx * D + D; i++) act[i] = spo_swiglu(gate[i], up[i]);
      }
    }
  }
  /* combine (moe_batch.go:163-192) */
  memset(out, 0, sizeof(float) * (size_t)(batch * H));
  for (int64_t t = 0; t < batch; t++)
    for (int64_t r = 0; r < K; r++) {
      int64_t idx = t * K + r;
      float wt = sel[idx].weight;
      if (wt <= 0.0f) continue;
      for (int64_t h = 0; h < H; h++) out[t * H + h] = fmaf(res[idx * H + h], wt, out[t * H + h]);
    }
  /* dispatch order: experts ascending, each list from its head */
  for (int64_t e = 0; e < E; e++) {
    int64_t n = 0;
    for (int64_t s = heads[e]; s >= 0; s = next[s]) {
      if (perm_out) perm_out[dispatched] = (int32_t)s;
      dispatched++;
      n++;
    }
    if (count_out) count_out[e] = (int32_t)n;
  }
  if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)(batch * E));
  if (sel_out) memcpy(sel_out, sel, sizeof(spo_selection) * (size_t)S);
  if (act_out) memcpy(act_out, act, sizeof(float) * (size_t)(S * D));
  if (results_out) memcpy(results_out, res, sizeof(float) * (size_t)(S * H));
  free(logits); free(sel); free(heads); free(next); free(gate); free(up); free(act); free(res);
  return dispatched;
}

/* ---- independent f64 oracle: moe_sparse_test.go:18-76 ------------------- */
static void project_f64(const uint8_t *mat, int64_t rows, int64_t input, const double *in,
                        double *out) {
  static const double lv[16] = {0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6};
  int64_t blocks = input / 32;
  for (int64_t r = 0; r < rows; r++) {
    double acc = 0.0;
    for (int64_t b = 0; b < blocks; b++) {
      const uint8_t *enc = mat + (r * blocks + b) * 17;
      double scale = ldexp(1.0, (int)enc[0] - 127);
      for (int i = 0; i < 16; i++) {
        uint8_t p = enc[1 + i];
        acc += scale * lv[p & 15] * in[b * 32 + i];
        acc += scale * lv[p >> 4] * in[b * 32 + i + 16];
      }
    }
    out[r] = acc;
  }
}

void spo_scalar_sparse_moe_f64(const spo_moe_weights *w, const float *x, float *result) {
  const int64_t H = w->hidden, D = w->expert_dim, E = w->experts, K = w->top_k;
  double *logits = (double *)calloc((size_t)E, sizeof(double));
  int64_t *order = (int64_t *)malloc(sizeof(int64_t) * (size_t)E);
  for (int64_t e = 0; e < E; e++) {
    order[e] = e;
    for (int64_t i = 0; i < H; i++)
      logits[e] += (double)load_f32_le(w->router + 4 * (e * H + i)) * (double)x[i];
  }
  /* stable sort descending (insertion sort keeps equal keys in order) */
  for (int64_t i = 1; i < E; i++) {
    int64_t v = order[i], j = i - 1;
    while (j >= 0 && logits[order[j]] < logits[v]) { order[j + 1] = order[j]; j--; }
    order[j + 1] = v;
  }
  double *wts = (double *)malloc(sizeof(double) * (size_t)K);
  double total = 0;
  for (int64_t r = 0; r < K; r++) {
    wts[r] = exp(logits[order[r]] - logits[order[0]]);
    total += wts[r];
  }
  double *in = (double *)malloc(sizeof(double) * (size_t)H);
  for (int64_t i = 0; i < H; i++) in[i] = (double)x[i];
  double *g = (double *)malloc(sizeof(double) * (size_t)D);
  double *u = (double *)malloc(sizeof(double) * (size_t)D);
  double *dn = (double *)malloc(sizeof(double) * (size_t)H);
  for (int64_t i = 0; i < H; i++) result[i] = 0.0f;
  for (int64_t r = 0; r < K; r++) {
    int64_t e = order[r];
    project_f64(w->gate + e * D * (H / 32 * 17), D, H, in, g);
    project_f64(w->up + e * D * (H / 32 * 17), D, H, in, u);
    for (int64_t i = 0; i < D; i++) {
      double gg = g[i] < 7 ? g[i] : 7;
      double uu = u[i] < 7 ? u[i] : 7;
      uu = uu > -7 ? uu : -7;
      g[i] = gg / (1 + exp(-1.702 * gg)) * (uu + 1);
    }
    project_f64(w->down + e * H * (D / 32 * 17), H, D, g, dn);
    for (int64_t i = 0; i < H; i++) result[i] += (float)(dn[i] * wts[r] / total);
  }
  free(logits); free(order); free(wts); free(in); free(g); free(u); free(dn);
}

/* ---- RMSNorm + residual: forward/layer_batch.go:139-195, layer.go:305-340 */
void spo_rmsnorm(const float *x, const float *weight, int64_t batch, int64_t dim, float eps,
                 float *y) {
  int L = g_lanes;
  for (int64_t t = 0; t < batch; t++) {
    const float *in = x + t * dim;
    float sq[64];
    for (int l = 0; l < L; l++) sq[l] = 0.0f;
    for (int64_t o = 0; o < dim; o += L)
      for (int l = 0; l < L; l++) {
        float v = (o + l < dim) ? in[o + l] : 0.0f;
        sq[l] = fmaf(v, v, sq[l]);
      }
    float sum = 0.0f;
    for (int l = 0; l < L; l++) sum += sq[l];
    float q = sum / (float)dim + eps;
    float f = 1.0f / (float)sqrt((double)q);
    for (int64_t i = 0; i < dim; i++) y[t * dim + i] = (in[i] * weight[i]) * f;
  }
}

void spo_add(float *dst, const float *src, int64_t n) {
  for (int64_t i = 0; i < n; i++) dst[i] = dst[i] + src[i];
}

/* ---- Q8_0: forward/quant_amd64.go:92-110, forward/q80.go:22-148 -------- */
/* The Q8_0 and Q4_0 dots are built twice (x86-64-v3 and baseline, chosen at
 * load time): with FMA in the instruction set each fmaf is one instruction
 * instead of a library call.  The arithmetic is the same either way (fmaf
 * is exact-rounded, and -ffp-contract=off keeps every other operation as
 * written), so only the speed of the CPU baseline changes. */
#define SPO_CLONES __attribute__((target_clones("arch=x86-64-v3", "default")))

SPO_CLONES float spo_dot_q80(const uint8_t *row, const float *x, int64_t input) {
  float a[32];
  for (int c = 0; c < 32; c++) a[c] = 0.0f;
  for (int64_t b = 0; b < input / 32; b++) {
    const uint8_t *enc = row + 34 * b;
    uint16_t hb; memcpy(&hb, enc, 2);
    float scale = spo_f16(hb);
    for (int c = 0; c < 32; c++) {
      float wv = (float)(int8_t)enc[2 + c] * scale;
      a[c] = fmaf(wv, x[32 * b + c], a[c]);
    }
  }
  return reduce32_scalar(a);
}

typedef struct { const uint8_t *data; int64_t input; const float *x; float *y; } q80_ctx;
static void q80_range(void *p, int64_t begin, int64_t end) {
  q80_ctx *c = (q80_ctx *)p;
  int64_t row_bytes = c->input / 32 * 34;
  for (int64_t r = begin; r < end; r++) c->y[r] = spo_dot_q80(c->data + r * row_bytes, c->x, c->input);
}

int64_t spo_mul_q80(const uint8_t *data, int64_t input, int64_t output, const float *x, float *y,
                    float *best_logit, int workers) {
  q80_ctx c = {data, input, x, y};
  spo_parallel(output, workers < 1 ? 1 : workers, q80_range, &c);
  int64_t best = 0;
  float bl = -INFINITY;
  for (int64_t r = 0; r < output; r++)
    if (y[r] > bl) { bl = y[r]; best = r; }
  if (best_logit) *best_logit = bl;
  return best;
}

/* ---- Q4_0: forward/quant_amd64.go:65-90 (one input), :118-148 (a batch),
 * forward/q40.go:35-101 ------------------------------------------------- */
/* quantQ40WeightsAVX2 (forward/quant_amd64.go:65-73): element c of a block is
 * the low nibble of byte c (c < 16) or the high nibble of byte c - 16, and
 * its weight is (nibble - 8) * scale, exact in fp32. */
static void q40_decode(const uint8_t *enc, float w[32]) {
  uint16_t hb; memcpy(&hb, enc, 2);
  const float scale = spo_f16(hb);
  for (int i = 0; i < 16; i++) {
    w[i] = (float)((int)(enc[2 + i] & 15) - 8) * scale;
    w[16 + i] = (float)((int)(enc[2 + i] >> 4) - 8) * scale;
  }
}

/* quantQ40AVX2 (forward/quant_amd64.go:75-90): chain c takes element c of
 * every block; a0+a1+a2+a3, then quantSumAVX2. */
SPO_CLONES float spo_dot_q40(const uint8_t *row, const float *x, int64_t input) {
  float a[32], w[32];
  for (int c = 0; c < 32; c++) a[c] = 0.0f;
  for (int64_t b = 0; b < input / 32; b++) {
    q40_decode(row + 18 * b, w);
    for (int c = 0; c < 32; c++) a[c] = fmaf(w[c], x[32 * b + c], a[c]);
  }
  return reduce32_scalar(a);
}

/* quantDotQ40Batch (forward/quant_amd64.go:118-148): one 8-lane accumulator
 * per item; lane l takes elements l, 8+l, 16+l, 24+l of each block in that
 * order, then quantSumAVX2.  Writes y[item * output + row_index]. */
SPO_CLONES void spo_dot_q40_batch(const uint8_t *row, const float *x, float *y, int64_t input, int64_t output,
                       int64_t row_index, int64_t batch) {
  float w[32];
  for (int64_t item = 0; item < batch; item++) {
    const float *v = x + item * input;
    float acc[8];
    for (int l = 0; l < 8; l++) acc[l] = 0.0f;
    for (int64_t b = 0; b < input / 32; b++) {
      q40_decode(row + 18 * b, w);
      for (int l = 0; l < 8; l++)
        for (int j = 0; j < 4; j++) acc[l] = fmaf(w[8 * j + l], v[32 * b + 8 * j + l], acc[l]);
    }
    y[item * output + row_index] = qsum8_scalar(acc);
  }
}

typedef struct { const uint8_t *data; int64_t input, output, batch; const float *x; float *y; } q40_ctx;
static void q40_range(void *p, int64_t begin, int64_t end) {
  q40_ctx *c = (q40_ctx *)p;
  const int64_t row_bytes = c->input / 32 * 18;
  for (int64_t r = begin; r < end; r++) {
    const uint8_t *row = c->data + r * row_bytes;
    if (c->batch == 1)
      c->y[r] = spo_dot_q40(row, c->x, c->input);
    else
      spo_dot_q40_batch(row, c->x, c->y, c->input, c->output, r, c->batch);
  }
}

void spo_mul_q40(const uint8_t *data, int64_t input, int64_t output, const float *x, int64_t batch, float *y,
                 int workers) {
  q40_ctx c = {data, input, output, batch, x, y};
  spo_parallel(output, workers < 1 ? 1 : workers, q40_range, &c);
}

void spo_fmaf_vec(const float *a, const float *b, const float *c, float *out, int64_t n) {
  for (int64_t i = 0; i < n; i++) out[i] = fmaf(a[i], b[i], c[i]);
}
