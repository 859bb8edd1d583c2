/*
 * spt_synth.c -- the benchmark's seeded synthetic GPT-OSS layer, generated on
 * the host by the oracle itself.
 *
 * TEST INFRASTRUCTURE ONLY (part of libspt_oracle.so).  The CPU baseline and
 * the reference arm of bench.py build their weights here, so that timing the
 * reference's arithmetic never loads the CUDA library under test.  The bytes
 * equal those of the product's own generator (spt_synth_layer_host and the
 * device arena); tests/test_oracle_synth.py checks that on every tensor.
 *
 * Generator (not reference code: the reference ships no synthetic weights):
 *   - Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers:
 *     as easy as 1, 2, 3", SC'11): 10 rounds, multipliers 0xD2511F53 and
 *     0xCD9E8D57, Weyl key increments 0x9E3779B9 and 0xBB67AE85; key = the
 *     seed's two 32-bit halves; counter = (index lo, index hi, tag, stream
 *     word).  tag = layer << 8 | tensor kind.
 *   - MXFP4 block i of a tensor: counter word 3 = 0 gives the 16 nibble
 *     bytes (little-endian words), word 3 = 1 the scale byte lo +
 *     floor(x * span / 2^32).
 *   - Gaussians: counter word 3 = 2, Box-Muller in double
 *     (u1 = (a + 1) / 2^32, u2 = b / 2^32, z = sqrt(-2 ln u1) cos(2 pi u2)),
 *     mean + std * z rounded to float.
 *   - Zipf skew of the router bias: a Fisher-Yates permutation of ranks
 *     1..E driven by the same generator (kind 8), bias[e] += beta * (-s *
 *     ln(rank[e])) in double.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "spt_oracle.h"

enum {
  kGate = 0,
  kUp = 1,
  kDown = 2,
  kRouter = 3,
  kRouterBias = 4,
  kGateBias = 5,
  kUpBias = 6,
  kDownBias = 7,
  kZipfPerm = 8,
  kNormWeight = 9
};

typedef struct {
  uint32_t v[4];
} word4;

static word4 philox(word4 c, uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c.v[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c.v[2];
    word4 n;
    n.v[0] = (uint32_t)(p1 >> 32) ^ c.v[1] ^ k0;
    n.v[1] = (uint32_t)p1;
    n.v[2] = (uint32_t)(p0 >> 32) ^ c.v[3] ^ k1;
    n.v[3] = (uint32_t)p0;
    c = n;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

static uint32_t tag_of(int64_t layer, uint32_t kind) { return ((uint32_t)layer << 8) | kind; }

static void block17(uint64_t seed, uint32_t tag, uint64_t index, uint8_t lo, uint8_t hi, uint8_t *out) {
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  word4 c = {{(uint32_t)index, (uint32_t)(index >> 32), tag, 0u}};
  const word4 nib = philox(c, k0, k1);
  c.v[3] = 1u;
  const word4 sc = philox(c, k0, k1);
  const uint32_t span = (uint32_t)hi - (uint32_t)lo + 1u;
  out[0] = (uint8_t)(lo + (uint32_t)(((uint64_t)sc.v[0] * span) >> 32));
  for (int i = 0; i < 16; ++i) out[1 + i] = (uint8_t)(nib.v[i >> 2] >> (8 * (i & 3)));
}

static float gaussian(uint64_t seed, uint32_t tag, uint64_t index, float mean, float sd) {
  word4 c = {{(uint32_t)index, (uint32_t)(index >> 32), tag, 2u}};
  const word4 r = philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const double u1 = ((double)r.v[0] + 1.0) / 4294967296.0;
  const double u2 = (double)r.v[1] / 4294967296.0;
  const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
  return (float)((double)mean + (double)sd * z);
}

void spo_synth_normal(uint64_t seed, uint32_t tag, float mean, float sd, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = gaussian(seed, tag, (uint64_t)i, mean, sd);
}

/* MXFP4 tensors are large (1.7 GB per GPT-OSS layer): split them over threads. */
typedef struct {
  uint64_t seed;
  uint32_t tag;
  uint8_t lo, hi;
  uint8_t *dst;
  int64_t begin, end;
} blocks_job;

static void *blocks_run(void *p) {
  const blocks_job *j = (const blocks_job *)p;
  for (int64_t i = j->begin; i < j->end; ++i) block17(j->seed, j->tag, (uint64_t)i, j->lo, j->hi, j->dst + 17 * i);
  return NULL;
}

static void synth_blocks(uint64_t seed, uint32_t tag, uint8_t lo, uint8_t hi, uint8_t *dst, int64_t n,
                         int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (n < 4096 || threads == 1) {
    blocks_job j = {seed, tag, lo, hi, dst, 0, n};
    blocks_run(&j);
    return;
  }
  pthread_t tid[256];
  int made[256];
  blocks_job job[256];
  for (int t = 0; t < threads; ++t) {
    job[t] = (blocks_job){seed, tag, lo, hi, dst, n * t / threads, n * (t + 1) / threads};
    made[t] = pthread_create(&tid[t], NULL, blocks_run, &job[t]) == 0;
    if (!made[t]) blocks_run(&job[t]);
  }
  for (int t = 0; t < threads; ++t)
    if (made[t]) pthread_join(tid[t], NULL);
}

void spo_synth_router_bias(const spo_synth_params *p, int64_t experts, int64_t layer, float *bias) {
  if (p->router_bias) spo_synth_normal(p->seed, tag_of(layer, kRouterBias), 0.0f, p->bias_std, bias, experts);
  else memset(bias, 0, sizeof(float) * (size_t)experts);
  if (p->zipf_s > 0.0f) {
    int64_t *rank = (int64_t *)malloc(sizeof(int64_t) * (size_t)experts);
    for (int64_t i = 0; i < experts; ++i) rank[i] = i + 1;
    for (int64_t i = experts - 1; i > 0; --i) {
      word4 c = {{(uint32_t)i, (uint32_t)((uint64_t)i >> 32), tag_of(layer, kZipfPerm), 2u}};
      const word4 r = philox(c, (uint32_t)p->seed, (uint32_t)(p->seed >> 32));
      const int64_t j = (int64_t)(((uint64_t)r.v[0] * (uint64_t)(i + 1)) >> 32);
      const int64_t t = rank[i];
      rank[i] = rank[j];
      rank[j] = t;
    }
    for (int64_t e = 0; e < experts; ++e)
      bias[e] = (float)((double)bias[e] + (double)p->zipf_beta * (-(double)p->zipf_s * log((double)rank[e])));
    free(rank);
  }
}

int spo_synth_layer(const spo_synth_params *p, int64_t hidden, int64_t expert_dim, int64_t experts, int64_t layer,
                    uint8_t *router, float *router_bias, uint8_t *gate, uint8_t *up, uint8_t *down,
                    float *gate_bias, float *up_bias, float *down_bias, int threads) {
  const int64_t H = hidden, D = expert_dim, E = experts;
  if (!p || H <= 0 || D <= 0 || E <= 0 || H % 32 != 0 || D % 32 != 0) return -1;
  if (router) {
    float *w = (float *)malloc(sizeof(float) * (size_t)(E * H));
    if (!w) return -1;
    spo_synth_normal(p->seed, tag_of(layer, kRouter), 0.0f, p->router_std, w, E * H);
    memcpy(router, w, sizeof(float) * (size_t)(E * H));
    free(w);
  }
  if (router_bias) spo_synth_router_bias(p, E, layer, router_bias);
  struct {
    uint32_t kind;
    int64_t n;
    float *dst;
  } biases[3] = {{kGateBias, E * D, gate_bias}, {kUpBias, E * D, up_bias}, {kDownBias, E * H, down_bias}};
  for (int i = 0; i < 3; ++i) {
    if (!biases[i].dst) continue;
    if (p->expert_bias) spo_synth_normal(p->seed, tag_of(layer, biases[i].kind), 0.0f, p->bias_std, biases[i].dst,
                                         biases[i].n);
    else memset(biases[i].dst, 0, sizeof(float) * (size_t)biases[i].n);
  }
  struct {
    uint32_t kind;
    int64_t blocks;
    uint8_t *dst;
  } mats[3] = {{kGate, E * D * (H / 32), gate}, {kUp, E * D * (H / 32), up}, {kDown, E * H * (D / 32), down}};
  for (int i = 0; i < 3; ++i)
    if (mats[i].dst)
      synth_blocks(p->seed, tag_of(layer, mats[i].kind), p->scale_lo, p->scale_hi, mats[i].dst, mats[i].blocks,
                   threads);
  return 0;
}

int spo_synth_experts(const spo_synth_params *p, int64_t hidden, int64_t expert_dim, int64_t experts, int64_t layer,
                      const int32_t *ids, int64_t n_ids, uint8_t *gate, uint8_t *up, uint8_t *down, int threads) {
  const int64_t H = hidden, D = expert_dim, E = experts;
  if (!p || H <= 0 || D <= 0 || E <= 0 || H % 32 != 0 || D % 32 != 0) return -1;
  const int64_t gu = D * (H / 32), dn = H * (D / 32);  // blocks per expert
  for (int64_t i = 0; i < n_ids; ++i) {
    const int64_t e = ids[i];
    if (e < 0 || e >= E) return -1;
    /* block b of expert e is block e * per + b of the tensor: same bytes as the whole-tensor generator */
    struct {
      uint32_t kind;
      int64_t per;
      uint8_t *dst;
    } mats[3] = {{kGate, gu, gate}, {kUp, gu, up}, {kDown, dn, down}};
    for (int m = 0; m < 3; ++m) {
      if (!mats[m].dst) continue;
      blocks_job j = {p->seed, tag_of(layer, mats[m].kind), p->scale_lo, p->scale_hi, mats[m].dst,
                      e * mats[m].per, (e + 1) * mats[m].per};
      if (threads > 1) {
        /* split this expert's blocks over threads */
        const int64_t n = mats[m].per;
        pthread_t tid[64];
        int made[64];
        blocks_job job[64];
        int th = threads > 64 ? 64 : threads;
        for (int t = 0; t < th; ++t) {
          job[t] = j;
          job[t].begin = e * n + n * t / th;
          job[t].end = e * n + n * (t + 1) / th;
          made[t] = pthread_create(&tid[t], NULL, blocks_run, &job[t]) == 0;
          if (!made[t]) blocks_run(&job[t]);
        }
        for (int t = 0; t < th; ++t)
          if (made[t]) pthread_join(tid[t], NULL);
      } else {
        blocks_run(&j);
      }
    }
  }
  return 0;
}

void spo_synth_norm(uint64_t seed, int64_t layer, int64_t dim, float *out) {
  spo_synth_normal(seed, tag_of(layer, kNormWeight), 1.0f, 0.02f, out, dim);
}
