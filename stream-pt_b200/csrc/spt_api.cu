// spt_api.cu -- C ABI (include/spt_moe.h): validation, HBM expert arena,
// orchestration of the MoE block on one CUDA stream, stage entry points.
//
// Validation follows forwardMoEBatch's checks in order
// (forward/moe_batch.go:81-136, forward/mxfp4_batch.go:17-27,
// forward/moe_batch.go:196-219, forward/layer.go:279-289,
// ggufmap/mmap_linux.go:318-334); each failure maps to one spt_status.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <initializer_list>
#include <limits>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/spt_moe.h"
#include "spt_gguf.h"
#include "spt_internal.cuh"
#include "spt_philox.h"

using namespace spt;

namespace {

thread_local std::string g_tls_error;

struct DevBuf {
  void *p = nullptr;
  size_t bytes = 0;
  cudaError_t ensure(size_t want) {
    if (want <= bytes) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    size_t cap = std::max<size_t>(want, 256);
    cudaError_t st = cudaMalloc(&p, cap);
    if (st == cudaSuccess) bytes = cap;
    return st;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  template <class T>
  T *as() const { return reinterpret_cast<T *>(p); }
};

}  // namespace

struct spt_context {
  int device = -1;
  bool has_device = false;
  int sm_count = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::string err;
  // per-call scratch
  DevBuf logits, sel_idx, sel_w, offsets, perm, slot_pos, act_list, meta, act, res, xdev, outdev;
  int64_t last_T = 0, last_E = 0, last_K = 0;
  bool have_routing = false;
  // optional per-stage timing (events on the launching stream)
  bool timing = false;
  cudaEvent_t ev[SPT_NUM_STAGES + 1] = {};
  // tensor-core path
  int path = SPT_PATH_AUTO;
  int kernels_last = 0;
  DevBuf dev_err, pad_off, tile_gu, tile_dn, pos_expert, qx, sfx, qa, sfa;
  DevBuf stack_norm, stack_ffn;  // layer stack: normed rows and block output [T][H]
  DevBuf g16_count;  // decode GEMV: arrivals per down row group of the fused combine (zero between launches)
  DevBuf route_count;  // router CTAs finished, for the selection + dispatch in its last CTA (zero between launches)
  DevBuf xq, xe, actq, act_off;  // decode GEMV: split x rows, their exponents, split SwiGLU rows,
                                 // first dispatch position of each active expert
  int32_t *err_host = nullptr;  // pinned copy of dev_err, read after the host path's single sync
  void *hx = nullptr, *hout = nullptr;  // pinned staging of pageable caller x / out (host entry points)
  size_t hx_bytes = 0, hout_bytes = 0;
  // tuning options (spt_context_set_option), seeded from the environment once
  int opt_tile_tokens = 0;      // tcgen05 token-tile width (0: from the batch)
  int opt_router_bulk = 1;      // the shared-memory router stages rows with bulk copies (SPT_ROUTER_BULK)
  int opt_fused_select = 1;     // 1: top-k + dispatch in the router's last CTA (T <= kRouterDispatchMaxTokens),
                                // else for T <= kSelectDispatchMaxTokens top-k in the dispatch kernel;
                                // 2: top-k in the dispatch kernel (T <= 8); 0: separate launches
  int opt_prefetch = 0;         // tcgen05 weight tiles prefetched into L2 ahead
  int opt_gemv16_slots = 16;    // SPT_PATH_AUTO: decode GEMV while batch x top-k <= this
  int opt_wait_shift = 31;      // bounded device waits give up after 2^shift clock cycles
  int opt_fault_stage = -1;     // failure injection: the tcgen05 producer skips this stage (tests)
  int opt_host_graphs = 1;      // replay repeated host calls from captured CUDA graphs
  int opt_prefill_fp8 = 0;      // 128-token tiles: e4m3 activation terms instead of e2m1
  // Host-call graphs: the block's kernels captured once per (arena, layer,
  // batch, path and options) and replayed by the host entry points; `bufs`
  // is the device buffers the capture used (a grown buffer invalidates it).
  struct HostGraph {
    uint64_t arena = 0;
    int64_t layer = 0, T = 0;
    std::vector<int64_t> opts;
    std::vector<const void *> bufs;
    cudaGraphExec_t exec = nullptr;
    bool warm = false;  // ran once uncaptured with this key (its buffers exist)
    uint64_t used = 0;
  };
  std::vector<HostGraph> graphs;
  uint64_t graph_clock = 0;
  int last_path = SPT_PATH_EXACT;  // expert path of the last forward (SPT_PATH_EXACT / _MMA / _GEMV16)
  bool timed_last = false;         // the last forward recorded stage events
  int last_bn = 0;                 // its tcgen05 token-tile width
  // activation tensor maps of the last call (re-encoded when the buffers or shape change)
  struct ActMaps {
    const void *q = nullptr;
    int kp = 0, rb = 0, bn = 0, ks = 0;
    ActFmt fmt = ActFmt::kFp4Stack;
    CUtensorMap m, m1;
  } act_maps[2];
};

struct spt_q80_matrix {
  spt_context *ctx = nullptr;
  int64_t input = 0, output = 0;
  DevBuf w;            // rows x input/32 x 34 bytes, + padding
  DevBuf best, err;    // argmax key, bounded-wait flag
  DevBuf res;          // argmax (int64) + logit (float) of the host path
  DevBuf xdev, ydev;   // host-path staging
};

struct spt_q40_matrix {
  spt_context *ctx = nullptr;
  int64_t input = 0, output = 0;
  DevBuf w;            // rows x input/32 x 18 bytes, + padding
  DevBuf err;          // bounded-wait flag of the one-input kernel
  DevBuf xdev, ydev;   // host-path staging
};

struct spt_arena {
  uint64_t id = 0;           // unique per arena in the process (keys the context's call graphs)
  int device = -1;
  spt_moe_config cfg{};
  int64_t expert_begin = 0;  // experts [expert_begin, expert_begin + expert_count) are resident
  int64_t expert_count = 0;  // (every expert unless the arena is one rank's expert-parallel shard)
  std::vector<LayerDev> layers;
  std::vector<void *> allocs;
  uint64_t bytes = 0;
  uint32_t flags = 0;
};

namespace {

constexpr float kSynthNormStd = 0.02f;  // RMSNorm weights ~ N(1, 0.02)

spt_arena *new_arena() {
  static std::atomic<uint64_t> next{1};
  spt_arena *a = new spt_arena();
  a->id = next.fetch_add(1);
  return a;
}

// Device address of the allocation-free entry point's static scratch on
// ctx's device (defined with that entry point below).
spt_status static_scratch(spt_context *ctx, unsigned char **out);

spt_status fail(spt_context *ctx, spt_status st, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx) ctx->err = buf;
  else g_tls_error = buf;
  return st;
}

spt_status cuda_fail(spt_context *ctx, cudaError_t e, const char *what) {
  return fail(ctx, SPT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

spt_status cuda_ok(spt_context *ctx, cudaError_t e, const char *what) {
  return e == cudaSuccess ? SPT_OK : cuda_fail(ctx, e, what);
}

#define SPT_CUDA(ctx, call)                                  \
  do {                                                       \
    cudaError_t _e = (call);                                 \
    if (_e != cudaSuccess) return cuda_fail((ctx), _e, #call); \
  } while (0)

bool canceled(const volatile int32_t *cancel) { return cancel && *cancel != 0; }

// moeBatchProduct (forward/moe_batch.go:29-38): every factor > 0, no
// overflow of Go's int (int64).
bool product(std::initializer_list<int64_t> vals, int64_t *out) {
  int64_t n = 1;
  for (int64_t v : vals) {
    if (v <= 0 || n > std::numeric_limits<int64_t>::max() / v) return false;
    n *= v;
  }
  if (out) *out = n;
  return true;
}

bool named(const spt_tensor &t) { return t.name && t.name[0] != '\0'; }
const char *tname(const spt_tensor &t) { return t.name ? t.name : ""; }

// validateMoEBatchExpert (forward/mxfp4_batch.go:17-27)
spt_status validate_expert(spt_context *ctx, const spt_tensor &t, int64_t input, int64_t output,
                           int64_t experts) {
  if (t.type != 39 || t.n_dims != 3 || t.shape[0] != (uint64_t)input ||
      t.shape[1] != (uint64_t)output || t.shape[2] != (uint64_t)experts || input % 32 != 0)
    return fail(ctx, SPT_ERR_EXPERT, "\"%s\": expected MXFP4 expert tensor [%lld %lld %lld]",
                tname(t), (long long)input, (long long)output, (long long)experts);
  int64_t n = 0;
  if (!product({input / 32, 17, output, experts}, &n) || t.end < t.start ||
      t.end - t.start != (uint64_t)n)
    return fail(ctx, SPT_ERR_EXPERT, "\"%s\": invalid expert range or overflow", tname(t));
  return SPT_OK;
}

// validateMoEBatchBias (forward/moe_batch.go:196-219)
spt_status validate_bias(spt_context *ctx, const spt_tensor &t, int64_t dim, int64_t count) {
  if (!named(t)) {
    if (t.end != t.start) return fail(ctx, SPT_ERR_BIAS, "unnamed MoE bias has nonempty range");
    return SPT_OK;
  }
  int64_t width = 4;
  if (t.type == 1 || t.type == 30) width = 2;
  else if (t.type != 0) return fail(ctx, SPT_ERR_BIAS, "\"%s\": unsupported bias type", tname(t));
  int64_t n = 0;
  const bool ok = product({dim, count, width}, &n);
  uint32_t want_dims = 2;
  if (count == 1 && t.n_dims == 1) want_dims = 1;
  if (!ok || t.n_dims != want_dims || t.shape[0] != (uint64_t)dim ||
      (want_dims == 2 && t.shape[1] != (uint64_t)count) || t.end < t.start ||
      t.end - t.start != (uint64_t)n)
    return fail(ctx, SPT_ERR_BIAS, "\"%s\": invalid bias shape or range", tname(t));
  return SPT_OK;
}

// validateRangeLocked (ggufmap/mmap_linux.go:318-334) for a tensor that the
// reference would map.
spt_status validate_file_range(spt_context *ctx, const spt_reader *r, const spt_tensor &t) {
  if (t.end <= t.start) return fail(ctx, SPT_ERR_FILE_RANGE, "tensor \"%s\": empty or invalid range", tname(t));
  if (t.end > r->size) return fail(ctx, SPT_ERR_FILE_RANGE, "tensor \"%s\": range exceeds file size", tname(t));
  return SPT_OK;
}

spt_status validate_config(spt_context *ctx, const spt_moe_config *cfg) {
  const int64_t h = cfg->hidden_dim, d = cfg->expert_hidden_dim, e = cfg->num_experts,
                k = cfg->num_experts_used;
  if (!product({h, 4}, nullptr) || k <= 0 || k > e || d <= 0)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  return SPT_OK;
}

spt_status validate_layer(spt_context *ctx, const spt_reader *reader, const spt_moe_config *cfg,
                          const spt_layer_weights *lw) {
  if (!reader || !cfg || !lw)
    return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE context, reader, configuration or weights");
  spt_status st = validate_config(ctx, cfg);
  if (st) return st;
  const int64_t h = cfg->hidden_dim, d = cfg->expert_hidden_dim, e = cfg->num_experts;
  const spt_tensor &router = lw->ffn_gate_inp;
  int64_t router_bytes = 0;
  const bool ok = product({h, e, 4}, &router_bytes);
  if (!ok || router.type != 0 || router.n_dims != 2 || router.shape[0] != (uint64_t)h ||
      router.shape[1] != (uint64_t)e || router.end < router.start ||
      router.end - router.start != (uint64_t)router_bytes)
    return fail(ctx, SPT_ERR_ROUTER, "\"%s\": invalid F32 router shape or range", tname(router));
  if ((st = validate_expert(ctx, lw->ffn_gate_exps, h, d, e))) return st;
  if ((st = validate_expert(ctx, lw->ffn_up_exps, h, d, e))) return st;
  if ((st = validate_expert(ctx, lw->ffn_down_exps, d, h, e))) return st;
  if ((st = validate_bias(ctx, lw->ffn_gate_inp_bias, e, 1))) return st;
  if ((st = validate_bias(ctx, lw->ffn_gate_exps_bias, d, e))) return st;
  if ((st = validate_bias(ctx, lw->ffn_up_exps_bias, d, e))) return st;
  if ((st = validate_bias(ctx, lw->ffn_down_exps_bias, h, e))) return st;
  // normBatch weight (layer_batch.go:145-155): F32, F16 or BF16 (tag 28), 1-D [hidden]
  if (named(lw->post_attention_norm)) {
    const spt_tensor &t = lw->post_attention_norm;
    const int64_t width = t.type == 0 ? 4 : 2;
    if (t.type != 0 && t.type != 1 && t.type != 28)
      return fail(ctx, SPT_ERR_BIAS, "\"%s\": unsupported normalization weight type %u", tname(t), t.type);
    if (t.n_dims != 1 || t.shape[0] != (uint64_t)h || t.end < t.start || t.end - t.start != (uint64_t)(h * width))
      return fail(ctx, SPT_ERR_BIAS, "\"%s\": invalid float vector shape or range", tname(t));
    if ((st = validate_file_range(ctx, reader, t))) return st;
  }
  // readFloatVector on the router bias needs a 1-D [E] tensor (layer.go:285-289)
  if (named(lw->ffn_gate_inp_bias) && lw->ffn_gate_inp_bias.n_dims != 1)
    return fail(ctx, SPT_ERR_BIAS, "\"%s\": invalid float vector shape or range",
                tname(lw->ffn_gate_inp_bias));
  const spt_tensor *mapped[] = {&lw->ffn_gate_inp_bias, &router, &lw->ffn_gate_exps,
                                &lw->ffn_up_exps, &lw->ffn_down_exps, &lw->ffn_gate_exps_bias,
                                &lw->ffn_up_exps_bias, &lw->ffn_down_exps_bias};
  for (const spt_tensor *t : mapped) {
    if (t != &router && t != &lw->ffn_gate_exps && t != &lw->ffn_up_exps &&
        t != &lw->ffn_down_exps && !named(*t))
      continue;
    if ((st = validate_file_range(ctx, reader, *t))) return st;
  }
  if (!reader->base && reader->size > 0)
    return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE context, reader, configuration or weights");
  return SPT_OK;
}

// readFloatVector element decode (forward/layer.go:291-301, q40.go:149-180).
float f16_to_f32(uint16_t bits) {
  uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
  uint32_t exponent = (bits >> 10) & 0x1fu;
  uint32_t mantissa = bits & 0x3ffu;
  uint32_t out;
  if (exponent == 0) {
    if (mantissa == 0) {
      out = sign;
    } else {
      uint32_t ex = 113;
      while ((mantissa & 0x400u) == 0) {
        mantissa <<= 1;
        ex--;
      }
      out = sign | ex << 23 | (mantissa & 0x3ffu) << 13;
    }
  } else if (exponent == 31) {
    out = sign | 0x7f800000u | mantissa << 13;
  } else {
    out = sign | (exponent + 112) << 23 | mantissa << 13;
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

void decode_floats(const uint8_t *src, uint32_t type, int64_t n, float *dst) {
  for (int64_t i = 0; i < n; ++i) {
    if (type == 0) {
      memcpy(&dst[i], src + 4 * i, 4);
    } else {
      uint16_t hbits;
      memcpy(&hbits, src + 2 * i, 2);
      if (type == 1) {
        dst[i] = f16_to_f32(hbits);
      } else {
        uint32_t u = (uint32_t)hbits << 16;
        memcpy(&dst[i], &u, 4);
      }
    }
  }
}

// ---- host synthetic generation (shared by the arena and the host copy) --
void synth_normal(uint64_t seed, uint32_t tag, float mean, float sd, float *out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t a, b;
    synth_uniform_pair(seed, tag, (uint64_t)i, &a, &b);
    const double u1 = ((double)a + 1.0) / 4294967296.0;
    const double u2 = (double)b / 4294967296.0;
    const double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    out[i] = (float)((double)mean + (double)sd * z);
  }
}

void synth_router_bias(const spt_moe_config *cfg, const spt_synth_params *p, int64_t layer,
                       float *bias) {
  const int64_t E = cfg->num_experts;
  if (p->router_bias) synth_normal(p->seed, synth_tag(layer, kSynthRouterBias), 0.0f, p->bias_std, bias, E);
  else std::fill(bias, bias + E, 0.0f);
  if (p->zipf_s > 0.0f) {
    // seeded permutation of ranks 1..E (Fisher-Yates), bias += beta*(-s*ln(rank))
    std::vector<int64_t> rank(E);
    for (int64_t i = 0; i < E; ++i) rank[i] = i + 1;
    for (int64_t i = E - 1; i > 0; --i) {
      uint32_t a, b;
      synth_uniform_pair(p->seed, synth_tag(layer, kSynthZipfPerm), (uint64_t)i, &a, &b);
      const int64_t j = (int64_t)(((uint64_t)a * (uint64_t)(i + 1)) >> 32);
      std::swap(rank[i], rank[j]);
    }
    for (int64_t e = 0; e < E; ++e)
      bias[e] = (float)((double)bias[e] +
                        (double)p->zipf_beta * (-(double)p->zipf_s * log((double)rank[e])));
  }
}

// ---- arena ----------------------------------------------------------------
template <class T>
spt_status arena_alloc(spt_context *ctx, spt_arena *a, size_t count, T **out) {
  void *p = nullptr;
  const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc(arena)");
  a->allocs.push_back(p);
  a->bytes += bytes;
  *out = reinterpret_cast<T *>(p);
  return SPT_OK;
}

spt_status upload(spt_context *ctx, void *dst, const void *src, size_t bytes) {
  // host -> device through a pinned staging buffer (the arena is uploaded once)
  static const size_t kChunk = 32u << 20;
  void *pinned = nullptr;
  SPT_CUDA(ctx, cudaMallocHost(&pinned, std::min(bytes, kChunk) + 16));
  for (size_t off = 0; off < bytes; off += kChunk) {
    const size_t n = std::min(kChunk, bytes - off);
    memcpy(pinned, (const uint8_t *)src + off, n);
    cudaError_t e = cudaMemcpyAsync((uint8_t *)dst + off, pinned, n, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
      cudaFreeHost(pinned);
      return cuda_fail(ctx, e, "upload");
    }
  }
  cudaFreeHost(pinned);
  return SPT_OK;
}

spt_status alloc_g8(spt_context *ctx, spt_arena *a, int64_t experts, int rows, int blocks,
                    MatrixG8 *m, uint4 **nib, uint32_t **scl) {
  spt_status st = arena_alloc(ctx, a, g8_nib_count(experts, rows, blocks), nib);
  if (st) return st;
  if ((st = arena_alloc(ctx, a, g8_scl_count(experts, rows, blocks), scl))) return st;
  SPT_CUDA(ctx, cudaMemsetAsync(*nib, 0, g8_nib_count(experts, rows, blocks) * sizeof(uint4), ctx->stream));
  SPT_CUDA(ctx, cudaMemsetAsync(*scl, 0, g8_scl_count(experts, rows, blocks) * sizeof(uint32_t), ctx->stream));
  m->nib = *nib;
  m->scl = *scl;
  m->rows = rows;
  m->blocks = blocks;
  m->groups = (rows + 7) / 8;
  m->quads = (blocks + 3) / 4;
  return SPT_OK;
}

spt_status stage_raw(spt_context *ctx, DevBuf *staging, const uint8_t *src, size_t raw) {
  SPT_CUDA(ctx, staging->ensure(raw));
  return upload(ctx, staging->p, src, raw);
}

spt_status repack_g8_from(spt_context *ctx, spt_arena *a, const uint8_t *dev_raw, int64_t experts,
                          int rows, int blocks, MatrixG8 *m) {
  uint4 *nib = nullptr;
  uint32_t *scl = nullptr;
  spt_status st = alloc_g8(ctx, a, experts, rows, blocks, m, &nib, &scl);
  if (st) return st;
  cudaError_t e = launch_repack_g8(dev_raw, experts, rows, blocks, nib, scl, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "repack");
  return SPT_OK;
}

spt_status upload_mxfp4(spt_context *ctx, spt_arena *a, const uint8_t *src, int64_t experts,
                        int rows, int blocks, MatrixG8 *m) {
  DevBuf staging;
  spt_status st = stage_raw(ctx, &staging, src, (size_t)experts * rows * blocks * 17);
  if (st == SPT_OK) st = repack_g8_from(ctx, a, staging.as<uint8_t>(), experts, rows, blocks, m);
  staging.release();
  return st;
}

// Allocate (zeroed) MMA planes for `experts` x `rows` x K and encode the TMA map.
spt_status alloc_mma(spt_context *ctx, spt_arena *a, int64_t experts, int rows, int k, MmaMatrix *m) {
  m->experts = experts;
  m->rows = rows;
  m->k = k;
  m->kp = (k + kMmaKT - 1) / kMmaKT * kMmaKT;
  m->mtiles = (rows + kMmaM - 1) / kMmaM;
  const size_t wb = mma_w_bytes(experts, rows, k), sb = mma_sf_bytes(experts, rows, k);
  spt_status st = arena_alloc(ctx, a, wb, &m->w);
  if (st) return st;
  if ((st = arena_alloc(ctx, a, sb, &m->sf))) return st;
  SPT_CUDA(ctx, cudaMemsetAsync(m->w, 0, wb, ctx->stream));
  SPT_CUDA(ctx, cudaMemsetAsync(m->sf, 0, sb, ctx->stream));
  if (!mma_encode_weights(m)) return fail(ctx, SPT_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed");
  return SPT_OK;
}

spt_status upload_floats(spt_context *ctx, spt_arena *a, const float *host, size_t n,
                         const float **out) {
  float *d = nullptr;
  spt_status st = arena_alloc(ctx, a, n, &d);
  if (st) return st;
  if ((st = upload(ctx, d, host, n * sizeof(float)))) return st;
  *out = d;
  return SPT_OK;
}

spt_status require_device(spt_context *ctx) {
  if (!ctx) return fail(nullptr, SPT_ERR_NULL_ARG, "nil context");
  if (!ctx->has_device) return fail(ctx, SPT_ERR_NO_DEVICE, "context has no CUDA device");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaSetDevice");
  return SPT_OK;
}

spt_status ensure_scratch(spt_context *ctx, int64_t T, const spt_moe_config &c) {
  const int64_t H = c.hidden_dim, D = c.expert_hidden_dim, E = c.num_experts, K = c.num_experts_used;
  const int64_t S = std::max<int64_t>(T * K, 1);
  SPT_CUDA(ctx, ctx->logits.ensure(sizeof(float) * std::max<int64_t>(T * E, 1)));
  SPT_CUDA(ctx, ctx->sel_idx.ensure(sizeof(int32_t) * S));
  SPT_CUDA(ctx, ctx->sel_w.ensure(sizeof(float) * S));
  SPT_CUDA(ctx, ctx->offsets.ensure(sizeof(int32_t) * (E + 1)));
  SPT_CUDA(ctx, ctx->perm.ensure(sizeof(int32_t) * S));
  SPT_CUDA(ctx, ctx->slot_pos.ensure(sizeof(int32_t) * S));
  SPT_CUDA(ctx, ctx->act_list.ensure(sizeof(int32_t) * E));
  SPT_CUDA(ctx, ctx->meta.ensure(sizeof(int32_t) * 4));
  SPT_CUDA(ctx, ctx->act.ensure(sizeof(float) * S * D));
  SPT_CUDA(ctx, ctx->res.ensure(sizeof(float) * S * H));
  return SPT_OK;
}

int pick_mt(int64_t T, int64_t K, int64_t E) {
  const double avg = (double)(T * K) / (double)E;
  if (T <= 1 || avg <= 0.5) return 1;
  if (avg <= 1.5) return 2;
  if (avg <= 3.0) return 4;
  return 8;
}

// Activation tensor maps for GEMM `which` (0 gate/up, 1 down), encoded only
// when the buffer or the shape differs from the previous call.
bool act_maps(spt_context *ctx, int which, uint8_t *q, int kp, int rb, int bn, int ks, CUtensorMap *m,
              CUtensorMap *m1) {
  auto &c = ctx->act_maps[which];
  const ActFmt f = mma_act_fmt(bn, ctx->opt_prefill_fp8 != 0);
  if (c.q != q || c.kp != kp || c.rb != rb || c.bn != bn || c.ks != ks || c.fmt != f) {
    c.q = nullptr;
    if (!mma_encode_acts(&c.m, q, kp, rb, bn, f, ks) || !mma_encode_acts(&c.m1, q, kp, rb, bn, f, 1)) return false;
    c.fmt = f;
    c.q = q;
    c.kp = kp;
    c.rb = rb;
    c.bn = bn;
    c.ks = ks;
  }
  *m = c.m;
  *m1 = c.m1;
  return true;
}

// Tokens per tensor-core tile from the mean tokens per expert: up to 5 per
// expert 8-token tiles (smaller activation stages; an expert with more tokens
// takes a second tile, whose weights mostly come from L2), up to 8 per expert
// 16-token tiles, larger batches 128-token tiles.  Measured on B200 (GPT-OSS
// layer, 8 vs 16 tokens): T=96 378.6 vs 410.5 us, T=128 389.1 vs 417.5,
// T=192 433.9 vs 434.6, T=256 514.9 vs 451.5.  The context option
// SPT_OPT_TILE_TOKENS (8, 16 or 128) fixes the choice.
int pick_bn(const spt_context *ctx, int64_t T, int64_t K, int64_t E) {
  if (ctx->opt_tile_tokens) return ctx->opt_tile_tokens;
  const int64_t S = T * K;
  return S <= 5 * E ? 8 : S <= 8 * E ? 16 : 128;
}

// Launch parameters of the two tensor-core GEMMs of one forward (T tokens,
// bn-token tiles); the tile tables they point at are the dispatch kernel's.
// ks_fixed > 0 fixes the K tiles per stage (the decode kernel's GEMMs).
spt_status build_gemms(spt_context *ctx, const LayerDev &L, const spt_moe_config &c, int64_t T, int bn,
                       MmaLaunch *gu, MmaLaunch *dn, int *rb_out, int ks_fixed = 0) {
  const int H = (int)c.hidden_dim, D = (int)c.expert_hidden_dim, E = (int)c.num_experts,
            K = (int)c.num_experts_used;
  const int64_t S = T * K;
  const int64_t na_max = std::min<int64_t>(E, S);
  const int rb = (int)((int64_t)kMmaM * (S / bn + na_max + 1));
  const int kph = L.gu_mma.kp, kpd = L.dn_mma.kp;
  const ActFmt fmt = mma_act_fmt(bn, ctx->opt_prefill_fp8 != 0);
  const bool fp4 = fmt == ActFmt::kFp4Stack;  // decode-sized tiles, several K tiles per stage
  // work units per token tile (row tiles, or groups of them for 128-token tiles)
  const int mt_gu = mma_row_units(bn, L.gu_mma.mtiles), mt_dn = mma_row_units(bn, L.dn_mma.mtiles);
  // one stage size for both GEMMs (they share the activation map cache), from
  // an estimate of the down GEMM's row tiles: its host bound halved (the bound
  // puts every slot on its own expert and counts partial token tiles twice)
  const int ks = ks_fixed > 0 ? ks_fixed
                              : mma_stage_tiles(bn, (int64_t)std::min(mt_gu, mt_dn) * (na_max + S / bn + 1) / 2,
                                                ctx->sm_count);
  const bool wide = ks == kMmaStageTilesWide && fp4;
  MmaLaunch &g = *gu;
  g.ks = ks;
  g.tmap_a = fp4 ? (wide ? L.gu_mma.tmap_pw : L.gu_mma.tmap_p)
                 : fmt == ActFmt::kFp4Planes ? L.gu_mma.tmap_gp : L.gu_mma.tmap_g;
  g.tmap_a1 = fp4 ? L.gu_mma.tmap_p1 : L.gu_mma.tmap;
  g.tmap_sfa = L.gu_mma.tmap_sfg;
  if (!act_maps(ctx, 0, ctx->qx.as<uint8_t>(), kph, rb, bn, ks, &g.tmap_b, &g.tmap_b1))
    return fail(ctx, SPT_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed");
  g.w = L.gu_mma.w;
  g.sfa = L.gu_mma.sf;
  g.sfb = ctx->sfx.as<uint8_t>();
  g.rows = L.gu_mma.rows;
  g.kp = kph;
  g.mtiles = L.gu_mma.mtiles;
  g.ktiles = kph / kMmaKT;
  g.rb = rb;
  g.offsets = ctx->offsets.as<int32_t>();
  g.pad_off = ctx->pad_off.as<int32_t>();
  g.act_list = ctx->act_list.as<int32_t>();
  g.tile_off = ctx->tile_gu.as<int32_t>();
  g.meta = ctx->meta.as<int32_t>();
  g.max_tiles = (int)std::min<int64_t>((int64_t)mt_gu * (na_max + S / bn + 1), 1 << 30);
  g.mode = 0;
  g.bias0 = L.gate_bias;
  g.bias1 = L.up_bias;
  g.y = ctx->act.as<float>();
  g.y_stride = D;
  g.out_rows = D;
  g.err = ctx->dev_err.as<int32_t>();
  g.prefetch = ctx->opt_prefetch;
  g.wait_shift = ctx->opt_wait_shift;
  g.fault_stage = ctx->opt_fault_stage;
  MmaLaunch &d = *dn;
  d = g;
  d.tmap_a = fp4 ? (wide ? L.dn_mma.tmap_pw : L.dn_mma.tmap_p)
                 : fmt == ActFmt::kFp4Planes ? L.dn_mma.tmap_gp : L.dn_mma.tmap_g;
  d.tmap_a1 = fp4 ? L.dn_mma.tmap_p1 : L.dn_mma.tmap;
  d.tmap_sfa = L.dn_mma.tmap_sfg;
  if (!act_maps(ctx, 1, ctx->qa.as<uint8_t>(), kpd, rb, bn, ks, &d.tmap_b, &d.tmap_b1))
    return fail(ctx, SPT_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed");
  d.w = L.dn_mma.w;
  d.sfa = L.dn_mma.sf;
  d.sfb = ctx->sfa.as<uint8_t>();
  d.rows = L.dn_mma.rows;
  d.kp = kpd;
  d.mtiles = L.dn_mma.mtiles;
  d.ktiles = kpd / kMmaKT;
  d.tile_off = ctx->tile_dn.as<int32_t>();
  d.max_tiles = (int)std::min<int64_t>((int64_t)mt_dn * (na_max + S / bn + 1), 1 << 30);
  d.mode = 1;
  d.bias0 = L.down_bias;
  d.bias1 = nullptr;
  d.y = ctx->res.as<float>();
  d.y_stride = H;
  d.out_rows = H;
  if (rb_out) *rb_out = rb;
  return SPT_OK;
}

// Expert GEMMs on the tensor cores (after router/select/dispatch):
// plan -> quantize x -> gate/up GEMM (+SwiGLU) -> quantize act -> down GEMM.
spt_status forward_mma(spt_context *ctx, const LayerDev &L, const spt_moe_config &c, const float *x,
                       int64_t T, cudaStream_t s, int bn) {
  const int H = (int)c.hidden_dim, D = (int)c.expert_hidden_dim, K = (int)c.num_experts_used;
  const int64_t S = T * K;
  // buffers: reserve_experts; pad_off, tile_gu, tile_dn and pos_expert come
  // from the dispatch kernel
  MmaLaunch g, dn;
  int rb = 0;
  spt_status st = build_gemms(ctx, L, c, T, bn, &g, &dn, &rb);
  if (st) return st;
  const ActFmt fmt = mma_act_fmt(bn, ctx->opt_prefill_fp8 != 0);
  // each token's row once, stored at every position it was dispatched to
  SPT_CUDA(ctx, launch_quantize_tokens(x, H, (int)T, K, ctx->slot_pos.as<int32_t>(), ctx->offsets.as<int32_t>(),
                                       ctx->pad_off.as<int32_t>(), ctx->pos_expert.as<int32_t>(), H, g.kp, rb, bn,
                                       fmt, ctx->qx.as<uint8_t>(), ctx->sfx.as<uint8_t>(), s));
  if (ctx->timing) SPT_CUDA(ctx, cudaEventRecord(ctx->ev[4], s));
  SPT_CUDA(ctx, launch_mma_gemm(g, bn, fmt, ctx->sm_count, s));
  if (ctx->timing) SPT_CUDA(ctx, cudaEventRecord(ctx->ev[5], s));
  SPT_CUDA(ctx, launch_quantize_act(ctx->act.as<float>(), D, nullptr, K, false, ctx->offsets.as<int32_t>(),
                                    ctx->pad_off.as<int32_t>(), ctx->pos_expert.as<int32_t>(),
                                    ctx->meta.as<int32_t>(), (int)S, D, dn.kp, rb, bn, fmt, ctx->qa.as<uint8_t>(),
                                    ctx->sfa.as<uint8_t>(), s));
  if (ctx->timing) SPT_CUDA(ctx, cudaEventRecord(ctx->ev[6], s));
  SPT_CUDA(ctx, launch_mma_gemm(dn, bn, fmt, ctx->sm_count, s));
  ctx->kernels_last = 8;  // router, select, dispatch, quantize, gate/up, quantize, down, combine
  return SPT_OK;
}

// What gave up, from the code a bounded device wait recorded.
const char *device_wait_name(int32_t code) {
  return code >= 20 ? "expert-parallel peer exchange" : code == 9 ? "router" : "tensor-core GEMM";
}

spt_status check_device_error(spt_context *ctx) {
  if (!ctx->dev_err.p) return SPT_OK;
  int32_t e = 0;
  SPT_CUDA(ctx, cudaMemcpy(&e, ctx->dev_err.p, sizeof e, cudaMemcpyDeviceToHost));
  if (e != 0) {
    cudaMemset(ctx->dev_err.p, 0, sizeof e);
    return fail(ctx, SPT_ERR_TIMEOUT, "%s: bounded wait %d gave up",
                device_wait_name(e), e);
  }
  return SPT_OK;
}

// Expert products of this call.  Arenas with the tensor-core planes run
// them there: the decode GEMV (k_gemv16) for batches of at most
// opt_gemv16_slots slots (batch x top-k), the tcgen05 GEMM above that
// (SPT_PATH_MMA and SPT_PATH_GEMV16 force one of the two); arenas with only
// the G8 planes, or SPT_PATH_EXACT, run the bit-exact CUDA-core GEMV.
enum ExpertPath { kPathExact = 0, kPathTcgen05 = 1, kPathGemv16 = 2 };

bool gemv16_fits(const LayerDev &L) {
  return L.has_mma && L.gemv16_ok && L.gu_mma.kp / kMmaKT <= kGemv16MaxKtiles &&
         L.dn_mma.kp / kMmaKT <= kGemv16MaxKtiles;
}

spt_status pick_path(spt_context *ctx, const LayerDev &L, const spt_moe_config &c, int64_t T, ExpertPath *path) {
  *path = kPathExact;
  if (ctx->path == SPT_PATH_MMA && !L.has_mma)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "arena was created without SPT_ARENA_MMA");
  if (ctx->path == SPT_PATH_GEMV16 && !gemv16_fits(L))
    return fail(ctx, SPT_ERR_UNSUPPORTED,
                "decode GEMV needs SPT_ARENA_MMA planes with every scale byte in [%d, %d] and K <= %d",
                kF16ScaleLo, kF16ScaleHi, kGemv16MaxKtiles * kMmaKT);
  if (ctx->path != SPT_PATH_EXACT && L.has_mma) {
    if (ctx->path == SPT_PATH_GEMV16) *path = kPathGemv16;
    else if (ctx->path == SPT_PATH_MMA) *path = kPathTcgen05;
    else *path = gemv16_fits(L) && T * c.num_experts_used <= (int64_t)ctx->opt_gemv16_slots ? kPathGemv16
                                                                                                 : kPathTcgen05;
  }
  if (*path == kPathExact && !L.has_g8)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "arena was created without SPT_ARENA_GEMV");
  return SPT_OK;
}

// Every device buffer experts_combine needs for T tokens of config c.  It
// allocates only here, so a caller can make the allocations before work that
// must not overlap a cudaMalloc/cudaFree (an NCCL exchange in flight: their
// implicit device synchronisation can deadlock against NCCL's progress).
spt_status reserve_experts(spt_context *ctx, const LayerDev &L, const spt_moe_config &c, int64_t T,
                           int bn_hint = 0) {
  spt_status st = ensure_scratch(ctx, T, c);
  if (st) return st;
  ExpertPath path;
  if ((st = pick_path(ctx, L, c, T, &path))) return st;
  if (path == kPathExact) return SPT_OK;
  const int64_t E = c.num_experts, K = c.num_experts_used, S = T * K;
  if (path == kPathGemv16) {
    const int64_t kph = L.gu_mma.kp, kpd = L.dn_mma.kp;
    SPT_CUDA(ctx, ctx->xq.ensure(sizeof(__half) * 2 * kph * std::max<int64_t>(T, 1)));
    SPT_CUDA(ctx, ctx->xe.ensure(sizeof(int32_t) * std::max<int64_t>(T, 1)));
    SPT_CUDA(ctx, ctx->act_off.ensure(sizeof(int32_t) * (E + 1)));
    const size_t cnt = sizeof(int32_t) * 4 * (size_t)L.dn_mma.mtiles;
    if (ctx->g16_count.bytes < cnt) {
      SPT_CUDA(ctx, ctx->g16_count.ensure(cnt));
      SPT_CUDA(ctx, cudaMemsetAsync(ctx->g16_count.p, 0, ctx->g16_count.bytes, ctx->stream));
    }
    SPT_CUDA(ctx, ctx->actq.ensure(sizeof(__half) * 2 * kpd * std::max<int64_t>(S, 1)));
    return SPT_OK;
  }
  SPT_CUDA(ctx, ctx->pad_off.ensure(sizeof(int32_t) * E));
  SPT_CUDA(ctx, ctx->tile_gu.ensure(sizeof(int32_t) * (E + 1)));
  SPT_CUDA(ctx, ctx->tile_dn.ensure(sizeof(int32_t) * (E + 1)));
  SPT_CUDA(ctx, ctx->pos_expert.ensure(sizeof(int32_t) * std::max<int64_t>(S, 1)));
  const int bn = bn_hint ? bn_hint : pick_bn(ctx, T, K, E);
  const int64_t na_max = std::min<int64_t>(E, S);
  const int rb = (int)((int64_t)kMmaM * (S / bn + na_max + 1));
  const int kph = L.gu_mma.kp, kpd = L.dn_mma.kp;
  if (!ctx->dev_err.p) {
    SPT_CUDA(ctx, ctx->dev_err.ensure(sizeof(int32_t)));
    SPT_CUDA(ctx, cudaMemsetAsync(ctx->dev_err.p, 0, sizeof(int32_t), ctx->stream));
  }
  const ActFmt fmt = mma_act_fmt(bn, ctx->opt_prefill_fp8 != 0);
  SPT_CUDA(ctx, ctx->qx.ensure(mma_act_bytes(fmt, rb, kph)));
  SPT_CUDA(ctx, ctx->sfx.ensure(mma_act_sf_bytes(fmt, rb, kph)));
  SPT_CUDA(ctx, ctx->qa.ensure(mma_act_bytes(fmt, rb, kpd)));
  SPT_CUDA(ctx, ctx->sfa.ensure(mma_act_sf_bytes(fmt, rb, kpd)));
  return SPT_OK;
}

#define SPT_MARK(i) \
  if (ctx->timing) SPT_CUDA(ctx, cudaEventRecord(ctx->ev[i], s))

// Dispatch, expert products and combine for selections already made
// (sel_idx/sel_w [T*K], expert ids local to the arena): out[t] = sum over
// ranks r of fma(result, weight, out[t]).  `c` gives the arena's experts
// and top-k (the expert-parallel receive side passes its shard and top-k 1).
// With `logits` (one device, T <= kSelectDispatchMaxTokens) the top-k
// selection runs inside the dispatch kernel and writes sel_idx / sel_w there.
// Decode GEMV batches of up to this many slots combine inside the down
// launch (one launch fewer; the last CTA of each row group does the sums).
constexpr int64_t kFusedCombineSlots = 64;

// The tensor-core tile layout (and the decode GEMV's position table) the
// dispatch lays out for this batch on `path`.
DispatchPlan dispatch_plan(spt_context *ctx, const LayerDev &L, int64_t T, int K, int E, ExpertPath path,
                           int bn_hint) {
  DispatchPlan plan;
  if (path == kPathGemv16) plan.act_off = ctx->act_off.as<int32_t>();
  if (path == kPathTcgen05) {
    plan.bn = bn_hint ? bn_hint : pick_bn(ctx, T, K, E);
    plan.mt_gu = mma_row_units(plan.bn, L.gu_mma.mtiles);
    plan.mt_dn = mma_row_units(plan.bn, L.dn_mma.mtiles);
    plan.pad_off = ctx->pad_off.as<int32_t>();
    plan.tile_gu = ctx->tile_gu.as<int32_t>();
    plan.tile_dn = ctx->tile_dn.as<int32_t>();
    plan.pos_expert = ctx->pos_expert.as<int32_t>();
  }
  return plan;
}

// dispatched: the router's last CTA already selected and dispatched (no
// dispatch launch here).
spt_status experts_combine(spt_context *ctx, const LayerDev &L, const spt_moe_config &c, const float *x,
                           int64_t T, const int32_t *sel_idx, const float *sel_w, float *out, int bn_hint = 0,
                           const float *logits = nullptr, bool x_split_done = false,
                           const float *resid = nullptr, bool dispatched = false) {
  const int H = (int)c.hidden_dim, D = (int)c.expert_hidden_dim, E = (int)c.num_experts,
            K = (int)c.num_experts_used;
  cudaStream_t s = ctx->stream;
  spt_status st = SPT_OK;
  const int max_active = (int)std::min<int64_t>(E, T * K);
  bool fused_combine = false;  // the decode GEMV's down launch also combines
  ExpertPath path;
  if ((st = pick_path(ctx, L, c, T, &path))) return st;
  if ((st = reserve_experts(ctx, L, c, T, bn_hint))) return st;
  const bool use_mma = path == kPathTcgen05;
  ctx->last_path = path == kPathGemv16 ? SPT_PATH_GEMV16 : use_mma ? SPT_PATH_MMA : SPT_PATH_EXACT;
  ctx->last_bn = 0;
  // tensor-core tile layout, made by the dispatch kernel
  const DispatchPlan plan = dispatch_plan(ctx, L, T, K, E, path, bn_hint);
  if (use_mma) ctx->last_bn = plan.bn;
  if (dispatched) {
    // made by the router's last CTA
  } else if (logits) {
    SPT_CUDA(ctx, launch_select_dispatch(logits, (int)T, E, K, const_cast<int32_t *>(sel_idx),
                                         const_cast<float *>(sel_w), ctx->offsets.as<int32_t>(),
                                         ctx->perm.as<int32_t>(), ctx->slot_pos.as<int32_t>(),
                                         ctx->act_list.as<int32_t>(), ctx->meta.as<int32_t>(), s,
                                         path != kPathExact ? &plan : nullptr));
  } else {
    SPT_CUDA(ctx, launch_dispatch(sel_idx, sel_w, (int)(T * K), E,
                                  ctx->offsets.as<int32_t>(), ctx->perm.as<int32_t>(),
                                  ctx->slot_pos.as<int32_t>(), ctx->act_list.as<int32_t>(),
                                  ctx->meta.as<int32_t>(), s, path != kPathExact ? &plan : nullptr));
  }
  SPT_MARK(3);
  if (path == kPathGemv16) {
    const int kph = L.gu_mma.kp, kpd = L.dn_mma.kp;
    __half *xq = ctx->xq.as<__half>(), *actq = ctx->actq.as<__half>();
    // the tokens' split operand, unless the router made it already
    if (!x_split_done)
      SPT_CUDA(ctx, launch_split_rows(x, H, (int)T, H, kph, nullptr, 1, nullptr, xq, ctx->xe.as<int32_t>(), s));
    Gemv16Launch g;
    g.w = L.gu_mma.w;
    g.sf = L.gu_mma.sf;
    g.rows = L.gu_mma.rows;
    g.out_rows = D;
    g.mtiles = L.gu_mma.mtiles;
    g.ktiles = kph / kMmaKT;
    g.kp = kph;
    g.xq = xq;
    g.xq_stride = 2 * (int64_t)kph;
    g.xe = ctx->xe.as<int32_t>();
    g.perm = ctx->perm.as<int32_t>();
    g.top_k = K;
    g.act_list = ctx->act_list.as<int32_t>();
    g.act_off = ctx->act_off.as<int32_t>();
    g.meta = ctx->meta.as<int32_t>();
    g.bias0 = L.gate_bias;
    g.bias1 = L.up_bias;
    g.actq = actq;
    g.actq_stride = 2 * (int64_t)kpd;
    g.actq_kp = kpd;
    SPT_MARK(4);
    SPT_CUDA(ctx, launch_gemv16(g, 0, max_active, s));
    SPT_MARK(5);
    Gemv16Launch d = g;
    d.w = L.dn_mma.w;
    d.sf = L.dn_mma.sf;
    d.rows = L.dn_mma.rows;
    d.out_rows = H;
    d.mtiles = L.dn_mma.mtiles;
    d.ktiles = kpd / kMmaKT;
    d.kp = kpd;
    d.xq = actq;
    d.xq_stride = 2 * (int64_t)kpd;
    d.xe = nullptr;
    d.perm = nullptr;
    d.top_k = 1;
    d.bias0 = L.down_bias;
    d.bias1 = nullptr;
    d.actq = nullptr;
    d.y = ctx->res.as<float>();
    d.y_stride = H;
    // decode batches: the combine runs in the down launch's last CTAs
    fused_combine = T * K <= kFusedCombineSlots;
    if (fused_combine) {
      d.cw = sel_w;
      d.cslot = ctx->slot_pos.as<int32_t>();
      d.ct = (int)T;
      d.ck = K;
      d.cout = out;
      d.cresid = resid;
      d.ccount = ctx->g16_count.as<int32_t>();
    }
    SPT_MARK(6);
    SPT_CUDA(ctx, launch_gemv16(d, 1, max_active, s));
    // router, select, dispatch, [split x], gate/up, down, [combine]
    ctx->kernels_last = (x_split_done ? 6 : 7) - (fused_combine ? 1 : 0);
  } else if (use_mma) {
    if ((st = forward_mma(ctx, L, c, x, T, s, plan.bn))) return st;
  } else {
    const int mt = pick_mt(T, K, E);
    GemvLaunch gu;
    gu.m0 = L.gate;
    gu.m1 = L.up;
    gu.bias0 = L.gate_bias;
    gu.bias1 = L.up_bias;
    gu.x = x;
    gu.x_stride = H;
    gu.y = ctx->act.as<float>();
    gu.y_stride = D;
    gu.perm = ctx->perm.as<int32_t>();
    gu.offsets = ctx->offsets.as<int32_t>();
    gu.act_list = ctx->act_list.as<int32_t>();
    gu.meta = ctx->meta.as<int32_t>();
    gu.top_k = K;
    gu.mode = kRowsMoEGateUp;
    gu.gate_up = true;
    gu.max_active = max_active;
    gu.mt = mt > 4 ? 4 : mt;
    SPT_MARK(4);
    SPT_CUDA(ctx, launch_gemv(gu, ctx->sm_count, s));
    SPT_MARK(5);
    SPT_MARK(6);
    GemvLaunch dn = gu;
    dn.m0 = L.down;
    dn.m1 = MatrixG8{};
    dn.bias0 = L.down_bias;
    dn.bias1 = nullptr;
    dn.x = ctx->act.as<float>();
    dn.x_stride = D;
    dn.y = ctx->res.as<float>();
    dn.y_stride = H;
    dn.mode = kRowsMoEDown;
    dn.gate_up = false;
    dn.mt = mt;
    SPT_CUDA(ctx, launch_gemv(dn, ctx->sm_count, s));
    ctx->kernels_last = 6;
  }
  SPT_MARK(7);
  if (!fused_combine)
    SPT_CUDA(ctx, launch_combine(ctx->res.as<float>(), sel_w, ctx->slot_pos.as<int32_t>(), (int)T, K, H, out, s,
                                 resid));
  SPT_MARK(8);
  if (logits || dispatched) ctx->kernels_last -= 1;  // no separate selection launch
  if (dispatched) ctx->kernels_last -= 1;            // nor a dispatch launch
  return SPT_OK;
}

// Router logits and top-k selections of T tokens (all experts of the layer).
// select = false leaves the selection to the fused dispatch kernel.
spt_status route_select(spt_context *ctx, const LayerDev &L, const spt_moe_config &c, const float *x,
                        int64_t T, int32_t *sel_idx, float *sel_w, bool select = true,
                        const RouterSplit *split = nullptr, bool *split_done = nullptr,
                        const RouterNorm *norm = nullptr, int *router_launches = nullptr,
                        const RouterDispatch *dispatch = nullptr, bool *dispatch_done = nullptr) {
  const int H = (int)c.hidden_dim, E = (int)c.num_experts, K = (int)c.num_experts_used;
  cudaStream_t s = ctx->stream;
  SPT_MARK(0);
  if (!ctx->dev_err.p) {  // the router's bounded wait reports here
    SPT_CUDA(ctx, ctx->dev_err.ensure(sizeof(int32_t)));
    SPT_CUDA(ctx, cudaMemsetAsync(ctx->dev_err.p, 0, sizeof(int32_t), ctx->stream));
  }
  SPT_CUDA(ctx, launch_router(L.router, x, L.router_bias, (int)T, H, E, ctx->logits.as<float>(), 8, s, split,
                              split_done, norm, router_launches, dispatch, dispatch_done,
                              ctx->opt_router_bulk ? ctx->dev_err.as<int32_t>() : nullptr, ctx->opt_wait_shift,
                              ctx->opt_fault_stage));
  SPT_MARK(1);
  if (select && !(dispatch_done && *dispatch_done))  // else the router's last CTA selected
    SPT_CUDA(ctx, launch_select(ctx->logits.as<float>(), (int)T, E, K, sel_idx, sel_w, s));
  SPT_MARK(2);
  return SPT_OK;
}

spt_status check_layer_limits(spt_context *ctx, const spt_moe_config &c) {
  if (c.num_experts > kDispatchMaxExperts || c.num_experts_used > kSelectMaxK)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "experts %lld > %d or top-k %lld > %d unsupported",
                (long long)c.num_experts, kDispatchMaxExperts, (long long)c.num_experts_used, kSelectMaxK);
  return SPT_OK;
}

// The whole block on device pointers (enqueue only).
// With resid, out = resid + block(x) (the layer stack's residual add; out
// may be resid).  With norm, the block's input is normBatch(x) (written to
// norm->out, by the router's prologue when it can), and x is only read.
spt_status forward_device(spt_context *ctx, spt_arena *arena, int64_t layer, const float *x,
                          float *out, int64_t T, const float *resid = nullptr, const RouterNorm *norm = nullptr) {
  const spt_moe_config &c = arena->cfg;
  spt_status st = check_layer_limits(ctx, c);
  if (st) return st;
  if (arena->expert_count != c.num_experts)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "arena holds experts [%lld, %lld) of %lld: use the expert-parallel entry point",
                (long long)arena->expert_begin, (long long)(arena->expert_begin + arena->expert_count),
                (long long)c.num_experts);
  if ((st = ensure_scratch(ctx, T, c))) return st;
  const LayerDev &L = arena->layers[(size_t)layer];
  const bool fuse = T <= kSelectDispatchMaxTokens && ctx->opt_fused_select;
  ctx->timed_last = ctx->timing;
  // the decode GEMV's split operand comes out of the router when it can
  ExpertPath path;
  if ((st = pick_path(ctx, L, c, T, &path))) return st;
  if ((st = reserve_experts(ctx, L, c, T))) return st;
  RouterSplit rs;
  if (path == kPathGemv16) {
    rs.xq = ctx->xq.as<__half>();
    rs.xe = ctx->xe.as<int32_t>();
    rs.kp = L.gu_mma.kp;
  }
  bool split_done = false, dispatched = false;
  int router_launches = 1;
  // decode batches: selection and dispatch in the router's last CTA when it
  // stages its rows (SPT_OPT_FUSED_SELECT 1), else inside the dispatch kernel
  RouterDispatch rd;
  const bool router_dispatch = T <= kRouterDispatchMaxTokens && ctx->opt_fused_select == 1;
  if (router_dispatch) {
    if (ctx->route_count.bytes < sizeof(unsigned)) {
      SPT_CUDA(ctx, ctx->route_count.ensure(sizeof(unsigned)));
      SPT_CUDA(ctx, cudaMemsetAsync(ctx->route_count.p, 0, ctx->route_count.bytes, ctx->stream));
    }
    rd.sel_idx = ctx->sel_idx.as<int32_t>();
    rd.sel_w = ctx->sel_w.as<float>();
    rd.offsets = ctx->offsets.as<int32_t>();
    rd.perm = ctx->perm.as<int32_t>();
    rd.slot_pos = ctx->slot_pos.as<int32_t>();
    rd.act_list = ctx->act_list.as<int32_t>();
    rd.meta = ctx->meta.as<int32_t>();
    rd.plan = path != kPathExact ? dispatch_plan(ctx, L, T, (int)c.num_experts_used, (int)c.num_experts, path, 0)
                                 : DispatchPlan{};
    rd.topk = (int)c.num_experts_used;
    rd.count = ctx->route_count.as<unsigned>();
  }
  if ((st = route_select(ctx, L, c, x, T, ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>(), !fuse,
                         path == kPathGemv16 ? &rs : nullptr, &split_done, norm, &router_launches,
                         router_dispatch ? &rd : nullptr, &dispatched)))
    return st;
  if ((st = experts_combine(ctx, L, c, norm ? norm->out : x, T, ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>(),
                            out, 0, fuse && !dispatched ? ctx->logits.as<float>() : nullptr, split_done, resid,
                            dispatched)))
    return st;
  ctx->kernels_last += router_launches - 1;
  ctx->last_T = T;
  ctx->last_E = c.num_experts;
  ctx->last_K = c.num_experts_used;
  ctx->have_routing = true;
  return SPT_OK;
}

spt_status check_batch(spt_context *ctx, const spt_moe_config &c, const float *x, int64_t x_len,
                       const float *out, int64_t out_len, int64_t batch) {
  int64_t n = 0;
  const bool ok = product({batch, c.hidden_dim, 4}, &n);
  if (!ok || x_len != n / 4 || out_len != n / 4 || c.num_experts_used <= 0 ||
      c.num_experts_used > c.num_experts || c.expert_hidden_dim <= 0)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  if (!x || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE input or output");
  const uintptr_t xs = (uintptr_t)x, ys = (uintptr_t)out;
  if ((xs <= ys && ys - xs < (uintptr_t)n) || (ys < xs && xs - ys < (uintptr_t)n))
    return fail(ctx, SPT_ERR_OVERLAP, "MoE input and output overlap");
  return SPT_OK;
}


// Device buffers a captured block touches.
std::vector<const void *> call_buffers(const spt_context *ctx) {
  std::vector<const void *> v;
  for (const DevBuf *b : {&ctx->logits, &ctx->sel_idx, &ctx->sel_w, &ctx->offsets, &ctx->perm, &ctx->slot_pos,
                          &ctx->act_list, &ctx->meta, &ctx->act, &ctx->res, &ctx->xdev, &ctx->outdev, &ctx->dev_err,
                          &ctx->pad_off, &ctx->tile_gu, &ctx->tile_dn, &ctx->pos_expert, &ctx->qx, &ctx->sfx,
                          &ctx->qa, &ctx->sfa, &ctx->xq, &ctx->xe, &ctx->actq, &ctx->act_off, &ctx->g16_count,
                          &ctx->route_count})
    v.push_back(b->p);
  return v;
}

std::vector<int64_t> call_options(const spt_context *ctx) {
  return {ctx->path, ctx->opt_tile_tokens, ctx->opt_fused_select, ctx->opt_prefetch, ctx->opt_gemv16_slots,
          ctx->opt_wait_shift, ctx->opt_fault_stage, ctx->opt_prefill_fp8, ctx->opt_router_bulk,
          (int64_t)(uintptr_t)ctx->stream};
}

// Capture the block on the context's device buffers into a graph (after a
// warm uncaptured run made every buffer).  On any failure the capture is
// dropped and the caller launches the kernels itself.
bool capture_block(spt_context *ctx, spt_arena *arena, int64_t layer, int64_t batch, cudaGraphExec_t *exec) {
  *exec = nullptr;
  if (cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const std::string saved = ctx->err;
  const spt_status st = forward_device(ctx, arena, layer, ctx->xdev.as<float>(), ctx->outdev.as<float>(), batch);
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  bool ok = st == SPT_OK && e == cudaSuccess && graph;
  if (ok) ok = cudaGraphInstantiate(exec, graph, 0) == cudaSuccess;
  if (graph) cudaGraphDestroy(graph);
  if (!ok) {
    cudaGetLastError();
    *exec = nullptr;
    ctx->err = saved;
  }
  return ok;
}

// Whether host memory p is page-locked (copies from it can be asynchronous).
bool host_pinned(const void *p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

spt_status ensure_pinned(spt_context *ctx, void **buf, size_t *have, size_t want) {
  if (*have >= want) return SPT_OK;
  if (*buf) cudaFreeHost(*buf);
  *buf = nullptr;
  *have = 0;
  SPT_CUDA(ctx, cudaHostAlloc(buf, want, cudaHostAllocDefault));
  *have = want;
  return SPT_OK;
}

spt_status forward_host(spt_context *ctx, spt_arena *arena, int64_t layer, const float *x,
                        int64_t x_len, float *out, int64_t out_len, int64_t batch,
                        const volatile int32_t *cancel) {
  if (!ctx || !arena) return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE context, reader, configuration or weights");
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  spt_status st = check_batch(ctx, arena->cfg, x, x_len, out, out_len, batch);
  if (st) return st;
  if (layer < 0 || layer >= (int64_t)arena->layers.size())
    return fail(ctx, SPT_ERR_DIMENSIONS, "layer %lld out of range", (long long)layer);
  if ((st = require_device(ctx))) return st;
  const size_t bytes = sizeof(float) * (size_t)x_len;
  SPT_CUDA(ctx, ctx->xdev.ensure(bytes));
  SPT_CUDA(ctx, ctx->outdev.ensure(bytes));
  if (!ctx->err_host) SPT_CUDA(ctx, cudaHostAlloc((void **)&ctx->err_host, sizeof(int32_t), cudaHostAllocDefault));
  // Pageable caller memory (a Go slice) goes through the context's pinned
  // buffers, so both copies are asynchronous and the call synchronises once.
  const bool x_pinned = host_pinned(x), out_pinned = host_pinned(out);
  const void *xsrc = x;
  if (!x_pinned) {
    if ((st = ensure_pinned(ctx, &ctx->hx, &ctx->hx_bytes, bytes))) return st;
    memcpy(ctx->hx, x, bytes);
    xsrc = ctx->hx;
  }
  if (!out_pinned && (st = ensure_pinned(ctx, &ctx->hout, &ctx->hout_bytes, bytes))) return st;
  SPT_CUDA(ctx, cudaMemcpyAsync(ctx->xdev.p, xsrc, bytes, cudaMemcpyHostToDevice, ctx->stream));
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  // The block: replayed from a captured graph on repeated calls (not while
  // stage timing records events), else launched kernel by kernel.
  spt_context::HostGraph *g = nullptr;
  if (ctx->opt_host_graphs && !ctx->timing) {
    const std::vector<int64_t> opts = call_options(ctx);
    for (auto &h : ctx->graphs)
      if (h.arena == arena->id && h.layer == layer && h.T == batch && h.opts == opts) g = &h;
    if (g && g->exec && g->bufs != call_buffers(ctx)) {  // a buffer moved: capture again
      cudaGraphExecDestroy(g->exec);
      g->exec = nullptr;
    }
    if (!g) {
      if (ctx->graphs.size() >= 16) {  // evict the least recently used
        auto lru = std::min_element(ctx->graphs.begin(), ctx->graphs.end(),
                                    [](const auto &p, const auto &q) { return p.used < q.used; });
        if (lru->exec) cudaGraphExecDestroy(lru->exec);
        ctx->graphs.erase(lru);
      }
      ctx->graphs.push_back({});
      g = &ctx->graphs.back();
      g->arena = arena->id;
      g->layer = layer;
      g->T = batch;
      g->opts = opts;
    }
    g->used = ++ctx->graph_clock;
    if (!g->exec && g->warm && capture_block(ctx, arena, layer, batch, &g->exec)) g->bufs = call_buffers(ctx);
  }
  if (g && g->exec) {
    SPT_CUDA(ctx, cudaGraphLaunch(g->exec, ctx->stream));
  } else {
    if ((st = forward_device(ctx, arena, layer, ctx->xdev.as<float>(), ctx->outdev.as<float>(), batch))) return st;
    if (g) g->warm = true;
  }
  SPT_CUDA(ctx, cudaMemcpyAsync(out_pinned ? (void *)out : ctx->hout, ctx->outdev.p, bytes, cudaMemcpyDeviceToHost,
                                ctx->stream));
  // the GEMM's error flag comes back with the output: one synchronisation
  if (ctx->dev_err.p)
    SPT_CUDA(ctx, cudaMemcpyAsync(ctx->err_host, ctx->dev_err.p, sizeof(int32_t), cudaMemcpyDeviceToHost,
                                  ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (!out_pinned) memcpy(out, ctx->hout, bytes);
  if (ctx->dev_err.p && *ctx->err_host != 0) {
    const int32_t e = *ctx->err_host;
    *ctx->err_host = 0;
    SPT_CUDA(ctx, cudaMemsetAsync(ctx->dev_err.p, 0, sizeof(int32_t), ctx->stream));
    SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return fail(ctx, SPT_ERR_TIMEOUT, "%s: bounded wait %d gave up",
                device_wait_name(e), e);
  }
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  return SPT_OK;
}

// Options from the environment, read once per context (spt_context_set_option
// changes them afterwards).
void seed_options(spt_context *ctx) {
  auto env = [](const char *name, int *dst, int lo, int hi) {
    const char *v = getenv(name);
    if (!v || !*v) return;
    const long x = strtol(v, nullptr, 10);
    if (x >= lo && x <= hi) *dst = (int)x;
  };
  env("SPT_MMA_BN", &ctx->opt_tile_tokens, 0, 128);
  if (ctx->opt_tile_tokens != 8 && ctx->opt_tile_tokens != 16 && ctx->opt_tile_tokens != 128) ctx->opt_tile_tokens = 0;
  env("SPT_FUSED_SELECT", &ctx->opt_fused_select, 0, 2);
  env("SPT_ROUTER_BULK", &ctx->opt_router_bulk, 0, 1);
  env("SPT_MMA_PREFETCH", &ctx->opt_prefetch, 0, 64);
  env("SPT_GEMV16_SLOTS", &ctx->opt_gemv16_slots, 0, 1 << 20);
  env("SPT_HOST_GRAPHS", &ctx->opt_host_graphs, 0, 1);
  env("SPT_PREFILL_FP8", &ctx->opt_prefill_fp8, 0, 1);
}

// Temporary device buffer for stage entry points.
struct Tmp {
  void *p = nullptr;
  ~Tmp() {
    if (p) cudaFree(p);
  }
  cudaError_t alloc(size_t n) { return cudaMalloc(&p, std::max<size_t>(n, 16)); }
  template <class T>
  T *as() const { return reinterpret_cast<T *>(p); }
};

}  // namespace

// =========================================================================
extern "C" {

const char *spt_status_string(spt_status s) {
  switch (s) {
    case SPT_OK: return "ok";
    case SPT_ERR_NULL_ARG: return "nil argument";
    case SPT_ERR_DIMENSIONS: return "invalid MoE batch dimensions";
    case SPT_ERR_OVERLAP: return "MoE input and output overlap";
    case SPT_ERR_ROUTER: return "invalid F32 router shape or range";
    case SPT_ERR_EXPERT: return "invalid MXFP4 expert tensor";
    case SPT_ERR_BIAS: return "invalid MoE bias";
    case SPT_ERR_FILE_RANGE: return "tensor range outside the file";
    case SPT_ERR_SCRATCH: return "MoE batch scratch dimensions mismatch";
    case SPT_ERR_CANCELED: return "context canceled";
    case SPT_ERR_CUDA: return "CUDA error";
    case SPT_ERR_NCCL: return "NCCL error";
    case SPT_ERR_TIMEOUT: return "device wait timed out";
    case SPT_ERR_UNSUPPORTED: return "unsupported";
    case SPT_ERR_NO_DEVICE: return "no CUDA device";
    case SPT_ERR_FORMAT: return "invalid GGUF model";
  }
  return "unknown status";
}

spt_status spt_context_create(int device, spt_context **out) {
  if (!out) return fail(nullptr, SPT_ERR_NULL_ARG, "nil output pointer");
  *out = nullptr;
  spt_context *ctx = new spt_context();
  if (device >= 0) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n) {
      cudaGetLastError();
      spt_status st = fail(nullptr, SPT_ERR_NO_DEVICE, "CUDA device %d unavailable", device);
      delete ctx;
      return st;
    }
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      spt_status st = fail(nullptr, SPT_ERR_NO_DEVICE, "CUDA device %d: %s", device, cudaGetErrorString(e));
      delete ctx;
      return st;
    }
    cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    seed_options(ctx);
    ctx->device = device;
    ctx->has_device = true;
    ctx->stream = ctx->own_stream;
    // Resolve the static scratch of spt_forward_moe_batch_device_static now:
    // it loads this library's device code on the device (CUDA loads modules
    // lazily) and with it the array, so a caller that creates its context
    // before reserving the rest of HBM has that memory in place from the start.
    unsigned char *scratch = nullptr;
    spt_status sst = static_scratch(ctx, &scratch);
    if (sst != SPT_OK) {
      const std::string why = ctx->err;
      cudaStreamDestroy(ctx->own_stream);
      delete ctx;
      return fail(nullptr, sst, "%s", why.c_str());
    }
  }
  *out = ctx;
  return SPT_OK;
}

void spt_context_destroy(spt_context *ctx) {
  if (!ctx) return;
  if (ctx->has_device) {
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (DevBuf *b : {&ctx->logits, &ctx->sel_idx, &ctx->sel_w, &ctx->offsets, &ctx->perm,
                      &ctx->slot_pos, &ctx->act_list, &ctx->meta, &ctx->act, &ctx->res,
                      &ctx->xdev, &ctx->outdev, &ctx->dev_err, &ctx->pad_off, &ctx->tile_gu,
                      &ctx->tile_dn, &ctx->pos_expert, &ctx->qx, &ctx->sfx, &ctx->qa, &ctx->sfa,
                      &ctx->stack_norm, &ctx->stack_ffn, &ctx->xq, &ctx->xe, &ctx->actq, &ctx->act_off,
                      &ctx->g16_count, &ctx->route_count})
      b->release();
    for (cudaEvent_t &e : ctx->ev)
      if (e) cudaEventDestroy(e);
    for (auto &g : ctx->graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    if (ctx->hx) cudaFreeHost(ctx->hx);
    if (ctx->hout) cudaFreeHost(ctx->hout);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  }
  delete ctx;
}

spt_status spt_set_stage_timing(spt_context *ctx, int enable) {
  spt_status st = require_device(ctx);
  if (st) return st;
  if (enable)
    for (cudaEvent_t &e : ctx->ev)
      if (!e) SPT_CUDA(ctx, cudaEventCreate(&e));
  ctx->timing = enable != 0;
  return SPT_OK;
}

int spt_stage_times(spt_context *ctx, float *ms, int n) {
  if (!ctx || !ctx->timing || !ctx->timed_last || !ms) return 0;
  if (cudaEventSynchronize(ctx->ev[SPT_NUM_STAGES]) != cudaSuccess) return 0;
  int w = 0;
  for (int i = 0; i < SPT_NUM_STAGES && i < n; ++i, ++w)
    if (cudaEventElapsedTime(&ms[i], ctx->ev[i], ctx->ev[i + 1]) != cudaSuccess) ms[i] = -1.0f;
  return w;
}

int spt_kernels_per_forward(spt_context *ctx) { return ctx ? ctx->kernels_last : 0; }

int spt_last_expert_path(spt_context *ctx, int *tile_tokens) {
  if (tile_tokens) *tile_tokens = ctx ? ctx->last_bn : 0;
  return ctx ? ctx->last_path : -1;
}

const char *spt_last_error(const spt_context *ctx) {
  return ctx ? ctx->err.c_str() : g_tls_error.c_str();
}

void *spt_context_stream(spt_context *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

spt_status spt_context_set_stream(spt_context *ctx, void *stream) {
  if (!ctx) return fail(nullptr, SPT_ERR_NULL_ARG, "nil context");
  ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
  return SPT_OK;
}

spt_status spt_context_sync(spt_context *ctx) {
  spt_status st = require_device(ctx);
  if (st) return st;
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return check_device_error(ctx);
}

spt_status spt_context_set_path(spt_context *ctx, int path) {
  if (!ctx) return fail(nullptr, SPT_ERR_NULL_ARG, "nil context");
  if (path < SPT_PATH_AUTO || path > SPT_PATH_GEMV16) return fail(ctx, SPT_ERR_UNSUPPORTED, "unknown path %d", path);
  ctx->path = path;
  return SPT_OK;
}

spt_status spt_context_set_option(spt_context *ctx, int option, int64_t v) {
  if (!ctx) return fail(nullptr, SPT_ERR_NULL_ARG, "nil context");
  switch (option) {
    case SPT_OPT_TILE_TOKENS:
      if (v != 0 && v != 8 && v != 16 && v != 128) break;
      ctx->opt_tile_tokens = (int)v;
      return SPT_OK;
    case SPT_OPT_FUSED_SELECT:
      if (v < 0 || v > 2) break;
      ctx->opt_fused_select = (int)v;
      return SPT_OK;
    case SPT_OPT_L2_PREFETCH:
      if (v < 0 || v > 64) break;
      ctx->opt_prefetch = (int)v;
      return SPT_OK;
    case SPT_OPT_GEMV16_SLOTS:
      if (v < 0 || v > (1 << 20)) break;
      ctx->opt_gemv16_slots = (int)v;
      return SPT_OK;
    case SPT_OPT_WAIT_LIMIT:
      if (v < 10 || v > 31) break;
      ctx->opt_wait_shift = (int)v;
      return SPT_OK;
    case SPT_OPT_FAULT_STAGE:
      if (v < -1 || v > (1 << 20)) break;
      ctx->opt_fault_stage = (int)v;
      return SPT_OK;
    case SPT_OPT_HOST_GRAPHS:
      if (v != 0 && v != 1) break;
      ctx->opt_host_graphs = (int)v;
      return SPT_OK;
    case SPT_OPT_PREFILL_FP8:
      if (v != 0 && v != 1) break;
      ctx->opt_prefill_fp8 = (int)v;
      return SPT_OK;
    default:
      return fail(ctx, SPT_ERR_UNSUPPORTED, "unknown option %d", option);
  }
  return fail(ctx, SPT_ERR_DIMENSIONS, "option %d: value %lld out of range", option, (long long)v);
}

int64_t spt_context_get_option(const spt_context *ctx, int option) {
  if (!ctx) return -1;
  switch (option) {
    case SPT_OPT_TILE_TOKENS: return ctx->opt_tile_tokens;
    case SPT_OPT_FUSED_SELECT: return ctx->opt_fused_select;
    case SPT_OPT_L2_PREFETCH: return ctx->opt_prefetch;
    case SPT_OPT_GEMV16_SLOTS: return ctx->opt_gemv16_slots;
    case SPT_OPT_WAIT_LIMIT: return ctx->opt_wait_shift;
    case SPT_OPT_FAULT_STAGE: return ctx->opt_fault_stage;
    case SPT_OPT_HOST_GRAPHS: return ctx->opt_host_graphs;
    case SPT_OPT_PREFILL_FP8: return ctx->opt_prefill_fp8;
  }
  return -1;
}

spt_status spt_validate_moe_layer(spt_context *ctx, const spt_reader *reader,
                                  const spt_moe_config *cfg, const spt_layer_weights *lw) {
  return validate_layer(ctx, reader, cfg, lw);
}

// With `views` (spt_arena_create_views) every tensor's bytes come from its
// own pointer instead of reader.base + start; the caller's reader validated
// the file ranges.
static spt_status arena_create_impl(spt_context *ctx, const spt_reader *readers, const spt_moe_config *cfg,
                             const spt_layer_weights *layers, int64_t n_layers, uint32_t flags, int64_t e0,
                             int64_t e1, spt_arena **out, const spt_layer_data *views = nullptr) {
  if (!out || (!readers && !views) || !cfg || !layers || n_layers <= 0)
    return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE context, reader, configuration or weights");
  *out = nullptr;
  for (int64_t l = 0; l < n_layers; ++l) {
    static const uint8_t kAny = 0;
    const spt_reader whole = {&kAny, UINT64_MAX};  // ranges were checked by the caller's reader
    spt_status st = validate_layer(ctx, views ? &whole : &readers[l], cfg, &layers[l]);
    if (st) return st;
    if (views) {
      const spt_layer_weights &w = layers[l];
      const spt_layer_data &v = views[l];
      const std::pair<const spt_tensor *, const uint8_t *> need[] = {
          {&w.ffn_gate_inp, v.ffn_gate_inp},         {&w.ffn_gate_inp_bias, v.ffn_gate_inp_bias},
          {&w.ffn_gate_exps, v.ffn_gate_exps},       {&w.ffn_gate_exps_bias, v.ffn_gate_exps_bias},
          {&w.ffn_up_exps, v.ffn_up_exps},           {&w.ffn_up_exps_bias, v.ffn_up_exps_bias},
          {&w.ffn_down_exps, v.ffn_down_exps},       {&w.ffn_down_exps_bias, v.ffn_down_exps_bias},
          {&w.post_attention_norm, v.post_attention_norm}};
      for (const auto &n : need)
        if (named(*n.first) && !n.second)
          return fail(ctx, SPT_ERR_NULL_ARG, "tensor \"%s\": no data", tname(*n.first));
    }
  }
  spt_status st = require_device(ctx);
  if (st) return st;
  if (flags == 0) flags = SPT_ARENA_GEMV;
  const int64_t H = cfg->hidden_dim, D = cfg->expert_hidden_dim, E = cfg->num_experts;
  if (H > (1 << 30) || D > (1 << 30)) return fail(ctx, SPT_ERR_UNSUPPORTED, "dimensions too large");
  if (e0 < 0 || e1 > E || e0 >= e1) return fail(ctx, SPT_ERR_DIMENSIONS, "expert range [%lld, %lld) outside [0, %lld)",
                                                (long long)e0, (long long)e1, (long long)E);
  const int64_t ne = e1 - e0;  // resident experts
  spt_arena *a = new_arena();
  a->device = ctx->device;
  a->cfg = *cfg;
  a->expert_begin = e0;
  a->expert_count = ne;
  a->flags = flags;
  a->layers.resize((size_t)n_layers);
  std::vector<float> tmp;
  DevBuf range;  // smallest and largest E8M0 byte of a layer's expert blocks
  for (int64_t l = 0; l < n_layers && st == SPT_OK; ++l) {
    const spt_layer_weights &w = layers[l];
    // first byte of tensor t of this layer (views: the caller's pointer)
    auto src = [&](const spt_tensor &t, const uint8_t *view) -> const uint8_t * {
      return views ? view : readers[l].base + t.start;
    };
    const spt_layer_data nov{};
    const spt_layer_data &v = views ? views[l] : nov;
    LayerDev &L = a->layers[(size_t)l];
    float *router = nullptr;
    if ((st = arena_alloc(ctx, a, (size_t)(E * H), &router))) break;
    if ((st = upload(ctx, router, src(w.ffn_gate_inp, v.ffn_gate_inp), (size_t)(E * H * 4)))) break;
    L.router = router;
    tmp.assign((size_t)E, 0.0f);
    if (named(w.ffn_gate_inp_bias))
      decode_floats(src(w.ffn_gate_inp_bias, v.ffn_gate_inp_bias), w.ffn_gate_inp_bias.type, E, tmp.data());
    if ((st = upload_floats(ctx, a, tmp.data(), (size_t)E, &L.router_bias))) break;
    if (named(w.post_attention_norm)) {
      tmp.assign((size_t)H, 0.0f);
      const uint32_t ty = w.post_attention_norm.type == 28 ? 30u : w.post_attention_norm.type;  // RMSNorm's BF16 tag
      decode_floats(src(w.post_attention_norm, v.post_attention_norm), ty, H, tmp.data());
      if ((st = upload_floats(ctx, a, tmp.data(), (size_t)H, &L.norm))) break;
    }
    struct {
      const spt_tensor *t;
      const uint8_t *view;
      int64_t dim;
      const float **dst;
    } biases[] = {{&w.ffn_gate_exps_bias, v.ffn_gate_exps_bias, D, &L.gate_bias},
                  {&w.ffn_up_exps_bias, v.ffn_up_exps_bias, D, &L.up_bias},
                  {&w.ffn_down_exps_bias, v.ffn_down_exps_bias, H, &L.down_bias}};
    for (auto &b : biases) {
      tmp.assign((size_t)(E * b.dim), 0.0f);
      if (named(*b.t)) decode_floats(src(*b.t, b.view), b.t->type, E * b.dim, tmp.data());
      if ((st = upload_floats(ctx, a, tmp.data() + e0 * b.dim, (size_t)(ne * b.dim), b.dst))) break;
    }
    if (st) break;
    if ((flags & SPT_ARENA_MMA) && (st = cuda_ok(ctx, range.ensure(2 * sizeof(int32_t)), "scale range")) == SPT_OK) {
      const int32_t init[2] = {255, 0};
      st = cuda_ok(ctx, cudaMemcpy(range.p, init, sizeof init, cudaMemcpyHostToDevice), "scale range");
    }
    if (st) break;
    {
      DevBuf sg, su;
      // expert e's matrix is the byte range [start + e * per_expert, + per_expert)
      const size_t gu_per = (size_t)D * (H / 32) * 17, gu_raw = (size_t)ne * gu_per;
      if ((st = stage_raw(ctx, &sg, src(w.ffn_gate_exps, v.ffn_gate_exps) + e0 * gu_per, gu_raw)) == SPT_OK &&
          (st = stage_raw(ctx, &su, src(w.ffn_up_exps, v.ffn_up_exps) + e0 * gu_per, gu_raw)) == SPT_OK) {
        if (flags & SPT_ARENA_GEMV) {
          if (st == SPT_OK) st = repack_g8_from(ctx, a, sg.as<uint8_t>(), ne, (int)D, (int)(H / 32), &L.gate);
          if (st == SPT_OK) st = repack_g8_from(ctx, a, su.as<uint8_t>(), ne, (int)D, (int)(H / 32), &L.up);
        }
        if (st == SPT_OK && (flags & SPT_ARENA_MMA)) {
          st = alloc_mma(ctx, a, ne, (int)(2 * D), (int)H, &L.gu_mma);
          if (st == SPT_OK) {
            cudaError_t e = launch_scale_range(sg.as<uint8_t>(), (int64_t)(gu_raw / 17), range.as<int32_t>(), ctx->stream);
            if (e == cudaSuccess)
              e = launch_scale_range(su.as<uint8_t>(), (int64_t)(gu_raw / 17), range.as<int32_t>(), ctx->stream);
            if (e == cudaSuccess)
              e = launch_repack_mma_gu(sg.as<uint8_t>(), su.as<uint8_t>(), ne, (int)D, (int)H, &L.gu_mma, ctx->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
            if (e != cudaSuccess) st = cuda_fail(ctx, e, "repack mma gate/up");
          }
        }
      }
      sg.release();
      su.release();
      if (st) break;
      DevBuf sd;
      const size_t dn_per = (size_t)H * (D / 32) * 17;
      if ((st = stage_raw(ctx, &sd, src(w.ffn_down_exps, v.ffn_down_exps) + e0 * dn_per, (size_t)ne * dn_per)) == SPT_OK) {
        if (flags & SPT_ARENA_GEMV) st = repack_g8_from(ctx, a, sd.as<uint8_t>(), ne, (int)H, (int)(D / 32), &L.down);
        if (st == SPT_OK && (flags & SPT_ARENA_MMA)) {
          st = alloc_mma(ctx, a, ne, (int)H, (int)D, &L.dn_mma);
          if (st == SPT_OK) {
            cudaError_t e = launch_scale_range(sd.as<uint8_t>(), (int64_t)(ne * dn_per / 17), range.as<int32_t>(),
                                               ctx->stream);
            if (e == cudaSuccess) e = launch_repack_mma(sd.as<uint8_t>(), ne, (int)H, (int)D, &L.dn_mma, ctx->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
            if (e != cudaSuccess) st = cuda_fail(ctx, e, "repack mma down");
          }
        }
      }
      sd.release();
      if (st) break;
      L.has_g8 = (flags & SPT_ARENA_GEMV) != 0;
      L.has_mma = (flags & SPT_ARENA_MMA) != 0;
      if (L.has_mma) {
        int32_t r[2] = {0, 255};
        if ((st = cuda_ok(ctx, cudaMemcpy(r, range.p, sizeof r, cudaMemcpyDeviceToHost), "scale range"))) break;
        L.gemv16_ok = r[0] >= kF16ScaleLo && r[1] <= kF16ScaleHi;
      }
    }
  }
  range.release();
  if (st) {
    spt_arena_destroy(a);
    return st;
  }
  *out = a;
  return SPT_OK;
}

spt_status spt_arena_create(spt_context *ctx, const spt_reader *readers, const spt_moe_config *cfg,
                            const spt_layer_weights *layers, int64_t n_layers, uint32_t flags,
                            spt_arena **out) {
  return arena_create_impl(ctx, readers, cfg, layers, n_layers, flags, 0, cfg ? cfg->num_experts : 0, out);
}

spt_status spt_arena_create_views(spt_context *ctx, const spt_moe_config *cfg, const spt_layer_weights *layers,
                                  const spt_layer_data *data, int64_t n_layers, uint32_t flags, int64_t expert_begin,
                                  int64_t expert_end, spt_arena **out) {
  if (!data) return fail(ctx, SPT_ERR_NULL_ARG, "nil tensor data");
  if (expert_end == 0 && cfg) expert_end = cfg->num_experts;
  return arena_create_impl(ctx, nullptr, cfg, layers, n_layers, flags, expert_begin, expert_end, out, data);
}

spt_status spt_arena_create_range(spt_context *ctx, const spt_reader *readers, const spt_moe_config *cfg,
                                  const spt_layer_weights *layers, int64_t n_layers, uint32_t flags,
                                  int64_t expert_begin, int64_t expert_end, spt_arena **out) {
  return arena_create_impl(ctx, readers, cfg, layers, n_layers, flags, expert_begin, expert_end, out);
}

static spt_status synth_create_impl(spt_context *ctx, const spt_moe_config *cfg, const spt_synth_params *p,
                             int64_t n_layers, uint32_t flags, int64_t e0, int64_t e1, spt_arena **out) {
  if (!out || !cfg || !p || n_layers <= 0)
    return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  *out = nullptr;
  spt_status st = validate_config(ctx, cfg);
  if (st) return st;
  const int64_t H = cfg->hidden_dim, D = cfg->expert_hidden_dim, E = cfg->num_experts;
  if (H % 32 != 0 || D % 32 != 0)
    return fail(ctx, SPT_ERR_EXPERT, "expected MXFP4 expert tensor dimensions divisible by 32");
  if ((st = require_device(ctx))) return st;
  if (e0 < 0 || e1 > E || e0 >= e1) return fail(ctx, SPT_ERR_DIMENSIONS, "expert range [%lld, %lld) outside [0, %lld)",
                                                (long long)e0, (long long)e1, (long long)E);
  const int64_t ne = e1 - e0;  // resident experts
  if (flags == 0) flags = SPT_ARENA_GEMV;
  spt_arena *a = new_arena();
  a->device = ctx->device;
  a->cfg = *cfg;
  a->expert_begin = e0;
  a->expert_count = ne;
  a->flags = flags;
  a->layers.resize((size_t)n_layers);
  std::vector<float> tmp;
  for (int64_t l = 0; l < n_layers && st == SPT_OK; ++l) {
    LayerDev &L = a->layers[(size_t)l];
    tmp.resize((size_t)(E * H));
    synth_normal(p->seed, synth_tag(l, kSynthRouter), 0.0f, p->router_std, tmp.data(), E * H);
    if ((st = upload_floats(ctx, a, tmp.data(), tmp.size(), &L.router))) break;
    tmp.resize((size_t)E);
    synth_router_bias(cfg, p, l, tmp.data());
    if ((st = upload_floats(ctx, a, tmp.data(), tmp.size(), &L.router_bias))) break;
    tmp.resize((size_t)H);
    synth_normal(p->seed, synth_tag(l, kSynthNormWeight), 1.0f, kSynthNormStd, tmp.data(), H);
    if ((st = upload_floats(ctx, a, tmp.data(), tmp.size(), &L.norm))) break;
    struct {
      uint32_t kind;
      int64_t dim;
      const float **dst;
    } biases[] = {{kSynthGateBias, D, &L.gate_bias}, {kSynthUpBias, D, &L.up_bias},
                  {kSynthDownBias, H, &L.down_bias}};
    for (auto &b : biases) {
      tmp.assign((size_t)(E * b.dim), 0.0f);
      if (p->expert_bias) synth_normal(p->seed, synth_tag(l, b.kind), 0.0f, p->bias_std, tmp.data(), E * b.dim);
      if ((st = upload_floats(ctx, a, tmp.data() + e0 * b.dim, (size_t)(ne * b.dim), b.dst))) break;
    }
    if (st) break;
    struct {
      uint32_t kind;
      int rows, blocks;
      MatrixG8 *m;
    } mats[] = {{kSynthGate, (int)D, (int)(H / 32), &L.gate},
                {kSynthUp, (int)D, (int)(H / 32), &L.up},
                {kSynthDown, (int)H, (int)(D / 32), &L.down}};
    for (auto &m : mats) {
      if (!(flags & SPT_ARENA_GEMV)) break;
      uint4 *nib = nullptr;
      uint32_t *scl = nullptr;
      if ((st = alloc_g8(ctx, a, ne, m.rows, m.blocks, m.m, &nib, &scl))) break;
      cudaError_t e = launch_synth_g8(p->seed, synth_tag(l, m.kind), e0, ne, m.rows, m.blocks,
                                      p->scale_lo, p->scale_hi, nib, scl, ctx->stream);
      if (e != cudaSuccess) {
        st = cuda_fail(ctx, e, "synth");
        break;
      }
    }
    if (st) break;
    if (flags & SPT_ARENA_MMA) {
      if ((st = alloc_mma(ctx, a, ne, (int)(2 * D), (int)H, &L.gu_mma))) break;
      cudaError_t e = launch_synth_mma_gu(p->seed, synth_tag(l, kSynthGate), synth_tag(l, kSynthUp), e0, ne, (int)D,
                                          (int)H, p->scale_lo, p->scale_hi, &L.gu_mma, ctx->stream);
      if (e != cudaSuccess) {
        st = cuda_fail(ctx, e, "synth mma");
        break;
      }
      if ((st = alloc_mma(ctx, a, ne, (int)H, (int)D, &L.dn_mma))) break;
      e = launch_synth_mma(p->seed, synth_tag(l, kSynthDown), e0, ne, (int)H, (int)D, p->scale_lo, p->scale_hi,
                           &L.dn_mma, ctx->stream);
      if (e != cudaSuccess) {
        st = cuda_fail(ctx, e, "synth mma");
        break;
      }
    }
    L.has_g8 = (flags & SPT_ARENA_GEMV) != 0;
    L.has_mma = (flags & SPT_ARENA_MMA) != 0;
    L.gemv16_ok = p->scale_lo >= kF16ScaleLo && p->scale_hi <= kF16ScaleHi;
  }
  if (st == SPT_OK) {
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) st = cuda_fail(ctx, e, "synth sync");
  }
  if (st) {
    spt_arena_destroy(a);
    return st;
  }
  *out = a;
  return SPT_OK;
}

spt_status spt_arena_create_synthetic(spt_context *ctx, const spt_moe_config *cfg, const spt_synth_params *p,
                                      int64_t n_layers, uint32_t flags, spt_arena **out) {
  return synth_create_impl(ctx, cfg, p, n_layers, flags, 0, cfg ? cfg->num_experts : 0, out);
}

spt_status spt_arena_create_synthetic_range(spt_context *ctx, const spt_moe_config *cfg,
                                            const spt_synth_params *p, int64_t n_layers, uint32_t flags,
                                            int64_t expert_begin, int64_t expert_end, spt_arena **out) {
  return synth_create_impl(ctx, cfg, p, n_layers, flags, expert_begin, expert_end, out);
}

void spt_arena_expert_range(const spt_arena *arena, int64_t *expert_begin, int64_t *expert_end) {
  if (expert_begin) *expert_begin = arena ? arena->expert_begin : 0;
  if (expert_end) *expert_end = arena ? arena->expert_begin + arena->expert_count : 0;
}

void spt_arena_destroy(spt_arena *a) {
  if (!a) return;
  if (a->device >= 0) cudaSetDevice(a->device);
  for (void *p : a->allocs) cudaFree(p);
  delete a;
}

uint64_t spt_arena_bytes(const spt_arena *a) { return a ? a->bytes : 0; }

spt_status spt_synth_layer_host(const spt_moe_config *cfg, const spt_synth_params *p, int64_t layer,
                                uint8_t *router, float *router_bias, uint8_t *gate, uint8_t *up,
                                uint8_t *down, float *gate_bias, float *up_bias, float *down_bias) {
  if (!cfg || !p) return fail(nullptr, SPT_ERR_NULL_ARG, "nil argument");
  spt_status st = validate_config(nullptr, cfg);
  if (st) return st;
  const int64_t H = cfg->hidden_dim, D = cfg->expert_hidden_dim, E = cfg->num_experts;
  if (H % 32 != 0 || D % 32 != 0) return fail(nullptr, SPT_ERR_EXPERT, "dimensions not divisible by 32");
  if (router) {
    std::vector<float> tmp((size_t)(E * H));
    synth_normal(p->seed, synth_tag(layer, kSynthRouter), 0.0f, p->router_std, tmp.data(), E * H);
    memcpy(router, tmp.data(), tmp.size() * 4);
  }
  if (router_bias) synth_router_bias(cfg, p, layer, router_bias);
  struct {
    uint32_t kind;
    int64_t dim;
    float *dst;
  } biases[] = {{kSynthGateBias, D, gate_bias}, {kSynthUpBias, D, up_bias}, {kSynthDownBias, H, down_bias}};
  for (auto &b : biases) {
    if (!b.dst) continue;
    if (p->expert_bias) synth_normal(p->seed, synth_tag(layer, b.kind), 0.0f, p->bias_std, b.dst, E * b.dim);
    else std::fill(b.dst, b.dst + E * b.dim, 0.0f);
  }
  struct {
    uint32_t kind;
    int64_t rows, blocks;
    uint8_t *dst;
  } mats[] = {{kSynthGate, D, H / 32, gate}, {kSynthUp, D, H / 32, up}, {kSynthDown, H, D / 32, down}};
  for (auto &m : mats) {
    if (!m.dst) continue;
    const int64_t n = E * m.rows * m.blocks;
    for (int64_t i = 0; i < n; ++i)
      synth_mxfp4_block(p->seed, synth_tag(layer, m.kind), (uint64_t)i, p->scale_lo, p->scale_hi, m.dst + 17 * i);
  }
  return SPT_OK;
}

spt_status spt_synth_norm_host(const spt_synth_params *p, int64_t layer, int64_t dim, float *out) {
  if (!p || !out || dim <= 0) return fail(nullptr, SPT_ERR_NULL_ARG, "nil argument");
  synth_normal(p->seed, synth_tag(layer, kSynthNormWeight), 1.0f, kSynthNormStd, out, dim);
  return SPT_OK;
}

spt_status spt_synth_normal_host(uint64_t seed, uint64_t stream, float mean, float sd, float *out,
                                 int64_t n) {
  if (!out && n > 0) return fail(nullptr, SPT_ERR_NULL_ARG, "nil output");
  synth_normal(seed, (uint32_t)stream, mean, sd, out, n);
  return SPT_OK;
}

spt_status spt_forward_moe_batch(spt_context *ctx, spt_arena *arena, int64_t layer, const float *x,
                                 int64_t x_len, float *out, int64_t out_len, int64_t batch,
                                 const volatile int32_t *cancel) {
  return forward_host(ctx, arena, layer, x, x_len, out, out_len, batch, cancel);
}

spt_status spt_forward_moe(spt_context *ctx, spt_arena *arena, int64_t layer, const float *x,
                           int64_t x_len, float *out, int64_t out_len,
                           const volatile int32_t *cancel) {
  return forward_host(ctx, arena, layer, x, x_len, out, out_len, 1, cancel);
}

spt_status spt_forward_moe_batch_device(spt_context *ctx, spt_arena *arena, int64_t layer,
                                        const float *x, float *out, int64_t batch) {
  if (!ctx || !arena || !x || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (batch <= 0 || layer < 0 || layer >= (int64_t)arena->layers.size())
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(ctx, SPT_ERR_DIMENSIONS, "device x and out must be 16-byte aligned");
  spt_status st = require_device(ctx);
  if (st) return st;
  return forward_device(ctx, arena, layer, x, out, batch);
}

spt_status spt_forward_moe_batch_reader(spt_context *ctx, const spt_reader *reader,
                                        const spt_moe_config *cfg, const spt_layer_weights *lw,
                                        const float *x, int64_t x_len, float *out, int64_t out_len,
                                        int64_t batch, const volatile int32_t *cancel) {
  if (!ctx || !reader || !cfg || !lw)
    return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE context, reader, configuration or weights");
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  spt_status st = validate_config(ctx, cfg);
  if (st) return st;
  if ((st = check_batch(ctx, *cfg, x, x_len, out, out_len, batch))) return st;
  if ((st = validate_layer(ctx, reader, cfg, lw))) return st;
  spt_arena *arena = nullptr;
  if ((st = spt_arena_create(ctx, reader, cfg, lw, 1, SPT_ARENA_GEMV, &arena))) return st;
  st = forward_host(ctx, arena, 0, x, x_len, out, out_len, batch, cancel);
  spt_arena_destroy(arena);
  return st;
}

spt_status spt_last_routing(spt_context *ctx, float *logits, int32_t *sel_index, float *sel_weight,
                            int32_t *perm, int32_t *expert_count, int64_t *dispatched) {
  spt_status st = require_device(ctx);
  if (st) return st;
  if (!ctx->have_routing) return fail(ctx, SPT_ERR_DIMENSIONS, "no forward call yet");
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  const int64_t T = ctx->last_T, E = ctx->last_E, K = ctx->last_K;
  int32_t meta[2];
  SPT_CUDA(ctx, cudaMemcpy(meta, ctx->meta.p, sizeof meta, cudaMemcpyDeviceToHost));
  if (logits) SPT_CUDA(ctx, cudaMemcpy(logits, ctx->logits.p, sizeof(float) * T * E, cudaMemcpyDeviceToHost));
  if (sel_index) SPT_CUDA(ctx, cudaMemcpy(sel_index, ctx->sel_idx.p, sizeof(int32_t) * T * K, cudaMemcpyDeviceToHost));
  if (sel_weight) SPT_CUDA(ctx, cudaMemcpy(sel_weight, ctx->sel_w.p, sizeof(float) * T * K, cudaMemcpyDeviceToHost));
  if (perm && meta[1] > 0) SPT_CUDA(ctx, cudaMemcpy(perm, ctx->perm.p, sizeof(int32_t) * meta[1], cudaMemcpyDeviceToHost));
  if (expert_count) {
    std::vector<int32_t> off((size_t)E + 1);
    SPT_CUDA(ctx, cudaMemcpy(off.data(), ctx->offsets.p, sizeof(int32_t) * (E + 1), cudaMemcpyDeviceToHost));
    for (int64_t e = 0; e < E; ++e) expert_count[e] = off[e + 1] - off[e];
  }
  if (dispatched) *dispatched = meta[1];
  return SPT_OK;
}

spt_status spt_route_moe_batch(spt_context *ctx, const uint8_t *data, uint64_t data_len,
                               const float *x, int64_t x_len, const float *router_bias,
                               int64_t batch, int64_t hidden, int64_t experts, float *logits,
                               const volatile int32_t *cancel) {
  if (!data || !x || !logits) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  int64_t nw = 0, nx = 0, nl = 0;
  if (!product({experts, hidden, 4}, &nw) || !product({batch, hidden}, &nx) ||
      !product({batch, experts}, &nl) || data_len != (uint64_t)nw || x_len != nx)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid router dimensions");
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  spt_status st = require_device(ctx);
  if (st) return st;
  Tmp dw, dx, db, dl;
  SPT_CUDA(ctx, dw.alloc((size_t)nw));
  SPT_CUDA(ctx, dx.alloc(sizeof(float) * (size_t)nx));
  SPT_CUDA(ctx, dl.alloc(sizeof(float) * (size_t)nl));
  SPT_CUDA(ctx, cudaMemcpyAsync(dw.p, data, (size_t)nw, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(dx.p, x, sizeof(float) * (size_t)nx, cudaMemcpyHostToDevice, ctx->stream));
  if (router_bias) {
    SPT_CUDA(ctx, db.alloc(sizeof(float) * (size_t)experts));
    SPT_CUDA(ctx, cudaMemcpyAsync(db.p, router_bias, sizeof(float) * (size_t)experts, cudaMemcpyHostToDevice, ctx->stream));
  }
  SPT_CUDA(ctx, launch_router(dw.as<float>(), dx.as<float>(), db.as<float>(), (int)batch, (int)hidden,
                              (int)experts, dl.as<float>(), 8, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(logits, dl.p, sizeof(float) * (size_t)nl, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  return SPT_OK;
}

spt_status spt_select_moe_batch(spt_context *ctx, const float *logits, int64_t batch, int64_t experts,
                                int64_t k, int32_t *index, float *weight) {
  if (!logits || !index || !weight) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (batch <= 0 || experts <= 0 || k <= 0) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid dimensions");
  if (k > kSelectMaxK) return fail(ctx, SPT_ERR_UNSUPPORTED, "top-k > %d", kSelectMaxK);
  spt_status st = require_device(ctx);
  if (st) return st;
  Tmp dl, di, dw;
  SPT_CUDA(ctx, dl.alloc(sizeof(float) * batch * experts));
  SPT_CUDA(ctx, di.alloc(sizeof(int32_t) * batch * k));
  SPT_CUDA(ctx, dw.alloc(sizeof(float) * batch * k));
  SPT_CUDA(ctx, cudaMemcpyAsync(dl.p, logits, sizeof(float) * batch * experts, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, launch_select(dl.as<float>(), (int)batch, (int)experts, (int)k, di.as<int32_t>(), dw.as<float>(), ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(index, di.p, sizeof(int32_t) * batch * k, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(weight, dw.p, sizeof(float) * batch * k, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return SPT_OK;
}

spt_status spt_dispatch_moe_batch(spt_context *ctx, const int32_t *index, const float *weight,
                                  int64_t batch, int64_t k, int64_t experts, int32_t *perm,
                                  int32_t *expert_offsets, int64_t *dispatched) {
  if (!index || !weight || !perm || !expert_offsets) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (batch <= 0 || k <= 0 || experts <= 0) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid dimensions");
  if (experts > kDispatchMaxExperts) return fail(ctx, SPT_ERR_UNSUPPORTED, "experts > %d", kDispatchMaxExperts);
  const int64_t S = batch * k;
  for (int64_t s = 0; s < S; ++s)
    if (index[s] < 0 || index[s] >= experts) return fail(ctx, SPT_ERR_DIMENSIONS, "expert index out of range");
  spt_status st = require_device(ctx);
  if (st) return st;
  Tmp di, dw, doff, dperm, dpos, dact, dmeta;
  SPT_CUDA(ctx, di.alloc(sizeof(int32_t) * S));
  SPT_CUDA(ctx, dw.alloc(sizeof(float) * S));
  SPT_CUDA(ctx, doff.alloc(sizeof(int32_t) * (experts + 1)));
  SPT_CUDA(ctx, dperm.alloc(sizeof(int32_t) * S));
  SPT_CUDA(ctx, dpos.alloc(sizeof(int32_t) * S));
  SPT_CUDA(ctx, dact.alloc(sizeof(int32_t) * experts));
  SPT_CUDA(ctx, dmeta.alloc(sizeof(int32_t) * 4));
  SPT_CUDA(ctx, cudaMemcpyAsync(di.p, index, sizeof(int32_t) * S, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(dw.p, weight, sizeof(float) * S, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, launch_dispatch(di.as<int32_t>(), dw.as<float>(), (int)S, (int)experts, doff.as<int32_t>(),
                                dperm.as<int32_t>(), dpos.as<int32_t>(), dact.as<int32_t>(),
                                dmeta.as<int32_t>(), ctx->stream));
  int32_t meta[2];
  SPT_CUDA(ctx, cudaMemcpyAsync(meta, dmeta.p, sizeof meta, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(expert_offsets, doff.p, sizeof(int32_t) * (experts + 1), cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (meta[1] > 0) SPT_CUDA(ctx, cudaMemcpy(perm, dperm.p, sizeof(int32_t) * meta[1], cudaMemcpyDeviceToHost));
  if (dispatched) *dispatched = meta[1];
  return SPT_OK;
}

spt_status spt_mul_moe_batch_expert(spt_context *ctx, const uint8_t *data, uint64_t data_len,
                                    int64_t input, int64_t output, const float *x, int64_t x_len,
                                    const int64_t *x_offsets, int64_t count, const float *bias,
                                    float *y, int64_t y_len, const int64_t *y_offsets,
                                    const volatile int32_t *cancel) {
  if (!data || !x || !y || !x_offsets || !y_offsets) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  int64_t nbytes = 0;
  if (input <= 0 || input % 32 != 0 || output <= 0 || count <= 0 ||
      !product({input / 32, 17, output}, &nbytes) || data_len != (uint64_t)nbytes)
    return fail(ctx, SPT_ERR_EXPERT, "expected MXFP4 expert matrix [%lld %lld]", (long long)input, (long long)output);
  for (int64_t j = 0; j < count; ++j) {
    if (x_offsets[j] < 0 || x_offsets[j] > x_len - input || y_offsets[j] < 0 ||
        y_offsets[j] > y_len - output)
      return fail(ctx, SPT_ERR_DIMENSIONS, "offset %lld out of range", (long long)j);
  }
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  spt_status st = require_device(ctx);
  if (st) return st;
  if (output > (1 << 30) || input > (1 << 30)) return fail(ctx, SPT_ERR_UNSUPPORTED, "matrix too large");
  const int rows = (int)output, blocks = (int)(input / 32);
  // one-expert G8 arena for this matrix
  spt_arena tmp_arena;
  tmp_arena.device = ctx->device;
  MatrixG8 m;
  if ((st = upload_mxfp4(ctx, &tmp_arena, data, 1, rows, blocks, &m))) {
    for (void *p : tmp_arena.allocs) cudaFree(p);
    return st;
  }
  std::vector<float> xg((size_t)(count * input));
  for (int64_t j = 0; j < count; ++j)
    memcpy(&xg[(size_t)(j * input)], x + x_offsets[j], sizeof(float) * (size_t)input);
  Tmp dx, dy, db, doff, dact, dmeta;
  cudaError_t e = dx.alloc(sizeof(float) * xg.size());
  if (e == cudaSuccess) e = dy.alloc(sizeof(float) * (size_t)(count * output));
  if (e == cudaSuccess) e = doff.alloc(sizeof(int32_t) * 2);
  if (e == cudaSuccess) e = dact.alloc(sizeof(int32_t));
  if (e == cudaSuccess) e = dmeta.alloc(sizeof(int32_t) * 4);
  if (e == cudaSuccess && bias) e = db.alloc(sizeof(float) * (size_t)output);
  const int32_t off_h[2] = {0, (int32_t)count}, act_h[1] = {0}, meta_h[4] = {1, (int32_t)count, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpyAsync(dx.p, xg.data(), sizeof(float) * xg.size(), cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(doff.p, off_h, sizeof off_h, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dact.p, act_h, sizeof act_h, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dmeta.p, meta_h, sizeof meta_h, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess && bias) e = cudaMemcpyAsync(db.p, bias, sizeof(float) * (size_t)output, cudaMemcpyHostToDevice, ctx->stream);
  std::vector<float> yg((size_t)(count * output));
  if (e == cudaSuccess) {
    GemvLaunch g;
    g.m0 = m;
    g.bias0 = db.as<float>();
    g.x = dx.as<float>();
    g.x_stride = input;
    g.y = dy.as<float>();
    g.y_stride = output;
    g.offsets = doff.as<int32_t>();
    g.act_list = dact.as<int32_t>();
    g.meta = dmeta.as<int32_t>();
    g.mode = kRowsMoEDown;
    g.gate_up = false;
    g.max_active = 1;
    g.mt = count >= 8 ? 8 : (count >= 4 ? 4 : (count >= 2 ? 2 : 1));
    e = launch_gemv(g, ctx->sm_count, ctx->stream);
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(yg.data(), dy.p, sizeof(float) * yg.size(), cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  for (void *p : tmp_arena.allocs) cudaFree(p);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "mul_moe_batch_expert");
  for (int64_t j = 0; j < count; ++j)
    memcpy(y + y_offsets[j], &yg[(size_t)(j * output)], sizeof(float) * (size_t)output);
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  return SPT_OK;
}

spt_status spt_swiglu(spt_context *ctx, const float *gate, const float *up, float *act, int64_t n) {
  if (!gate || !up || !act) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (n <= 0) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid length");
  spt_status st = require_device(ctx);
  if (st) return st;
  Tmp dg, du, da;
  SPT_CUDA(ctx, dg.alloc(sizeof(float) * n));
  SPT_CUDA(ctx, du.alloc(sizeof(float) * n));
  SPT_CUDA(ctx, da.alloc(sizeof(float) * n));
  SPT_CUDA(ctx, cudaMemcpyAsync(dg.p, gate, sizeof(float) * n, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(du.p, up, sizeof(float) * n, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, launch_swiglu(dg.as<float>(), du.as<float>(), da.as<float>(), n, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(act, da.p, sizeof(float) * n, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return SPT_OK;
}

spt_status spt_combine_moe_batch(spt_context *ctx, const float *results, const float *weight,
                                 int64_t batch, int64_t k, int64_t hidden, float *out) {
  if (!results || !weight || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (batch <= 0 || k <= 0 || hidden <= 0 || hidden % 4 != 0)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid dimensions");
  spt_status st = require_device(ctx);
  if (st) return st;
  Tmp dr, dw, dout;
  SPT_CUDA(ctx, dr.alloc(sizeof(float) * batch * k * hidden));
  SPT_CUDA(ctx, dw.alloc(sizeof(float) * batch * k));
  SPT_CUDA(ctx, dout.alloc(sizeof(float) * batch * hidden));
  SPT_CUDA(ctx, cudaMemcpyAsync(dr.p, results, sizeof(float) * batch * k * hidden, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(dw.p, weight, sizeof(float) * batch * k, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, launch_combine(dr.as<float>(), dw.as<float>(), nullptr, (int)batch, (int)k, (int)hidden,
                               dout.as<float>(), ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(out, dout.p, sizeof(float) * batch * hidden, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return SPT_OK;
}

spt_status spt_rmsnorm(spt_context *ctx, const float *x, const float *weight, int64_t batch,
                       int64_t dim, float eps, float *y) {
  if (!x || !weight || !y) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (batch <= 0 || dim <= 0) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid dimensions");
  if (eps < 0 || isnan(eps) || isinf(eps)) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid epsilon: %g", (double)eps);
  spt_status st = require_device(ctx);
  if (st) return st;
  Tmp dx, dw, dy;
  SPT_CUDA(ctx, dx.alloc(sizeof(float) * batch * dim));
  SPT_CUDA(ctx, dw.alloc(sizeof(float) * dim));
  SPT_CUDA(ctx, dy.alloc(sizeof(float) * batch * dim));
  SPT_CUDA(ctx, cudaMemcpyAsync(dx.p, x, sizeof(float) * batch * dim, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(dw.p, weight, sizeof(float) * dim, cudaMemcpyHostToDevice, ctx->stream));
  SPT_CUDA(ctx, launch_rmsnorm(dx.as<float>(), dw.as<float>(), (int)batch, (int)dim, eps, dy.as<float>(), 8, ctx->stream));
  SPT_CUDA(ctx, cudaMemcpyAsync(y, dy.p, sizeof(float) * batch * dim, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return SPT_OK;
}

spt_status spt_q80_matrix_create(spt_context *ctx, const uint8_t *data, uint64_t data_len, int64_t input,
                                 int64_t output, spt_q80_matrix **out) {
  if (!ctx || !data || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil context, data or output");
  *out = nullptr;
  // q80Shape (forward/q80.go:150-170)
  if (input <= 0 || output <= 0 || input % 32 != 0)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid Q8_0 shape [%lld %lld]", (long long)input, (long long)output);
  if (input > (1 << 24) || output > 0xffffffffll)
    return fail(ctx, SPT_ERR_DIMENSIONS, "matrix dimensions exceed platform limits");
  const uint64_t row_bytes = (uint64_t)input / 32 * 34;
  if (data_len != row_bytes * (uint64_t)output) return fail(ctx, SPT_ERR_FILE_RANGE, "invalid byte range");
  if (q80_rows_per_chunk((int)input) <= 0)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "Q8_0 rows of %lld elements exceed the shared-memory ring", (long long)input);
  spt_status st = require_device(ctx);
  if (st) return st;
  spt_q80_matrix *m = new spt_q80_matrix();
  m->ctx = ctx;
  m->input = input;
  m->output = output;
  // the file's rows go up once and are repacked into four-row groups in HBM
  const uint64_t packed = q80_packed_bytes(output, (int)input);
  Tmp raw;
  cudaError_t e = m->w.ensure(packed);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->w.p, 0, packed, ctx->stream);
  if (e == cudaSuccess) e = raw.alloc(data_len);
  if (e == cudaSuccess) e = cudaMemcpyAsync(raw.p, data, data_len, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = launch_q80_repack(raw.as<uint8_t>(), output, (int)input, m->w.as<uint8_t>(), ctx->stream);
  if (e == cudaSuccess) e = m->best.ensure(sizeof(unsigned long long));
  if (e == cudaSuccess) e = m->err.ensure(sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemsetAsync(m->err.p, 0, sizeof(int32_t), ctx->stream);
  if (e == cudaSuccess) e = m->res.ensure(16);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    spt_q80_matrix_destroy(m);
    return cuda_fail(ctx, e, "Q8_0 matrix upload");
  }
  *out = m;
  return SPT_OK;
}

void spt_q80_matrix_destroy(spt_q80_matrix *m) {
  if (!m) return;
  if (m->ctx && m->ctx->has_device) {
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
  }
  for (DevBuf *b : {&m->w, &m->best, &m->err, &m->res, &m->xdev, &m->ydev}) b->release();
  delete m;
}

spt_status spt_mul_q80_matrix_device(spt_context *ctx, spt_q80_matrix *m, const float *x, float *y, int64_t *argmax,
                                     float *best_logit) {
  if (!ctx || !m || !x) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (m->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "Q8_0 matrix belongs to another context");
  spt_status st = require_device(ctx);
  if (st) return st;
  SPT_CUDA(ctx, launch_q80(m->w.as<uint8_t>(), m->output, (int)m->input, x, y, m->best.as<unsigned long long>(),
                           argmax, best_logit, m->err.as<int32_t>(), ctx->sm_count, ctx->stream));
  ctx->kernels_last = 3;  // key init, GEMV, decode
  return SPT_OK;
}

spt_status spt_mul_q80_matrix(spt_context *ctx, spt_q80_matrix *m, const float *x, float *y, int64_t *argmax,
                              float *best_logit) {
  if (!ctx || !m || !x) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (m->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "Q8_0 matrix belongs to another context");
  spt_status st = require_device(ctx);
  if (st) return st;
  cudaStream_t s = ctx->stream;
  SPT_CUDA(ctx, m->xdev.ensure(sizeof(float) * m->input));
  if (y) SPT_CUDA(ctx, m->ydev.ensure(sizeof(float) * m->output));
  SPT_CUDA(ctx, cudaMemcpyAsync(m->xdev.p, x, sizeof(float) * m->input, cudaMemcpyHostToDevice, s));
  int64_t *d_arg = m->res.as<int64_t>();
  float *d_logit = reinterpret_cast<float *>(m->res.as<uint8_t>() + 8);
  if ((st = spt_mul_q80_matrix_device(ctx, m, m->xdev.as<float>(), y ? m->ydev.as<float>() : nullptr, d_arg,
                                      d_logit)))
    return st;
  if (y) SPT_CUDA(ctx, cudaMemcpyAsync(y, m->ydev.p, sizeof(float) * m->output, cudaMemcpyDeviceToHost, s));
  uint8_t res[16];
  SPT_CUDA(ctx, cudaMemcpyAsync(res, m->res.p, 16, cudaMemcpyDeviceToHost, s));
  int32_t err = 0;
  SPT_CUDA(ctx, cudaMemcpyAsync(&err, m->err.p, sizeof err, cudaMemcpyDeviceToHost, s));
  SPT_CUDA(ctx, cudaStreamSynchronize(s));
  if (err) {
    SPT_CUDA(ctx, cudaMemset(m->err.p, 0, sizeof err));
    return fail(ctx, SPT_ERR_TIMEOUT, "Q8_0 GEMV: bounded wait gave up");
  }
  if (argmax) memcpy(argmax, res, 8);
  if (best_logit) memcpy(best_logit, res + 8, 4);
  return SPT_OK;
}

spt_status spt_mul_q80(spt_context *ctx, const uint8_t *data, uint64_t data_len, int64_t input,
                       int64_t output, const float *x, float *y, int64_t *argmax, float *best_logit) {
  spt_q80_matrix *m = nullptr;
  spt_status st = spt_q80_matrix_create(ctx, data, data_len, input, output, &m);
  if (st) return st;
  st = spt_mul_q80_matrix(ctx, m, x, y, argmax, best_logit);
  spt_q80_matrix_destroy(m);
  return st;
}


// ---- Q4_0 (forward/q40.go:35-130) -------------------------------------------

namespace {

// q40Shape (forward/q40.go:105-130): type 2, two dimensions, input a nonzero
// multiple of 32, output nonzero, byte range = output rows of input/32
// 18-byte blocks; then the reader's range check.
spt_status q40_shape(spt_context *ctx, const spt_reader *reader, const spt_tensor *t, int64_t *input,
                     int64_t *output) {
  if (!reader || !reader->base) return fail(ctx, SPT_ERR_NULL_ARG, "nil GGUF reader");
  if (!t) return fail(ctx, SPT_ERR_NULL_ARG, "nil tensor");
  if (t->type != 2)
    return fail(ctx, SPT_ERR_DIMENSIONS, "\"%s\": GGML type %u instead of Q4_0 (2)", tname(*t), t->type);
  if (t->n_dims != 2) return fail(ctx, SPT_ERR_DIMENSIONS, "\"%s\": expected a two-dimensional matrix", tname(*t));
  const uint64_t in = t->shape[0], out = t->shape[1];
  if (in == 0 || out == 0 || in % 32 != 0)
    return fail(ctx, SPT_ERR_DIMENSIONS, "\"%s\": invalid Q4_0 matrix shape [%llu %llu]", tname(*t),
                (unsigned long long)in, (unsigned long long)out);
  const uint64_t max_int = (uint64_t)INT64_MAX;
  if (in > max_int || out > max_int || in / 32 > max_int / 18)
    return fail(ctx, SPT_ERR_DIMENSIONS, "\"%s\": matrix dimensions exceed platform limits", tname(*t));
  const uint64_t bytes = in / 32 * 18;
  if (out > UINT64_MAX / bytes || t->end <= t->start || t->end - t->start != out * bytes)
    return fail(ctx, SPT_ERR_FILE_RANGE, "\"%s\": invalid tensor byte range for shape [%llu %llu]", tname(*t),
                (unsigned long long)in, (unsigned long long)out);
  spt_status st = validate_file_range(ctx, reader, *t);
  if (st) return st;
  // this build: the one-input kernel's shared-memory ring and 32-bit grids
  if (!q40_supported((int)std::min<uint64_t>(in, 1u << 30)) || out > 0x7fffffffull)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "\"%s\": Q4_0 matrix [%llu %llu] exceeds this build's limits", tname(*t),
                (unsigned long long)in, (unsigned long long)out);
  *input = (int64_t)in;
  *output = (int64_t)out;
  return SPT_OK;
}

// MulQ40BatchInto's argument checks (forward/q40.go:58-71).
spt_status q40_args(spt_context *ctx, int64_t input, int64_t output, const float *x, int64_t x_len,
                    const float *y, int64_t y_len, int64_t batch, bool lengths) {
  if (batch < 1 || batch > INT64_MAX / input || batch > INT64_MAX / output)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid or oversized batch: %lld", (long long)batch);
  if (batch > INT64_MAX / 4 / std::max(input, output))
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid or oversized batch: %lld", (long long)batch);
  if (lengths && (x_len != batch * input || y_len != batch * output))
    return fail(ctx, SPT_ERR_DIMENSIONS, "expected %lld input and %lld output elements, got %lld and %lld",
                (long long)(batch * input), (long long)(batch * output), (long long)x_len, (long long)y_len);
  if (!x || !y) return fail(ctx, SPT_ERR_NULL_ARG, "nil input or output");
  const uintptr_t a = (uintptr_t)x, b = (uintptr_t)y;
  const uintptr_t na = (uintptr_t)(batch * input) * 4, nb = (uintptr_t)(batch * output) * 4;
  if (a < b + nb && b < a + na) return fail(ctx, SPT_ERR_OVERLAP, "input and output must not overlap");
  return SPT_OK;
}

}  // namespace

spt_status spt_q40_matrix_create(spt_context *ctx, const spt_reader *reader, const spt_tensor *tensor,
                                 spt_q40_matrix **out) {
  if (!ctx || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil context or output");
  *out = nullptr;
  int64_t input = 0, output = 0;
  spt_status st = q40_shape(ctx, reader, tensor, &input, &output);
  if (st) return st;
  if ((st = require_device(ctx))) return st;
  const uint64_t len = tensor->end - tensor->start;
  spt_q40_matrix *m = new spt_q40_matrix();
  m->ctx = ctx;
  m->input = input;
  m->output = output;
  cudaError_t e = m->w.ensure(len + 64);  // the last chunk's copy rounds up to 16 bytes
  if (e == cudaSuccess) e = cudaMemsetAsync(m->w.p, 0, len + 64, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(m->w.p, reader->base + tensor->start, len, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = m->err.ensure(sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemsetAsync(m->err.p, 0, sizeof(int32_t), ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    spt_q40_matrix_destroy(m);
    return cuda_fail(ctx, e, "Q4_0 matrix upload");
  }
  *out = m;
  return SPT_OK;
}

void spt_q40_matrix_destroy(spt_q40_matrix *m) {
  if (!m) return;
  if (m->ctx && m->ctx->has_device) {
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
  }
  for (DevBuf *b : {&m->w, &m->err, &m->xdev, &m->ydev}) b->release();
  delete m;
}

spt_status spt_q40_matrix_shape(const spt_q40_matrix *m, int64_t *input, int64_t *output) {
  if (!m) return SPT_ERR_NULL_ARG;
  if (input) *input = m->input;
  if (output) *output = m->output;
  return SPT_OK;
}

spt_status spt_mul_q40_matrix_device(spt_context *ctx, spt_q40_matrix *m, const float *x, float *y, int64_t batch) {
  if (!ctx || !m) return fail(ctx, SPT_ERR_NULL_ARG, "nil context or matrix");
  if (m->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "Q4_0 matrix belongs to another context");
  spt_status st = q40_args(ctx, m->input, m->output, x, 0, y, 0, batch, false);
  if (st) return st;
  if ((st = require_device(ctx))) return st;
  SPT_CUDA(ctx, launch_q40(m->w.as<uint8_t>(), m->output, (int)m->input, x, batch, y, m->err.as<int32_t>(),
                           ctx->sm_count, ctx->stream));
  ctx->kernels_last = 1;
  return SPT_OK;
}

spt_status spt_mul_q40_matrix(spt_context *ctx, spt_q40_matrix *m, const float *x, int64_t x_len, float *y,
                              int64_t y_len, int64_t batch, const volatile int32_t *cancel) {
  if (!ctx || !m) return fail(ctx, SPT_ERR_NULL_ARG, "nil context or matrix");
  if (m->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "Q4_0 matrix belongs to another context");
  spt_status st = q40_args(ctx, m->input, m->output, x, x_len, y, y_len, batch, true);
  if (st) return st;
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  if ((st = require_device(ctx))) return st;
  cudaStream_t s = ctx->stream;
  const size_t xb = sizeof(float) * (size_t)(batch * m->input), yb = sizeof(float) * (size_t)(batch * m->output);
  SPT_CUDA(ctx, m->xdev.ensure(xb));
  SPT_CUDA(ctx, m->ydev.ensure(yb));
  SPT_CUDA(ctx, cudaMemcpyAsync(m->xdev.p, x, xb, cudaMemcpyHostToDevice, s));
  if ((st = spt_mul_q40_matrix_device(ctx, m, m->xdev.as<float>(), m->ydev.as<float>(), batch))) return st;
  SPT_CUDA(ctx, cudaMemcpyAsync(y, m->ydev.p, yb, cudaMemcpyDeviceToHost, s));
  int32_t err = 0;
  SPT_CUDA(ctx, cudaMemcpyAsync(&err, m->err.p, sizeof err, cudaMemcpyDeviceToHost, s));
  SPT_CUDA(ctx, cudaStreamSynchronize(s));
  if (err) {
    SPT_CUDA(ctx, cudaMemset(m->err.p, 0, sizeof err));
    return fail(ctx, SPT_ERR_TIMEOUT, "Q4_0 GEMV: bounded wait gave up");
  }
  return SPT_OK;
}

spt_status spt_mul_q40_batch(spt_context *ctx, const spt_reader *reader, const spt_tensor *tensor, const float *x,
                             int64_t x_len, float *y, int64_t y_len, int64_t batch, const volatile int32_t *cancel) {
  if (!ctx) return fail(ctx, SPT_ERR_NULL_ARG, "nil context");
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  int64_t input = 0, output = 0;
  spt_status st = q40_shape(ctx, reader, tensor, &input, &output);
  if (st) return st;
  if ((st = q40_args(ctx, input, output, x, x_len, y, y_len, batch, true))) return st;
  spt_q40_matrix *m = nullptr;
  if ((st = spt_q40_matrix_create(ctx, reader, tensor, &m))) return st;
  st = spt_mul_q40_matrix(ctx, m, x, x_len, y, y_len, batch, cancel);
  spt_q40_matrix_destroy(m);
  return st;
}

spt_status spt_mul_q40(spt_context *ctx, const spt_reader *reader, const spt_tensor *tensor, const float *x,
                       int64_t x_len, float *y, int64_t y_len, const volatile int32_t *cancel) {
  return spt_mul_q40_batch(ctx, reader, tensor, x, x_len, y, y_len, 1, cancel);
}

}  // extern "C"

// =========================================================================
// Allocation-free forward.  Some callers cannot let this library call
// cudaMalloc once they are running: an engine that reserved all of HBM for
// the expert arena and its own caching allocator at load time (a late
// cudaMalloc would fail or evict), and latency-critical decode loops, where
// cudaMalloc/cudaFree synchronise the whole device.  This entry point runs the
// exact path with every intermediate in one file-scope device array instead
// of the context's grow-on-demand buffers.
namespace {

constexpr int64_t kStaticMaxSlots = 64;     // tokens x top-k per call
constexpr int64_t kStaticMaxDim = 4096;     // hidden and expert dimension
constexpr int64_t kStaticMaxExperts = 256;  // experts (the dispatch kernel's limit too)

constexpr size_t align256(size_t n) { return (n + 255) / 256 * 256; }
constexpr size_t kOffLogits = 0;
constexpr size_t kOffSelIdx = kOffLogits + align256(sizeof(float) * kStaticMaxSlots * kStaticMaxExperts);
constexpr size_t kOffSelW = kOffSelIdx + align256(sizeof(int32_t) * kStaticMaxSlots);
constexpr size_t kOffOffsets = kOffSelW + align256(sizeof(float) * kStaticMaxSlots);
constexpr size_t kOffPerm = kOffOffsets + align256(sizeof(int32_t) * (kStaticMaxExperts + 1));
constexpr size_t kOffSlotPos = kOffPerm + align256(sizeof(int32_t) * kStaticMaxSlots);
constexpr size_t kOffActList = kOffSlotPos + align256(sizeof(int32_t) * kStaticMaxSlots);
constexpr size_t kOffMeta = kOffActList + align256(sizeof(int32_t) * kStaticMaxExperts);
constexpr size_t kOffAct = kOffMeta + 256;
constexpr size_t kOffRes = kOffAct + align256(sizeof(float) * kStaticMaxSlots * kStaticMaxDim);
constexpr size_t kStaticBytes = kOffRes + align256(sizeof(float) * kStaticMaxSlots * kStaticMaxDim);

}  // namespace

// About 2.2 MB; every GPU that loads the library holds it until the process exits.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

namespace {

std::mutex g_static_mu;
void *g_static_addr[64] = {};

// Device address of g_static_scratch on ctx's device.  The host-side name
// is only a stand-in, so the address is looked up once per device (with that
// device current) and cached.
spt_status static_scratch(spt_context *ctx, unsigned char **out) {
  if (ctx->device < 0 || ctx->device >= 64) return fail(ctx, SPT_ERR_UNSUPPORTED, "device index %d", ctx->device);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_addr[ctx->device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGetSymbolAddress(static scratch)");
    g_static_addr[ctx->device] = p;
  }
  *out = static_cast<unsigned char *>(g_static_addr[ctx->device]);
  return SPT_OK;
}

}  // namespace

extern "C" spt_status spt_forward_moe_batch_device_static(spt_context *ctx, spt_arena *arena,
                                                          int64_t layer, const float *x, float *out,
                                                          int64_t batch) {
  if (!ctx || !arena || !x || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (batch <= 0 || layer < 0 || layer >= (int64_t)arena->layers.size())
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(ctx, SPT_ERR_DIMENSIONS, "device x and out must be 16-byte aligned");
  const spt_moe_config &c = arena->cfg;
  const int64_t H = c.hidden_dim, D = c.expert_hidden_dim, E = c.num_experts, K = c.num_experts_used;
  if (batch * K > kStaticMaxSlots || H > kStaticMaxDim || D > kStaticMaxDim || E > kStaticMaxExperts ||
      K > kSelectMaxK)
    return fail(ctx, SPT_ERR_UNSUPPORTED,
                "batch %lld x top-k %lld, hidden %lld, expert dim %lld or %lld experts exceed the static "
                "scratch (tokens x top-k <= %lld, dimensions <= %lld, experts <= %lld)",
                (long long)batch, (long long)K, (long long)H, (long long)D, (long long)E,
                (long long)kStaticMaxSlots, (long long)kStaticMaxDim, (long long)kStaticMaxExperts);
  spt_status st = require_device(ctx);
  if (st) return st;
  if (arena->expert_count != E)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "arena holds only some of the experts (an expert-parallel shard)");
  const LayerDev &L = arena->layers[(size_t)layer];
  if (!L.has_g8) return fail(ctx, SPT_ERR_UNSUPPORTED, "arena was created without SPT_ARENA_GEMV");
  unsigned char *base = nullptr;
  if ((st = static_scratch(ctx, &base))) return st;
  // Nothing here needs zeroing: every word is written before it is read within
  // one call (the dispatch kernel counts in shared memory), so the previous
  // call's contents are harmless.  Calls that overlap on the GPU (two streams,
  // or two host threads on different contexts of one device) share this array
  // and race: serialise them.
  float *logits = reinterpret_cast<float *>(base + kOffLogits);
  int32_t *sel_idx = reinterpret_cast<int32_t *>(base + kOffSelIdx);
  float *sel_w = reinterpret_cast<float *>(base + kOffSelW);
  int32_t *offsets = reinterpret_cast<int32_t *>(base + kOffOffsets);
  int32_t *perm = reinterpret_cast<int32_t *>(base + kOffPerm);
  int32_t *slot_pos = reinterpret_cast<int32_t *>(base + kOffSlotPos);
  int32_t *act_list = reinterpret_cast<int32_t *>(base + kOffActList);
  int32_t *meta = reinterpret_cast<int32_t *>(base + kOffMeta);
  float *act = reinterpret_cast<float *>(base + kOffAct);
  float *res = reinterpret_cast<float *>(base + kOffRes);
  const int T = (int)batch;
  cudaStream_t s = ctx->stream;
  SPT_CUDA(ctx, launch_router(L.router, x, L.router_bias, T, (int)H, (int)E, logits, 8, s));
  SPT_CUDA(ctx, launch_select(logits, T, (int)E, (int)K, sel_idx, sel_w, s));
  SPT_CUDA(ctx, launch_dispatch(sel_idx, sel_w, (int)(T * K), (int)E, offsets, perm, slot_pos, act_list, meta, s));
  const int mt = pick_mt(T, K, E);
  GemvLaunch gu;
  gu.m0 = L.gate;
  gu.m1 = L.up;
  gu.bias0 = L.gate_bias;
  gu.bias1 = L.up_bias;
  gu.x = x;
  gu.x_stride = H;
  gu.y = act;
  gu.y_stride = D;
  gu.perm = perm;
  gu.offsets = offsets;
  gu.act_list = act_list;
  gu.meta = meta;
  gu.top_k = (int)K;
  gu.mode = kRowsMoEGateUp;
  gu.gate_up = true;
  gu.max_active = (int)std::min<int64_t>(E, T * K);
  gu.mt = mt > 4 ? 4 : mt;
  SPT_CUDA(ctx, launch_gemv(gu, ctx->sm_count, s));
  GemvLaunch dn = gu;
  dn.m0 = L.down;
  dn.m1 = MatrixG8{};
  dn.bias0 = L.down_bias;
  dn.bias1 = nullptr;
  dn.x = act;
  dn.x_stride = D;
  dn.y = res;
  dn.y_stride = H;
  dn.mode = kRowsMoEDown;
  dn.gate_up = false;
  dn.mt = mt;
  SPT_CUDA(ctx, launch_gemv(dn, ctx->sm_count, s));
  SPT_CUDA(ctx, launch_combine(res, sel_w, slot_pos, T, (int)K, (int)H, out, s));
  // This call's routing lives in the static array, not in the context's
  // buffers, and it records no stage events: spt_last_routing and
  // spt_stage_times refuse until the next allocating forward.
  ctx->have_routing = false;
  ctx->timed_last = false;
  ctx->kernels_last = 6;  // router, select, dispatch, gate/up, down, combine
  ctx->last_path = SPT_PATH_EXACT;
  ctx->last_bn = 0;
  return SPT_OK;
}

// =========================================================================
// Expert parallelism.  Rank r of `world` holds experts [r*E/world,
// (r+1)*E/world) of every layer and the whole router; each rank routes its
// own tokens, sends every dispatched slot's token row to the owner of its
// expert, runs the expert products for the rows it receives, and returns the
// result rows, which the sender combines in rank order exactly as the
// single-GPU block does.  The exchange runs on NCCL point-to-point calls on
// the context's stream; libnccl is opened at run time, so a process that has
// already loaded one (a PyTorch process) shares it.

#include <dlfcn.h>
#include <nccl.h>
#include <time.h>
#include <unistd.h>

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
  std::string why;  // empty when loaded
};

const NcclApi &nccl() {
  static NcclApi api = [] {
    NcclApi a;
    // An NCCL already in the process (PyTorch's) is found by its soname and
    // shared.
    // SPT_NCCL_LIBRARY names the NCCL to use (the Python mirror points it at
    // PyTorch's, so that a later `import torch` finds the same one already
    // loaded under the soname it links against).
    void *h = nullptr;
    if (const char *path = getenv("SPT_NCCL_LIBRARY")) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      a.why = std::string("cannot open libnccl.so.2: ") + dlerror();
      return a;
    }
    bool ok = true;
    auto sym = [&](const char *name) {
      void *f = dlsym(h, name);
      if (!f) ok = false;
      return f;
    };
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(sym("ncclGetUniqueId"));
    a.comm_init_rank_config = reinterpret_cast<decltype(a.comm_init_rank_config)>(sym("ncclCommInitRankConfig"));
    a.comm_get_async_error = reinterpret_cast<decltype(a.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
    a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(sym("ncclCommAbort"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(sym("ncclCommDestroy"));
    a.send = reinterpret_cast<decltype(a.send)>(sym("ncclSend"));
    a.recv = reinterpret_cast<decltype(a.recv)>(sym("ncclRecv"));
    a.group_start = reinterpret_cast<decltype(a.group_start)>(sym("ncclGroupStart"));
    a.group_end = reinterpret_cast<decltype(a.group_end)>(sym("ncclGroupEnd"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(sym("ncclGetErrorString"));
    if (!ok) a.why = "libnccl is missing an expected symbol";
    return a;
  }();
  return api;
}

}  // namespace

struct spt_ep {
  spt_context *ctx = nullptr;
  int rank = 0, world = 1;
  ncclComm_t comm = nullptr;
  bool broken = false;   // aborted after a wait ran out; every later call fails
  bool pending = false;  // the last result exchange may still be in flight
  int64_t cap_tokens = 0;  // > 0: fixed-capacity exchange, at most this many tokens per rank and call
  int64_t t_max = 0;     // largest batch so far (no buffer grows below it)
  int64_t timeout_ms = 60000;
  // send side (this rank's tokens)
  DevBuf sel_w;          // [S] selection weights kept for the final combine
  DevBuf send_off;       // [world+1] first send row of each destination rank
  DevBuf send_perm;      // [S] send row -> slot
  DevBuf send_pos;       // [S] slot -> send row, -1 if not dispatched
  DevBuf dest_list, send_meta;
  DevBuf xs, ms;         // send rows [S][H] and their local expert ids [S]
  DevBuf ret;            // result rows returned to this rank [S][H]
  DevBuf counts;         // [2*world] rows sent to / received from each rank
  // receive side (rows other ranks send here)
  DevBuf xr, mr;         // received rows [R][H] and local expert ids [R]
  DevBuf rows_out;       // their results [R][H]
  int32_t *counts_host = nullptr;  // pinned [2*world]
  std::vector<int64_t> soff, roff;  // prefix offsets (rows) per rank
  // peer-memory exchange of the fixed-capacity layout (one GPU per rank)
  int exchange = SPT_EP_EXCHANGE_PEER;  // transport of the fixed-capacity exchange
  bool peer_tried = false;  // set-up attempted for the current window shape
  bool peer_ok = false;     // windows mapped: the fixed-capacity calls use them
  EpPeerLayout lay;         // base[] = every rank's window in this process
  void *win = nullptr;      // this rank's window (cudaMalloc, shared by IPC)
  DevBuf arrive;            // [2] arrival counters of the send and return kernels
  uint64_t seq = 0;         // calls made through the windows
};

namespace {

#define SPT_NCCL(ctx, call)                                                                        \
  do {                                                                                             \
    ncclResult_t _r = (call);                                                                      \
    if (_r != ncclSuccess)                                                                         \
      return fail((ctx), SPT_ERR_NCCL, "%s: %s", #call, nccl().error_string(_r));                  \
  } while (0)

// Bounded waits.  The communicator is non-blocking, so NCCL calls return
// while their setup is in progress; a peer that never arrives would leave
// both that and the exchange kernels on the stream waiting forever.  Each
// wait below gives up after ep->timeout_ms, aborts the communicator (which
// also ends its kernels) and marks the group broken.
int64_t now_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (int64_t)ts.tv_sec * 1000 + ts.tv_nsec / 1000000;
}

spt_status ep_abort(spt_ep *ep, const char *what) {
  if (ep->comm && !ep->broken) nccl().comm_abort(ep->comm);
  ep->broken = true;
  return fail(ep->ctx, SPT_ERR_NCCL, "expert-parallel %s: no progress within %lld ms; group aborted", what,
              (long long)ep->timeout_ms);
}

// The waits spin for their first couple of milliseconds (an exchange's
// enqueue normally completes within microseconds, and a sleep would put tens
// of microseconds on every call), then back off to short sleeps.
constexpr int64_t kSpinMs = 2;

spt_status wait_comm(spt_ep *ep, const char *what) {
  const int64_t start = now_ms(), deadline = start + ep->timeout_ms;
  for (;;) {
    ncclResult_t state = ncclSuccess;
    ncclResult_t r = nccl().comm_get_async_error(ep->comm, &state);
    if (r != ncclSuccess) return fail(ep->ctx, SPT_ERR_NCCL, "ncclCommGetAsyncError: %s", nccl().error_string(r));
    if (state == ncclSuccess) return SPT_OK;
    if (state != ncclInProgress) {
      spt_status st = fail(ep->ctx, SPT_ERR_NCCL, "%s: %s", what, nccl().error_string(state));
      nccl().comm_abort(ep->comm);
      ep->broken = true;
      return st;
    }
    const int64_t t = now_ms();
    if (t > deadline) return ep_abort(ep, what);
    if (t - start >= kSpinMs) usleep(50);
  }
}

spt_status wait_stream(spt_ep *ep, const char *what) {
  const int64_t start = now_ms(), deadline = start + ep->timeout_ms;
  for (;;) {
    cudaError_t e = cudaStreamQuery(ep->ctx->stream);
    if (e == cudaSuccess) return SPT_OK;
    if (e != cudaErrorNotReady) return cuda_fail(ep->ctx, e, what);
    const int64_t t = now_ms();
    if (t > deadline) return ep_abort(ep, what);
    if (t - start >= kSpinMs) usleep(20);
  }
}

// One grouped exchange: for every peer, send cnt_s rows of `width` elements
// starting at row soff and receive cnt_r rows at roff.
spt_status exchange(spt_ep *ep, const void *send, void *recv, int64_t width, size_t elem, ncclDataType_t type,
                    const std::vector<int64_t> &soff, const std::vector<int64_t> &roff) {
  spt_context *ctx = ep->ctx;
  const NcclApi &api = nccl();
  if (ep->broken) return fail(ctx, SPT_ERR_NCCL, "expert-parallel group was aborted");
  SPT_NCCL(ctx, api.group_start());
  for (int j = 0; j < ep->world; ++j) {
    const int64_t ns = soff[j + 1] - soff[j], nr = roff[j + 1] - roff[j];
    if (ns > 0)
      SPT_NCCL(ctx, api.send(static_cast<const uint8_t *>(send) + (size_t)soff[j] * width * elem,
                             (size_t)(ns * width), type, j, ep->comm, ctx->stream));
    if (nr > 0)
      SPT_NCCL(ctx, api.recv(static_cast<uint8_t *>(recv) + (size_t)roff[j] * width * elem, (size_t)(nr * width),
                             type, j, ep->comm, ctx->stream));
  }
  ncclResult_t r = api.group_end();
  if (r == ncclSuccess) return SPT_OK;
  if (r != ncclInProgress) return fail(ctx, SPT_ERR_NCCL, "ncclGroupEnd: %s", api.error_string(r));
  return wait_comm(ep, "exchange");
}

// SPT_EP_TRACE=1 prints each phase of an expert-parallel call to stderr.
void ep_trace(const spt_ep *ep, const char *fmt, ...) {
  static const bool on = [] {
    const char *v = getenv("SPT_EP_TRACE");
    return v && v[0] == '1';
  }();
  if (!on) return;
  char buf[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  fprintf(stderr, "[spt ep %d/%d %lld ms] %s\n", ep->rank, ep->world, (long long)(now_ms() % 1000000), buf);
  fflush(stderr);
}

// One grouped exchange of fixed-size pieces: for every peer j and every item,
// send `count` elements at send + j*count and receive them at recv + j*count.
struct FixedItem {
  const void *send;
  void *recv;
  size_t count, elem;
  ncclDataType_t type;
};
spt_status exchange_fixed(spt_ep *ep, std::initializer_list<FixedItem> items) {
  spt_context *ctx = ep->ctx;
  const NcclApi &api = nccl();
  if (ep->broken) return fail(ctx, SPT_ERR_NCCL, "expert-parallel group was aborted");
  SPT_NCCL(ctx, api.group_start());
  for (int j = 0; j < ep->world; ++j)
    for (const FixedItem &it : items) {
      SPT_NCCL(ctx, api.send(static_cast<const uint8_t *>(it.send) + (size_t)j * it.count * it.elem, it.count,
                             it.type, j, ep->comm, ctx->stream));
      SPT_NCCL(ctx, api.recv(static_cast<uint8_t *>(it.recv) + (size_t)j * it.count * it.elem, it.count, it.type, j,
                             ep->comm, ctx->stream));
    }
  ncclResult_t r = api.group_end();
  if (r == ncclSuccess) return SPT_OK;
  if (r != ncclInProgress) return fail(ctx, SPT_ERR_NCCL, "ncclGroupEnd: %s", api.error_string(r));
  return wait_comm(ep, "exchange");
}

// ---- peer-memory windows ---------------------------------------------------
// One record per rank, exchanged once over the communicator: its window's
// IPC handle and its device's UUID (peer mode needs one GPU per rank).
struct PeerRecord {
  cudaIpcMemHandle_t handle;
  unsigned char uuid[16];
  int64_t bytes;
  unsigned char pad[128 - sizeof(cudaIpcMemHandle_t) - 16 - sizeof(int64_t)];
};
static_assert(sizeof(PeerRecord) == 128, "peer record");

void ep_peer_release(spt_ep *ep) {
  if (!ep->win) return;
  if (ep->ctx && ep->ctx->stream) cudaStreamSynchronize(ep->ctx->stream);
  for (int r = 0; r < ep->world; ++r)
    if (r != ep->rank && ep->lay.base[r]) cudaIpcCloseMemHandle(ep->lay.base[r]);
  cudaFree(ep->win);
  ep->win = nullptr;
  ep->peer_ok = false;
  for (int r = 0; r < kEpMaxPeers; ++r) ep->lay.base[r] = nullptr;
}

// Collective (every rank at the same call): windows for cap rows per peer and
// hidden width H, mapped into every process.  Leaves peer_ok false (the NCCL
// exchange is used) when two ranks share a GPU or the set-up fails on a rank;
// every rank reaches the same decision from the same records.
spt_status ep_peer_setup(spt_ep *ep, int64_t cap, int64_t H) {
  spt_context *ctx = ep->ctx;
  const int W = ep->world;
  if (ep->peer_tried && (!ep->peer_ok || (ep->lay.cap >= cap && ep->lay.hidden == H))) return SPT_OK;
  ep_peer_release(ep);
  ep->peer_tried = true;
  if (W > kEpMaxPeers || ep->exchange != SPT_EP_EXCHANGE_PEER) return SPT_OK;
  EpPeerLayout L;
  L.world = W;
  L.rank = ep->rank;
  L.cap = (int)cap;
  L.hidden = (int)H;
  auto align = [](int64_t v) { return (v + 255) / 256 * 256; };
  int64_t off = 0;
  L.rows_off = off;
  off = align(off + 2 * W * cap * H * (int64_t)sizeof(float));
  L.ret_off = off;
  off = align(off + 2 * W * cap * H * (int64_t)sizeof(float));
  L.ids_off = off;
  off = align(off + 2 * W * cap * (int64_t)sizeof(int32_t));
  L.cnt_off = off;
  off = align(off + 2 * W * (int64_t)sizeof(int32_t));
  L.ffwd_off = off;
  off = align(off + W * (int64_t)sizeof(uint64_t));
  L.fret_off = off;
  off = align(off + W * (int64_t)sizeof(uint64_t));
  L.bytes = off;
  // this rank's record; a failed allocation still takes part (bytes = 0)
  PeerRecord mine;
  memset(&mine, 0, sizeof mine);
  cudaDeviceProp prop;
  SPT_CUDA(ctx, cudaGetDeviceProperties(&prop, ctx->device));
  memcpy(mine.uuid, &prop.uuid, 16);
  if (cudaMalloc(&ep->win, (size_t)L.bytes) == cudaSuccess &&
      cudaMemset(ep->win, 0, (size_t)L.bytes) == cudaSuccess &&
      cudaIpcGetMemHandle(&mine.handle, ep->win) == cudaSuccess) {
    mine.bytes = L.bytes;
  } else {
    cudaGetLastError();
    if (ep->win) cudaFree(ep->win);
    ep->win = nullptr;
  }
  SPT_CUDA(ctx, cudaDeviceSynchronize());
  DevBuf send, recv;
  SPT_CUDA(ctx, send.ensure(sizeof(PeerRecord) * W));
  SPT_CUDA(ctx, recv.ensure(sizeof(PeerRecord) * W));
  for (int r = 0; r < W; ++r)
    SPT_CUDA(ctx, cudaMemcpy(send.as<uint8_t>() + sizeof(PeerRecord) * r, &mine, sizeof mine, cudaMemcpyHostToDevice));
  spt_status st = exchange_fixed(ep, {{send.p, recv.p, sizeof(PeerRecord), 1, ncclUint8}});
  if (!st) st = wait_stream(ep, "peer window exchange");
  std::vector<PeerRecord> rec(W);
  if (!st) SPT_CUDA(ctx, cudaMemcpy(rec.data(), recv.p, sizeof(PeerRecord) * W, cudaMemcpyDeviceToHost));
  send.release();
  recv.release();
  if (st) return st;
  bool usable = true;
  for (int r = 0; r < W; ++r) {
    usable = usable && rec[r].bytes == L.bytes;
    for (int q = 0; q < r; ++q) usable = usable && memcmp(rec[r].uuid, rec[q].uuid, 16) != 0;
  }
  if (usable) {
    for (int r = 0; r < W; ++r) {
      if (r == ep->rank) {
        L.base[r] = static_cast<uint8_t *>(ep->win);
        continue;
      }
      void *p = nullptr;
      if (cudaIpcOpenMemHandle(&p, rec[r].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        usable = false;  // (a rank that fails here fails every later peer call: see below)
        break;
      }
      L.base[r] = static_cast<uint8_t *>(p);
    }
  }
  ep->lay = L;
  if (!usable) {
    // a mapping that failed on one rank only would leave the ranks on
    // different transports; keep the group consistent by failing instead
    bool all_distinct = true;
    for (int r = 0; r < W; ++r)
      for (int q = 0; q < r; ++q) all_distinct = all_distinct && memcmp(rec[r].uuid, rec[q].uuid, 16) != 0;
    bool all_alloc = true;
    for (int r = 0; r < W; ++r) all_alloc = all_alloc && rec[r].bytes == L.bytes;
    ep_peer_release(ep);
    ep->lay.cap = (int)cap;
    ep->lay.hidden = (int)H;
    if (all_distinct && all_alloc)
      return fail(ctx, SPT_ERR_CUDA, "cudaIpcOpenMemHandle failed for a peer's expert-parallel window");
    return SPT_OK;  // shared GPU or an allocation failed: every rank falls back to NCCL
  }
  SPT_CUDA(ctx, ep->arrive.ensure(sizeof(int32_t) * 2));
  SPT_CUDA(ctx, cudaMemset(ep->arrive.p, 0, sizeof(int32_t) * 2));
  ep->seq = 0;
  ep->peer_ok = true;
  ep_trace(ep, "peer windows mapped: %lld bytes each", (long long)L.bytes);
  return SPT_OK;
}

// The fixed-capacity call through the peer windows: no NCCL call and no host
// synchronisation; only live rows cross NVLink.
spt_status forward_ep_peer(spt_context *ctx, spt_ep *ep, const LayerDev &L, const spt_moe_config &c, const float *x,
                           float *out, int64_t T) {
  const int64_t H = c.hidden_dim, E = c.num_experts, K = c.num_experts_used;
  const int W = ep->world;
  const int64_t ne = E / W, cap = ep->cap_tokens * K, rows = W * cap, S = T * K;
  cudaStream_t s = ctx->stream;
  spt_moe_config lc = c;  // receive side: top-1 over this rank's experts
  lc.num_experts = ne;
  lc.num_experts_used = 1;
  const int bn_hint = pick_bn(ctx, S, 1, ne);
  spt_status st = ensure_scratch(ctx, ep->cap_tokens, c);
  if (st) return st;
  if ((st = reserve_experts(ctx, L, lc, rows, bn_hint))) return st;
  SPT_CUDA(ctx, ep->sel_w.ensure(sizeof(float) * cap));
  SPT_CUDA(ctx, ep->send_off.ensure(sizeof(int32_t) * (W + 1)));
  SPT_CUDA(ctx, ep->send_perm.ensure(sizeof(int32_t) * cap));
  SPT_CUDA(ctx, ep->send_pos.ensure(sizeof(int32_t) * cap));
  SPT_CUDA(ctx, ep->dest_list.ensure(sizeof(int32_t) * W));
  SPT_CUDA(ctx, ep->send_meta.ensure(sizeof(int32_t) * 4));
  SPT_CUDA(ctx, ep->rows_out.ensure(sizeof(float) * rows * H));
  if (!ctx->dev_err.p) {  // the device waits' error flag
    SPT_CUDA(ctx, ctx->dev_err.ensure(sizeof(int32_t)));
    SPT_CUDA(ctx, cudaMemsetAsync(ctx->dev_err.p, 0, sizeof(int32_t), ctx->stream));
  }
  const EpPeerLayout &lay = ep->lay;
  const uint64_t seq = ++ep->seq;
  const int par = (int)(seq & 1u);
  int32_t *err = ctx->dev_err.as<int32_t>();
  ep_trace(ep, "peer call %llu T=%lld, %lld rows per peer", (unsigned long long)seq, (long long)T, (long long)cap);
  // 1. route, group by owner rank, rows straight into the owners' windows
  if ((st = route_select(ctx, L, c, x, T, ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>()))) return st;
  SPT_CUDA(ctx, cudaMemcpyAsync(ep->sel_w.p, ctx->sel_w.p, sizeof(float) * S, cudaMemcpyDeviceToDevice, s));
  SPT_CUDA(ctx, launch_dispatch(ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>(), (int)S, W,
                                ep->send_off.as<int32_t>(), ep->send_perm.as<int32_t>(), ep->send_pos.as<int32_t>(),
                                ep->dest_list.as<int32_t>(), ep->send_meta.as<int32_t>(), s, nullptr, (int)ne));
  SPT_CUDA(ctx, launch_ep_send_peer(x, ctx->sel_idx.as<int32_t>(), ep->send_perm.as<int32_t>(),
                                    ep->send_off.as<int32_t>(), ep->send_meta.as<int32_t>(), (int)K, (int)ne, (int)S,
                                    lay, par, seq, ep->send_pos.as<int32_t>(), ep->arrive.as<int32_t>(), s));
  // 2. every sender's rows for this call have landed here
  SPT_CUDA(ctx, launch_ep_wait(lay, lay.ffwd_off, seq, ctx->opt_wait_shift, err, 20, s));
  // 3. expert products for the live received rows
  const float *xr = reinterpret_cast<const float *>(lay.base[lay.rank] + lay.rows_off) + (size_t)par * rows * H;
  const int32_t *mr = reinterpret_cast<const int32_t *>(lay.base[lay.rank] + lay.ids_off) + (size_t)par * rows;
  SPT_CUDA(ctx, launch_ep_recv_weights_peer(lay, par, ctx->sel_w.as<float>(), s));
  if ((st = experts_combine(ctx, L, lc, xr, rows, mr, ctx->sel_w.as<float>(), ep->rows_out.as<float>(), bn_hint)))
    return st;
  const int recv_kernels = 2 + ctx->kernels_last - 2;  // wait, weights + experts_combine's (no router/select)
  // 4. results straight back into the senders' windows, then the rank-ordered
  //    combine once every owner's results have landed here
  SPT_CUDA(ctx, launch_ep_return_peer(ep->rows_out.as<float>(), lay, par, seq, ep->arrive.as<int32_t>() + 1, s));
  SPT_CUDA(ctx, launch_ep_wait(lay, lay.fret_off, seq, ctx->opt_wait_shift, err, 21, s));
  ep->pending = true;
  const float *ret = reinterpret_cast<const float *>(lay.base[lay.rank] + lay.ret_off) + (size_t)par * rows * H;
  SPT_CUDA(ctx, launch_combine(ret, ep->sel_w.as<float>(), ep->send_pos.as<int32_t>(), (int)T, (int)K, (int)H, out, s));
  ctx->kernels_last = 6 + recv_kernels;  // router, select, rank grouping, send, return, wait, combine + receive side
  return SPT_OK;
}

// Fixed-capacity variant: every rank sends every peer a slot of cap =
// cap_tokens * K rows (the live count travels in the same group), so no count
// reaches the host and the call never synchronises.  The receiving rank
// weights padding rows 0, which the dispatch kernel never dispatches.
spt_status forward_ep_cap(spt_context *ctx, spt_ep *ep, const LayerDev &L, const spt_moe_config &c, const float *x,
                          float *out, int64_t T) {
  const int64_t H = c.hidden_dim, E = c.num_experts, K = c.num_experts_used;
  const int W = ep->world;
  const int64_t ne = E / W, cap = ep->cap_tokens * K, rows = W * cap, S = T * K;
  cudaStream_t s = ctx->stream;
  spt_moe_config lc = c;  // receive side: top-1 over this rank's experts
  lc.num_experts = ne;
  lc.num_experts_used = 1;
  // token tiles sized for the rows a rank receives on average (its own slot count)
  const int bn_hint = pick_bn(ctx, S, 1, ne);
  // every buffer at its full size before anything is enqueued: none grows later
  spt_status st = ensure_scratch(ctx, ep->cap_tokens, c);
  if (st) return st;
  if ((st = reserve_experts(ctx, L, lc, rows, bn_hint))) return st;
  SPT_CUDA(ctx, ep->sel_w.ensure(sizeof(float) * cap));
  SPT_CUDA(ctx, ep->send_off.ensure(sizeof(int32_t) * (W + 1)));
  SPT_CUDA(ctx, ep->send_perm.ensure(sizeof(int32_t) * cap));
  SPT_CUDA(ctx, ep->send_pos.ensure(sizeof(int32_t) * cap));
  SPT_CUDA(ctx, ep->dest_list.ensure(sizeof(int32_t) * W));
  SPT_CUDA(ctx, ep->send_meta.ensure(sizeof(int32_t) * 4));
  SPT_CUDA(ctx, ep->counts.ensure(sizeof(int32_t) * 2 * W));
  for (DevBuf *b : {&ep->xs, &ep->xr, &ep->rows_out, &ep->ret}) SPT_CUDA(ctx, b->ensure(sizeof(float) * rows * H));
  for (DevBuf *b : {&ep->ms, &ep->mr}) SPT_CUDA(ctx, b->ensure(sizeof(int32_t) * rows));
  ep_trace(ep, "fixed-capacity call T=%lld, %lld rows per peer", (long long)T, (long long)cap);
  // 1. route, group by owner rank, gather into each rank's slot
  if ((st = route_select(ctx, L, c, x, T, ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>()))) return st;
  SPT_CUDA(ctx, cudaMemcpyAsync(ep->sel_w.p, ctx->sel_w.p, sizeof(float) * S, cudaMemcpyDeviceToDevice, s));
  SPT_CUDA(ctx, launch_dispatch(ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>(), (int)S, W,
                                ep->send_off.as<int32_t>(), ep->send_perm.as<int32_t>(), ep->send_pos.as<int32_t>(),
                                ep->dest_list.as<int32_t>(), ep->send_meta.as<int32_t>(), s, nullptr, (int)ne));
  SPT_CUDA(ctx, launch_ep_gather_cap(x, ctx->sel_idx.as<int32_t>(), ep->send_perm.as<int32_t>(),
                                     ep->send_off.as<int32_t>(), ep->send_meta.as<int32_t>(), (int)K, (int)ne, (int)H,
                                     (int)S, W, (int)cap, ep->xs.as<float>(), ep->ms.as<int32_t>(),
                                     ep->counts.as<int32_t>(), ep->send_pos.as<int32_t>(), s));
  // 2. rows, local expert ids and counts to every peer, one group
  if ((st = exchange_fixed(ep, {{ep->xs.p, ep->xr.p, (size_t)(cap * H), sizeof(float), ncclFloat32},
                                {ep->ms.p, ep->mr.p, (size_t)cap, sizeof(int32_t), ncclInt32},
                                {ep->counts.p, ep->counts.as<int32_t>() + W, 1, sizeof(int32_t), ncclInt32}})))
    return st;
  // 3. expert products for the live received rows
  SPT_CUDA(ctx, launch_ep_recv_weights(ep->counts.as<int32_t>() + W, (int)cap, W, ctx->sel_w.as<float>(), s));
  if ((st = experts_combine(ctx, L, lc, ep->xr.as<float>(), rows, ep->mr.as<int32_t>(), ctx->sel_w.as<float>(),
                            ep->rows_out.as<float>(), bn_hint)))
    return st;
  const int recv_kernels = 1 + ctx->kernels_last - 2;  // weights + experts_combine's (no router/select)
  // 4. result rows back into each sender's slot, rank-ordered combine
  if ((st = exchange_fixed(ep, {{ep->rows_out.p, ep->ret.p, (size_t)(cap * H), sizeof(float), ncclFloat32}})))
    return st;
  ep->pending = true;
  SPT_CUDA(ctx, launch_combine(ep->ret.as<float>(), ep->sel_w.as<float>(), ep->send_pos.as<int32_t>(), (int)T, (int)K,
                               (int)H, out, s));
  ctx->kernels_last = 5 + recv_kernels;  // router, select, rank grouping, gather, combine + receive side
  return SPT_OK;
}

spt_status forward_ep_device(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t layer, const float *x,
                             float *out, int64_t T) {
  const spt_moe_config &c = arena->cfg;
  spt_status st = check_layer_limits(ctx, c);
  if (st) return st;
  const int64_t H = c.hidden_dim, E = c.num_experts, K = c.num_experts_used;
  const int W = ep->world;
  if (E % W != 0)
    return fail(ctx, SPT_ERR_UNSUPPORTED, "%lld experts do not divide evenly over %d ranks", (long long)E, W);
  const int64_t ne = E / W;
  if (arena->expert_begin != ep->rank * ne || arena->expert_count != ne)
    return fail(ctx, SPT_ERR_DIMENSIONS, "arena holds experts [%lld, %lld), rank %d of %d owns [%lld, %lld)",
                (long long)arena->expert_begin, (long long)(arena->expert_begin + arena->expert_count), ep->rank, W,
                (long long)(ep->rank * ne), (long long)((ep->rank + 1) * ne));
  if (H % 4 != 0) return fail(ctx, SPT_ERR_UNSUPPORTED, "hidden size %lld not a multiple of 4", (long long)H);
  cudaStream_t s = ctx->stream;
  const LayerDev &L = arena->layers[(size_t)layer];
  ctx->timed_last = ctx->timing;
  ctx->have_routing = false;  // the context's dispatch buffers describe the rows this rank received
  const int64_t S = T * K;
  if (ep->cap_tokens > 0) {
    if (T > ep->cap_tokens)
      return fail(ctx, SPT_ERR_DIMENSIONS, "batch %lld exceeds the group's capacity of %lld tokens per rank",
                  (long long)T, (long long)ep->cap_tokens);
    if ((st = ep_peer_setup(ep, ep->cap_tokens * K, H))) return st;
    return ep->peer_ok ? forward_ep_peer(ctx, ep, L, c, x, out, T) : forward_ep_cap(ctx, ep, L, c, x, out, T);
  }
  // A previous call's result exchange may still be in flight (device entry
  // point): let it finish before this call's buffers can grow.
  if (ep->pending && T > ep->t_max && (st = wait_stream(ep, "previous exchange"))) return st;
  ep->t_max = std::max(ep->t_max, T);
  ep_trace(ep, "start T=%lld pending=%d", (long long)T, (int)ep->pending);
  // 1. route this rank's tokens over all experts
  if ((st = ensure_scratch(ctx, T, c))) return st;
  if ((st = route_select(ctx, L, c, x, T, ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>()))) return st;
  // 2. group the dispatched slots by owner rank, gather their rows
  SPT_CUDA(ctx, ep->sel_w.ensure(sizeof(float) * std::max<int64_t>(S, 1)));
  SPT_CUDA(ctx, ep->send_off.ensure(sizeof(int32_t) * (W + 1)));
  SPT_CUDA(ctx, ep->send_perm.ensure(sizeof(int32_t) * std::max<int64_t>(S, 1)));
  SPT_CUDA(ctx, ep->send_pos.ensure(sizeof(int32_t) * std::max<int64_t>(S, 1)));
  SPT_CUDA(ctx, ep->dest_list.ensure(sizeof(int32_t) * W));
  SPT_CUDA(ctx, ep->send_meta.ensure(sizeof(int32_t) * 4));
  SPT_CUDA(ctx, ep->xs.ensure(sizeof(float) * std::max<int64_t>(S, 1) * H));
  SPT_CUDA(ctx, ep->ms.ensure(sizeof(int32_t) * std::max<int64_t>(S, 1)));
  SPT_CUDA(ctx, ep->ret.ensure(sizeof(float) * std::max<int64_t>(S, 1) * H));
  SPT_CUDA(ctx, ep->counts.ensure(sizeof(int32_t) * 2 * W));
  if (!ep->counts_host)
    SPT_CUDA(ctx, cudaHostAlloc((void **)&ep->counts_host, sizeof(int32_t) * 2 * W, cudaHostAllocDefault));
  SPT_CUDA(ctx, cudaMemcpyAsync(ep->sel_w.p, ctx->sel_w.p, sizeof(float) * S, cudaMemcpyDeviceToDevice, s));
  SPT_CUDA(ctx, launch_dispatch(ctx->sel_idx.as<int32_t>(), ctx->sel_w.as<float>(), (int)S, W,
                                ep->send_off.as<int32_t>(), ep->send_perm.as<int32_t>(), ep->send_pos.as<int32_t>(),
                                ep->dest_list.as<int32_t>(), ep->send_meta.as<int32_t>(), s, nullptr, (int)ne));
  SPT_CUDA(ctx, launch_ep_gather(x, ctx->sel_idx.as<int32_t>(), ep->send_perm.as<int32_t>(),
                                 ep->send_meta.as<int32_t>(), (int)K, (int)ne, (int)H, (int)S, ep->xs.as<float>(),
                                 ep->ms.as<int32_t>(), s));
  SPT_CUDA(ctx, launch_ep_counts(ep->send_off.as<int32_t>(), W, ep->counts.as<int32_t>(), s));
  // 3. exchange the row counts; the one host synchronisation of the call
  {
    std::vector<int64_t> one(W + 1);
    for (int j = 0; j <= W; ++j) one[j] = j;
    if ((st = exchange(ep, ep->counts.as<int32_t>(), ep->counts.as<int32_t>() + W, 1, sizeof(int32_t), ncclInt32,
                       one, one)))
      return st;
  }
  SPT_CUDA(ctx, cudaMemcpyAsync(ep->counts_host, ep->counts.p, sizeof(int32_t) * 2 * W, cudaMemcpyDeviceToHost, s));
  if ((st = wait_stream(ep, "row-count exchange"))) return st;
  ep->pending = false;
  ep->soff.assign(W + 1, 0);
  ep->roff.assign(W + 1, 0);
  for (int j = 0; j < W; ++j) {
    ep->soff[j + 1] = ep->soff[j] + ep->counts_host[j];
    ep->roff[j + 1] = ep->roff[j] + ep->counts_host[W + j];
  }
  const int64_t R = ep->roff[W];
  ep_trace(ep, "counts exchanged: send %lld rows, receive %lld", (long long)ep->soff[W], (long long)R);
  bool counts_ok = ep->soff[W] <= S;  // a rank receives up to every other rank's slots
  for (int j = 0; j < W; ++j) counts_ok = counts_ok && ep->counts_host[j] >= 0 && ep->counts_host[W + j] >= 0;
  if (!counts_ok) {
    // the peers post their row exchanges next: abort so that they fail too
    // instead of waiting for this rank
    if (ep->comm) nccl().comm_abort(ep->comm);
    ep->broken = true;
    return fail(ctx, SPT_ERR_NCCL, "expert-parallel row counts out of range (sent %lld of %lld slots); group aborted",
                (long long)ep->soff[W], (long long)S);
  }
  // 4. token rows and local expert ids to their owners
  // every allocation of the call happens before the exchanges below
  spt_moe_config lc = c;  // receive side: top-1 over this rank's experts
  lc.num_experts = ne;
  lc.num_experts_used = 1;
  SPT_CUDA(ctx, ep->xr.ensure(sizeof(float) * std::max<int64_t>(R, 1) * H));
  SPT_CUDA(ctx, ep->mr.ensure(sizeof(int32_t) * std::max<int64_t>(R, 1)));
  SPT_CUDA(ctx, ep->rows_out.ensure(sizeof(float) * std::max<int64_t>(R, 1) * H));
  if (R > 0 && (st = reserve_experts(ctx, L, lc, R))) return st;
  ep_trace(ep, "buffers reserved");
  if ((st = exchange(ep, ep->xs.p, ep->xr.p, H, sizeof(float), ncclFloat32, ep->soff, ep->roff))) return st;
  if ((st = exchange(ep, ep->ms.p, ep->mr.p, 1, sizeof(int32_t), ncclInt32, ep->soff, ep->roff))) return st;
  ep_trace(ep, "rows exchange enqueued");
  // 5. expert products for the received rows: top-1 selections of weight 1
  //    over this rank's experts, "combined" into one result row each
  if (R > 0) {
    SPT_CUDA(ctx, launch_fill(ctx->sel_w.as<float>(), R, 1.0f, s));
    if ((st = experts_combine(ctx, L, lc, ep->xr.as<float>(), R, ep->mr.as<int32_t>(), ctx->sel_w.as<float>(),
                              ep->rows_out.as<float>())))
      return st;
  }
  // 6. results back to the ranks that sent the rows, then the rank-ordered
  //    combine over this rank's slots
  ep_trace(ep, "experts enqueued");
  if ((st = exchange(ep, ep->rows_out.p, ep->ret.p, H, sizeof(float), ncclFloat32, ep->roff, ep->soff))) return st;
  ep->pending = true;
  ep_trace(ep, "results exchange enqueued");
  const int recv_kernels = R > 0 ? 1 + ctx->kernels_last - 2 : 0;  // fill + experts_combine's (no router/select)
  SPT_CUDA(ctx, launch_combine(ep->ret.as<float>(), ep->sel_w.as<float>(), ep->send_pos.as<int32_t>(), (int)T, (int)K,
                               (int)H, out, s));
  // router, select, rank grouping, gather, counts, combine + the receive side
  ctx->kernels_last = 6 + recv_kernels;
  return SPT_OK;
}

}  // namespace

extern "C" {

void spt_ep_expert_range(int64_t num_experts, int32_t world, int32_t rank, int64_t *begin, int64_t *end) {
  const bool ok = world > 0 && rank >= 0 && rank < world && num_experts > 0;
  if (begin) *begin = ok ? rank * num_experts / world : 0;
  if (end) *end = ok ? (rank + 1) * num_experts / world : 0;
}

spt_status spt_ep_unique_id(uint8_t id[SPT_EP_UNIQUE_ID_BYTES]) {
  if (!id) return fail(nullptr, SPT_ERR_NULL_ARG, "nil id");
  const NcclApi &api = nccl();
  if (!api.why.empty()) return fail(nullptr, SPT_ERR_NCCL, "%s", api.why.c_str());
  static_assert(sizeof(ncclUniqueId) == SPT_EP_UNIQUE_ID_BYTES, "ncclUniqueId size");
  ncclUniqueId u;
  ncclResult_t r = api.get_unique_id(&u);
  if (r != ncclSuccess) return fail(nullptr, SPT_ERR_NCCL, "ncclGetUniqueId: %s", api.error_string(r));
  memcpy(id, &u, sizeof u);
  return SPT_OK;
}

spt_status spt_ep_create(spt_context *ctx, const uint8_t id[SPT_EP_UNIQUE_ID_BYTES], int32_t rank, int32_t world,
                         spt_ep **out) {
  if (!ctx || !id || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return fail(ctx, SPT_ERR_DIMENSIONS, "rank %d of world %d", rank, world);
  spt_status st = require_device(ctx);
  if (st) return st;
  const NcclApi &api = nccl();
  if (!api.why.empty()) return fail(ctx, SPT_ERR_NCCL, "%s", api.why.c_str());
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  spt_ep *ep = new spt_ep();
  ep->ctx = ctx;
  ep->rank = rank;
  ep->world = world;
  if (const char *t = getenv("SPT_EP_TIMEOUT_MS")) ep->timeout_ms = std::max<int64_t>(1, atoll(t));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclResult_t r = api.comm_init_rank_config(&ep->comm, world, u, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    delete ep;
    return fail(ctx, SPT_ERR_NCCL, "ncclCommInitRankConfig: %s", api.error_string(r));
  }
  if ((st = wait_comm(ep, "communicator set-up"))) {
    ep->comm = nullptr;  // aborted (freed) by the wait
    delete ep;
    return st;
  }
  *out = ep;
  return SPT_OK;
}

void spt_ep_destroy(spt_ep *ep) {
  if (!ep) return;
  spt_context *ctx = ep->ctx;
  if (ctx && ctx->has_device) {
    cudaSetDevice(ctx->device);
    // an exchange a peer never joins is aborted after the group's timeout
    if (ctx->stream && !ep->broken) (void)wait_stream(ep, "exchange before destroy");
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  }
  ep_peer_release(ep);
  if (ep->comm && !ep->broken) nccl().comm_destroy(ep->comm);
  for (DevBuf *b : {&ep->sel_w, &ep->send_off, &ep->send_perm, &ep->send_pos, &ep->dest_list, &ep->send_meta,
                    &ep->xs, &ep->ms, &ep->ret, &ep->counts, &ep->xr, &ep->mr, &ep->rows_out, &ep->arrive})
    b->release();
  if (ep->counts_host) cudaFreeHost(ep->counts_host);
  delete ep;
}

spt_status spt_ep_set_capacity(spt_ep *ep, int64_t max_tokens_per_rank) {
  if (!ep) return fail(nullptr, SPT_ERR_NULL_ARG, "nil expert-parallel group");
  if (max_tokens_per_rank < 0 || max_tokens_per_rank > (1 << 20))
    return fail(ep->ctx, SPT_ERR_DIMENSIONS, "capacity %lld tokens out of range", (long long)max_tokens_per_rank);
  if (ep->pending) {  // the previous call's buffers may still be in use
    spt_status st = wait_stream(ep, "exchange before a capacity change");
    if (st) return st;
    ep->pending = false;
  }
  ep->cap_tokens = max_tokens_per_rank;
  return SPT_OK;
}

spt_status spt_ep_set_exchange(spt_ep *ep, int32_t exchange) {
  if (!ep) return fail(nullptr, SPT_ERR_NULL_ARG, "nil expert-parallel group");
  if (exchange != SPT_EP_EXCHANGE_PEER && exchange != SPT_EP_EXCHANGE_NCCL)
    return fail(ep->ctx, SPT_ERR_UNSUPPORTED, "unknown exchange %d", exchange);
  if (exchange == ep->exchange) return SPT_OK;
  if (ep->pending) {
    spt_status st = wait_stream(ep, "exchange before a transport change");
    if (st) return st;
    ep->pending = false;
  }
  ep->exchange = exchange;
  ep->peer_tried = false;  // the next fixed-capacity call sets up (or drops) the windows
  ep_peer_release(ep);
  return SPT_OK;
}

spt_status spt_last_dispatch(spt_context *ctx, int64_t *active_experts, int64_t *dispatched) {
  spt_status st = require_device(ctx);
  if (st) return st;
  if (!ctx->meta.p) return fail(ctx, SPT_ERR_DIMENSIONS, "no forward call yet");
  int32_t meta[2];
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  SPT_CUDA(ctx, cudaMemcpy(meta, ctx->meta.p, sizeof meta, cudaMemcpyDeviceToHost));
  if (active_experts) *active_experts = meta[0];
  if (dispatched) *dispatched = meta[1];
  return SPT_OK;
}

spt_status spt_forward_moe_batch_ep_device(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t layer,
                                           const float *x, float *out, int64_t batch) {
  if (!ctx || !ep || !arena || !x || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (ep->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "expert-parallel group belongs to another context");
  if (batch <= 0 || layer < 0 || layer >= (int64_t)arena->layers.size())
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(ctx, SPT_ERR_DIMENSIONS, "device x and out must be 16-byte aligned");
  spt_status st = require_device(ctx);
  if (st) return st;
  return forward_ep_device(ctx, ep, arena, layer, x, out, batch);
}

spt_status spt_forward_moe_batch_ep(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t layer, const float *x,
                                    int64_t x_len, float *out, int64_t out_len, int64_t batch,
                                    const volatile int32_t *cancel) {
  if (!ctx || !ep || !arena) return fail(ctx, SPT_ERR_NULL_ARG, "nil MoE context, reader, configuration or weights");
  if (ep->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "expert-parallel group belongs to another context");
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  spt_status st = check_batch(ctx, arena->cfg, x, x_len, out, out_len, batch);
  if (st) return st;
  if (layer < 0 || layer >= (int64_t)arena->layers.size())
    return fail(ctx, SPT_ERR_DIMENSIONS, "layer %lld out of range", (long long)layer);
  if ((st = require_device(ctx))) return st;
  const size_t bytes = sizeof(float) * (size_t)x_len;
  SPT_CUDA(ctx, ctx->xdev.ensure(bytes));
  SPT_CUDA(ctx, ctx->outdev.ensure(bytes));
  SPT_CUDA(ctx, cudaMemcpyAsync(ctx->xdev.p, x, bytes, cudaMemcpyHostToDevice, ctx->stream));
  if ((st = forward_ep_device(ctx, ep, arena, layer, ctx->xdev.as<float>(), ctx->outdev.as<float>(), batch)))
    return st;
  // bounded wait for the exchanges first: a copy into pageable host memory
  // would block until the stream drains, however long that takes
  if ((st = wait_stream(ep, "result exchange"))) return st;
  ep->pending = false;
  SPT_CUDA(ctx, cudaMemcpyAsync(out, ctx->outdev.p, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if ((st = check_device_error(ctx))) return st;
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  return SPT_OK;
}

}  // extern "C"

// =========================================================================
// Layer stack: the MoE half of forwardLayerBatch (forward/layer_batch.go:
// 102-120) repeated over consecutive layers on the residual stream x.
namespace {

spt_status forward_stack_device(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t first, int64_t n, float *x,
                                int64_t T, float eps) {
  const spt_moe_config &c = arena->cfg;
  const int64_t H = c.hidden_dim;
  if (first < 0 || n <= 0 || first + n > (int64_t)arena->layers.size())
    return fail(ctx, SPT_ERR_DIMENSIONS, "layers [%lld, %lld) outside the arena's %zu", (long long)first,
                (long long)(first + n), arena->layers.size());
  if (!(eps >= 0.0f) || isinf(eps)) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid epsilon: %g", (double)eps);
  for (int64_t l = first; l < first + n; ++l)
    if (!arena->layers[(size_t)l].norm)
      return fail(ctx, SPT_ERR_BIAS, "layer %lld has no post-attention norm weights", (long long)l);
  // both buffers exist before any work is enqueued; growing them while an
  // expert-parallel exchange is in flight could deadlock, so wait for it first
  const size_t need = sizeof(float) * (size_t)(T * H);
  if (ep && ep->pending && (ctx->stack_norm.bytes < need || ctx->stack_ffn.bytes < need)) {
    spt_status st = wait_stream(ep, "previous exchange");
    if (st) return st;
    ep->pending = false;
  }
  SPT_CUDA(ctx, ctx->stack_norm.ensure(need));
  SPT_CUDA(ctx, ctx->stack_ffn.ensure(need));
  float *normed = ctx->stack_norm.as<float>(), *ffn = ctx->stack_ffn.as<float>();
  int kernels = 0;
  for (int64_t l = first; l < first + n; ++l) {
    const LayerDev &L = arena->layers[(size_t)l];
    if (ep) {
      SPT_CUDA(ctx, launch_rmsnorm(x, L.norm, (int)T, (int)H, eps, normed, 8, ctx->stream));
      spt_status st = forward_ep_device(ctx, ep, arena, l, normed, ffn, T);
      if (st) return st;
      SPT_CUDA(ctx, launch_add(x, ffn, T * H, ctx->stream));
      kernels += 2 + ctx->kernels_last;
    } else {
      // normBatch happens in the router's prologue (the block's input goes to
      // `normed`), the residual add in the block's combine: x = x + block(norm(x))
      RouterNorm rn;
      rn.w = L.norm;
      rn.eps = eps;
      rn.out = normed;
      spt_status st = forward_device(ctx, arena, l, x, x, T, x, &rn);
      if (st) return st;
      kernels += ctx->kernels_last;
    }
  }
  ctx->kernels_last = kernels;
  return SPT_OK;
}

}  // namespace

extern "C" {

spt_status spt_forward_stack_device(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t first_layer,
                                    int64_t n_layers, float *x, int64_t batch, float eps) {
  if (!ctx || !arena || !x) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (ep && ep->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "expert-parallel group belongs to another context");
  if (batch <= 0) return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  if (reinterpret_cast<uintptr_t>(x) & 15u) return fail(ctx, SPT_ERR_DIMENSIONS, "device x must be 16-byte aligned");
  spt_status st = require_device(ctx);
  if (st) return st;
  return forward_stack_device(ctx, ep, arena, first_layer, n_layers, x, batch, eps);
}

spt_status spt_forward_stack(spt_context *ctx, spt_ep *ep, spt_arena *arena, int64_t first_layer, int64_t n_layers,
                             float *x, int64_t x_len, int64_t batch, float eps, const volatile int32_t *cancel) {
  if (!ctx || !arena || !x) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (ep && ep->ctx != ctx) return fail(ctx, SPT_ERR_DIMENSIONS, "expert-parallel group belongs to another context");
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  int64_t n = 0;
  if (batch <= 0 || !product({batch, arena->cfg.hidden_dim}, &n) || x_len != n)
    return fail(ctx, SPT_ERR_DIMENSIONS, "invalid MoE batch dimensions");
  spt_status st = require_device(ctx);
  if (st) return st;
  const size_t bytes = sizeof(float) * (size_t)x_len;
  SPT_CUDA(ctx, ctx->xdev.ensure(bytes));
  SPT_CUDA(ctx, cudaMemcpyAsync(ctx->xdev.p, x, bytes, cudaMemcpyHostToDevice, ctx->stream));
  if ((st = forward_stack_device(ctx, ep, arena, first_layer, n_layers, ctx->xdev.as<float>(), batch, eps))) return st;
  if (ep) {
    if ((st = wait_stream(ep, "result exchange"))) return st;
    ep->pending = false;
  }
  SPT_CUDA(ctx, cudaMemcpyAsync(x, ctx->xdev.p, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  SPT_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if ((st = check_device_error(ctx))) return st;
  if (canceled(cancel)) return fail(ctx, SPT_ERR_CANCELED, "context canceled");
  return SPT_OK;
}

}  // extern "C"

// =========================================================================
// GGUF model files (the parser is in spt_gguf.cpp).
struct spt_gguf {
  spt::GgufModel m;
};

namespace {

spt_tensor tensor_fact(const spt::GgufModel &m, size_t idx) {
  const spt::GgufTensor &t = m.tensors[idx];
  spt_tensor c{};
  c.name = t.name.c_str();
  c.type = t.type;
  c.n_dims = (uint32_t)t.shape.size();
  for (size_t i = 0; i < t.shape.size() && i < 4; ++i) c.shape[i] = t.shape[i];
  c.start = t.start;
  c.end = t.end;
  return c;
}

bool ends_with(const std::string &s, const char *suffix) {
  const size_t n = strlen(suffix);
  return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

}  // namespace

extern "C" {

spt_status spt_gguf_open(const char *const *paths, int64_t n_paths, spt_gguf **out) {
  if (!out || (!paths && n_paths > 0) || n_paths < 0) return fail(nullptr, SPT_ERR_NULL_ARG, "nil argument");
  *out = nullptr;
  std::vector<std::string> ps;
  for (int64_t i = 0; i < n_paths; ++i) {
    if (!paths[i]) return fail(nullptr, SPT_ERR_NULL_ARG, "nil path");
    ps.emplace_back(paths[i]);
  }
  spt_gguf *g = new spt_gguf();
  std::string err;
  if (!spt::gguf_open(ps, &g->m, &err)) {
    delete g;
    return fail(nullptr, SPT_ERR_FORMAT, "%s", err.c_str());
  }
  *out = g;
  return SPT_OK;
}

void spt_gguf_close(spt_gguf *g) {
  if (!g) return;
  spt::gguf_close(&g->m);
  delete g;
}

int64_t spt_gguf_layer_count(const spt_gguf *g) { return g ? g->m.layer_count : 0; }

spt_status spt_gguf_config(const spt_gguf *g, spt_moe_config *cfg, float *rms_eps) {
  if (!g || !cfg) return fail(nullptr, SPT_ERR_NULL_ARG, "nil argument");
  int64_t v = 0;
  cfg->hidden_dim = 2880;  // NewConfig defaults (forward/config.go:57-75)
  cfg->expert_hidden_dim = 2880;
  cfg->num_experts = 128;
  cfg->num_experts_used = 4;
  if (spt::gguf_meta_int(g->m, "gpt-oss.embedding_length", &v) && v > 0) cfg->hidden_dim = v;
  if (spt::gguf_meta_int(g->m, "gpt-oss.expert_count", &v) && v > 0) cfg->num_experts = v;
  if (spt::gguf_meta_int(g->m, "gpt-oss.expert_used_count", &v) && v > 0) cfg->num_experts_used = v;
  if (spt::gguf_meta_int(g->m, "gpt-oss.expert_feed_forward_length", &v) && v > 0) cfg->expert_hidden_dim = v;
  if (rms_eps) {
    double e = 0;
    *rms_eps = 1e-5f;
    if (spt::gguf_meta_float(g->m, "gpt-oss.attention.layer_norm_rms_epsilon", &e) && (float)e > 0) *rms_eps = (float)e;
  }
  return SPT_OK;
}

spt_status spt_gguf_layer(const spt_gguf *g, int64_t layer, spt_layer_weights *lw, spt_reader *reader) {
  if (!g || !lw) return fail(nullptr, SPT_ERR_NULL_ARG, "nil argument");
  if (layer < 0 || layer >= g->m.layer_count)
    return fail(nullptr, SPT_ERR_DIMENSIONS, "layer %lld out of range", (long long)layer);
  *lw = spt_layer_weights{};
  int file = -1;
  // NewLayerWeights' suffix cases (forward/layer.go:42-83), MoE tensors only
  struct Case {
    const char *suffix;
    spt_tensor *dst;
  } cases[] = {{"post_attention_norm.weight", &lw->post_attention_norm},
               {"ffn_gate_inp.weight", &lw->ffn_gate_inp},
               {"ffn_gate_inp.bias", &lw->ffn_gate_inp_bias},
               {"ffn_gate_exps.weight", &lw->ffn_gate_exps},
               {"ffn_gate_exps.bias", &lw->ffn_gate_exps_bias},
               {"ffn_up_exps.weight", &lw->ffn_up_exps},
               {"ffn_up_exps.bias", &lw->ffn_up_exps_bias},
               {"ffn_down_exps.weight", &lw->ffn_down_exps},
               {"ffn_down_exps.bias", &lw->ffn_down_exps_bias}};
  for (size_t idx : g->m.layers[(size_t)layer]) {
    const spt::GgufTensor &t = g->m.tensors[idx];
    for (const Case &c : cases) {
      if (!ends_with(t.name, c.suffix)) continue;
      if (t.shape.size() > 4)
        return fail(nullptr, SPT_ERR_FORMAT, "tensor \"%s\": more than 4 dimensions", t.name.c_str());
      if (file >= 0 && t.file != file)
        return fail(nullptr, SPT_ERR_FILE_RANGE, "layer %lld: MoE tensors span several files", (long long)layer);
      file = t.file;
      *c.dst = tensor_fact(g->m, idx);
      break;
    }
  }
  if (reader) {
    const spt::GgufFile &f = g->m.files[(size_t)(file < 0 ? 0 : file)];
    reader->base = f.base;
    reader->size = f.size;
  }
  return SPT_OK;
}

spt_status spt_gguf_tensor(const spt_gguf *g, const char *name, spt_tensor *t, spt_reader *reader) {
  if (!g || !name || !t) return fail(nullptr, SPT_ERR_NULL_ARG, "nil argument");
  auto it = g->m.by_name.find(name);
  if (it == g->m.by_name.end()) return fail(nullptr, SPT_ERR_FORMAT, "no tensor \"%s\"", name);
  *t = tensor_fact(g->m, it->second);
  if (reader) {
    const spt::GgufFile &f = g->m.files[(size_t)g->m.tensors[it->second].file];
    reader->base = f.base;
    reader->size = f.size;
  }
  return SPT_OK;
}

spt_status spt_arena_create_gguf(spt_context *ctx, const spt_gguf *g, int64_t first_layer, int64_t n_layers,
                                 uint32_t flags, int64_t expert_begin, int64_t expert_end, spt_arena **out) {
  if (!ctx || !g || !out) return fail(ctx, SPT_ERR_NULL_ARG, "nil argument");
  if (first_layer < 0 || n_layers <= 0 || first_layer + n_layers > g->m.layer_count)
    return fail(ctx, SPT_ERR_DIMENSIONS, "layers [%lld, %lld) outside the model's %lld", (long long)first_layer,
                (long long)(first_layer + n_layers), (long long)g->m.layer_count);
  spt_moe_config cfg;
  spt_status st = spt_gguf_config(g, &cfg, nullptr);
  if (st) return st;
  std::vector<spt_reader> readers((size_t)n_layers);
  std::vector<spt_layer_weights> lws((size_t)n_layers);
  for (int64_t l = 0; l < n_layers; ++l)
    if ((st = spt_gguf_layer(g, first_layer + l, &lws[(size_t)l], &readers[(size_t)l])))
      return fail(ctx, st, "%s", spt_last_error(nullptr));
  if (expert_end == 0) expert_end = cfg.num_experts;
  return arena_create_impl(ctx, readers.data(), &cfg, lws.data(), n_layers, flags, expert_begin, expert_end, out);
}

}  // extern "C"
