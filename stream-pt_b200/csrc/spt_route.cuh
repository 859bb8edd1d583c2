// spt_route.cuh -- device functions of the routing stage shared by the
// separate router/selection kernels and the single-launch decode kernel.
#pragma once
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "spt_internal.cuh"

namespace spt {

// Router logit of one (token, expert) pair from rows in shared memory, one
// warp, the order of the AVX2 dot product (vector_amd64.go:28-56) that the
// router kernels follow: lane l runs chains l (a) and l+32 (b) over 64-element
// chunks, the 32-element tail feeds the a chains, then the fixed shuffle tree.
// The result is valid in lane 0.
__device__ __forceinline__ float router_dot(const float *w, const float *x, int H, int lane) {
  float a = 0.0f, b = 0.0f;
  const int full = H / 64;
  int o = 0;
#pragma unroll 4
  for (int c = 0; c < full; ++c, o += 64) {
    a = fmaf(w[o + lane], x[o + lane], a);
    b = fmaf(w[o + 32 + lane], x[o + 32 + lane], b);
  }
  if (o < H) a = fmaf(w[o + lane], x[o + lane], a);
  const unsigned m = 0xffffffffu;
  const float a8 = __shfl_sync(m, a, (lane + 8) & 31);
  const float a16 = __shfl_sync(m, a, (lane + 16) & 31);
  const float a24 = __shfl_sync(m, a, (lane + 24) & 31);
  const float b8 = __shfl_sync(m, b, (lane + 8) & 31);
  const float b16 = __shfl_sync(m, b, (lane + 16) & 31);
  const float b24 = __shfl_sync(m, b, (lane + 24) & 31);
  const float s0 = ((a + a8) + a16) + a24;
  const float s1 = ((b + b8) + b16) + b24;
  const float sv = s0 + s1;
  const float p = sv + __shfl_sync(m, sv, (lane + 4) & 31);
  const float qv = p + __shfl_sync(m, p, (lane + 1) & 31);
  return qv + __shfl_sync(m, qv, (lane + 2) & 31);
}

// ---------------------------------------------------------------------------
// selectMoEBatch: one warp per token, the token's logits held in registers
// (expert lane + 32i in slot i).  Each pass takes the first strictly greater
// logit among experts not yet chosen (lowest index wins ties, NaN and -Inf
// never win); no candidate gives (index = pass, value 0), and that index
// counts as chosen for the later passes.
// kCG: read the logits through L2 only (ld.global.cg), for logits written by
// other CTAs of the same kernel (the router's last CTA selects).
template <bool kCG = false>
__device__ __forceinline__ void select_token(const float *__restrict__ logits, int t, int E, int K, int lane,
                                             int32_t *__restrict__ sel_idx, float *__restrict__ sel_w) {
  constexpr int kPer = kDispatchMaxExperts / 32;
  const float *lg = logits + (size_t)t * E;
  const bool in_regs = E <= 32 * kPer;  // else every pass reads the logits again
  float lv[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    lv[i] = (in_regs && lane + 32 * i < E) ? (kCG ? __ldcg(lg + lane + 32 * i) : lg[lane + 32 * i]) : 0.0f;
  uint32_t taken = 0;  // bit i: expert lane + 32i already chosen
  int chosen[kSelectMaxK];
  float val[kSelectMaxK];
  for (int r = 0; r < K; ++r) {
    int best = -1;
    float v = -INFINITY;
    if (in_regs) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !((taken >> i) & 1u) && lv[i] > v) {
          v = lv[i];
          best = e;
        }
      }
    } else {
      for (int e = lane; e < E; e += 32) {
        bool already = false;
        for (int p = 0; p < r; ++p) already |= (chosen[p] == e);
        const float l = kCG ? __ldcg(lg + e) : lg[e];
        if (!already && l > v) {
          v = l;
          best = e;
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int ob = __shfl_xor_sync(0xffffffffu, best, off);
      if (ob >= 0 && (best < 0 || ov > v || (ov == v && ob < best))) {
        v = ov;
        best = ob;
      }
    }
    if (best < 0) {
      best = r;
      v = 0.0f;
    }
    if ((best & 31) == lane && best < 32 * kPer) taken |= 1u << (best >> 5);
    chosen[r] = best;
    val[r] = v;
  }
  // Softmax over the chosen logits (every lane holds the same chosen/val):
  // lane r < K takes exp of pass r's logit, the sum runs in pass order in
  // every lane, and lane r writes pass r.  Same operations as a serial loop.
  float m = -INFINITY;
  for (int r = 0; r < K; ++r)
    if (val[r] > m) m = val[r];
  float ex = 0.0f;
  int my_idx = 0;
  if (lane < K) {
    ex = (float)exp((double)__fsub_rn(val[lane], m));
    my_idx = chosen[lane];
  }
  float sum = 0.0f;
  for (int r = 0; r < K; ++r) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, ex, r));
  if (sum > 0.0f) ex = __fmul_rn(ex, __fdiv_rn(1.0f, sum));
  if (lane < K) {
    sel_idx[(size_t)t * K + lane] = my_idx;
    sel_w[(size_t)t * K + lane] = ex;
  }
}

}  // namespace spt
