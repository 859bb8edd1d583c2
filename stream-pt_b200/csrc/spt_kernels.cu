// spt_kernels.cu -- sm_100a kernels of the MoE FFN block (CUDA cores).
//
// Every kernel reproduces the reference's arithmetic order so the GPU result
// is bit-identical to the Go AVX2 path (paths relative to the Stream-PT
// repository root):
//   * router:   64 FMA chains + fixed tree, forward/vector_amd64.go:28-56
//   * select:   k strict-> argmax passes + f64-exp softmax, forward/moe_batch.go:305-342
//   * dispatch: per-expert push-front lists, forward/moe_batch.go:142-159
//   * GEMV:     32 FMA chains over MXFP4 blocks + fixed tree,
//               forward/mxfp4_amd64.go:11-26 and forward/quant_amd64.go:112-116
//   * SwiGLU:   forward/moe.go:66-70
//   * combine:  fma(result, weight, out) in rank order, forward/moe_batch.go:163-192
// The file is compiled with -fmad=false: every fused multiply-add is an
// explicit fmaf / fma.rn.f32x2, all other operations round separately.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <map>
#include <mutex>

#include "spt_device.cuh"
#include "spt_internal.cuh"
#include "spt_philox.h"
#include "spt_ptx.cuh"
#include "spt_route.cuh"

namespace spt {

namespace {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Packed fp32 pair arithmetic (sm_100a f32x2): two independent IEEE
// round-to-nearest operations per instruction.
__device__ __forceinline__ void fma2(float &c0, float &c1, float a0, float a1, float b0,
                                     float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\tmov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ void mul2(float &a0, float &a1, float f) {
  asm("{\n\t.reg .b64 ra, rb;\n\t"
      "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %2};\n\t"
      "mul.rn.f32x2 ra, ra, rb;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(f));
}

// quantSumAVX2 of an 8-lane vector (forward/quant_amd64.go:112-116).
__device__ __forceinline__ float qsum8(const float s[8]) {
  float p0 = s[0] + s[4], p1 = s[1] + s[5], p2 = s[2] + s[6], p3 = s[3] + s[7];
  return (p0 + p1) + (p2 + p3);
}

// Decode 8 MXFP4 elements (nibble j of `w` = element 8q+j) with E8M0 byte s
// into exactly fl(level * 2^(s-127)), the value of scaledFP4Table
// (forward/mxfp4.go:24).  Bits (m<<22)|(sign<<31) form the float
// +-level * 2^-126 (e2m1's exponent lands in the fp32 exponent, its mantissa
// bit in the top mantissa bit, subnormals included), so one exact multiply
// by 2^(s-1) gives the scaled level for s <= 128.  Larger s take a second
// exact multiply (overflow rounds to Inf as in the reference) and s = 255
// multiplies by +Inf (0 * Inf = NaN, as the reference table holds).
__device__ __forceinline__ void decode8(uint32_t w, uint32_t s, float out[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t c = (((w >> (4 * j)) & 7u) << 22) | (((w >> (4 * j + 3)) & 1u) << 31);
    out[j] = __uint_as_float(c);
  }
  float f = __uint_as_float((s + 126u) << 23);
  if (s > 128u) f = (s == 255u) ? __uint_as_float(0x7f800000u) : 0x1p127f;
#pragma unroll
  for (int j = 0; j < 8; j += 2) mul2(out[j], out[j + 1], f);
  if (s > 128u && s < 255u) {
    const float f2 = __uint_as_float((s - 1u) << 23);  // 2^(s-128)
#pragma unroll
    for (int j = 0; j < 8; j += 2) mul2(out[j], out[j + 1], f2);
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int t) {
  return t == 0 ? v.x : (t == 1 ? v.y : (t == 2 ? v.z : v.w));
}

// Cross-thread part of the AVX2 reduction: thread q of a row holds the 8
// lanes of accumulator a_q; s[l] = ((a0[l]+a1[l])+a2[l])+a3[l], then
// quantSum.  Valid in the q == 0 lane.
__device__ __forceinline__ float reduce_row(const float acc[8], int lane) {
  const int base = lane & ~3;
  float s[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    const float v1 = __shfl_sync(kFull, acc[l], base + 1);
    const float v2 = __shfl_sync(kFull, acc[l], base + 2);
    const float v3 = __shfl_sync(kFull, acc[l], base + 3);
    s[l] = ((acc[l] + v1) + v2) + v3;
  }
  return qsum8(s);
}

// ---------------------------------------------------------------------------
// Router: logits[t,e] = dotF32AVX2(W[e], x[t]) + bias[e].
// One warp per (ME experts, MTR tokens).  Lane l runs chains l and l+32 of
// the 64 chains (a_j[l'] with chain = 8j+l'); a 32-element tail
// (hidden%64 == 32) feeds chains 0..31 (vector_amd64.go:45-52).  The chunk
// loop is unrolled UNR times so the loads of UNR chunks are in flight
// together; x values are reused across the ME experts of the warp.
template <int MTR, int ME, int UNR>
__global__ void __launch_bounds__(32) k_router(const float *__restrict__ W,
                                               const float *__restrict__ x,
                                               const float *__restrict__ bias, int T, int H,
                                               int E, float *__restrict__ logits) {
  pdl_wait();
  pdl_trigger();
  const int e0 = blockIdx.x * ME, t0 = blockIdx.y * MTR, lane = threadIdx.x;
  const int nt = min(MTR, T - t0);
  const int ne = min(ME, E - e0);
  float a[ME][MTR], b[ME][MTR];
#pragma unroll
  for (int m = 0; m < ME; ++m)
#pragma unroll
    for (int j = 0; j < MTR; ++j) a[m][j] = b[m][j] = 0.0f;
  const float *xr[MTR];
#pragma unroll
  for (int j = 0; j < MTR; ++j) xr[j] = x + (size_t)(t0 + min(j, nt - 1)) * H;
  const float *wr[ME];
#pragma unroll
  for (int m = 0; m < ME; ++m) wr[m] = W + (size_t)(e0 + min(m, ne - 1)) * H;
  const int full = H / 64;
  int o = 0;
#pragma unroll UNR
  for (int c = 0; c < full; ++c, o += 64) {
    float w0[ME], w1[ME], x0[MTR], x1[MTR];
#pragma unroll
    for (int m = 0; m < ME; ++m) {
      w0[m] = __ldg(wr[m] + o + lane);
      w1[m] = __ldg(wr[m] + o + 32 + lane);
    }
#pragma unroll
    for (int j = 0; j < MTR; ++j) {
      x0[j] = __ldg(xr[j] + o + lane);
      x1[j] = __ldg(xr[j] + o + 32 + lane);
    }
#pragma unroll
    for (int m = 0; m < ME; ++m)
#pragma unroll
      for (int j = 0; j < MTR; ++j) {
        a[m][j] = fmaf(w0[m], x0[j], a[m][j]);
        b[m][j] = fmaf(w1[m], x1[j], b[m][j]);
      }
  }
  if (o < H) {
#pragma unroll
    for (int m = 0; m < ME; ++m) {
      const float w0 = __ldg(wr[m] + o + lane);
#pragma unroll
      for (int j = 0; j < MTR; ++j) a[m][j] = fmaf(w0, __ldg(xr[j] + o + lane), a[m][j]);
    }
  }
#pragma unroll
  for (int m = 0; m < ME; ++m) {
    const float be = (bias && m < ne) ? bias[e0 + m] : 0.0f;
#pragma unroll
    for (int j = 0; j < MTR; ++j) {
      const float a8 = __shfl_sync(kFull, a[m][j], (lane + 8) & 31);
      const float a16 = __shfl_sync(kFull, a[m][j], (lane + 16) & 31);
      const float a24 = __shfl_sync(kFull, a[m][j], (lane + 24) & 31);
      const float b8 = __shfl_sync(kFull, b[m][j], (lane + 8) & 31);
      const float b16 = __shfl_sync(kFull, b[m][j], (lane + 16) & 31);
      const float b24 = __shfl_sync(kFull, b[m][j], (lane + 24) & 31);
      const float s0 = ((a[m][j] + a8) + a16) + a24;
      const float s1 = ((b[m][j] + b8) + b16) + b24;
      const float sv = s0 + s1;
      const float p = sv + __shfl_sync(kFull, sv, (lane + 4) & 31);
      const float qv = p + __shfl_sync(kFull, p, (lane + 1) & 31);
      const float r = qv + __shfl_sync(kFull, qv, (lane + 2) & 31);
      if (lane == 0 && j < nt && m < ne) logits[(size_t)(t0 + j) * E + e0 + m] = r + be;
    }
  }
}

// Router with its operands staged in shared memory.  The CTA copies EG rows
// of W and TG rows of x with cp.async, all in flight together (one memory
// latency instead of one per 64-element chunk), then each warp computes one
// token against up to four experts from shared memory, in k_router's order:
// lane l runs chains l and l+32, the 32-element tail feeds chains 0..31, and
// the same shuffle tree reduces them (vector_amd64.go:28-56).
constexpr int kRouterSmemMax = 200 * 1024;


constexpr int kRouterSmemDispatchMax = 180 * 1024;  // leaves room for dispatch_cta's static tables

template <bool kCG>
__device__ __forceinline__ void dispatch_cta(int32_t *sel_idx, float *sel_w, int S, int E,
                                             int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                                             int32_t *__restrict__ slot_pos, int32_t *__restrict__ act_list,
                                             int32_t *__restrict__ meta, const DispatchPlan &plan, int key_div,
                                             const float *__restrict__ logits, int T, int topk);

template <bool DISPATCH>
__global__ void __launch_bounds__(512) k_router_smem(const float *__restrict__ W,
                                                     const float *__restrict__ x,
                                                     const float *__restrict__ bias, int T, int H,
                                                     int E, int EG, int TG,
                                                     float *__restrict__ logits, __half *__restrict__ xq,
                                                     int32_t *__restrict__ xe, int KP,
                                                     const float *__restrict__ norm_w, float eps,
                                                     float *__restrict__ normed, RouterDispatch rd,
                                                     int32_t *err, int wait_shift, int fault) {
  extern __shared__ float4 router_smem[];
  float *ws = reinterpret_cast<float *>(router_smem);  // [EG][H]
  float *xs = ws + (size_t)EG * H;                     // [TG][H]
  __shared__ uint64_t s_rows_full;
  const int e0 = blockIdx.x * EG, t0 = blockIdx.y * TG;
  const int ne = min(EG, E - e0), nt = min(TG, T - t0);
  if (err) {
    // every row is one bulk copy on an mbarrier (rows are 16-byte multiples):
    // the expert rows do not depend on earlier kernels and go out before the
    // wait for the predecessor grid, the token rows after it
    if (threadIdx.x == 0) {
      mbar_init(&s_rows_full, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      mbar_expect_tx(&s_rows_full, (uint32_t)((ne + nt) * H * (int)sizeof(float)));
      // test hook (kRouterFault): CTA 0 leaves out its first row's copy, so
      // the wait below runs out -- the failure path without a fault
      const int r_first = (fault && blockIdx.x == 0 && blockIdx.y == 0) ? 1 : 0;
      for (int r = r_first; r < ne; ++r)
        bulk_load(ws + (size_t)r * H, W + (size_t)(e0 + r) * H, (uint32_t)(H * sizeof(float)), &s_rows_full);
    }
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0)
      for (int r = 0; r < nt; ++r)
        bulk_load(xs + (size_t)r * H, x + (size_t)(t0 + r) * H, (uint32_t)(H * sizeof(float)), &s_rows_full);
    __syncthreads();  // the barrier is initialised before anyone waits on it
    // on a timeout (here or recorded by another kernel) the whole CTA leaves
    // -- the host reports SPT_ERR_TIMEOUT -- once thread 0's copies have
    // landed or a second bound has passed
    const bool ok = mbar_wait(&s_rows_full, 0, err, 9, wait_shift);
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) {
        mbar_wait_own(&s_rows_full, 0, wait_shift);
        if constexpr (DISPATCH) {  // still counted, so the counter is 0 again for the next launch
          if (atomicAdd(rd.count, 1u) == gridDim.x * gridDim.y - 1) atomicExch(rd.count, 0u);
        }
      }
      return;
    }
  } else {
    pdl_wait();
    pdl_trigger();
    const int q = H / 4;  // 16-byte pieces per row
    for (int i = threadIdx.x; i < (ne + nt) * q; i += blockDim.x) {
      const int r = i / q, c = i - r * q;
      const float *src = r < ne ? W + (size_t)(e0 + r) * H : x + (size_t)(t0 + r - ne) * H;
      float *dst = r < ne ? ws + (size_t)r * H : xs + (size_t)(r - ne) * H;
      cp_async16(dst + 4 * c, src + 4 * c);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (norm_w) {
    // normBatch (forward/layer_batch.go:139-195) on the staged token rows, in
    // k_rmsnorm's order: 8 lanes of sequential squares, summed lane by lane;
    // then the rows are replaced by (x * w) * f, and this CTA's share of them
    // (every gridDim.x-th element) goes to `normed` for the expert kernels
    __shared__ float s_f[8];
    for (int j = warp; j < nt; j += blockDim.x >> 5) {
      const float *xr = xs + (size_t)j * H;
      float acc = 0.0f;
      if (lane < 8) {  // H % 32 == 0 here: no zero-padded tail
#pragma unroll 8
        for (int o = lane; o < H; o += 8) acc = fmaf(xr[o], xr[o], acc);
      }
      float sum = 0.0f;
      for (int l = 0; l < 8; ++l) sum = __fadd_rn(sum, __shfl_sync(kFull, acc, l));
      if (lane == 0) s_f[j] = __fdiv_rn(1.0f, (float)sqrt((double)__fadd_rn(__fdiv_rn(sum, (float)H), eps)));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nt * H; i += blockDim.x) {
      const int j = i / H, k = i - j * H;
      xs[i] = __fmul_rn(__fmul_rn(xs[i], __ldg(norm_w + k)), s_f[j]);
    }
    __syncthreads();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nt * H; i += gridDim.x * blockDim.x)
      normed[(size_t)t0 * H + i] = xs[i];
  }
  if (xq) {
    // The decode GEMV's split operand of these tokens (spt_gemv16.cuh), made
    // here from the staged rows: CTA bx writes K tiles bx, bx + gridDim.x, ...
    __shared__ float s_red[16];  // one per warp (256 or 512 threads)
    for (int j = 0; j < nt; ++j) {
      const float *xr = xs + (size_t)j * H;
      float m = 0.0f;
      for (int k = threadIdx.x; k < H; k += blockDim.x) m = fmaxf(m, fabsf(xr[k]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
      if (lane == 0) s_red[warp] = m;
      __syncthreads();
      m = s_red[0];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, s_red[w]);
      __syncthreads();
      const int ex = split_exponent(m);
      const float f = __int_as_float((127 - ex) << 23);
      if (blockIdx.x == 0 && threadIdx.x == 0) xe[t0 + j] = ex;
      __half *hi = xq + (size_t)(t0 + j) * 2 * KP, *lo = hi + KP;
      for (int kt = blockIdx.x; kt * kMmaKT < KP; kt += gridDim.x)
        for (int i = threadIdx.x; i < kMmaKT; i += blockDim.x) {
          const int k = kt * kMmaKT + i;
          __half h, l;
          split_f16(k < H ? __fmul_rn(xr[k], f) : 0.0f, &h, &l);
          hi[k] = h;
          lo[k] = l;
        }
    }
  }
  const int groups = (ne + 3) / 4;
  for (int item = warp; item < nt * groups; item += blockDim.x >> 5) {
    const int j = item / groups, mb = (item - j * groups) * 4;
    const float *xr = xs + (size_t)j * H;
    const float *wr[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) wr[m] = ws + (size_t)min(mb + m, ne - 1) * H;
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f}, b[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int full = H / 64;
    int o = 0;
#pragma unroll 3
    for (int c = 0; c < full; ++c, o += 64) {
      const float x0 = xr[o + lane], x1 = xr[o + 32 + lane];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        a[m] = fmaf(wr[m][o + lane], x0, a[m]);
        b[m] = fmaf(wr[m][o + 32 + lane], x1, b[m]);
      }
    }
    if (o < H) {
      const float x0 = xr[o + lane];
#pragma unroll
      for (int m = 0; m < 4; ++m) a[m] = fmaf(wr[m][o + lane], x0, a[m]);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float a8 = __shfl_sync(kFull, a[m], (lane + 8) & 31);
      const float a16 = __shfl_sync(kFull, a[m], (lane + 16) & 31);
      const float a24 = __shfl_sync(kFull, a[m], (lane + 24) & 31);
      const float b8 = __shfl_sync(kFull, b[m], (lane + 8) & 31);
      const float b16 = __shfl_sync(kFull, b[m], (lane + 16) & 31);
      const float b24 = __shfl_sync(kFull, b[m], (lane + 24) & 31);
      const float s0 = ((a[m] + a8) + a16) + a24;
      const float s1 = ((b[m] + b8) + b16) + b24;
      const float sv = s0 + s1;
      const float p = sv + __shfl_sync(kFull, sv, (lane + 4) & 31);
      const float qv = p + __shfl_sync(kFull, p, (lane + 1) & 31);
      const float r = qv + __shfl_sync(kFull, qv, (lane + 2) & 31);
      if (lane == 0 && mb + m < ne) logits[(size_t)(t0 + j) * E + e0 + mb + m] = r + (bias ? bias[e0 + mb + m] : 0.0f);
    }
  }
  if constexpr (DISPATCH) {
    // the last CTA to finish selects and dispatches: this CTA's logits are
    // made visible device-wide before it counts itself
    __shared__ bool s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(rd.count, 1u);
      s_last = prev == gridDim.x * gridDim.y - 1;
      if (s_last) atomicExch(rd.count, 0u);  // every other CTA has counted itself
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    dispatch_cta<true>(rd.sel_idx, rd.sel_w, T * rd.topk, E, rd.offsets, rd.perm, rd.slot_pos, rd.act_list,
                       rd.meta, rd.plan, 1, logits, T, rd.topk);
  }
}

// Router for hidden % 32 != 0: the portable simd.Float32s order with `lanes`
// lanes (forward/moe_batch.go:228-302): lane l accumulates elements l,
// l+lanes, ... (zero-padded tail), then the lanes are summed in order.
__global__ void k_router_portable(const float *__restrict__ W, const float *__restrict__ x,
                                  const float *__restrict__ bias, int T, int H, int E,
                                  int lanes, float *__restrict__ logits) {
  pdl_wait();
  pdl_trigger();
  const int e = blockIdx.x, t = blockIdx.y, lane = threadIdx.x;
  float acc = 0.0f;
  if (lane < lanes) {
    for (int o = 0; o < H; o += lanes) {
      const float wv = (o + lane < H) ? W[(size_t)e * H + o + lane] : 0.0f;
      const float xv = (o + lane < H) ? x[(size_t)t * H + o + lane] : 0.0f;
      acc = fmaf(wv, xv, acc);
    }
  }
  float sum = 0.0f;
  for (int l = 0; l < lanes; ++l) sum += __shfl_sync(kFull, acc, l);
  if (lane == 0) logits[(size_t)t * E + e] = sum + (bias ? bias[e] : 0.0f);
}

__global__ void __launch_bounds__(128) k_select(const float *__restrict__ logits, int T, int E,
                                                int K, int32_t *__restrict__ sel_idx,
                                                float *__restrict__ sel_w) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t < T) select_token(logits, t, E, K, threadIdx.x & 31, sel_idx, sel_w);
}

// ---------------------------------------------------------------------------
// Dispatch: the reference pushes slot t*k+r (weight > 0 or NaN) onto the
// front of its expert's list (moe_batch.go:142-159), so walking a list visits
// that expert's slots in descending slot order.  One CTA turns that into a
// stable counting sort: histogram, block scan over experts, then chunks of
// 1024 slots taken in descending order, ranked within a warp by
// __match_any_sync and across warps by a per-warp count table.
//
// The sort key is sel_idx / key_div: 1 groups slots by expert; the expert-
// parallel path passes the experts per rank, grouping slots by owner rank.
//
// With plan.bn > 0 the same CTA also lays out the tensor-core GEMM tiles:
// each active expert's tokens form ceil(n/bn) token tiles, each owning one
// 128-row activation slot (pad_off), and gate/up and down tile prefixes over
// the active experts (tile_gu, tile_dn), plus pos -> expert (pos_expert).
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(kFull, v, d);
    if (lane >= d) v += o;
  }
  return v;
}

// The whole dispatch, run by one CTA of any size up to 1024 threads (the
// dispatch kernel's, or the router's last CTA).  kCG: the logits were written
// by other CTAs of the running kernel and are read through L2 only.
template <bool kCG>
__device__ __forceinline__ void dispatch_cta(int32_t *sel_idx, float *sel_w, int S, int E,
                                             int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                                             int32_t *__restrict__ slot_pos, int32_t *__restrict__ act_list,
                                             int32_t *__restrict__ meta, const DispatchPlan &plan, int key_div,
                                             const float *__restrict__ logits, int T, int topk) {
  constexpr int kScanWarps = kDispatchMaxExperts / 32;
  constexpr int kVals = 5;  // tokens, active flag, slot rows, gate/up tiles, down tiles
  __shared__ int s_cnt[kDispatchMaxExperts];
  __shared__ int s_off[kDispatchMaxExperts + 1];
  __shared__ int s_run[kDispatchMaxExperts];
  __shared__ int s_w[32 * kDispatchMaxExperts];
  __shared__ int s_tot[kScanWarps][kVals];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (logits) {
    // selectMoEBatch for small batches (single device, key_div 1), one warp
    // per token, before the sort; the selections also go to global memory for
    // the later kernels, and __syncthreads makes them visible to this block.
    // sel_idx / sel_w are plain pointers here: no read-only cache path.
    for (int t = warp; t < T; t += (int)(blockDim.x >> 5))
      select_token<kCG>(logits, t, E, topk, lane, sel_idx, sel_w);
    __syncthreads();
  }
  for (int e = tid; e < E; e += blockDim.x) {
    s_cnt[e] = 0;
    s_run[e] = 0;
  }
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x)
    if (!(sel_w[s] <= 0.0f)) atomicAdd(&s_cnt[sel_idx[s] / key_div], 1);
  __syncthreads();
  int v[kVals] = {0, 0, 0, 0, 0}, inc[kVals] = {0, 0, 0, 0, 0};
  if (tid < kDispatchMaxExperts) {
    const int cnt = tid < E ? s_cnt[tid] : 0;
    const int nt = plan.bn > 0 ? (cnt + plan.bn - 1) / plan.bn : 0;
    v[0] = cnt;
    v[1] = cnt > 0 ? 1 : 0;
    v[2] = nt * 128;
    v[3] = nt * plan.mt_gu;
    v[4] = nt * plan.mt_dn;
#pragma unroll
    for (int k = 0; k < kVals; ++k) inc[k] = warp_incl_scan(v[k], lane);
    if (lane == 31)
#pragma unroll
      for (int k = 0; k < kVals; ++k) s_tot[warp][k] = inc[k];
  }
  __syncthreads();
  if (tid < kDispatchMaxExperts) {
#pragma unroll
    for (int k = 0; k < kVals; ++k)
      for (int w = 0; w < warp; ++w) inc[k] += s_tot[w][k];
    const int e = tid;
    if (e < E) {
      const int off = inc[0] - v[0];
      s_off[e] = off;
      offsets[e] = off;
      if (v[1]) {
        const int ai = inc[1] - 1;
        act_list[ai] = e;
        if (plan.act_off) plan.act_off[ai] = off;
        if (plan.bn > 0) {
          plan.pad_off[e] = inc[2] - v[2];
          plan.tile_gu[ai] = inc[3] - v[3];
          plan.tile_dn[ai] = inc[4] - v[4];
        }
      }
    }
    if (e == kDispatchMaxExperts - 1) {  // inclusive totals over every expert
      s_off[E] = inc[0];
      offsets[E] = inc[0];
      meta[0] = inc[1];
      meta[1] = inc[0];
      if (plan.act_off) plan.act_off[inc[1]] = inc[0];
      if (plan.bn > 0) {
        plan.tile_gu[inc[1]] = inc[3];
        plan.tile_dn[inc[1]] = inc[4];
      }
    }
  }
  __syncthreads();
  const int total = s_off[E];
  if (plan.bn > 0) {
    for (int p = tid; p < total; p += blockDim.x) {
      int lo = 0, hi = E - 1;  // largest expert with offsets[e] <= p
      while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (s_off[mid] <= p) lo = mid;
        else hi = mid - 1;
      }
      plan.pos_expert[p] = lo;
    }
  }
  for (int base = 0; base < S; base += blockDim.x) {
    const int s = S - 1 - (base + tid);
    const bool valid = s >= 0;
    int e = -1;
    bool disp = false;
    if (valid) {
      disp = !(sel_w[s] <= 0.0f);
      e = sel_idx[s] / key_div;
    }
    const int key = disp ? e : -1;
    const unsigned m = __match_any_sync(kFull, key);
    const int rank = __popc(m & ((1u << lane) - 1u));
    for (int k = tid; k < 32 * E; k += blockDim.x) s_w[k] = 0;
    __syncthreads();
    if (disp && rank == 0) s_w[warp * E + e] = __popc(m);
    __syncthreads();
    if (disp) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += s_w[w * E + e];
      const int pos = s_off[e] + s_run[e] + before + rank;
      perm[pos] = s;
      slot_pos[s] = pos;
    } else if (valid) {
      slot_pos[s] = -1;
    }
    __syncthreads();
    for (int k = tid; k < E; k += blockDim.x) {
      int tot = 0;
      for (int w = 0; w < 32; ++w) tot += s_w[w * E + k];
      s_run[k] += tot;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(1024) k_dispatch(int32_t *sel_idx, float *sel_w, int S, int E,
                                                   int32_t *__restrict__ offsets,
                                                   int32_t *__restrict__ perm,
                                                   int32_t *__restrict__ slot_pos,
                                                   int32_t *__restrict__ act_list,
                                                   int32_t *__restrict__ meta, DispatchPlan plan,
                                                   int key_div, const float *__restrict__ logits, int T,
                                                   int topk) {
  pdl_wait();
  pdl_trigger();
  dispatch_cta<false>(sel_idx, sel_w, S, E, offsets, perm, slot_pos, act_list, meta, plan, key_div, logits, T, topk);
}

// ---------------------------------------------------------------------------
// Expert-parallel exchange helpers.
//
// Send-side gather: row p of the send buffer is the token of slot perm[p]
// (slots grouped by owner rank), with the expert id local to that rank.
__global__ void __launch_bounds__(256) k_ep_gather(const float *__restrict__ x,
                                                   const int32_t *__restrict__ sel_idx,
                                                   const int32_t *__restrict__ perm,
                                                   const int32_t *__restrict__ meta, int K,
                                                   int experts_per_rank, int H, int S,
                                                   float *__restrict__ xs, int32_t *__restrict__ ms) {
  pdl_wait();
  pdl_trigger();
  const int n = min(meta[1], S);
  for (int p = blockIdx.x; p < n; p += gridDim.x) {
    const int slot = perm[p];
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(slot / K) * H);
    float4 *dst = reinterpret_cast<float4 *>(xs + (size_t)p * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) ms[p] = sel_idx[slot] % experts_per_rank;
  }
}

// Fixed-capacity layout (no host round trip): rank `dest`'s rows go to send
// rows [dest*cap, dest*cap + count).  Writes the rows, their local expert
// ids, the per-rank counts, and rewrites slot_pos (the dispatch kernel's
// compact position) to the row in this layout.
__global__ void __launch_bounds__(256) k_ep_gather_cap(const float *__restrict__ x,
                                                       const int32_t *__restrict__ sel_idx,
                                                       const int32_t *__restrict__ perm,
                                                       const int32_t *__restrict__ offsets,
                                                       const int32_t *__restrict__ meta, int K,
                                                       int experts_per_rank, int H, int S, int world,
                                                       int cap, float *__restrict__ xs,
                                                       int32_t *__restrict__ ms, int32_t *__restrict__ counts,
                                                       int32_t *__restrict__ slot_pos) {
  pdl_wait();
  pdl_trigger();
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < world; r += blockDim.x) counts[r] = offsets[r + 1] - offsets[r];
  const int n = min(meta[1], S);
  for (int p = blockIdx.x; p < n; p += gridDim.x) {
    int lo = 0, hi = world - 1;  // destination rank: largest r with offsets[r] <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (offsets[mid] <= p) lo = mid;
      else hi = mid - 1;
    }
    const int row = lo * cap + (p - offsets[lo]);
    const int slot = perm[p];
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(slot / K) * H);
    float4 *dst = reinterpret_cast<float4 *>(xs + (size_t)row * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) {
      ms[row] = sel_idx[slot] % experts_per_rank;
      slot_pos[slot] = row;
    }
  }
}

// Receive side of the fixed-capacity layout: row j (from rank j / cap) is
// live when j % cap < that rank's count; live rows get weight 1, padding 0
// (never dispatched).
__global__ void k_ep_recv_weights(const int32_t *__restrict__ counts, int cap, int world,
                                  float *__restrict__ w) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = (int64_t)cap * world;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
    w[j] = (j % cap) < counts[j / cap] ? 1.0f : 0.0f;
}

// ---------------------------------------------------------------------------
// Peer-memory exchange of the fixed-capacity layout.  Every rank's window
// (EpPeerLayout) is mapped into every other rank's address space (CUDA IPC,
// one GPU per rank); a sender writes its live rows straight into the owner's
// window over NVLink and then publishes the call's sequence number in the
// owner's flag for it, a receiver waits (bounded) until every sender's flag
// has reached the sequence number.  Windows are double-buffered by call
// parity.

// 64-bit flag store with release semantics at system scope.
__device__ __forceinline__ void flag_release(uint8_t *p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(reinterpret_cast<uint64_t *>(p)), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t flag_acquire(const uint8_t *p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(reinterpret_cast<const uint64_t *>(p)) : "memory");
  return v;
}

// The CTA that arrives last (counted in *arrive, which it resets) after
// every CTA's peer writes: sets flag[me] = seq in every rank's window.
__device__ __forceinline__ void signal_peers(const EpPeerLayout &L, int64_t flag_off, uint64_t seq, int32_t *arrive) {
  __shared__ int s_last;
  __threadfence_system();  // this thread's writes to the peers, before the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(arrive, 1);
    s_last = prev == (int)gridDim.x - 1;
    if (s_last) *arrive = 0;
  }
  __syncthreads();
  if (s_last && threadIdx.x < L.world) {
    __threadfence_system();
    flag_release(L.base[threadIdx.x] + flag_off + 8 * (int64_t)L.rank, seq);
  }
}

// Send side: slot groups by owner rank (the dispatch kernel keyed by expert /
// experts-per-rank), row j of the group for rank `dest` into dest's window at
// rows[par][me][j], its local expert id, this rank's count in dest's window,
// and slot_pos[slot] = dest*cap + j (where the result comes back).
__global__ void __launch_bounds__(256) k_ep_send_peer(const float *__restrict__ x, const int32_t *__restrict__ sel_idx,
                                                      const int32_t *__restrict__ perm,
                                                      const int32_t *__restrict__ offsets,
                                                      const int32_t *__restrict__ meta, int K, int experts_per_rank,
                                                      int S, EpPeerLayout L, int par, uint64_t seq,
                                                      int32_t *__restrict__ slot_pos, int32_t *arrive) {
  pdl_wait();
  pdl_trigger();
  const int W = L.world, me = L.rank, cap = L.cap, H = L.hidden;
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < W; r += blockDim.x)
      reinterpret_cast<int32_t *>(L.base[r] + L.cnt_off)[par * W + me] = offsets[r + 1] - offsets[r];
  const int n = min(meta[1], S);
  for (int p = blockIdx.x; p < n; p += gridDim.x) {
    int lo = 0, hi = W - 1;  // destination rank: largest r with offsets[r] <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (offsets[mid] <= p) lo = mid;
      else hi = mid - 1;
    }
    const int j = p - offsets[lo];
    const int slot = perm[p];
    const int64_t row = ((int64_t)par * W + me) * cap + j;
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(slot / K) * H);
    float4 *dst = reinterpret_cast<float4 *>(L.base[lo] + L.rows_off) + row * (H / 4);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) {
      reinterpret_cast<int32_t *>(L.base[lo] + L.ids_off)[row] = sel_idx[slot] % experts_per_rank;
      slot_pos[slot] = lo * cap + j;
    }
  }
  signal_peers(L, L.ffwd_off, seq, arrive);
}

// Receive side, results: row src*cap + j of rows_out (j < src's count) back
// into src's window at ret[par][me][j].
__global__ void __launch_bounds__(256) k_ep_return_peer(const float *__restrict__ rows_out, EpPeerLayout L, int par,
                                                        uint64_t seq, int32_t *arrive) {
  pdl_wait();
  pdl_trigger();
  const int W = L.world, me = L.rank, cap = L.cap, H = L.hidden;
  const int32_t *cnt = reinterpret_cast<const int32_t *>(L.base[me] + L.cnt_off) + par * W;
  for (int64_t p = blockIdx.x; p < (int64_t)W * cap; p += gridDim.x) {
    const int src = (int)(p / cap), j = (int)(p - (int64_t)src * cap);
    if (j >= cnt[src]) continue;
    const float4 *from = reinterpret_cast<const float4 *>(rows_out + (size_t)p * H);
    float4 *dst = reinterpret_cast<float4 *>(L.base[src] + L.ret_off) + (((int64_t)par * W + me) * cap + j) * (H / 4);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = from[i];
  }
  signal_peers(L, L.fret_off, seq, arrive);
}

// Wait until every rank's flag in this rank's window has reached seq, at most
// about 2^shift clock cycles; then *err = code and return.
__global__ void k_ep_wait(EpPeerLayout L, int64_t flag_off, uint64_t seq, int shift, int32_t *err, int code) {
  pdl_wait();
  pdl_trigger();
  const int r = threadIdx.x;
  if (r < L.world) {
    const uint8_t *f = L.base[L.rank] + flag_off + 8 * (int64_t)r;
    const long long t0 = clock64();
    for (uint32_t i = 0;; ++i) {
      if (flag_acquire(f) >= seq) break;
      if ((i & 63u) == 0u && clock64() - t0 > (1ll << shift)) {
        atomicCAS(err, 0, code);
        break;
      }
    }
  }
  __syncthreads();
}

// Receive side weights of the peer layout: row j of rank j / cap is live when
// j % cap < that rank's count in this rank's window.
__global__ void k_ep_recv_weights_peer(EpPeerLayout L, int par, float *__restrict__ w) {
  pdl_wait();
  pdl_trigger();
  const int32_t *cnt = reinterpret_cast<const int32_t *>(L.base[L.rank] + L.cnt_off) + par * L.world;
  const int64_t n = (int64_t)L.cap * L.world;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
    w[j] = (j % L.cap) < cnt[j / L.cap] ? 1.0f : 0.0f;
}

// counts[r] = offsets[r+1] - offsets[r]: rows sent to each rank.
__global__ void k_ep_counts(const int32_t *__restrict__ offsets, int world, int32_t *__restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  for (int r = threadIdx.x; r < world; r += blockDim.x) counts[r] = offsets[r + 1] - offsets[r];
}

__global__ void k_fill(float *__restrict__ p, int64_t n, float v) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ---------------------------------------------------------------------------
// Grouped MXFP4 GEMV on CUDA cores, bit-exact with dotMXFP4Fast.
// A warp owns (active expert, group of 8 rows); lane 4i+q runs FMA chains
// 8q..8q+7 of row 8g+i for up to MT tokens of the expert at once, so each
// decoded weight is reused across the tokens.  GU fuses gate and up and
// writes SwiGLU(gate+bias, up+bias).
template <int MT, bool GU>
__global__ void __launch_bounds__(128) k_gemv(const GemvLaunch a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, i = lane >> 2, q = lane & 3;
  const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const int G = a.m0.groups, NQ = a.m0.quads, NB = a.m0.blocks, R = a.m0.rows;
  const long long n_items = (long long)a.meta[0] * G;
  for (long long item = gw; item < n_items; item += nw) {
    const int ai = (int)(item / G), g = (int)(item - (long long)ai * G);
    const int e = a.act_list[ai];
    const int p0 = a.offsets[e], n = a.offsets[e + 1] - p0;
    const int row = g * 8 + i;
    const size_t base = ((size_t)e * G + g) * NQ;
    const uint4 *nb0 = a.m0.nib + base * 32 + lane;
    const uint32_t *sb0 = a.m0.scl + base * 8 + i;
    const uint4 *nb1 = GU ? a.m1.nib + base * 32 + lane : nullptr;
    const uint32_t *sb1 = GU ? a.m1.scl + base * 8 + i : nullptr;
    for (int t0 = 0; t0 < n; t0 += MT) {
      const int nt = min(MT, n - t0);
      const float *xr[MT];
#pragma unroll
      for (int j = 0; j < MT; ++j) {
        const int p = p0 + t0 + min(j, nt - 1);
        const int src = (a.mode == kRowsMoEGateUp) ? a.perm[p] / a.top_k : p;
        xr[j] = a.x + (size_t)src * a.x_stride + 8 * q;
      }
      float acc0[MT][8];
      float acc1[GU ? MT : 1][8];
#pragma unroll
      for (int j = 0; j < MT; ++j)
#pragma unroll
        for (int l = 0; l < 8; ++l) acc0[j][l] = 0.0f;
      if (GU) {
#pragma unroll
        for (int j = 0; j < (GU ? MT : 1); ++j)
#pragma unroll
          for (int l = 0; l < 8; ++l) acc1[j][l] = 0.0f;
      }
      uint4 w0 = __ldg(nb0);
      uint32_t s0 = __ldg(sb0);
      uint4 w1 = make_uint4(0, 0, 0, 0);
      uint32_t s1 = 0;
      if (GU) {
        w1 = __ldg(nb1);
        s1 = __ldg(sb1);
      }
      for (int Q = 0; Q < NQ; ++Q) {
        // software pipeline: fetch the next quad before decoding this one
        uint4 nw0 = w0, nw1 = w1;
        uint32_t ns0 = s0, ns1 = s1;
        if (Q + 1 < NQ) {
          nw0 = __ldg(nb0 + (size_t)(Q + 1) * 32);
          ns0 = __ldg(sb0 + (size_t)(Q + 1) * 8);
          if (GU) {
            nw1 = __ldg(nb1 + (size_t)(Q + 1) * 32);
            ns1 = __ldg(sb1 + (size_t)(Q + 1) * 8);
          }
        }
        const int nbq = min(4, NB - 4 * Q);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (t < nbq) {
            float d0[8], d1[8];
            decode8(word_of(w0, t), (s0 >> (8 * t)) & 0xffu, d0);
            if (GU) decode8(word_of(w1, t), (s1 >> (8 * t)) & 0xffu, d1);
            const int b = 4 * Q + t;
#pragma unroll
            for (int j = 0; j < MT; ++j) {
              if (j < nt) {
                const float4 xa = __ldg(reinterpret_cast<const float4 *>(xr[j] + 32 * b));
                const float4 xb = __ldg(reinterpret_cast<const float4 *>(xr[j] + 32 * b + 4));
                fma2(acc0[j][0], acc0[j][1], d0[0], d0[1], xa.x, xa.y);
                fma2(acc0[j][2], acc0[j][3], d0[2], d0[3], xa.z, xa.w);
                fma2(acc0[j][4], acc0[j][5], d0[4], d0[5], xb.x, xb.y);
                fma2(acc0[j][6], acc0[j][7], d0[6], d0[7], xb.z, xb.w);
                if (GU) {
                  fma2(acc1[j][0], acc1[j][1], d1[0], d1[1], xa.x, xa.y);
                  fma2(acc1[j][2], acc1[j][3], d1[2], d1[3], xa.z, xa.w);
                  fma2(acc1[j][4], acc1[j][5], d1[4], d1[5], xb.x, xb.y);
                  fma2(acc1[j][6], acc1[j][7], d1[6], d1[7], xb.z, xb.w);
                }
              }
            }
          }
        }
        w0 = nw0;
        s0 = ns0;
        w1 = nw1;
        s1 = ns1;
      }
#pragma unroll
      for (int j = 0; j < MT; ++j) {
        if (j < nt) {
          const float r0 = reduce_row(acc0[j], lane);
          float r1 = 0.0f;
          if (GU) r1 = reduce_row(acc1[GU ? j : 0], lane);
          if (q == 0 && row < R) {
            const float v0 = r0 + (a.bias0 ? a.bias0[(size_t)e * R + row] : 0.0f);
            float outv = v0;
            if (GU) {
              const float v1 = r1 + (a.bias1 ? a.bias1[(size_t)e * R + row] : 0.0f);
              outv = swiglu_ref(v0, v1);
            }
            a.y[(size_t)(p0 + t0 + j) * a.y_stride + row] = outv;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Combine: out[t,h] = 0, then for r = 0..K-1 with weight > 0 or NaN,
// out = fma(res[slot], w, out) (forward/moe_batch.go:163-192).
// With resid the sum is added to resid (the residual stream of the layer
// stack, addVector forward/layer.go:305-340: out = resid + sum, one rounding);
// out may be resid itself (each element is read and written by one thread).
__global__ void k_combine(const float *__restrict__ res, const float *__restrict__ sel_w,
                          const int32_t *__restrict__ slot_pos, int T, int K, int H,
                          const float *resid, float *out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (t >= T || h >= H) return;
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int r = 0; r < K; ++r) {
    const int s = t * K + r;
    const float w = sel_w[s];
    if (w <= 0.0f) continue;
    const int pos = slot_pos ? slot_pos[s] : s;
    const float4 v = *reinterpret_cast<const float4 *>(res + (size_t)pos * H + h);
    o.x = fmaf(v.x, w, o.x);
    o.y = fmaf(v.y, w, o.y);
    o.z = fmaf(v.z, w, o.z);
    o.w = fmaf(v.w, w, o.w);
  }
  if (resid) {
    const float4 x = *reinterpret_cast<const float4 *>(resid + (size_t)t * H + h);
    o = make_float4(__fadd_rn(x.x, o.x), __fadd_rn(x.y, o.y), __fadd_rn(x.z, o.z), __fadd_rn(x.w, o.w));
  }
  *reinterpret_cast<float4 *>(out + (size_t)t * H + h) = o;
}

__global__ void k_swiglu(const float *__restrict__ g, const float *__restrict__ u,
                         float *__restrict__ act, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    act[i] = swiglu_ref(g[i], u[i]);
}

// normBatch RMSNorm (forward/layer_batch.go:160-193) with `lanes`
// accumulation lanes: squares[l] = fma(v, v, squares[l]) over offsets step
// lanes (zero-padded), sequential lane sum, f = 1/float32(sqrt(float64(
// sum/float32(dim)+eps))), y = (x*w)*f.
__global__ void k_rmsnorm(const float *__restrict__ x, const float *__restrict__ w, int T,
                          int dim, float eps, int lanes, float *__restrict__ y) {
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  if (t >= T) return;
  const float *in = x + (size_t)t * dim;
  __shared__ float s_f;
  if (threadIdx.x < 32) {
    float acc = 0.0f;
    if (lane < lanes)
      for (int o = 0; o < dim; o += lanes) {
        const float v = (o + lane < dim) ? in[o + lane] : 0.0f;
        acc = fmaf(v, v, acc);
      }
    float sum = 0.0f;
    for (int l = 0; l < lanes; ++l) sum = __fadd_rn(sum, __shfl_sync(kFull, acc, l));
    if (lane == 0) {
      const float qv = __fadd_rn(__fdiv_rn(sum, (float)dim), eps);
      s_f = __fdiv_rn(1.0f, (float)sqrt((double)qv));
    }
  }
  __syncthreads();
  const float f = s_f;
  for (int i2 = threadIdx.x; i2 < dim; i2 += blockDim.x)
    y[(size_t)t * dim + i2] = __fmul_rn(__fmul_rn(in[i2], w[i2]), f);
}

__global__ void k_add(float *__restrict__ dst, const float *__restrict__ src, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __fadd_rn(dst[i], src[i]);
}

// ---------------------------------------------------------------------------
// GGUF 17-byte blocks -> G8 planes.  One thread per block.
__device__ __forceinline__ void block_to_g8(const uint8_t blk[17], int64_t e, int r, int b,
                                            int R, int NB, uint4 *nib, uint32_t *scl) {
  uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int qq = 0; qq < 4; ++qq)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int el = 8 * qq + j;
      const uint32_t nbl = el < 16 ? (blk[1 + el] & 15u) : (uint32_t)(blk[1 + el - 16] >> 4);
      words[qq] |= nbl << (4 * j);
    }
  const int G = (R + 7) / 8, NQ = (NB + 3) / 4;
  const int g = r / 8, ii = r % 8, Q = b / 4, t = b % 4;
  const size_t slot = (((size_t)e * G + g) * NQ + Q);
  uint32_t *nw = reinterpret_cast<uint32_t *>(nib);
#pragma unroll
  for (int qq = 0; qq < 4; ++qq) nw[((slot * 32) + ii * 4 + qq) * 4 + t] = words[qq];
  reinterpret_cast<uint8_t *>(scl)[((slot * 8) + ii) * 4 + t] = blk[0];
}

__global__ void k_repack_g8(const uint8_t *__restrict__ gguf, int64_t experts, int R, int NB,
                            uint4 *nib, uint32_t *scl) {
  const int64_t total = experts * R * NB;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx % NB);
    const int64_t er = idx / NB;
    const int r = (int)(er % R);
    const int64_t e = er / R;
    uint8_t blk[17];
    const uint8_t *src = gguf + idx * 17;
#pragma unroll
    for (int k = 0; k < 17; ++k) blk[k] = src[k];
    block_to_g8(blk, e, r, b, R, NB, nib, scl);
  }
}

__global__ void k_synth_g8(uint64_t seed, uint32_t tag, int64_t experts, int R, int NB,
                           uint8_t lo, uint8_t hi, uint64_t counter0, uint4 *nib, uint32_t *scl) {
  const int64_t total = experts * R * NB;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx % NB);
    const int64_t er = idx / NB;
    const int r = (int)(er % R);
    const int64_t e = er / R;
    uint8_t blk[17];
    synth_mxfp4_block(seed, tag, counter0 + (uint64_t)idx, lo, hi, blk);
    block_to_g8(blk, e, r, b, R, NB, nib, scl);
  }
}

inline unsigned grid_for(int64_t n, int threads, int64_t cap = 148 * 32) {
  int64_t g = (n + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

}  // namespace

// ---------------------------------------------------------------------------
// launchers

bool pdl_launches_enabled() {
  static const bool on = [] {
    const char *v = getenv("SPT_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

cudaError_t opt_in_smem_raw(const void *kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, int> done;  // (device, kernel) -> bytes set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({dev, kernel});
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[{dev, kernel}] = bytes;
  return e;
}

bool router_wide() {
  static const bool on = [] {
    const char *v = getenv("SPT_ROUTER_WIDE");
    return !(v && v[0] == '0');
  }();
  return on;
}

cudaError_t launch_router(const float *W, const float *x, const float *bias, int T, int H, int E,
                          float *logits, int portable_lanes, cudaStream_t stream, const RouterSplit *split,
                          bool *split_done, const RouterNorm *norm, int *launches, const RouterDispatch *dispatch,
                          bool *dispatch_done, int32_t *err, int wait_shift, int fault_stage) {
  const int fault = fault_stage == kRouterFault ? 1 : 0;
  if (split_done) *split_done = false;
  if (dispatch_done) *dispatch_done = false;
  if (launches) *launches = 1;
  if (T <= 0) return cudaSuccess;
  // the normalisation is folded into k_router_smem's prologue when that kernel
  // runs; otherwise it is its own launch and the router reads its output
  auto separate_norm = [&]() -> cudaError_t {
    if (!norm) return cudaSuccess;
    if (launches) *launches = 2;
    cudaError_t e = launch_rmsnorm(x, norm->w, T, H, norm->eps, norm->out, 8, stream);
    x = norm->out;
    return e;
  };
  if (H % 32 != 0) {
    cudaError_t e = separate_norm();
    if (e != cudaSuccess) return e;
    return launch_pdl(k_router_portable, dim3(E, T), dim3(32), 0, stream, W, x, bias, T, H, E, portable_lanes,
                      logits);
    return cudaGetLastError();
  }
  // Shared-memory staged router when the rows are 16-byte aligned and fit.
  int TG = T < 8 ? T : 8;
  const int n_tg = (T + TG - 1) / TG;
  int EG = 1;
  while (EG < 8 && (int64_t)(E / (EG * 2)) * n_tg >= 120) EG *= 2;
  auto bytes = [&](int eg, int tg) { return (int64_t)(eg + tg) * H * (int64_t)sizeof(float); };
  const bool with_dispatch = dispatch && dispatch->count && T <= kRouterDispatchMaxTokens &&
                             E <= kDispatchMaxExperts && dispatch->topk >= 1 && dispatch->topk <= E &&
                             dispatch->topk <= kSelectMaxK;
  const int64_t cap = with_dispatch ? kRouterSmemDispatchMax : kRouterSmemMax;
  while (EG > 1 && bytes(EG, TG) > cap) EG /= 2;
  while (TG > 1 && bytes(EG, TG) > cap) TG /= 2;
  // Beyond 64 tokens every CTA would restage the same rows many times over;
  // the register-blocked kernel reads them through L1/L2 instead.
  const bool aligned = ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
  if (T <= 64 && aligned && bytes(EG, TG) <= cap) {
    const bool do_split = split && split->xq && (E + EG - 1) / EG > 0;
    if (split_done) *split_done = do_split;
    const dim3 grid((E + EG - 1) / EG, (T + TG - 1) / TG);
    // above decode sizes a CTA has 8 tokens x EG experts of dots: 16 warps
    // take one token x 4 experts each (SPT_ROUTER_WIDE=0: 8 warps, two each)
    const int threads = (T > kRouterDispatchMaxTokens && router_wide()) ? 512 : 256;
    __half *sx = do_split ? split->xq : (__half *)nullptr;
    int32_t *se = do_split ? split->xe : (int32_t *)nullptr;
    const int skp = do_split ? split->kp : 0;
    const float *nw = norm ? norm->w : (const float *)nullptr;
    float *nout = norm ? norm->out : (float *)nullptr;
    const float neps = norm ? norm->eps : 0.0f;
    if (with_dispatch) {
      cudaError_t e = opt_in_smem(k_router_smem<true>, kRouterSmemDispatchMax);
      if (e != cudaSuccess) return e;
      if (dispatch_done) *dispatch_done = true;
      return launch_pdl(k_router_smem<true>, grid, dim3(threads), (size_t)bytes(EG, TG), stream, W, x, bias, T, H, E,
                        EG, TG, logits, sx, se, skp, nw, neps, nout, *dispatch, err, wait_shift, fault);
    }
    cudaError_t e = opt_in_smem(k_router_smem<false>, kRouterSmemMax);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_router_smem<false>, grid, dim3(threads), (size_t)bytes(EG, TG), stream, W, x, bias, T, H, E, EG,
                      TG, logits, sx, se, skp, nw, neps, nout, RouterDispatch{}, err, wait_shift, fault);
  } else {
    cudaError_t e = separate_norm();
    if (e != cudaSuccess) return e;
    return launch_pdl(k_router<8, 4, 1>, dim3((E + 3) / 4, (T + 7) / 8), dim3(32), 0, stream, W, x, bias, T, H, E,
                      logits);
  }
  return cudaGetLastError();
}

cudaError_t launch_select(const float *logits, int T, int E, int K, int32_t *sel_idx,
                          float *sel_w, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  return launch_pdl(k_select, dim3((T + 3) / 4), dim3(128), 0, stream, logits, T, E, K, sel_idx, sel_w);
}

cudaError_t launch_dispatch(const int32_t *sel_idx, const float *sel_w, int S, int E,
                            int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                            int32_t *act_list, int32_t *meta, cudaStream_t stream,
                            const DispatchPlan *plan, int key_div) {
  if (E > kDispatchMaxExperts || key_div < 1) return cudaErrorInvalidValue;
  // the kernel only writes sel_idx / sel_w when given logits
  return launch_pdl(k_dispatch, dim3(1), dim3(1024), 0, stream, const_cast<int32_t *>(sel_idx),
                    const_cast<float *>(sel_w), S, E, offsets, perm, slot_pos, act_list, meta,
                    plan ? *plan : DispatchPlan{}, key_div, (const float *)nullptr, 0, 0);
}

cudaError_t launch_select_dispatch(const float *logits, int T, int E, int K, int32_t *sel_idx, float *sel_w,
                                   int32_t *offsets, int32_t *perm, int32_t *slot_pos, int32_t *act_list,
                                   int32_t *meta, cudaStream_t stream, const DispatchPlan *plan) {
  if (E > kDispatchMaxExperts || T < 0 || T > kSelectDispatchMaxTokens || K < 1 || K > E || K > kSelectMaxK)
    return cudaErrorInvalidValue;
  return launch_pdl(k_dispatch, dim3(1), dim3(1024), 0, stream, sel_idx, sel_w, T * K, E, offsets, perm,
                    slot_pos, act_list, meta, plan ? *plan : DispatchPlan{}, 1, logits, T, K);
}

cudaError_t launch_ep_gather(const float *x, const int32_t *sel_idx, const int32_t *perm, const int32_t *meta,
                             int K, int experts_per_rank, int H, int S, float *xs, int32_t *ms,
                             cudaStream_t stream) {
  if (S <= 0) return cudaSuccess;
  if (H % 4 != 0) return cudaErrorInvalidValue;
  const int grid = S < 148 * 8 ? S : 148 * 8;
  return launch_pdl(k_ep_gather, dim3(grid), dim3(256), 0, stream, x, sel_idx, perm, meta, K, experts_per_rank, H,
                    S, xs, ms);
}

cudaError_t launch_ep_gather_cap(const float *x, const int32_t *sel_idx, const int32_t *perm, const int32_t *offsets,
                                 const int32_t *meta, int K, int experts_per_rank, int H, int S, int world, int cap,
                                 float *xs, int32_t *ms, int32_t *counts, int32_t *slot_pos, cudaStream_t stream) {
  if (H % 4 != 0 || world < 1) return cudaErrorInvalidValue;
  const int grid = S < 1 ? 1 : (S < 148 * 8 ? S : 148 * 8);
  return launch_pdl(k_ep_gather_cap, dim3(grid), dim3(256), 0, stream, x, sel_idx, perm, offsets, meta, K,
                    experts_per_rank, H, S, world, cap, xs, ms, counts, slot_pos);
}

cudaError_t launch_ep_recv_weights(const int32_t *counts, int cap, int world, float *w, cudaStream_t stream) {
  const int64_t n = (int64_t)cap * world;
  if (n <= 0) return cudaSuccess;
  const int64_t g = (n + 255) / 256;
  return launch_pdl(k_ep_recv_weights, dim3((unsigned)(g < 148 * 8 ? g : 148 * 8)), dim3(256), 0, stream, counts,
                    cap, world, w);
}

cudaError_t launch_ep_counts(const int32_t *offsets, int world, int32_t *counts, cudaStream_t stream) {
  return launch_pdl(k_ep_counts, dim3(1), dim3(256), 0, stream, offsets, world, counts);
}

cudaError_t launch_ep_send_peer(const float *x, const int32_t *sel_idx, const int32_t *perm, const int32_t *offsets,
                                const int32_t *meta, int K, int experts_per_rank, int S, const EpPeerLayout &L, int par,
                                uint64_t seq, int32_t *slot_pos, int32_t *arrive, cudaStream_t stream) {
  if (L.hidden % 4 != 0 || L.world < 1 || L.world > kEpMaxPeers) return cudaErrorInvalidValue;
  const int grid = S < 1 ? 1 : (S < 148 * 8 ? S : 148 * 8);
  return launch_pdl(k_ep_send_peer, dim3(grid), dim3(256), 0, stream, x, sel_idx, perm, offsets, meta, K,
                    experts_per_rank, S, L, par, seq, slot_pos, arrive);
}

cudaError_t launch_ep_return_peer(const float *rows_out, const EpPeerLayout &L, int par, uint64_t seq, int32_t *arrive,
                                  cudaStream_t stream) {
  if (L.hidden % 4 != 0 || L.world < 1 || L.world > kEpMaxPeers) return cudaErrorInvalidValue;
  const int64_t n = (int64_t)L.world * L.cap;
  const int grid = (int)(n < 1 ? 1 : (n < 148 * 8 ? n : 148 * 8));
  return launch_pdl(k_ep_return_peer, dim3(grid), dim3(256), 0, stream, rows_out, L, par, seq, arrive);
}

cudaError_t launch_ep_wait(const EpPeerLayout &L, int64_t flag_off, uint64_t seq, int shift, int32_t *err, int code,
                           cudaStream_t stream) {
  if (L.world < 1 || L.world > kEpMaxPeers) return cudaErrorInvalidValue;
  return launch_pdl(k_ep_wait, dim3(1), dim3(32), 0, stream, L, flag_off, seq, shift, err, code);
}

cudaError_t launch_ep_recv_weights_peer(const EpPeerLayout &L, int par, float *w, cudaStream_t stream) {
  const int64_t n = (int64_t)L.cap * L.world;
  if (n <= 0) return cudaSuccess;
  const int64_t g = (n + 255) / 256;
  return launch_pdl(k_ep_recv_weights_peer, dim3((unsigned)(g < 148 * 8 ? g : 148 * 8)), dim3(256), 0, stream, L,
                    par, w);
}

cudaError_t launch_fill(float *p, int64_t n, float v, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const int64_t g = (n + 255) / 256;
  return launch_pdl(k_fill, dim3((unsigned)(g < 148 * 16 ? g : 148 * 16)), dim3(256), 0, stream, p, n, v);
}

template <int MT, bool GU>
static cudaError_t gemv_inst(const GemvLaunch &a, unsigned grid, cudaStream_t stream) {
  cudaError_t e = launch_pdl(k_gemv<MT, GU>, dim3(grid), dim3(128), 0, stream, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_gemv(const GemvLaunch &a, int sm_count, cudaStream_t stream) {
  const int64_t items = (int64_t)a.max_active * a.m0.groups;
  int64_t ctas = (items + 3) / 4;
  const int64_t cap = (int64_t)(sm_count > 0 ? sm_count : 148) * 8;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  const unsigned grid = (unsigned)ctas;
  switch (a.mt) {
    case 1: return a.gate_up ? gemv_inst<1, true>(a, grid, stream) : gemv_inst<1, false>(a, grid, stream);
    case 2: return a.gate_up ? gemv_inst<2, true>(a, grid, stream) : gemv_inst<2, false>(a, grid, stream);
    case 4: return a.gate_up ? gemv_inst<4, true>(a, grid, stream) : gemv_inst<4, false>(a, grid, stream);
    default: return a.gate_up ? gemv_inst<8, true>(a, grid, stream) : gemv_inst<8, false>(a, grid, stream);
  }
}

cudaError_t launch_combine(const float *res, const float *sel_w, const int32_t *slot_pos, int T,
                           int K, int H, float *out, cudaStream_t stream, const float *resid) {
  if (T <= 0) return cudaSuccess;
  const int threads = 128;
  dim3 grid((H / 4 + threads - 1) / threads, T);
  cudaError_t e = launch_pdl(k_combine, dim3(grid), dim3(threads), 0, stream, res, sel_w, slot_pos, T, K, H, resid,
                             out);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const float *g, const float *u, float *act, int64_t n,
                          cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  k_swiglu<<<grid_for(n, 256), 256, 0, stream>>>(g, u, act, n);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float *x, const float *w, int T, int dim, float eps, float *y,
                           int lanes, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  k_rmsnorm<<<T, 256, 0, stream>>>(x, w, T, dim, eps, lanes, y);
  return cudaGetLastError();
}

cudaError_t launch_add(float *dst, const float *src, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  k_add<<<grid_for(n, 256), 256, 0, stream>>>(dst, src, n);
  return cudaGetLastError();
}

cudaError_t launch_repack_g8(const uint8_t *gguf, int64_t experts, int rows, int blocks,
                             uint4 *nib, uint32_t *scl, cudaStream_t stream) {
  const int64_t n = experts * rows * blocks;
  if (n <= 0) return cudaSuccess;
  k_repack_g8<<<grid_for(n, 256), 256, 0, stream>>>(gguf, experts, rows, blocks, nib, scl);
  return cudaGetLastError();
}

cudaError_t launch_synth_g8(uint64_t seed, uint32_t tag, int64_t first_expert, int64_t experts, int rows,
                            int blocks, uint8_t scale_lo, uint8_t scale_hi, uint4 *nib, uint32_t *scl,
                            cudaStream_t stream) {
  const int64_t n = experts * rows * blocks;
  if (n <= 0) return cudaSuccess;
  k_synth_g8<<<grid_for(n, 256), 256, 0, stream>>>(seed, tag, experts, rows, blocks, scale_lo, scale_hi,
                                                   (uint64_t)(first_expert * rows * blocks), nib, scl);
  return cudaGetLastError();
}

}  // namespace spt
