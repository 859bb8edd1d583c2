// spt_gemv16.cu -- decode-sized expert products: an HBM-streaming grouped
// GEMV over the packed MXFP4 planes of the tensor-core arena, with the
// dequantisation done in registers.
//
// At decode sizes (a few tokens per active expert) each weight byte is used
// by one to four tokens, so the expert products are bound by the weight
// stream, and what decides the time is how evenly and how early every SM
// starts streaming.  This path has no TMA descriptors, tensor memory or
// mbarrier rings to set up and no activation-quantisation launches: a CTA
// takes 32 rows of one active expert, its eight warps split K, and every
// lane issues all of its 16-byte weight loads (and the activation fragments
// it needs) before the first multiply.
//
// Arithmetic.  The GGUF MXFP4 weights are exact in f16 once scaled:
// e2m1 level (0..6) x 2^(s-127) is representable for scale bytes s in
// [kF16ScaleLo, kF16ScaleHi] (the arena records whether every scale of a
// layer is in that range).  Each byte of two e2m1 codes is converted to an
// f16 pair (cvt.rn.f16x2.e2m1x2) and multiplied by the f16 block scale
// (exact).  The activations enter as two f16 terms, hi = f16(v) and lo =
// f16(v - hi) ("split operand", about 22 significant bits), so every product
// is exact and the sums run in fp32 on the tensor cores' mma.sync
// m16n8k16 f16 -> f32 path, used here as the dot-product engine of a
// memory-bound GEMV: the 8 MMA columns are 4 tokens x (hi, lo).  Block
// outputs agree with the fp32 reference to about 1e-6 relative.
//
// Split operand layout (per row: token for gate/up, dispatch position for
// down): halves [row][term][KP], term 0 = hi, 1 = lo, natural element order,
// K padded to KP = 128 * ktiles with zeros.  x rows carry a power-of-two
// exponent xe[row] (x = (hi + lo) * 2^xe) chosen so that max|x| lands in
// [2^14, 2^15) and nothing overflows f16; SwiGLU outputs are bounded
// (|act| <= 56) and carry none.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "spt_device.cuh"
#include "spt_gemv16.cuh"
#include "spt_internal.cuh"

namespace spt {

namespace {

constexpr int kWarps = 8;             // K is split over the CTA's warps
constexpr int kRowsPerCta = 32;       // two m16 MMA tiles
constexpr int kMaxKtPerWarp = 3;      // ceil(23 / 8) for GPT-OSS; larger K loops
constexpr int kTokPerPass = 4;        // MMA N = 8 = 4 tokens x (hi, lo)

// E8M0 byte -> the f16 pair (2^(s-127), 2^(s-127)), exact for s in
// [kF16ScaleLo, kF16ScaleHi] (2^-23 .. 2^13, subnormal below 2^-14).  Bytes
// outside it occur only in the zero padding of the planes (rows beyond the
// matrix, K beyond its length), whose levels are 0: they map to 0.
__device__ __forceinline__ uint32_t scale_h2(uint32_t s) {
  const int k = (int)s - 127;
  uint32_t h = 0;
  if (k >= -14) h = (uint32_t)min(k + 15, 30) << 10;
  else if (k >= -24) h = 1u << (k + 24);
  return h | (h << 16);
}

// Eight e2m1 codes (one word; in each byte the low nibble is the lower
// element) -> four f16 pairs, byte i to h[i].
__device__ __forceinline__ void e2m1x8_h2(uint32_t w, uint32_t h[4]) {
  asm volatile(
      "{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void mma16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t word_at(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}


// ---------------------------------------------------------------------------
// fp32 rows -> split operand, one CTA per output row p: the source row is
// perm[p] / top_k (the token of dispatch position p) when perm is given,
// else p; rows at or past meta[1] (the dispatched count) are skipped when
// meta is given.  The row's values are loaded once (16-byte loads, all in
// flight together), then max |v|, the exponent xe with max|v| * 2^-xe in
// [2^14, 2^15) (0 when the row is all zeros or its maximum is not finite),
// hi/lo halves of v * 2^-xe, and zeros for the K padding.
constexpr int kSplitThreads = 256;
constexpr int kSplitVec = 4;  // float4 loads per thread: K <= 4096
__global__ void __launch_bounds__(kSplitThreads) k_split_rows(const float *__restrict__ src, int64_t stride, int K,
                                                              int KP, const int32_t *__restrict__ perm, int top_k,
                                                              const int32_t *__restrict__ meta,
                                                              __half *__restrict__ dst, int32_t *__restrict__ xe) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  if (meta && row >= meta[1]) return;
  const int srow = perm ? perm[row] / top_k : row;
  const float4 *s4 = reinterpret_cast<const float4 *>(src + (size_t)srow * stride);
  float4 v[kSplitVec];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < kSplitVec; ++i) {
    const int q = threadIdx.x + i * kSplitThreads;  // float4 index
    v[i] = 4 * q < K ? s4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < kSplitVec; ++i)
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
  __shared__ float red[kSplitThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < kSplitThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const int e = split_exponent(amax);
  const float f = __int_as_float((127 - e) << 23);  // 2^-e
  __half *hi = dst + (size_t)row * 2 * KP, *lo = hi + KP;
#pragma unroll
  for (int i = 0; i < kSplitVec; ++i) {
    const int q = threadIdx.x + i * kSplitThreads;
    if (4 * q >= KP) break;
    const float vals[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    __half h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split_f16(__fmul_rn(vals[j], f), &h[j], &l[j]);  // zeros past K
    *reinterpret_cast<uint2 *>(hi + 4 * q) = *reinterpret_cast<const uint2 *>(h);
    *reinterpret_cast<uint2 *>(lo + 4 * q) = *reinterpret_cast<const uint2 *>(l);
  }
  if (threadIdx.x == 0 && xe) xe[row] = e;
}

// ---------------------------------------------------------------------------
// The grouped GEMV.  CTA (blockIdx.x = 32-row group of the expert's MMA
// rows, blockIdx.y = active-expert index).  Warp w takes K tiles w, w+8, ...
// Lane (g = lane/4, c = lane%4) loads, per K tile, the 16-byte pieces of rows
// g, g+8, g+16, g+24 of the group (block c of the K tile) and the 32 split-
// operand halves of elements [32c, 32c+32) of its MMA column n = g (token
// n/2, term n%2).  The MMA's 16 logical k per step are elements
// 32c + 4j + {0,1,2,3} of every c, taken identically on both sides.
// MODE 0: gate/up (rows interleaved gate d / up d), bias, SwiGLU, the
//         result as split operand of the down GEMM (actq[pos]).
// MODE 1: down, bias, fp32 result rows y[pos][H].
template <int MODE>
__global__ void __launch_bounds__(256, 2) k_gemv16(const __grid_constant__ Gemv16Launch a) {
  pdl_wait();
  pdl_trigger();
  const int ai = blockIdx.y;
  const int grp = blockIdx.x;
  const int mt = grp >> 2, q = grp & 3;
  const int row0 = mt * kMmaM + q * kRowsPerCta;  // first MMA row of the group
  if (row0 >= a.rows) return;
  // the unit's expert and token range: independent loads, one latency
  const int n_active = a.meta[0];
  const int e_raw = a.act_list[ai];  // ai < max_active <= E: in bounds, stale when ai >= n_active
  const int p0 = a.act_off[ai];
  const int p1 = a.act_off[ai + 1];
  if (ai >= n_active) return;
  const int e = e_raw;  // expert ids are local to the arena's planes (an expert-parallel shard's too)
  const int n_tok = p1 - p0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int nkt = a.ktiles > warp ? (a.ktiles - warp + kWarps - 1) / kWarps : 0;
  const int nk = min(nkt, kMaxKtPerWarp);  // the launcher refuses longer K
  __shared__ float red[kWarps][2][32][4];

  const uint8_t *wt = a.w + (((size_t)e * a.mtiles + mt) * a.ktiles) * (kMmaM * 64) +
                      (size_t)(q * kRowsPerCta + g) * 64 + c * 16;
  const uint8_t *st = a.sf + (((size_t)e * a.mtiles + mt) * a.ktiles) * 512 + (size_t)lane * 16 + q * 4;

  // epilogue operands of warps 0-1 (tile = warp), loaded ahead: the biases
  // of rows 16*tile + g and + 8
  float bias_r[2] = {0.0f, 0.0f};
  if (warp < 2) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = row0 + 16 * warp + g + 8 * h;
      if (MODE == 0) {
        const int d = min(r >> 1, a.out_rows - 1);
        const float *b = (r & 1) ? a.bias1 : a.bias0;
        bias_r[h] = b ? __ldg(b + (size_t)e * a.out_rows + d) : 0.0f;
      } else {
        bias_r[h] = (a.bias0 && r < a.out_rows) ? __ldg(a.bias0 + (size_t)e * a.out_rows + r) : 0.0f;
      }
    }
  }

  // Tokens in passes of four (the MMA's 8 columns).  Each pass streams the
  // weights again (from L2 after the first): keeping them in registers across
  // passes would spill, and decode batches rarely put more than four tokens
  // on one expert.
  for (int pass = 0; pass < n_tok; pass += kTokPerPass) {
    // this warp's K tiles: weight pieces and scale words, all in flight
    uint4 raw[kMaxKtPerWarp][4];
    uint32_t sw[kMaxKtPerWarp];
#pragma unroll
    for (int i = 0; i < kMaxKtPerWarp; ++i) {
      if (i < nk) {
        const int kt = warp + i * kWarps;
        const uint8_t *p = wt + (size_t)kt * (kMmaM * 64);
#pragma unroll
        for (int s = 0; s < 4; ++s) raw[i][s] = ldg_stream(p + s * 8 * 64);
        sw[i] = __ldg(reinterpret_cast<const uint32_t *>(st + (size_t)kt * 512));
      }
    }
    // activation fragments: column n = g -> token pass + g/2, term g%2
    const int tj = pass + (g >> 1);
    const bool live = tj < n_tok;
    int xrow = 0;  // gate/up: the token of the position; down: the position
    if (live) xrow = MODE == 0 ? __ldg(a.perm + p0 + tj) / a.top_k : p0 + tj;
    const __half *xb = a.xq + (size_t)xrow * a.xq_stride + (size_t)(g & 1) * a.kp + c * 32;
    auto load_b = [&](int i, uint4 (&bq)[4]) {
      const uint4 *src = reinterpret_cast<const uint4 *>(xb + (size_t)(warp + i * kWarps) * kMmaKT);
#pragma unroll
      for (int s = 0; s < 4; ++s) bq[s] = live ? __ldg(src + s) : make_uint4(0, 0, 0, 0);
    };
    // the exponent of this lane's epilogue token (warps 0-1: token pass + c)
    const int etok = pass + c;
    const float fexp = (MODE == 0 && a.xe && warp < 2 && etok < n_tok)
                           ? __int_as_float((127 + __ldg(a.xe + __ldg(a.perm + p0 + etok) / a.top_k)) << 23)
                           : 1.0f;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    uint4 bnext[4];
    if (nk > 0) load_b(0, bnext);
#pragma unroll
    for (int i = 0; i < kMaxKtPerWarp; ++i) {
      if (i < nk) {
        uint4 bq[4];
#pragma unroll
        for (int s = 0; s < 4; ++s) bq[s] = bnext[s];
        if (i + 1 < nk) load_b(i + 1, bnext);  // next K tile's fragments in flight meanwhile
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
          // scales of rows 16*tile + g and + 8, block c
          const uint32_t s_lo = (__shfl_sync(0xffffffffu, sw[i], 16 * tile + g) >> (8 * c)) & 0xffu;
          const uint32_t s_hi = (__shfl_sync(0xffffffffu, sw[i], 16 * tile + g + 8) >> (8 * c)) & 0xffu;
          const uint32_t m_lo = scale_h2(s_lo), m_hi = scale_h2(s_hi);
          const uint4 ra = raw[i][2 * tile], rb = raw[i][2 * tile + 1];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi) {
            // word wi of each row's piece: bytes 4wi..4wi+3 = elements 8wi..8wi+7,
            // the A operands of MMA steps j = 2wi (bytes 0, 1) and 2wi+1 (bytes 2, 3)
            uint32_t ha[4], hb[4];
            e2m1x8_h2(word_at(ra, wi), ha);
            e2m1x8_h2(word_at(rb, wi), hb);
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int j = 2 * wi + jj;
              const uint32_t a0 = hmul2(ha[2 * jj], m_lo);
              const uint32_t a1 = hmul2(hb[2 * jj], m_hi);
              const uint32_t a2 = hmul2(ha[2 * jj + 1], m_lo);
              const uint32_t a3 = hmul2(hb[2 * jj + 1], m_hi);
              const uint32_t b0 = word_at(bq[j >> 1], (j & 1) * 2);
              const uint32_t b1 = word_at(bq[j >> 1], (j & 1) * 2 + 1);
              mma16816(acc[tile], a0, a1, a2, a3, b0, b1);
            }
          }
        }
      }
    }
    // sum the warps' K parts in warp order
#pragma unroll
    for (int tile = 0; tile < 2; ++tile)
      *reinterpret_cast<float4 *>(red[warp][tile][lane]) =
          make_float4(acc[tile][0], acc[tile][1], acc[tile][2], acc[tile][3]);
    __syncthreads();
    if (warp < 2) {
      const int tile = warp;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float4 r = *reinterpret_cast<const float4 *>(red[w][tile][lane]);
        v[0] += r.x;
        v[1] += r.y;
        v[2] += r.z;
        v[3] += r.w;
      }
      // lane (g, c): rows 16*tile + g (v0 hi, v1 lo) and + 8 (v2, v3), token pass + c
      const bool tlive = etok < n_tok;
      const int pos = p0 + etok;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = row0 + 16 * tile + g + 8 * h;
        const float y = __fmul_rn(__fadd_rn(v[2 * h], v[2 * h + 1]), fexp);
        if (MODE == 0) {
          const int d = r >> 1;
          const bool is_up = (r & 1) != 0;
          const float val = __fadd_rn(y, bias_r[h]);
          const float other = __shfl_xor_sync(0xffffffffu, val, 4);  // row r ^ 1 (lane g ^ 1)
          if (!is_up && tlive && d < a.out_rows) {
            __half hh, ll;
            split_f16(swiglu_ref(val, other), &hh, &ll);
            __half *dst = a.actq + (size_t)pos * a.actq_stride;
            dst[d] = hh;
            dst[a.actq_kp + d] = ll;
          }
        } else if (tlive && r < a.out_rows) {
          a.y[(size_t)pos * a.y_stride + r] = __fadd_rn(y, bias_r[h]);
        }
      }
      // the group holding the last output column zeroes the down operand's K padding
      if (MODE == 0 && tlive && row0 + kRowsPerCta >= 2 * a.out_rows && g < 2) {
        __half *dst = a.actq + (size_t)pos * a.actq_stride;
        const __half z = __float2half_rn(0.0f);
        for (int k = a.out_rows + (tile * 2 + g); k < a.actq_kp; k += 4) {
          dst[k] = z;
          dst[a.actq_kp + k] = z;
        }
      }
    }
    __syncthreads();
  }
  // Fused combine (down GEMV): the CTA that finishes its row group last
  // combines that group's rows of every token, in k_combine's arithmetic.
  if (MODE == 1 && a.cout) {
    __shared__ int s_last;
    __threadfence();  // this CTA's y rows, before its arrival is counted
    __syncthreads();
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(a.ccount + grp, 1);
      s_last = prev == n_active - 1;
      if (s_last) a.ccount[grp] = 0;  // every arrival counted: ready for the next launch
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      for (int i = threadIdx.x; i < a.ct * kRowsPerCta; i += blockDim.x) {
        const int t = i / kRowsPerCta, r = row0 + i % kRowsPerCta;
        if (r >= a.out_rows) continue;
        float o = 0.0f;
        for (int k = 0; k < a.ck; ++k) {
          const int s = t * a.ck + k;
          const float w = a.cw[s];
          if (w <= 0.0f) continue;
          o = fmaf(__ldcg(a.y + (size_t)a.cslot[s] * a.y_stride + r), w, o);
        }
        if (a.cresid) o = __fadd_rn(a.cresid[(size_t)t * a.out_rows + r], o);
        a.cout[(size_t)t * a.out_rows + r] = o;
      }
    }
  }
}

// Smallest and largest E8M0 byte of n 17-byte GGUF blocks (byte 0 of each):
// range[0] = atomicMin, range[1] = atomicMax (initialised by the caller).
__global__ void __launch_bounds__(256) k_scale_range(const uint8_t *__restrict__ blocks, int64_t n,
                                                     int32_t *range) {
  int lo = 255, hi = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int s = blocks[i * 17];
    lo = min(lo, s);
    hi = max(hi, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&range[0], lo);
    atomicMax(&range[1], hi);
  }
}

}  // namespace

cudaError_t launch_scale_range(const uint8_t *blocks, int64_t n, int32_t *range, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  int64_t g = (n + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  k_scale_range<<<(unsigned)g, 256, 0, s>>>(blocks, n, range);
  return cudaGetLastError();
}

cudaError_t launch_split_rows(const float *src, int64_t stride, int rows, int K, int KP, const int32_t *perm,
                              int top_k, const int32_t *meta, __half *dst, int32_t *xe, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  if (KP > 4 * kSplitVec * kSplitThreads || K > KP || K % 4 != 0 || KP % 4 != 0 || stride % 4 != 0)
    return cudaErrorInvalidValue;
  return launch_pdl(k_split_rows, dim3(rows), dim3(kSplitThreads), 0, s, src, stride, K, KP, perm, top_k, meta, dst,
                    xe);
}

cudaError_t launch_gemv16(const Gemv16Launch &a, int mode, int max_active, cudaStream_t s) {
  if (max_active <= 0) return cudaSuccess;
  if ((a.ktiles + kWarps - 1) / kWarps > kMaxKtPerWarp || a.kp != a.ktiles * kMmaKT) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)(a.mtiles * (kMmaM / kRowsPerCta)), (unsigned)max_active);
  return mode == 0 ? launch_pdl(k_gemv16<0>, grid, dim3(256), 0, s, a)
                   : launch_pdl(k_gemv16<1>, grid, dim3(256), 0, s, a);
}

}  // namespace spt
