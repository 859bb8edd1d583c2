// spt_mma.cu -- tcgen05 block-scaled grouped GEMM for the MoE experts
// (layouts and numerics: spt_mma.cuh).
//
// One persistent CTA per SM, 6 warps (GemmCta):
//   warp 0  TMA producer: per stage `ks` K tiles of the weight tile (packed
//           e2m1 for kind::mxf4, or unpacked to 16-byte groups by the TMA for
//           kind::mxf8f6f4), the activation terms and their E8M0 scale atoms,
//           into a shared-memory ring guarded by mbarriers;
//   warp 1  TMEM owner and single-thread MMA issuer: per stage it copies the
//           scale atoms to TMEM (tcgen05.cp) and issues the block-scaled MMAs
//           (kind::mxf4: the terms stacked along N; kind::mxf8f6f4: one MMA
//           per term) into a double-buffered fp32 accumulator;
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (lane = output row),
//           the term sums, bias, fused SwiGLU (gate/up rows are interleaved,
//           so a row pair sits in neighbouring lanes) or the down projection,
//           fp32 stores.
// Every mbarrier wait is bounded (~2^wait_shift clocks); on timeout the CTA
// records an error code in `err`, waits for its own copies and tensor-core
// work in flight, frees its tensor memory and exits.
#include <cuda.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "spt_device.cuh"
#include "spt_mma.cuh"
#include "spt_ptx.cuh"
#include "spt_internal.cuh"
#include "spt_philox.h"
#include "spt_route.cuh"

namespace spt {

size_t mma_w_bytes(int64_t experts, int rows, int k) {
  const int kp = (k + kMmaKT - 1) / kMmaKT * kMmaKT;
  const int mtiles = (rows + kMmaM - 1) / kMmaM;
  return (size_t)experts * mtiles * (kp / kMmaKT) * kMmaM * (kMmaKT / 2);
}

size_t mma_sf_bytes(int64_t experts, int rows, int k) {
  const int kp = (k + kMmaKT - 1) / kMmaKT * kMmaKT;
  return (size_t)experts * ((rows + kMmaM - 1) / kMmaM) * (kp / kMmaKT) * 512;
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

bool mma_encode_weights(MmaMatrix *m) {
  auto fn = encode_fn();
  if (!fn || !m->w || !m->sf) return false;
  if (m->kp % 128 != 0 || ((reinterpret_cast<uintptr_t>(m->w) | reinterpret_cast<uintptr_t>(m->sf)) & 31) != 0)
    return false;
  // Tile-major: every 128-row x 128-element box is one contiguous 8 KB block,
  // so the map is [rows = boxes * 128][128 elements] with a 64-byte pitch.
  const uint64_t boxes = (uint64_t)m->experts * m->mtiles * (m->kp / kMmaKT);
  cuuint64_t dims[2] = {(cuuint64_t)kMmaKT, (cuuint64_t)(boxes * kMmaM)};
  cuuint64_t strides[1] = {(cuuint64_t)(kMmaKT / 2)};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m->tmap, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 2, m->w, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  // Packed view for kind::mxf4: [boxes][128 rows][64 B], the 64-byte rows
  // land in shared memory as they are (SW64).
  cuuint64_t dims3[3] = {(cuuint64_t)(kMmaKT / 2), (cuuint64_t)kMmaM, (cuuint64_t)boxes};
  cuuint64_t strides3[2] = {(cuuint64_t)(kMmaKT / 2), (cuuint64_t)(kMmaKT / 2) * kMmaM};
  cuuint32_t estr3[3] = {1, 1, 1};
  for (int which = 0; which < 3; ++which) {
    const cuuint32_t nbox = which == 0 ? kMmaStageTilesFp4 : which == 1 ? 1u : (cuuint32_t)kMmaStageTilesWide;
    cuuint32_t box3[3] = {(cuuint32_t)(kMmaKT / 2), (cuuint32_t)kMmaM, nbox};
    CUtensorMap *map = which == 0 ? &m->tmap_p : which == 1 ? &m->tmap_p1 : &m->tmap_pw;
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, m->w, dims3, strides3, box3, estr3,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
  }
  // Row-tile groups for 128-token tiles: the same bytes as [row tiles][K
  // tiles][128 rows][64 B]; a box takes one K tile of kPrefillRowTiles row
  // tiles (past the last row tile of the matrix the copy fills zeros).
  const cuuint64_t kt_n = (cuuint64_t)(m->kp / kMmaKT), runs = (cuuint64_t)m->experts * m->mtiles;
  cuuint64_t dims4[4] = {(cuuint64_t)kMmaKT, (cuuint64_t)kMmaM, kt_n, runs};
  cuuint64_t strides4[3] = {(cuuint64_t)(kMmaKT / 2), (cuuint64_t)(kMmaKT / 2) * kMmaM,
                            kt_n * (kMmaKT / 2) * kMmaM};
  cuuint32_t box4[4] = {128, 128, 1, (cuuint32_t)kPrefillRowTiles};
  cuuint32_t estr4[4] = {1, 1, 1, 1};
  r = fn(&m->tmap_g, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 4, m->w, dims4, strides4, box4, estr4,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  // the same groups packed (kind::mxf4): 64-byte rows as they are (SW64)
  cuuint64_t dims4p[4] = {(cuuint64_t)(kMmaKT / 2), (cuuint64_t)kMmaM, kt_n, runs};
  cuuint32_t box4p[4] = {(cuuint32_t)(kMmaKT / 2), 128, 1, (cuuint32_t)kPrefillRowTiles};
  r = fn(&m->tmap_gp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, m->w, dims4p, strides4, box4p, estr4,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  cuuint64_t sdims[3] = {128, kt_n, runs};  // 32-bit words: an atom is 128 of them
  cuuint64_t sstrides[2] = {512, kt_n * 512};
  cuuint32_t sbox[3] = {128, 1, (cuuint32_t)kPrefillRowTiles};
  r = fn(&m->tmap_sfg, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, m->sf, sdims, sstrides, sbox, estr4,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool mma_encode_acts(CUtensorMap *map, uint8_t *q, int kp, int rb, int bn, ActFmt f, int ktiles) {
  auto fn = encode_fn();
  const int box_rows = mma_box_rows(f, bn);
  if (!fn || !q || box_rows < 1 || box_rows > 256 || ktiles < 1) return false;
  const cuuint64_t kt_n = (cuuint64_t)(kp / kMmaKT);
  CUresult r;
  if (f == ActFmt::kFp4Planes) {
    cuuint64_t dims[4] = {kMmaKT / 2, (cuuint64_t)rb, (cuuint64_t)kFp4Terms, kt_n};
    cuuint64_t strides[3] = {kMmaKT / 2, (cuuint64_t)rb * (kMmaKT / 2), (cuuint64_t)rb * (kMmaKT / 2) * kFp4Terms};
    cuuint32_t box[4] = {kMmaKT / 2, (cuuint32_t)box_rows, (cuuint32_t)kFp4Terms, (cuuint32_t)ktiles};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, q, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (f == ActFmt::kFp4Stack) {
    cuuint64_t dims[3] = {kMmaKT / 2, (cuuint64_t)rb, kt_n};
    cuuint64_t strides[2] = {kMmaKT / 2, (cuuint64_t)rb * (kMmaKT / 2)};
    cuuint32_t box[3] = {kMmaKT / 2, (cuuint32_t)box_rows, (cuuint32_t)ktiles};
    cuuint32_t estr[3] = {1, 1, 1};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, q, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[4] = {kMmaKT, (cuuint64_t)rb, (cuuint64_t)kActTerms, kt_n};
    cuuint64_t strides[3] = {kMmaKT, (cuuint64_t)rb * kMmaKT, (cuuint64_t)rb * kMmaKT * kActTerms};
    cuuint32_t box[4] = {kMmaKT, (cuuint32_t)box_rows, (cuuint32_t)kActTerms, (cuuint32_t)ktiles};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, q, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS;
}

namespace {

// ---------------------------------------------------------------------------
// MMA arena repack: GGUF 17-byte blocks -> packed e2m1 rows + scale atoms.

// Write block b (32 elements, GGUF order: byte 1+i = element i | element
// i+16 << 4) of MMA row `row` of expert e.
__device__ __forceinline__ void put_mma_block(const uint8_t blk[17], int64_t e, int row, int b,
                                              int rows, int kp, uint8_t *w, uint8_t *sf) {
  const int mtiles_ = (rows + kMmaM - 1) / kMmaM, ktiles_ = kp / kMmaKT;
  const size_t box = ((size_t)e * mtiles_ + row / kMmaM) * ktiles_ + (size_t)(b / 4);
  uint8_t *dst = w + (box * kMmaM + (size_t)(row % kMmaM)) * (kMmaKT / 2) + (size_t)(b % 4) * 16;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int e0 = 2 * i, e1 = 2 * i + 1;  // natural order: element 2i low nibble
    const uint32_t n0 = e0 < 16 ? (blk[1 + e0] & 15u) : (uint32_t)(blk[1 + e0 - 16] >> 4);
    const uint32_t n1 = e1 < 16 ? (blk[1 + e1] & 15u) : (uint32_t)(blk[1 + e1 - 16] >> 4);
    dst[i] = (uint8_t)(n0 | (n1 << 4));
  }
  const int mtiles = (rows + kMmaM - 1) / kMmaM, ktiles = kp / kMmaKT;
  const int mt = row / kMmaM, m = row % kMmaM, kt = b / 4, kb = b % 4;
  sf[(((size_t)e * mtiles + mt) * ktiles + kt) * 512 + (m % 32) * 16 + (m / 32) * 4 + kb] = blk[0];
}

// gate/up: MMA row 2d = gate row d, 2d+1 = up row d.
__global__ void k_repack_mma_gu(const uint8_t *__restrict__ gate, const uint8_t *__restrict__ up,
                                int64_t E, int D, int NB, int kp, uint8_t *w, uint8_t *sf) {
  const int64_t total = E * D * NB;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx % NB);
    const int64_t ed = idx / NB;
    const int d = (int)(ed % D);
    const int64_t e = ed / D;
    uint8_t blk[17];
#pragma unroll
    for (int k = 0; k < 17; ++k) blk[k] = gate[idx * 17 + k];
    put_mma_block(blk, e, 2 * d, b, 2 * D, kp, w, sf);
#pragma unroll
    for (int k = 0; k < 17; ++k) blk[k] = up[idx * 17 + k];
    put_mma_block(blk, e, 2 * d + 1, b, 2 * D, kp, w, sf);
  }
}

__global__ void k_repack_mma(const uint8_t *__restrict__ src, int64_t E, int R, int NB, int kp,
                             uint8_t *w, uint8_t *sf) {
  const int64_t total = E * R * NB;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx % NB);
    const int64_t er = idx / NB;
    const int r = (int)(er % R);
    const int64_t e = er / R;
    uint8_t blk[17];
#pragma unroll
    for (int k = 0; k < 17; ++k) blk[k] = src[idx * 17 + k];
    put_mma_block(blk, e, r, b, R, kp, w, sf);
  }
}

__global__ void k_synth_mma_gu(uint64_t seed, uint32_t tg, uint32_t tu, int64_t E, int D, int NB,
                               uint8_t lo, uint8_t hi, uint64_t counter0, int kp, uint8_t *w, uint8_t *sf) {
  const int64_t total = E * D * NB;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx % NB);
    const int64_t ed = idx / NB;
    const int d = (int)(ed % D);
    const int64_t e = ed / D;
    uint8_t blk[17];
    synth_mxfp4_block(seed, tg, counter0 + (uint64_t)idx, lo, hi, blk);
    put_mma_block(blk, e, 2 * d, b, 2 * D, kp, w, sf);
    synth_mxfp4_block(seed, tu, counter0 + (uint64_t)idx, lo, hi, blk);
    put_mma_block(blk, e, 2 * d + 1, b, 2 * D, kp, w, sf);
  }
}

__global__ void k_synth_mma(uint64_t seed, uint32_t tag, int64_t E, int R, int NB, uint8_t lo,
                            uint8_t hi, uint64_t counter0, int kp, uint8_t *w, uint8_t *sf) {
  const int64_t total = E * R * NB;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(idx % NB);
    const int64_t er = idx / NB;
    const int r = (int)(er % R);
    const int64_t e = er / R;
    uint8_t blk[17];
    synth_mxfp4_block(seed, tag, counter0 + (uint64_t)idx, lo, hi, blk);
    put_mma_block(blk, e, r, b, R, kp, w, sf);
  }
}

unsigned grid_of(int64_t n) {
  int64_t g = (n + 255) / 256;
  if (g > 148 * 32) g = 148 * 32;
  return (unsigned)(g < 1 ? 1 : g);
}

// ---------------------------------------------------------------------------
// Activations -> block-scaled multi-term operands.  Each 32-element block is
// written as a sum of terms q_t * 2^e_t, each term quantizing the residual
// left by the previous ones; every residual is exact in fp32.  Term scale:
// the smallest power of two 2^e with max|residual| / 2^e <= the format's
// largest finite value, so no element saturates.
//   FP4 (token tiles of <= 16): kFp4Terms e2m1 terms, stacked along N
//     (term t, token j at slot row t*bn + j%bn); q [KP/128][RB][64 B].
//   FP8 (128-token tiles): kActTerms e4m3 terms, each in its own plane of RB
//     rows; q [KP/128][kActTerms][RB][128 B].
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

// Smallest e with amax / 2^e <= qmax, clamped to the E8M0 range the scale
// atoms hold (-126 for amax 0, subnormal or NaN, 120 for Inf).  qmax =
// qm * 2^QE with qm = 1 + QF/2^23 (e2m1: 6 = 1.5 * 2^2; e4m3: 448 = 1.75 *
// 2^8): for amax = 1.f * 2^E the answer is E - QE, plus one when 1.f > qm.
template <int QE, uint32_t QF>
__device__ __forceinline__ int term_exponent(float amax) {
  if (!(amax > 0.0f)) return -126;
  const uint32_t bits = __float_as_uint(amax);
  const int E = (int)(bits >> 23) - 127;
  if (E == 128) return 120;
  const int ex = E - QE + ((bits & 0x7fffffu) > QF ? 1 : 0);
  return max(-126, min(ex, 120));
}

// Two floats -> one byte of two e2m1 codes (lo in the low nibble), round to
// nearest, saturating at 6.
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t out;
  asm("{\n\t.reg .b8 b;\n\tcvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\tcvt.u32.u8 %0, b;\n\t}"
      : "=r"(out)
      : "f"(hi), "f"(lo));
  return out;
}

// The terms of elements kt*128 + (lane/8)*32 + (lane%8)*4 + [0, 4) of one row
// (values v): per term the four codes (FP4: two bytes, FP8: four) and the
// block's E8M0 exponent (shared by the 8 lanes of the block).
template <bool FP4>
struct Terms {
  static constexpr int kN = FP4 ? kFp4Terms : kActTerms;
  uint32_t code[kN];
  int ex[kN];
};

// Byte of two e2m1 codes -> their values (lo: low nibble) as two floats.
__device__ __forceinline__ float2 e2m1x2_values(uint32_t byte) {
  uint32_t h2;
  asm("{\n\t.reg .b8 b;\n\tcvt.u8.u32 b, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b;\n\t}" : "=r"(h2) : "r"(byte));
  return __half22float2(*reinterpret_cast<const __half2 *>(&h2));
}

// The terms of N independent (row, K tile) items at once: term t of every
// item before term t + 1 of any, so the items' shuffle and conversion chains
// overlap.
template <bool FP4, int N>
__device__ __forceinline__ void quantize_term(float4 (&v)[N], Terms<FP4> (&r)[N], int t) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float amax = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
#pragma unroll
      for (int off = 4; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const int ex = FP4 ? term_exponent<2, 0x400000u>(amax) : term_exponent<8, 0x600000u>(amax);
      const float inv = exp2i(-ex), sc = exp2i(ex);
      float vv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      if constexpr (FP4) {
        const uint32_t c01 = e2m1x2(__fmul_rn(vv[0], inv), __fmul_rn(vv[1], inv));
        const uint32_t c23 = e2m1x2(__fmul_rn(vv[2], inv), __fmul_rn(vv[3], inv));
        // the residuals v - q * 2^ex are exact in fp32: one rounding-free FMA each
        const float2 q01 = e2m1x2_values(c01), q23 = e2m1x2_values(c23);
        vv[0] = __fmaf_rn(-q01.x, sc, vv[0]);
        vv[1] = __fmaf_rn(-q01.y, sc, vv[1]);
        vv[2] = __fmaf_rn(-q23.x, sc, vv[2]);
        vv[3] = __fmaf_rn(-q23.y, sc, vv[3]);
        r[i].code[t] = c01 | (c23 << 8);
      } else {
        uint32_t packed = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const __nv_fp8_storage_t code = __nv_cvt_float_to_fp8(__fmul_rn(vv[k], inv), __NV_SATFINITE, __NV_E4M3);
          const __half_raw hr = __nv_cvt_fp8_to_halfraw(code, __NV_E4M3);
          vv[k] = __fsub_rn(vv[k], __fmul_rn(__half2float(__half(hr)), sc));
          packed |= (uint32_t)code << (8 * k);
        }
        r[i].code[t] = packed;
      }
      r[i].ex[t] = ex;
      v[i] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    }
}

template <bool FP4, int N>
__device__ __forceinline__ void quantize_terms_n(float4 (&v)[N], Terms<FP4> (&r)[N]) {
  if constexpr (N > 1) {
    // large batches: every term unrolled (the terms stay in registers)
#pragma unroll
    for (int t = 0; t < Terms<FP4>::kN; ++t) quantize_term<FP4, N>(v, r, t);
  } else {
    // decode sizes: one copy of the body, the code a cold instruction cache
    // fetches
#pragma unroll 1
    for (int t = 0; t < Terms<FP4>::kN; ++t) quantize_term<FP4, N>(v, r, t);
  }
}

// Store the terms of one (dispatch row, 128-element K tile): row j of its
// token tile, whose 128-row activation slot starts at `slot`; 8 lanes per
// 32-element block, 4 elements per lane (the layouts of spt_mma.cuh: FP4
// terms stacked along the slot for bn <= 16, else one plane per term).
template <bool FP4>
__device__ __forceinline__ void store_terms(const Terms<FP4> &r, int kt, int kt_n, int j, int slot, int bn, int rb,
                                            uint8_t *__restrict__ q, uint8_t *__restrict__ sf, int lane) {
  const int sub = lane & 7;
  const int b = kt * 4 + (lane >> 3);
  const int64_t atom = (int64_t)(slot / kMmaM) * kt_n + kt;
  const bool stacked = FP4 && bn <= 16;
#pragma unroll
  for (int t = 0; t < Terms<FP4>::kN; ++t) {
    const int m = stacked ? t * bn + (j % bn) : (j % bn);  // row within the slot
    if constexpr (FP4) {
      const int64_t row = stacked ? (int64_t)kt * rb + slot + m : ((int64_t)kt * kFp4Terms + t) * rb + slot + m;
      *reinterpret_cast<uint16_t *>(q + row * (kMmaKT / 2) + (b % 4) * 16 + sub * 2) = (uint16_t)r.code[t];
    } else {
      const int64_t row = ((int64_t)kt * kActTerms + t) * rb + slot + m;
      *reinterpret_cast<uint32_t *>(q + row * kMmaKT + (b % 4) * 32 + sub * 4) = r.code[t];
    }
    if (sub == 0) {
      const int64_t a2 = stacked ? atom : atom * Terms<FP4>::kN + t;
      sf[a2 * 512 + (m % 32) * 16 + (m / 32) * 4 + (b % 4)] = (uint8_t)(r.ex[t] + 127);
    }
  }
}

constexpr int kQuantKt = 4;  // K tiles per warp for large batches

// The tokens' rows, each quantized once and stored at every dispatch
// position of the token (top_k slots, each in its expert's token tile): one
// warp per (token, group of KTW 128-element K tiles).
template <bool FP4, int KTW>
__global__ void k_quantize_tokens(const float *__restrict__ x, int64_t stride, int T, int top_k,
                                  const int32_t *__restrict__ slot_pos, const int32_t *__restrict__ offsets,
                                  const int32_t *__restrict__ pad_off, const int32_t *__restrict__ pos_expert,
                                  int K, int kp, int rb, int bn, uint8_t *__restrict__ q, uint8_t *__restrict__ sf) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int kt_n = kp / kMmaKT, groups = (kt_n + KTW - 1) / KTW;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int t = (int)(gw / groups), kt0 = (int)(gw - (int64_t)t * groups) * KTW;
  if (t >= T) return;
  float4 v[KTW];
  Terms<FP4> r[KTW];
#pragma unroll
  for (int i = 0; i < KTW; ++i) {
    const int b = (kt0 + i) * 4 + (lane >> 3);
    v[i] = (kt0 + i < kt_n && b * 32 < K)
               ? *reinterpret_cast<const float4 *>(x + (int64_t)t * stride + b * 32 + (lane & 7) * 4)
               : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  quantize_terms_n<FP4, KTW>(v, r);
  for (int k = 0; k < top_k; ++k) {
    const int pos = slot_pos[(int64_t)t * top_k + k];
    if (pos < 0) continue;
    const int e = pos_expert[pos];
    const int j = pos - offsets[e];
#pragma unroll
    for (int i = 0; i < KTW; ++i)
      if (kt0 + i < kt_n) store_terms<FP4>(r[i], kt0 + i, kt_n, j, pad_off[e] + (j / bn) * kMmaM, bn, rb, q, sf, lane);
  }
}

template <bool FP4, int KTW>
__global__ void k_quantize_act(const float *__restrict__ src, int64_t stride,
                               const int32_t *__restrict__ perm, int top_k, int gather,
                               const int32_t *__restrict__ offsets, const int32_t *__restrict__ pad_off,
                               const int32_t *__restrict__ pos_expert, const int32_t *__restrict__ meta,
                               int S_max, int K, int kp, int rb, int bn,
                               uint8_t *__restrict__ q, uint8_t *__restrict__ sf) {
  pdl_wait();
  pdl_trigger();
  // One warp per (dispatch position, group of KTW K tiles): the group's loads
  // are all in flight, and its term chains interleaved.
  const int lane = threadIdx.x & 31;
  const int kt_n = kp / kMmaKT, groups = (kt_n + KTW - 1) / KTW;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int pos = (int)(gw / groups), kt0 = (int)(gw - (int64_t)pos * groups) * KTW;
  if (pos >= S_max || pos >= meta[1]) return;
  const int e = pos_expert[pos];
  const int j = pos - offsets[e];
  const int slot = pad_off[e] + (j / bn) * kMmaM;  // this token tile's 128-row slot
  const int64_t srow = gather ? (int64_t)(perm[pos] / top_k) : (int64_t)pos;
  const float *row = src + srow * stride;
  float4 v[KTW];
  Terms<FP4> r[KTW];
#pragma unroll
  for (int i = 0; i < KTW; ++i) {
    const int b = (kt0 + i) * 4 + (lane >> 3);
    v[i] = (kt0 + i < kt_n && b * 32 < K) ? __ldcs(reinterpret_cast<const float4 *>(row + b * 32 + (lane & 7) * 4))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  quantize_terms_n<FP4, KTW>(v, r);
#pragma unroll
  for (int i = 0; i < KTW; ++i)
    if (kt0 + i < kt_n) store_terms<FP4>(r[i], kt0 + i, kt_n, j, slot, bn, rb, q, sf, lane);
}

// ---------------------------------------------------------------------------
// GEMM-specific PTX helpers (sm_100a); the generic ones are in spt_ptx.cuh.

__device__ __forceinline__ void tma_load_2d(const CUtensorMap *map, void *dst, uint64_t *bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap *map, void *dst, uint64_t *bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(const CUtensorMap *map, void *dst, uint64_t *bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}


__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// K-major shared-memory matrix descriptor (tcgen05): start address, leading
// byte offset (unused with swizzling), stride byte offset between 8-row
// groups, descriptor version 1, layout type (2 = 128-byte swizzle, 0 = none).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                                 // LBO (16 B)
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;       // SBO
  d |= (uint64_t)1u << 46;                                 // version
  d |= (uint64_t)(layout & 7u) << 61;                      // layout type
  return d;
}

// Block-scaled instruction descriptor: A = E2M1, B = E4M3, scales E8M0,
// K-major A and B, M = 128, N = n, scale-factor byte ids.
__device__ __forceinline__ uint32_t idesc_mxf8f6f4(int n, uint32_t sfa_id, uint32_t sfb_id) {
  uint32_t d = 0;
  d |= (sfb_id & 3u) << 4;
  d |= 5u << 7;                      // a_format E2M1
  d |= 0u << 10;                     // b_format E4M3
  d |= (uint32_t)(n >> 3) << 17;     // N
  d |= 1u << 23;                     // scale format E8M0
  d |= (uint32_t)(kMmaM >> 4) << 24; // M
  d |= (sfa_id & 3u) << 29;
  return d;
}

// kind::mxf4: A and B e2m1 (format 1), E8M0 scales, K = 64 per MMA.
__device__ __forceinline__ uint32_t idesc_mxf4(int n, uint32_t sfa_id, uint32_t sfb_id) {
  uint32_t d = 0;
  d |= (sfb_id & 3u) << 4;
  d |= 1u << 7;                      // a_format E2M1
  d |= 1u << 10;                     // b_format E2M1
  d |= (uint32_t)(n >> 3) << 17;     // N
  d |= 1u << 23;                     // scale format E8M0
  d |= (uint32_t)(kMmaM >> 4) << 24; // M
  d |= (sfa_id & 3u) << 29;
  return d;                          // bit 31 = 0: K = 64
}
__device__ __forceinline__ void tc_mma_fp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc_ld8(uint32_t taddr, float v[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float v[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 columns of this warp's 32 TMEM lanes in one load (and its wait).
__device__ __forceinline__ void tc_ld64(uint32_t taddr, float v[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float v[16]);
// Columns [taddr, taddr + C) of this warp's 32 TMEM lanes, C = 8 or 16.
template <int C>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float *v) {
  static_assert(C == 8 || C == 16, "TMEM load width");
  if constexpr (C == 8) tc_ld8(taddr, v);
  else tc_ld16(taddr, v);
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

struct TileInfo {
  int e, mt, p0, nvalid, rowb;
};

constexpr int kMaxActive = 256;  // active experts per launch (the dispatch kernel's limit)

// Per-launch tile tables, copied to shared memory once per CTA so that the
// producer, MMA and epilogue roles decode tiles without global loads.
struct TileTables {
  int tile_off[kMaxActive + 1];  // first tile of each active expert
  int e[kMaxActive];             // expert id
  int p0[kMaxActive];            // first dispatch position
  int n[kMaxActive];             // tokens
  int pad[kMaxActive];           // first 128-row activation slot
};

template <int BN>
__device__ __forceinline__ TileInfo tile_info(const TileTables &tt, int tile, int n_active, int mtiles) {
  int lo = 0, hi = n_active - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (tt.tile_off[mid] <= tile) lo = mid;
    else hi = mid - 1;
  }
  TileInfo t;
  t.e = tt.e[lo];
  const int local = tile - tt.tile_off[lo];
  const int n_e = tt.n[lo];
  const int ntn = (n_e + BN - 1) / BN;
  t.mt = local / ntn;
  const int nt = local - t.mt * ntn;
  t.p0 = tt.p0[lo] + nt * BN;
  t.nvalid = min(BN, n_e - nt * BN);
  t.rowb = tt.pad[lo] + nt * kMmaM;
  (void)mtiles;
  return t;
}

// FP4: kind::mxf4, packed weights (SW64), kFp4Terms e2m1 activation terms:
// for BN <= 16 stacked along N (N = kFp4Terms*BN, one scale atom per K tile,
// the term partial sums added in the epilogue), for 128-token tiles one
// N = BN operand and atom per term, all into one accumulator; two K = 64
// MMAs (per term) per K tile.  FP8: kind::mxf8f6f4, weights unpacked by the
// TMA (SW128), kActTerms e4m3 terms each its own N = BN operand with its own
// atom (four K = 32 MMAs per term per K tile).  KS: K tiles per pipeline
// stage.  MG row tiles share each activation K tile (128-token tiles:
// kPrefillRowTiles; their MG accumulators are single-buffered), else one row
// tile per unit with a double-buffered accumulator.
template <int BN, bool FP4, int KS, int MG = 1>
struct MmaShape {
  static constexpr bool kStacked = FP4 && BN <= 16;              // FP4 terms stacked along N
  static constexpr int kA = FP4 ? kMmaM * 64 : kMmaM * 128;     // smem bytes of one weight K tile
  static constexpr int kATx = kMmaM * 64;                        // its transaction bytes (packed source)
  static constexpr int kBTerm = FP4 ? BN * 64 : BN * 128;        // smem bytes of one term's K tile
  static constexpr int kTerms = FP4 ? kFp4Terms : kActTerms;
  static constexpr int kBt = kTerms * kBTerm;                    // all terms of one K tile
  static constexpr int kSfb = kStacked ? 1 : kTerms;             // activation scale atoms per K tile
  static constexpr int kN = kStacked ? kFp4Terms * BN : BN;      // MMA N
  static constexpr int kKSteps = FP4 ? 2 : 4;                    // MMAs (per term) per K tile
  static constexpr uint32_t kLayout = FP4 ? 4u : 2u;             // smem descriptor: SW64 / SW128
  static constexpr uint32_t kSbo = FP4 ? 512u : 1024u;           // 8-row swizzle atom
  // stage: A[KS][MG] | B[KS] | SFA[MG][KS] | SFB[KS][kSfb]
  static constexpr int kOffB = KS * MG * kA;
  static constexpr int kOffSfa = kOffB + KS * kBt;
  static constexpr int kOffSfb = kOffSfa + KS * MG * 512;
  static constexpr int kStage = ((kOffSfb + KS * kSfb * 512) + 1023) / 1024 * 1024;
  static constexpr int kStages = (200 * 1024) / kStage > 16 ? 16 : (200 * 1024) / kStage;
  static constexpr int kAccStride = (kN + 31) / 32 * 32;  // TMEM columns of one accumulator
  static constexpr int kAccBufs = MG > 1 ? 1 : 2;         // accumulator sets (double-buffered with one row tile)
  static constexpr int kAccCols = kAccBufs * MG * kAccStride;
  static constexpr int kSfCols = KS * (4 * MG + 4 * kSfb);  // SFA + SFB atoms of every K tile of a stage
  static constexpr int kCols = (kAccCols + kSfCols <= 32) ? 32
                               : (kAccCols + kSfCols <= 64) ? 64
                               : (kAccCols + kSfCols <= 128) ? 128
                               : (kAccCols + kSfCols <= 256) ? 256 : 512;
  // transaction bytes of one K tile of a unit with nm row tiles
  static __device__ __forceinline__ int tx_ktile(int nm) { return nm * (kATx + 512) + kBt + kSfb * 512; }
  static constexpr int kRing = kStages * kStage;
  static constexpr int kSmem = kRing + 1024 /*align*/ + 256 /*barriers*/ + (int)sizeof(TileTables);
  static_assert(kBTerm % 512 == 0 && kA % 1024 == 0, "swizzle atoms must stay aligned");
  static_assert(kAccCols + kSfCols <= 512, "TMEM columns");
  static_assert(kStages >= 2, "stage ring");
  static_assert(MG == 1 || (KS == 1 && BN == 128), "row-tile groups: one K tile per stage, 128-token tiles");
  // epilogue warps: with row-tile groups, whose single-buffered accumulators
  // make the next unit's MMAs wait for the epilogue, four per TMEM lane
  // quadrant (each takes a quarter of the columns); one per quadrant otherwise
  static constexpr int kEpiWarps = MG > 1 ? 16 : 4;
  static constexpr int kThreads = 32 * (2 + kEpiWarps);
  static_assert(kSmem <= 227 * 1024, "shared memory");
};

// One GEMM CTA: the shared-memory stage ring, its mbarriers, the TMEM
// accumulators, and the three roles.  Each role runs in its own thread(s)
// and keeps its ring slot, parity and tile count in that thread's copy of
// this struct.
template <int BN, bool FP4, int KS, int MG = 1>
struct GemmCta {
  using S = MmaShape<BN, FP4, KS, MG>;
  static constexpr int kBarBytes = 256;
  static_assert((2 * S::kStages + 5) * 8 + 4 <= kBarBytes, "mbarrier area");
  uint8_t *smem;  // 1024-byte aligned ring
  uint64_t *full, *empty, *accf, *acce, *drain;
  uint32_t *tmem_slot;
  uint32_t tmem = 0;
  int s = 0;           // ring slot (producer, MMA issuer)
  uint32_t phase = 0;  // ring parity (producer, MMA issuer)
  int local = 0;       // tiles handled by this CTA so far (MMA issuer, epilogue)

  __device__ explicit GemmCta(uint8_t *ring) : smem(ring) {
    full = reinterpret_cast<uint64_t *>(smem + S::kStages * S::kStage);
    empty = full + S::kStages;
    accf = empty + S::kStages;
    acce = accf + 2;
    drain = acce + 2;
    tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  }

  // thread 0
  __device__ void init_barriers() {
    for (int i = 0; i < S::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 32 * S::kEpiWarps);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // one whole warp
  __device__ void alloc_tmem() {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)S::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __device__ void dealloc_tmem() {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)S::kCols)
                 : "memory");
  }

  // ---------------- TMA producer (one thread) ----------------
  // Tile-major storage makes the kt_n weight boxes (and scale atoms) of one
  // (expert, row tile) a single contiguous run, so one bulk L2 prefetch per
  // tile, issued a.prefetch tiles ahead, can have the next tiles' weights on
  // their way from HBM while the ring streams the current one.
  // On an error (a wait that ran out, here or in another role) the producer
  // stops issuing and waits for the copies it already started, so that none
  // lands in shared memory after the CTA has gone.  a.fault_stage >= 0 (a
  // test of that path) makes CTA 0 skip the whole of that stage: the MMA
  // issuer's wait for it runs out.
  __device__ bool produce(const MmaLaunch &a, const TileTables &tt, int n_active, int n_tiles) {
    const int kt_n = a.ktiles;
    const uint32_t w_tile_bytes = (uint32_t)kt_n * kMmaM * (kMmaKT / 2);
    auto prefetch_tile = [&](int tile) {
      if (tile >= n_tiles) return;
      const TileInfo ti = tile_info<BN>(tt, tile, n_active, a.mtiles);
      const size_t run = (size_t)ti.e * a.mtiles + ti.mt;
      bulk_prefetch_l2(a.w + run * w_tile_bytes, w_tile_bytes);
      bulk_prefetch_l2(a.sfa + run * kt_n * 512, (uint32_t)kt_n * 512);
    };
    uint32_t issued = 0;  // bit i: ring slot i holds a stage whose copies may still be in flight
    uint32_t slot_phase = 0;  // bit i: the parity of that stage
    int stage = 0;
    bool ok = true;
    const int pf = MG == 1 ? a.prefetch : 0;  // whole-tile prefetch: one row tile per unit only
    for (int d = 1; d < pf; ++d) prefetch_tile(blockIdx.x + d * gridDim.x);
    for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
      const TileInfo t = tile_info<BN>(tt, tile, n_active, a.mtiles);
      const int mt0 = t.mt * MG;                    // first row tile of the unit
      const int nm = min(MG, a.mtiles - mt0);       // its row tiles
      const uint8_t *sfa = a.sfa + (((size_t)t.e * a.mtiles + mt0) * a.ktiles) * 512;
      const uint8_t *sfb = a.sfb + ((size_t)(t.rowb / kMmaM) * a.ktiles) * (S::kSfb * 512);
      const int box0 = (t.e * a.mtiles + mt0) * kt_n;
      if (pf > 0) prefetch_tile(tile + pf * gridDim.x);
      for (int kt = 0; kt < kt_n; kt += KS, ++stage) {
        if (!mbar_wait(&empty[s], phase ^ 1u, a.err, 1, a.wait_shift)) {
          ok = false;
          break;
        }
        const int nk = min(KS, kt_n - kt);
        if (!(a.fault_stage == stage && blockIdx.x == 0)) {
          uint8_t *st = smem + s * S::kStage;
          // a group short of MG row tiles still copies MG (the extra ones,
          // zeros or the next expert's rows, are never multiplied)
          mbar_expect_tx(&full[s], MG > 1 ? S::tx_ktile(MG) : nk * S::tx_ktile(nm));
          // one operation per operand for the whole stage; single K tiles with
          // the one-box maps at the end of an odd K
          const bool whole = nk == KS;
          const CUtensorMap *ma = whole ? &a.tmap_a : &a.tmap_a1;
          const CUtensorMap *mb = whole ? &a.tmap_b : &a.tmap_b1;
          if constexpr (MG > 1) {
            // one K tile (KS == 1) of MG row tiles and their scale atoms in
            // one copy each
            tma_load_4d(&a.tmap_a, st, &full[s], 0, 0, kt, t.e * a.mtiles + mt0);
            tma_load_4d(mb, st + S::kOffB, &full[s], 0, t.rowb, 0, kt);
            tma_load_3d(&a.tmap_sfa, st + S::kOffSfa, &full[s], 0, kt, t.e * a.mtiles + mt0);
          } else {
            for (int j = 0; j < (whole ? 1 : nk); ++j) {
              uint8_t *aj = st + j * S::kA;
              uint8_t *bj = st + S::kOffB + j * S::kBt;
              if (FP4) {
                tma_load_3d(ma, aj, &full[s], 0, 0, box0 + kt + j);
                tma_load_3d(mb, bj, &full[s], 0, t.rowb, kt + j);
              } else {
                tma_load_2d(ma, aj, &full[s], 0, (box0 + kt + j) * kMmaM);
                tma_load_4d(mb, bj, &full[s], 0, t.rowb, 0, kt + j);
              }
            }
            bulk_load(st + S::kOffSfa, sfa + (size_t)kt * 512, nk * 512, &full[s]);
          }
          bulk_load(st + S::kOffSfb, sfb + (size_t)kt * S::kSfb * 512, nk * S::kSfb * 512, &full[s]);
          issued |= 1u << s;
          slot_phase = (slot_phase & ~(1u << s)) | (phase << s);
        } else {
          issued &= ~(1u << s);  // nothing of this stage is in flight
        }
        if (++s == S::kStages) {
          s = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok) {
      // the last stage issued into each slot is the only one that can still
      // be in flight there (an earlier one was consumed before the slot was
      // reused); its full barrier completes when its bytes have landed
      for (int i = 0; i < S::kStages; ++i)
        if ((issued >> i) & 1u) mbar_wait_own(&full[i], (slot_phase >> i) & 1u, a.wait_shift);
    }
    return ok;
  }

  // ---------------- MMA issuer (one thread) ----------------
  // Descriptors are built once; per stage and K-step only their 14-bit start
  // address fields advance (stage bases are 1024-byte aligned and the whole
  // ring lies below 256 KB, so the adds never carry out of the field).
  __device__ bool mma(const MmaLaunch &a, const TileTables &tt, int n_active, int n_tiles) {
    const uint32_t sfa_t = tmem + S::kAccCols;  // scale-factor columns after the accumulators
    const uint32_t base = smem_u32(smem);
    const uint64_t a_desc0 = smem_desc(base, S::kSbo, S::kLayout);
    const uint64_t b_desc0 = smem_desc(base + S::kOffB, S::kSbo, S::kLayout);
    const uint64_t sfa_desc0 = smem_desc(base + S::kOffSfa, 128, 0);
    const uint64_t sfb_desc0 = smem_desc(base + S::kOffSfb, 128, 0);
    constexpr uint64_t kStage16 = S::kStage >> 4, kA16 = S::kA >> 4, kBt16 = S::kBt >> 4, kBTerm16 = S::kBTerm >> 4;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++local) {
      const int kt_lo = 0, kt_hi = a.ktiles;
      const TileInfo ti = tile_info<BN>(tt, tile, n_active, a.mtiles);
      const int nm = MG == 1 ? 1 : min(MG, a.mtiles - ti.mt * MG);
      // K step ks reads 32 bytes further along each row; FP4 steps use scale
      // bytes 2ks and 2ks+1 of the atom (two 32-blocks), FP8 steps byte ks.
      // With one operand per term the MMAs cover only the unit's tokens,
      // rounded up to 16 (the last token tile of an expert is often short).
      const int n_mma = S::kStacked ? S::kN : min(S::kN, (ti.nvalid + 15) & ~15);
      uint32_t idesc[S::kKSteps];
#pragma unroll
      for (int ks = 0; ks < S::kKSteps; ++ks)
        idesc[ks] = FP4 ? idesc_mxf4(n_mma, 2 * ks, 2 * ks) : idesc_mxf8f6f4(n_mma, ks, ks);
      const int buf = local % S::kAccBufs;
      const uint32_t accph = (uint32_t)(local / S::kAccBufs) & 1u;
      if (!mbar_wait(&acce[buf], accph ^ 1u, a.err, 2, a.wait_shift)) return false;
      tc_fence_after();
      const uint32_t d_tmem = tmem + buf * MG * S::kAccStride;
      for (int kt = kt_lo; kt < kt_hi; kt += KS) {
        if (!mbar_wait(&full[s], phase, a.err, 3, a.wait_shift)) return false;
        tc_fence_after();
        const int nk = min(KS, kt_hi - kt);
        const uint64_t so = (uint64_t)s * kStage16;
        // All scale-factor copies of the stage first, each K tile into its own
        // TMEM columns, then the MMAs: the copies' latency overlaps instead
        // of sitting between dependent MMAs.
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          if (j < nk) {
            const uint32_t sf_j = sfa_t + j * (4 * MG + 4 * S::kSfb), sfb_j = sf_j + 4 * MG;
#pragma unroll
            for (int m = 0; m < MG; ++m)
              if (m < nm) tc_cp_sf(sf_j + 4 * m, sfa_desc0 + so + 32 * (m * KS + j));
#pragma unroll
            for (int term = 0; term < S::kSfb; ++term)
              tc_cp_sf(sfb_j + 4 * term, sfb_desc0 + so + 32 * (j * S::kSfb + term));
          }
        }
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          if (j < nk) {
            const uint32_t sf_j = sfa_t + j * (4 * MG + 4 * S::kSfb), sfb_j = sf_j + 4 * MG;
            const uint64_t bd = b_desc0 + so + (uint64_t)j * kBt16;
#pragma unroll
            for (int m = 0; m < MG; ++m) {
              if (m >= nm) continue;
              const uint64_t ad = a_desc0 + so + (uint64_t)(j * MG + m) * kA16;
              const uint32_t dm = d_tmem + m * S::kAccStride, sfa_m = sf_j + 4 * m;
#pragma unroll
              for (int ks = 0; ks < S::kKSteps; ++ks) {
                const uint32_t id = FP4 ? 2u * ks : (uint32_t)ks;
#pragma unroll
                for (int term = 0; term < (S::kStacked ? 1 : S::kTerms); ++term) {
                  // the unit's first product into each accumulator overwrites it
                  const uint32_t acc = (kt == kt_lo && j == 0 && ks == 0 && term == 0) ? 0u : 1u;
                  if (FP4)
                    tc_mma_fp4(dm, ad + 2 * ks, bd + term * kBTerm16 + 2 * ks, idesc[ks], sfa_m | (id << 30),
                               (sfb_j + 4 * term) | (id << 30), acc);
                  else
                    tc_mma(dm, ad + 2 * ks, bd + term * kBTerm16 + 2 * ks, idesc[ks], sfa_m | (id << 30),
                           (sfb_j + 4 * term) | (id << 30), acc);
                }
              }
            }
          }
        }
        tc_commit(&empty[s]);
        if (++s == S::kStages) {
          s = 0;
          phase ^= 1u;
        }
      }
      tc_commit(&accf[buf]);
    }
    return true;
  }

  // Wait until every tensor-core operation this thread issued has finished
  // (also after an error: the accumulators' TMEM is freed after this).
  __device__ void drain_mma(int32_t *err, int shift) {
    tc_commit(drain);
    if (!mbar_wait_own(drain, 0, shift)) atomicCAS(err, 0, 4);
  }

  // ---------------- epilogue (warps 2-5) ----------------
  // tcgen05.ld of the accumulator (lane = output row), bias, fused SwiGLU
  // (gate/up rows are interleaved, so a row pair sits in neighbouring lanes)
  // or the down projection, fp32 stores.
  __device__ bool epilogue(const MmaLaunch &a, const TileTables &tt, int n_active, int n_tiles, int warp,
                           int lane) {
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_local = quad * 32 + lane;
    constexpr int kParts = S::kEpiWarps / 4;  // epilogue warps per TMEM lane quadrant
    const int half = (warp - 2) / 4;          // this warp's share of the columns
    constexpr int kCols = BN / kParts;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++local) {
      const TileInfo t = tile_info<BN>(tt, tile, n_active, a.mtiles);
      const int buf = local % S::kAccBufs;
      const uint32_t accph = (uint32_t)(local / S::kAccBufs) & 1u;
      if (!mbar_wait(&accf[buf], accph, a.err, 5, a.wait_shift)) return false;
      tc_fence_after();
      const int nm = min(MG, a.mtiles - t.mt * MG);
      if constexpr (!S::kStacked) {
        // Prefill tiles: this warp's share of the columns in one TMEM load per
        // row tile.  Gate/up: rows 2d (gate) and 2d+1 (up) sit in neighbouring
        // lanes; per pair of columns (c, c+1) each lane sends its partner the
        // value the partner lacks, the gate lane finishes column c and the up
        // lane column c+1 -- every lane computes SwiGLU, for half the columns.
        constexpr int kG = kCols >= 64 ? 64 : 32;
        static_assert(kCols % kG == 0, "epilogue column groups");
        for (int m = 0; m < nm; ++m) {
          const int r = (t.mt * MG + m) * kMmaM + row_local;
          const bool is_up = (r & 1) != 0;
          const int d = a.mode == 0 ? r >> 1 : r;
          const float *bsrc = a.mode == 0 ? (is_up ? a.bias1 : a.bias0) : a.bias0;
          const float bias = (bsrc && d < a.out_rows) ? bsrc[(size_t)t.e * a.out_rows + d] : 0.0f;
          for (int c0 = half * kCols; c0 < (half + 1) * kCols && c0 < t.nvalid; c0 += kG) {
            float v[kG];
            const uint32_t col =
                tmem + (uint32_t)((buf * MG + m) * S::kAccStride + c0) + ((uint32_t)(quad * 32) << 16);
            if constexpr (kG == 64) tc_ld64(col, v);
            else tc_ld32(col, v);
            if (a.mode == 0) {
#pragma unroll
              for (int j = 0; j < kG; j += 2) {
                const float v0 = v[j] + bias, v1 = v[j + 1] + bias;
                const float recv = __shfl_xor_sync(0xffffffffu, is_up ? v0 : v1, 1);
                const float g = is_up ? recv : v0, u = is_up ? v1 : recv;
                const int c = c0 + j + (is_up ? 1 : 0);
                if (c < t.nvalid && d < a.out_rows)
                  a.y[(size_t)(t.p0 + c) * a.y_stride + d] = swiglu_f32(g, u);
              }
            } else if (r < a.out_rows) {
#pragma unroll
              for (int j = 0; j < kG; ++j)
                if (c0 + j < t.nvalid) a.y[(size_t)(t.p0 + c0 + j) * a.y_stride + r] = v[j] + bias;
            }
          }
        }
      } else
      for (int m = 0; m < nm; ++m) {
      const int r = (t.mt * MG + m) * kMmaM + row_local;
      constexpr int kC = BN < 16 ? BN : 16;  // accumulator columns per TMEM load
      // columns past the unit's tokens were not written by the MMAs
      for (int c0 = half * kCols; c0 < (half + 1) * kCols && c0 < t.nvalid; c0 += kC) {
        float v[kC];
        const uint32_t col = tmem + (uint32_t)((buf * MG + m) * S::kAccStride + c0) + ((uint32_t)(quad * 32) << 16);
        if constexpr (FP4 && BN == 8 && kFp4Terms == 4) {
          // the term partial sums are consecutive columns: one round trip
          float w[kFp4Terms * 8];
          tc_ld32(col, w);
#pragma unroll
          for (int j = 0; j < kC; ++j) v[j] = w[j];
#pragma unroll
          for (int term = 1; term < kFp4Terms; ++term)
#pragma unroll
            for (int j = 0; j < kC; ++j) v[j] += w[term * BN + j];
        } else {
          tc_ld<kC>(col, v);
          if (S::kStacked) {  // the term partial sums sit BN columns apart
#pragma unroll
            for (int term = 1; term < kFp4Terms; ++term) {
              float w[kC];
              tc_ld<kC>(col + term * BN, w);
#pragma unroll
              for (int j = 0; j < kC; ++j) v[j] += w[j];
            }
          }
        }
        if (a.mode == 0) {
          const int d = r >> 1;
          const bool is_up = (r & 1) != 0;
          const float bias = is_up ? (a.bias1 ? a.bias1[(size_t)t.e * a.out_rows + d] : 0.0f)
                                   : (a.bias0 ? a.bias0[(size_t)t.e * a.out_rows + d] : 0.0f);
#pragma unroll
          for (int j = 0; j < kC; ++j) {
            const float val = v[j] + bias;
            const float other = __shfl_xor_sync(0xffffffffu, val, 1);
            if (!is_up && c0 + j < t.nvalid && d < a.out_rows)
              a.y[(size_t)(t.p0 + c0 + j) * a.y_stride + d] = swiglu_f32(val, other);
          }
        } else if (r < a.out_rows) {
          const float bias = a.bias0 ? a.bias0[(size_t)t.e * a.out_rows + r] : 0.0f;
#pragma unroll
          for (int j = 0; j < kC; ++j)
            if (c0 + j < t.nvalid) a.y[(size_t)(t.p0 + c0 + j) * a.y_stride + r] = v[j] + bias;
        }
      }
      }
      tc_fence_before();
      mbar_arrive(&acce[buf]);
    }
    return true;
  }
};

template <int BN, bool FP4, int KS, int MG>
__global__ void __launch_bounds__(MmaShape<BN, FP4, KS, MG>::kThreads, 1) k_mma_gemm(const __grid_constant__ MmaLaunch a) {
  using G = GemmCta<BN, FP4, KS, MG>;
  using S = typename G::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  G g(smem);
  TileTables &tt = *reinterpret_cast<TileTables *>(smem + S::kStages * S::kStage + G::kBarBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) g.init_barriers();
  if (warp == 1) g.alloc_tmem();
  // Barriers and TMEM above need nothing from the previous kernel; the tile
  // tables below are the dispatch kernel's output.
  pdl_wait();
  pdl_trigger();
  {
    const int na = a.meta[0];
    for (int i = threadIdx.x; i < na && i < kMaxActive; i += blockDim.x) {
      const int e = a.act_list[i];
      tt.e[i] = e;
      tt.p0[i] = a.offsets[e];
      tt.n[i] = a.offsets[e + 1] - a.offsets[e];
      tt.pad[i] = a.pad_off[e];
      tt.tile_off[i] = a.tile_off[i];
    }
    if (threadIdx.x == 0) tt.tile_off[min(na, kMaxActive)] = a.tile_off[min(na, kMaxActive)];
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  g.tmem = *g.tmem_slot;
  const int n_active = min(a.meta[0], kMaxActive);
  const int n_tiles = n_active > 0 ? tt.tile_off[n_active] : 0;

  if (warp == 0 && lane == 0) {
    g.produce(a, tt, n_active, n_tiles);
  } else if (warp == 1 && lane == 0) {
    g.mma(a, tt, n_active, n_tiles);
    g.drain_mma(a.err, a.wait_shift);
  } else if (warp >= 2) {
    g.epilogue(a, tt, n_active, n_tiles, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) g.dealloc_tmem();
}

template <int BN, bool FP4, int KS, int MG = 1>
cudaError_t launch_gemm_bn(const MmaLaunch &a, int sm_count, cudaStream_t s) {
  using Sh = MmaShape<BN, FP4, KS, MG>;
  cudaError_t e = opt_in_smem(k_mma_gemm<BN, FP4, KS, MG>, Sh::kSmem);
  if (e != cudaSuccess) return e;
  int grid = a.max_tiles < sm_count ? a.max_tiles : sm_count;
  if (grid < 1) grid = 1;
  return launch_pdl(k_mma_gemm<BN, FP4, KS, MG>, dim3(grid), dim3(Sh::kThreads), (size_t)Sh::kSmem, s, a);
}

}  // namespace

cudaError_t launch_repack_mma_gu(const uint8_t *gate, const uint8_t *up, int64_t E, int D, int K,
                                 MmaMatrix *m, cudaStream_t s) {
  const int NB = K / 32;
  k_repack_mma_gu<<<grid_of(E * D * NB), 256, 0, s>>>(gate, up, E, D, NB, m->kp, m->w, m->sf);
  return cudaGetLastError();
}

cudaError_t launch_repack_mma(const uint8_t *src, int64_t E, int R, int K, MmaMatrix *m, cudaStream_t s) {
  const int NB = K / 32;
  k_repack_mma<<<grid_of(E * R * NB), 256, 0, s>>>(src, E, R, NB, m->kp, m->w, m->sf);
  return cudaGetLastError();
}

cudaError_t launch_synth_mma_gu(uint64_t seed, uint32_t tg, uint32_t tu, int64_t first_expert, int64_t E, int D,
                                int K, uint8_t lo, uint8_t hi, MmaMatrix *m, cudaStream_t s) {
  const int NB = K / 32;
  k_synth_mma_gu<<<grid_of(E * D * NB), 256, 0, s>>>(seed, tg, tu, E, D, NB, lo, hi,
                                                     (uint64_t)(first_expert * D * NB), m->kp, m->w, m->sf);
  return cudaGetLastError();
}

cudaError_t launch_synth_mma(uint64_t seed, uint32_t tag, int64_t first_expert, int64_t E, int R, int K,
                             uint8_t lo, uint8_t hi, MmaMatrix *m, cudaStream_t s) {
  const int NB = K / 32;
  k_synth_mma<<<grid_of(E * R * NB), 256, 0, s>>>(seed, tag, E, R, NB, lo, hi, (uint64_t)(first_expert * R * NB),
                                                  m->kp, m->w, m->sf);
  return cudaGetLastError();
}

cudaError_t launch_quantize_tokens(const float *x, int64_t stride, int T, int top_k, const int32_t *slot_pos,
                                   const int32_t *offsets, const int32_t *pad_off, const int32_t *pos_expert, int K,
                                   int kp, int rb, int bn, ActFmt f, uint8_t *q, uint8_t *sf, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const int threads = 256;
  // large batches: several K tiles per warp (their chains overlap); small
  // ones one (more warps)
  const bool wide = T >= 512;
  const int ktw = wide ? kQuantKt : 1;
  const int64_t warps = (int64_t)T * ((kp / kMmaKT + ktw - 1) / ktw);
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  auto k = mma_fp4(f) ? (wide ? k_quantize_tokens<true, kQuantKt> : k_quantize_tokens<true, 1>)
                      : (wide ? k_quantize_tokens<false, kQuantKt> : k_quantize_tokens<false, 1>);
  return launch_pdl(k, dim3((unsigned)blocks), dim3(threads), 0, s, x, stride, T, top_k, slot_pos, offsets, pad_off,
                    pos_expert, K, kp, rb, bn, q, sf);
}

cudaError_t launch_quantize_act(const float *src, int64_t stride, const int32_t *perm, int top_k,
                                bool gather, const int32_t *offsets, const int32_t *pad_off,
                                const int32_t *pos_expert, const int32_t *meta, int S_max, int K, int kp,
                                int rb, int bn, ActFmt f, uint8_t *q, uint8_t *sf, cudaStream_t s) {
  if (S_max <= 0) return cudaSuccess;
  const int threads = 256;
  // large batches: several K tiles per warp (memory parallelism); small ones
  // one (more warps)
  const bool wide = S_max >= 2048;
  const int ktw = wide ? kQuantKt : 1;
  const int64_t warps = (int64_t)S_max * ((kp / kMmaKT + ktw - 1) / ktw);
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  auto k = mma_fp4(f) ? (wide ? k_quantize_act<true, kQuantKt> : k_quantize_act<true, 1>)
                      : (wide ? k_quantize_act<false, kQuantKt> : k_quantize_act<false, 1>);
  return launch_pdl(k, dim3((unsigned)blocks), dim3(threads), 0, s, src, stride, perm, top_k, gather ? 1 : 0, offsets,
                    pad_off, pos_expert, meta, S_max, K, kp, rb, bn, q, sf);
}

cudaError_t launch_mma_gemm(const MmaLaunch &a, int bn, ActFmt f, int sm_count, cudaStream_t s) {
  if (bn == 8 && a.ks == kMmaStageTilesWide) return launch_gemm_bn<8, true, kMmaStageTilesWide>(a, sm_count, s);
  if (bn == 8 && a.ks == kMmaStageTilesFp4) return launch_gemm_bn<8, true, kMmaStageTilesFp4>(a, sm_count, s);
  if (bn == 16 && a.ks == kMmaStageTilesFp4) return launch_gemm_bn<16, true, kMmaStageTilesFp4>(a, sm_count, s);
  if (bn == 128 && f == ActFmt::kFp4Planes) return launch_gemm_bn<128, true, 1, kPrefillRowTiles>(a, sm_count, s);
  if (bn == 128 && f == ActFmt::kFp8Planes) return launch_gemm_bn<128, false, 1, kPrefillRowTiles>(a, sm_count, s);
  return cudaErrorInvalidValue;
}

}  // namespace spt
