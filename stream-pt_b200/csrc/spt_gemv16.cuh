// spt_gemv16.cuh -- decode-sized expert products on the packed MXFP4 planes
// (spt_gemv16.cu): split-operand f16 GEMV with fp32 sums.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace spt {

// Scale bytes whose levels stay exact in f16 (e2m1 level x 2^(s-127)).
constexpr int kF16ScaleLo = 104;
constexpr int kF16ScaleHi = 140;
// K tiles (128 elements) one launch handles: 3 per warp over 8 warps.
constexpr int kGemv16MaxKtiles = 24;

// One split-operand value pair: hi = f16(v), lo = f16(v - hi).
__device__ __forceinline__ void split_f16(float v, __half *hi, __half *lo) {
  const __half h = __float2half_rn(v);
  *hi = h;
  *lo = __float2half_rn(__fsub_rn(v, __half2float(h)));
}

// Exponent e of a row with largest magnitude amax: amax * 2^-e lands in
// [2^14, 2^15), so the row's f16 terms neither overflow nor lose more than
// the f16 subnormal range at the bottom; 0 when amax is 0 or not finite.
__device__ __forceinline__ int split_exponent(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 0;
  int ex;
  frexpf(amax, &ex);  // amax = m * 2^ex, m in [0.5, 1)
  return max(-120, min(ex - 15, 120));
}

struct Gemv16Launch {
  const uint8_t *w = nullptr;    // MmaMatrix::w, tile-major packed e2m1
  const uint8_t *sf = nullptr;   // MmaMatrix::sf, scale atoms
  int rows = 0;                  // MMA rows per expert (2D for gate/up, H for down)
  int out_rows = 0;              // D (gate/up) or H (down)
  int mtiles = 0, ktiles = 0, kp = 0;
  const __half *xq = nullptr;    // split operand rows: gate/up per token, down per dispatch position
  int64_t xq_stride = 0;         // halves per row (2 * kp)
  const int32_t *xe = nullptr;   // per-row exponents of x (gate/up), or null
  const int32_t *perm = nullptr; // gate/up: the token of position p is perm[p] / top_k
  int top_k = 1;
  const int32_t *act_list = nullptr;  // [E] active experts (dispatch kernel)
  const int32_t *act_off = nullptr;   // [E+1] their first dispatch positions (DispatchPlan::act_off)
  const int32_t *meta = nullptr;      // [0] active experts
  const float *bias0 = nullptr;  // gate bias [E][D] or down bias [E][H]
  const float *bias1 = nullptr;  // up bias [E][D]
  __half *actq = nullptr;        // gate/up output: split operand of the down GEMM [pos][2][actq_kp]
  int64_t actq_stride = 0;
  int actq_kp = 0;
  float *y = nullptr;            // down output rows [pos][y_stride]
  int64_t y_stride = 0;
  // down only, optional: the combine of k_combine fused in.  The last CTA
  // of each 32-row group (counted in ccount[group], which it resets to 0)
  // writes out[t][rows] = sum over ranks r in order of fma(y[slot_pos[t*K+r]],
  // sel_w[t*K+r], .) for the ct tokens.
  const float *cw = nullptr;        // sel_w [ct * ck]
  const int32_t *cslot = nullptr;   // slot_pos [ct * ck]
  int ct = 0, ck = 0;
  float *cout = nullptr;            // [ct][out_rows]
  const float *cresid = nullptr;    // optional [ct][out_rows] added to the sums (may be cout)
  int32_t *ccount = nullptr;        // [mtiles * 4], zero between launches
};

// mode 0: gate/up + SwiGLU -> actq; mode 1: down -> y.  Grid: (32-row groups,
// max_active); CTAs of inactive experts exit at once.
cudaError_t launch_gemv16(const Gemv16Launch &a, int mode, int max_active, cudaStream_t s);
// fp32 rows (K used of each stride) -> split operand [rows][2][KP] with
// per-row exponents xe (may be null).  Output row p reads source row
// perm[p] / top_k (perm may be null: row p); with meta, rows >= meta[1] are
// skipped.  K <= 4096.
cudaError_t launch_split_rows(const float *src, int64_t stride, int rows, int K, int KP, const int32_t *perm,
                              int top_k, const int32_t *meta, __half *dst, int32_t *xe, cudaStream_t s);
// Scale-byte range of n GGUF MXFP4 blocks into range[0] (min), range[1] (max).
cudaError_t launch_scale_range(const uint8_t *blocks, int64_t n, int32_t *range, cudaStream_t s);

}  // namespace spt
