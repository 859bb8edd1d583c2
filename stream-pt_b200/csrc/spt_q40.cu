// spt_q40.cu -- Q4_0 matrix-vector and matrix-batch products (MulQ40Into /
// MulQ40BatchInto, forward/q40.go:35-101) on sm_100a, bit-exact with the
// reference's two AVX2 orders.
//
// A Q4_0 row is input/32 blocks of 18 bytes: a float16 scale, then 16 bytes
// whose low nibbles are elements 0..15 and high nibbles elements 16..31;
// weight = (nibble - 8) * scale, exact in fp32 (quantQ40WeightsAVX2,
// forward/quant_amd64.go:65-73).
//
// One input (quantQ40AVX2, quant_amd64.go:75-90): 32 FMA chains per row,
// chain c = element c of every block, summed ((a0+a1)+a2)+a3 over the four
// 8-lane accumulators and reduced with quantSumAVX2.  k_q40_gemv streams the
// matrix through a four-stage shared-memory ring (a producer warp issuing
// bulk copies of 4-row chunks, placed 32 bytes apart modulo 128 so the four
// rows a warp reads at once sit in different banks) and runs each row on 8
// lanes: lane j loads the two bytes 2j, 2j+1 of a block as one 16-bit word
// and owns chains 2j, 2j+1, 16+2j, 17+2j.  Each nibble becomes a float
// without a shift or a convert: masked in place and OR-ed with an exponent
// that gives its bit position weight 1 (2^23, 2^19, 2^15, 2^11 for bits
// 0, 4, 8, 12), then the exponent's value plus 8 is subtracted -- exact.
//
// A batch (quantDotQ40Batch, quant_amd64.go:118-148): one 8-lane accumulator
// per item; lane l takes elements l, 8+l, 16+l, 24+l of each block in that
// order, i.e. every k = l (mod 8) in increasing k, then quantSumAVX2.  That
// is a matrix product whose K dimension splits into 8 interleaved chains
// with a fixed final tree.  k_q40_batch tiles it like an fp32 GEMM: warp l
// of the CTA runs chain l for the whole tile (lane = an 8-row x TN-item
// micro-tile), weights decoded once per CTA into shared memory and reused
// by every item of the tile, and the 8 chains of an output meet in shared
// memory for the quantSumAVX2 tree.
#include <algorithm>

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spt_device.cuh"
#include "spt_internal.cuh"
#include "spt_ptx.cuh"

namespace spt {

namespace {

// =========================================================================
// One input
// =========================================================================
constexpr int kQ40Threads = 544;  // 16 consumer warps + 1 producer warp
constexpr int kQ40Stages = 4;
constexpr int kQ40Consumers = 16;
constexpr int kQ40Group = 4;      // consumer warps per stage
constexpr int kQ40Groups = kQ40Consumers / kQ40Group;
constexpr int kQ40Rows = 16;      // rows per stage: 4 warps x 4 sub-groups of 8 lanes

struct Q40Layout {
  int nb, rb;  // blocks and bytes per row
  int cr;      // rows per bulk copy (16-byte aligned: 4 when nb is even, else 8)
  int cs;      // shared-memory stride of one copy: cr*rb rounded so starts fall 32 B apart mod 128
  int stage;   // bytes of one stage
};

Q40Layout q40_layout(int input) {
  Q40Layout l;
  l.nb = input / 32;
  l.rb = l.nb * 18;
  l.cr = (l.nb % 2 == 0) ? 4 : 8;
  const int span = l.cr * l.rb;  // 72*nb or 144*nb: a multiple of 16
  l.cs = span + ((32 - span % 128) % 128 + 128) % 128;
  l.stage = (kQ40Rows / l.cr) * l.cs;
  return l;
}

struct Q40Launch {
  const uint8_t *w;  // rows x row bytes (+ at least 16 bytes of padding)
  int64_t rows;
  Q40Layout lay;
  const float *x;    // [input]
  float *y;          // [rows]
  int32_t *err;
};

// Warp roles as in the Q8_0 head: warps 0..15 consume in four groups of four
// that take the stages in turn; warp 16 produces.  Within a consumer warp,
// sub-group g (lanes 8g..8g+7) runs stage row wi + 4g (wi = the warp's index
// in its group), which is row wi of copy g when a copy holds 4 rows.
__global__ void __launch_bounds__(kQ40Threads, 1) k_q40_gemv(const __grid_constant__ Q40Launch a) {
  extern __shared__ __align__(128) uint8_t q40_smem[];
  const Q40Layout L = a.lay;
  const int nb = L.nb, rb = L.rb;
  float4 *xs = reinterpret_cast<float4 *>(q40_smem + (size_t)kQ40Stages * L.stage);  // [nb][8]
  float *wscale = reinterpret_cast<float *>(xs + (size_t)nb * 8);                    // [16][nb][4]
  uint64_t *full = reinterpret_cast<uint64_t *>(wscale + (size_t)kQ40Consumers * 4 * nb);
  uint64_t *empty = full + kQ40Stages;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n_chunks = (a.rows + kQ40Rows - 1) / kQ40Rows;
  if (tid == 0) {
    for (int s = 0; s < kQ40Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kQ40Group);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();
  if (warp == kQ40Consumers) {
    // ---- producer: the matrix does not depend on earlier kernels, so its
    // copies start before the wait for the predecessor grid ----
    if (lane == 0) {
      int it = 0;
      for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x, ++it) {
        const int s = it % kQ40Stages, use = it / kQ40Stages;
        if (use > 0 && !mbar_wait(&empty[s], (uint32_t)(use - 1) & 1u, a.err, 2)) break;
        const int64_t r0 = chunk * kQ40Rows;
        const int nr = (int)(a.rows - r0 < kQ40Rows ? a.rows - r0 : kQ40Rows);
        uint32_t tx = 0;
        for (int p = 0; p < nr; p += L.cr) tx += (uint32_t)((min(L.cr, nr - p) * rb + 15) & ~15);
        mbar_expect_tx(&full[s], tx);
        uint8_t *dst = q40_smem + (size_t)s * L.stage;
        for (int p = 0; p < nr; p += L.cr) {
          // the last copy rounds up to 16 bytes: the matrix buffer is padded
          const uint32_t bytes = (uint32_t)((min(L.cr, nr - p) * rb + 15) & ~15);
          bulk_load(dst + (size_t)(p / L.cr) * L.cs, a.w + (r0 + p) * rb, bytes, &full[s]);
        }
      }
      // if a wait gave up, copies may still be in flight: they land before
      // the CTA leaves (bounded wait for the last phase issued on each stage)
      for (int s = 0; s < kQ40Stages && s < it; ++s)
        mbar_wait_own(&full[s], (uint32_t)((it - 1 - s) / kQ40Stages) & 1u);
    }
    return;
  }
  // ---- consumers ----
  pdl_wait();
  for (int i = tid; i < nb * 8; i += kQ40Consumers * 32) {
    const int b = i >> 3, j = i & 7;
    const float *xb = a.x + 32 * b + 2 * j;
    xs[i] = make_float4(xb[0], xb[1], xb[16], xb[17]);  // chains 2j, 2j+1, 16+2j, 17+2j
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kQ40Consumers * 32) : "memory");
  const int group = warp / kQ40Group, wi = warp % kQ40Group, g = lane >> 3, j = lane & 7;
  float *sc = wscale + (size_t)warp * nb * 4;  // [nb][4 sub-groups]
  int it = group;
  for (int64_t chunk = blockIdx.x + (int64_t)group * gridDim.x; chunk < n_chunks;
       chunk += (int64_t)kQ40Groups * gridDim.x, it += kQ40Groups) {
    const int s = it % kQ40Stages, use = it / kQ40Stages;
    if (!mbar_wait(&full[s], (uint32_t)use & 1u, a.err, 1)) break;
    const uint8_t *cb = q40_smem + (size_t)s * L.stage;
    const int64_t r0 = chunk * kQ40Rows;
    const int nr = (int)(a.rows - r0 < kQ40Rows ? a.rows - r0 : kQ40Rows);
    if (wi < nr) {
      // rows past the end repeat row wi (computed, not stored)
      auto row_at = [&](int gg) -> const uint8_t * {
        const int r = wi + 4 * gg < nr ? wi + 4 * gg : wi;
        return cb + (size_t)(r / L.cr) * L.cs + (size_t)(r % L.cr) * rb;
      };
      for (int b = lane; b < nb; b += 32) {
        // float16 -> float32 is exact for every finite value and infinity
        // (quantFloat16Bits, forward/quant_portable.go:20-35); NaN stays NaN
        float4 v;
        v.x = __half2float(*reinterpret_cast<const __half *>(row_at(0) + b * 18));
        v.y = __half2float(*reinterpret_cast<const __half *>(row_at(1) + b * 18));
        v.z = __half2float(*reinterpret_cast<const __half *>(row_at(2) + b * 18));
        v.w = __half2float(*reinterpret_cast<const __half *>(row_at(3) + b * 18));
        reinterpret_cast<float4 *>(sc)[b] = v;
      }
      __syncwarp();
      const uint8_t *q = row_at(g) + 2 + 2 * j;
      float2 clo = make_float2(0.0f, 0.0f), chi = make_float2(0.0f, 0.0f);  // chains 2j, 2j+1 | 16+2j, 17+2j
      const float2 sub_lo = make_float2(-8388616.0f, -32776.0f), sub_hi = make_float2(-524296.0f, -2056.0f);
#pragma unroll 6
      for (int b = 0; b < nb; ++b) {
        const float4 xv = xs[b * 8 + j];
        const float s = sc[b * 4 + g];
        const uint32_t v = *reinterpret_cast<const uint16_t *>(q + b * 18);
        // nibble n at bits 0/8 (low nibbles of bytes 2j, 2j+1) and 4/12 (high
        // nibbles): (2^e + n) - (2^e + 8) = n - 8, exact
        float2 wl = make_float2(__uint_as_float((v & 0x000Fu) | 0x4B000000u),   // 2^23 + n
                                __uint_as_float((v & 0x0F00u) | 0x47000000u));  // 2^15 + n
        float2 wh = make_float2(__uint_as_float((v & 0x00F0u) | 0x49000000u),   // 2^19 + n
                                __uint_as_float((v & 0xF000u) | 0x45000000u));  // 2^11 + n
        const float2 ss = make_float2(s, s);
        wl = __fmul2_rn(__fadd2_rn(wl, sub_lo), ss);  // weight = (n - 8) * scale (exact); packed f32x2:
        wh = __fmul2_rn(__fadd2_rn(wh, sub_hi), ss);  // two independent IEEE operations
        clo = __ffma2_rn(wl, make_float2(xv.x, xv.y), clo);
        chi = __ffma2_rn(wh, make_float2(xv.z, xv.w), chi);
      }
      const float c0 = clo.x, c1 = clo.y, c2 = chi.x, c3 = chi.y;
      // a0+a1+a2+a3 then quantSumAVX2 over the sub-group's 8 lanes:
      // s_m = ((a_m + a_{8+m}) + a_{16+m}) + a_{24+m}; lane j < 4 holds
      // a_{2j+e} and a_{16+2j+e}, lane j+4 holds a_{8+2j+e} and a_{24+2j+e}
      const float t0 = __shfl_down_sync(0xffffffffu, c0, 4, 8), t1 = __shfl_down_sync(0xffffffffu, c1, 4, 8);
      const float t2 = __shfl_down_sync(0xffffffffu, c2, 4, 8), t3 = __shfl_down_sync(0xffffffffu, c3, 4, 8);
      const float s0 = __fadd_rn(__fadd_rn(__fadd_rn(c0, t0), c2), t2);  // s_{2j}
      const float s1 = __fadd_rn(__fadd_rn(__fadd_rn(c1, t1), c3), t3);  // s_{2j+1}
      // p_i = s_i + s_{4+i}: lane j < 2 gets p_{2j}, p_{2j+1}
      const float p0 = __fadd_rn(s0, __shfl_down_sync(0xffffffffu, s0, 2, 8));
      const float p1 = __fadd_rn(s1, __shfl_down_sync(0xffffffffu, s1, 2, 8));
      const float qv = __fadd_rn(p0, p1);  // lane 0: p0+p1, lane 1: p2+p3
      const float total = __fadd_rn(qv, __shfl_down_sync(0xffffffffu, qv, 1, 8));
      if (j == 0 && wi + 4 * g < nr && a.y) a.y[r0 + wi + 4 * g] = total;
      __syncwarp();  // the next chunk's scales overwrite these
    }
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

// =========================================================================
// A batch
// =========================================================================
constexpr int kQ40BatchThreads = 256;  // 8 warps = the 8 chains
constexpr int kQ40BatchK = 64;         // k per stage (two blocks)

// Position of tile row r in a shared-memory weight row: with TM = 8 the
// eight rows of lane pm are split in two float4 halves 128 bytes apart, so
// each warp-wide 16-byte load covers 128 contiguous bytes.
template <int TM>
__device__ __forceinline__ int q40_wpos(int r) {
  if (TM == 8) return ((r & 7) >> 2) * 32 + (r >> 3) * 4 + (r & 3);
  return r;
}

template <int N>
__device__ __forceinline__ void lds_vec(float *v, const float *p) {
  if constexpr (N == 1) {
    v[0] = p[0];
  } else if constexpr (N == 2) {
    const float2 t = *reinterpret_cast<const float2 *>(p);
    v[0] = t.x, v[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 t = *reinterpret_cast<const float4 *>(p + i);
      v[i] = t.x, v[i + 1] = t.y, v[i + 2] = t.z, v[i + 3] = t.w;
    }
  }
}

// CTA tile: BM = 8*TM rows x BN = 4*TN items; lane = (pm = lane & 7,
// pn = lane >> 3) owns rows pm*TM.. and items pn*TN.. of chain `warp`.
template <int TM, int TN>
__global__ void __launch_bounds__(kQ40BatchThreads, TM * TN <= 16 ? 3 : 2)
    k_q40_batch(const uint8_t *__restrict__ w, int64_t rows, int input, const float *__restrict__ x,
                int64_t batch, float *__restrict__ y) {
  constexpr int BM = 8 * TM, BN = 4 * TN;
  constexpr int EPT = kQ40BatchK * BM / kQ40BatchThreads;  // weights decoded per thread per stage (8 or 16)
  constexpr int XPT = kQ40BatchK * BN / kQ40BatchThreads;  // x values staged per thread per stage
  static_assert(EPT == 8 || EPT == 16, "a thread decodes half a block's nibble plane at most");
  static_assert(XPT >= 1, "tile too narrow");
  __shared__ __align__(16) float ws[2][kQ40BatchK][BM];
  __shared__ __align__(16) float xs[2][kQ40BatchK][BN];
  static_assert(sizeof(ws) >= 4u * TM * TN * 32 * sizeof(float), "reduction space");

  const int tid = threadIdx.x, chain = tid >> 5, lane = tid & 31;
  const int pm = lane & 7, pn = lane >> 3;
  const int nb = input / 32;
  const int64_t rb = (int64_t)nb * 18;
  const int64_t row0 = (int64_t)blockIdx.x * BM, item0 = (int64_t)blockIdx.y * BN;

  // decode role: tile row drow, stage elements [dk, dk + EPT) = one nibble
  // plane (low: elements 0..15, high: 16..31) of one block.  With TM = 8 the
  // 32 rows a warp decodes are those whose shared-memory positions fill one
  // 128-byte half (dpos = half*32 + lane), so its stores are conflict-free.
  const int dloc = tid % BM, dk = (tid / BM) * EPT;
  const int drow = TM == 8 ? ((dloc & 31) >> 2) * 8 + (dloc >> 5) * 4 + (dloc & 3) : dloc;
  const int dblk = dk >> 5, dhalf = (dk & 31) >> 4, dbyte = dk & 15;
  const int dpos = q40_wpos<TM>(drow);
  // staging role for x: item xitem, stage elements [xk, xk + XPT)
  const int xitem = tid % BN, xk = (tid / BN) * XPT;

  uint32_t wraw[EPT / 2];
  uint32_t wsc = 0;
  float xr[XPT];
  auto fetch = [&](int st) {
    const int blk = 2 * st + dblk;
    const int64_t grow = row0 + drow;
    if (blk < nb && grow < rows) {
      const uint8_t *p = w + grow * rb + (int64_t)blk * 18;
      wsc = __ldg(reinterpret_cast<const unsigned short *>(p));
#pragma unroll
      for (int i = 0; i < EPT / 2; ++i) wraw[i] = __ldg(reinterpret_cast<const unsigned short *>(p + 2 + dbyte + 2 * i));
    } else {
      wsc = 0;
#pragma unroll
      for (int i = 0; i < EPT / 2; ++i) wraw[i] = 0x8888u;  // zero weights (never used: k past the end is skipped)
    }
    const int64_t gi = item0 + xitem;
#pragma unroll
    for (int i = 0; i < XPT; ++i) {
      const int k = kQ40BatchK * st + xk + i;
      xr[i] = (gi < batch && k < input) ? __ldg(x + gi * input + k) : 0.0f;
    }
  };
  auto stage_in = [&](int buf) {
    const float s = __half2float(__ushort_as_half((unsigned short)wsc));
#pragma unroll
    for (int i = 0; i < EPT / 2; ++i) {
      // nibble of byte dbyte+2i (bits 0-7) and dbyte+2i+1 (bits 8-15) as
      // 2^23 + n, then - (2^23 + 8) and * scale: exact (no int->float convert)
      const uint32_t v = dhalf ? (wraw[i] >> 4) : wraw[i];
      const float n0 = __uint_as_float(0x4B000000u | (v & 15u)), n1 = __uint_as_float(0x4B000000u | ((v >> 8) & 15u));
      ws[buf][dk + 2 * i][dpos] = __fmul_rn(__fsub_rn(n0, 8388616.0f), s);
      ws[buf][dk + 2 * i + 1][dpos] = __fmul_rn(__fsub_rn(n1, 8388616.0f), s);
    }
#pragma unroll
    for (int i = 0; i < XPT; ++i) xs[buf][xk + i][xitem] = xr[i];
  };

  pdl_wait();
  pdl_trigger();
  // accumulators in row pairs: accp[i][jj] = (row 2i, row 2i+1) of item jj,
  // updated by one packed f32x2 fma (two independent IEEE fmas)
  float2 accp[TM / 2][TN];
#pragma unroll
  for (int i = 0; i < TM / 2; ++i)
#pragma unroll
    for (int jj = 0; jj < TN; ++jj) accp[i][jj] = make_float2(0.0f, 0.0f);
  const int nst = (nb + 1) / 2;
  fetch(0);
  stage_in(0);
  __syncthreads();
  for (int st = 0; st < nst; ++st) {
    const int buf = st & 1;
    if (st + 1 < nst) fetch(st + 1);
    const int kn = (2 * st + 1 < nb) ? kQ40BatchK : 32;
    // chain `chain` takes k = chain, chain + 8, ... of the stage: with the
    // stages in order that is every k = chain (mod 8) in increasing k
    for (int kk = chain; kk < kn; kk += 8) {
      float wv[TM], xv[TN];
      if constexpr (TM == 8) {
        lds_vec<4>(wv, &ws[buf][kk][pm * 4]);
        lds_vec<4>(wv + 4, &ws[buf][kk][32 + pm * 4]);
      } else {
        lds_vec<TM>(wv, &ws[buf][kk][pm * TM]);
      }
      lds_vec<TN>(xv, &xs[buf][kk][pn * TN]);
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) {
        const float2 xx = make_float2(xv[jj], xv[jj]);
#pragma unroll
        for (int i = 0; i < TM / 2; ++i) accp[i][jj] = __ffma2_rn(make_float2(wv[2 * i], wv[2 * i + 1]), xx, accp[i][jj]);
      }
    }
    if (st + 1 < nst) stage_in(buf ^ 1);
    __syncthreads();
  }

  // quantSumAVX2 over the 8 chains: p_i = a_i + a_{4+i}, then
  // (p_0 + p_1) + (p_2 + p_3); chains meet through shared memory
  float *red = &ws[0][0][0];  // [slot][TM*TN][32 lanes]
  constexpr int A = TM * TN;
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM / 2; ++i)
#pragma unroll
    for (int jj = 0; jj < TN; ++jj) acc[2 * i][jj] = accp[i][jj].x, acc[2 * i + 1][jj] = accp[i][jj].y;
  auto put = [&](int slot) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) red[(slot * A + i * TN + jj) * 32 + lane] = acc[i][jj];
  };
  auto add_from = [&](int slot) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) acc[i][jj] = __fadd_rn(acc[i][jj], red[(slot * A + i * TN + jj) * 32 + lane]);
  };
  if (chain >= 4) put(chain - 4);
  __syncthreads();
  if (chain < 4) add_from(chain);  // p_chain
  __syncthreads();
  if (chain == 1 || chain == 3) put(chain >> 1);
  __syncthreads();
  if (chain == 0 || chain == 2) add_from(chain >> 1);  // warp 0: p0 + p1, warp 2: p2 + p3
  __syncthreads();
  if (chain == 2) put(0);
  __syncthreads();
  if (chain == 0) {
    add_from(0);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t r = row0 + pm * TM + i;
      if (r >= rows) continue;
#pragma unroll
      for (int jj = 0; jj < TN; ++jj) {
        const int64_t it = item0 + pn * TN + jj;
        if (it < batch) y[it * rows + r] = acc[i][jj];
      }
    }
  }
}

// Relative time of one tile shape: the busiest SM's tiles x tile work / the
// share of the FMA pipe the tile can keep busy.  A lane's k step is TM*TN
// FMAs (TM*TN/4 cycles of the SM's FMA pipe per warp) against TM + TN
// shared-memory wavefronts (128-bit loads are served a quarter-warp at a
// time, so the w and x vectors cost TM and TN wavefronts), and the SM serves
// one wavefront per cycle; 1.5x when an SM would hold a single tile (too few
// warps to hide latency).
template <int TM, int TN>
double batch_tile_cost(int64_t rows, int64_t batch, int sm_count) {
  constexpr int BM = 8 * TM, BN = 4 * TN;
  const int64_t tiles = ((rows + BM - 1) / BM) * ((batch + BN - 1) / BN);
  const int64_t per_sm = (tiles + sm_count - 1) / sm_count;
  const double eff = std::min(1.0, (double)(TM * TN) / (4.0 * (TM + TN)));
  return (double)per_sm * BM * BN / eff * (per_sm < 2 ? 1.5 : 1.0);
}

template <int TM, int TN>
cudaError_t launch_batch_tile(const uint8_t *w, int64_t rows, int input, const float *x, int64_t batch, float *y,
                              cudaStream_t stream) {
  constexpr int BM = 8 * TM, BN = 4 * TN;
  const int64_t gx = (rows + BM - 1) / BM, gy = (batch + BN - 1) / BN;
  if (gx > 0x7fffffffll || gy > 65535) return cudaErrorInvalidValue;
  return launch_pdl(k_q40_batch<TM, TN>, dim3((unsigned)gx, (unsigned)gy), dim3(kQ40BatchThreads), 0, stream, w,
                    rows, input, x, batch, y);
}

}  // namespace

size_t q40_smem_bytes(int input) {
  const Q40Layout l = q40_layout(input);
  return (size_t)kQ40Stages * l.stage + (size_t)l.nb * 8 * 16 + (size_t)kQ40Consumers * 4 * l.nb * 4 +
         16 * kQ40Stages;
}

bool q40_supported(int input) {
  return input > 0 && input % 32 == 0 && input <= (1 << 24) && q40_smem_bytes(input) <= 226 * 1024;
}

cudaError_t launch_q40(const uint8_t *w, int64_t rows, int input, const float *x, int64_t batch, float *y,
                       int32_t *err, int sm_count, cudaStream_t stream) {
  if (!q40_supported(input) || rows <= 0 || batch <= 0) return cudaErrorInvalidValue;
  if (batch > 1) {
    const double c[5] = {batch_tile_cost<4, 1>(rows, batch, sm_count), batch_tile_cost<4, 2>(rows, batch, sm_count),
                         batch_tile_cost<4, 4>(rows, batch, sm_count), batch_tile_cost<8, 4>(rows, batch, sm_count),
                         batch_tile_cost<8, 8>(rows, batch, sm_count)};
    int best = 0;
    for (int i = 1; i < 5; ++i)
      if (c[i] < c[best]) best = i;
    switch (best) {
      case 0: return launch_batch_tile<4, 1>(w, rows, input, x, batch, y, stream);
      case 1: return launch_batch_tile<4, 2>(w, rows, input, x, batch, y, stream);
      case 2: return launch_batch_tile<4, 4>(w, rows, input, x, batch, y, stream);
      case 3: return launch_batch_tile<8, 4>(w, rows, input, x, batch, y, stream);
      default: return launch_batch_tile<8, 8>(w, rows, input, x, batch, y, stream);
    }
  }
  const size_t smem = q40_smem_bytes(input);
  cudaError_t e = opt_in_smem(k_q40_gemv, (int)smem);
  if (e != cudaSuccess) return e;
  Q40Launch a;
  a.w = w;
  a.rows = rows;
  a.lay = q40_layout(input);
  a.x = x;
  a.y = y;
  a.err = err;
  const int64_t chunks = (rows + kQ40Rows - 1) / kQ40Rows;
  const int grid = (int)(chunks < sm_count ? chunks : sm_count);
  return launch_pdl(k_q40_gemv, dim3(grid), dim3(kQ40Threads), smem, stream, a);
}

}  // namespace spt
