// spt_q80.cu -- Q8_0 LM-head GEMV + argmax (MulQ80Into / MulQ80Argmax,
// forward/q80.go:22-148) on sm_100a, bit-exact with the reference's AVX2
// path (quantQ80AVX2 / quantQ80PairAVX2, forward/quant_amd64.go:17-45,92-110).
//
// A Q8_0 row is input/32 blocks of 34 bytes: a float16 scale, then 32 int8
// values.  The reference keeps 32 FMA chains per row (chain c = element c of
// every block, weight = int8 * scale, exact in fp32), sums them as
// ((a0+a1)+a2)+a3 over its four 8-lane accumulators and reduces the 8 lanes
// with quantSumAVX2.  Here one lane runs one chain.
//
// The matrix (615 MB for GPT-OSS's 201,088 x 2,880 output head) is repacked
// once at upload into groups of four rows, the same bytes in another order:
// per group, the blocks' float16 scales [nb][4 rows], then the quants
// [nb][32 elements][4 rows] with the sign bit flipped (byte ^ 0x80), so one
// 32-bit shared load gives a lane its element of all four rows.  The packed
// matrix streams through a four-stage shared-memory ring of 16-row stages,
// filled by a producer warp with 8-row bulk copies (up to eight in flight) and
// released per stage through mbarriers; four groups of four consumer warps
// take the stages in turn, each warp decoding its row group's block scales
// (float16 -> float32, exact like the reference's decode) and running the four
// rows at once on packed fp32 pairs (one x load per four rows).  int8 -> float
// is the exact magic-number form: a byte permute builds 0x4B000000 | (b ^ 0x80),
// from which 8388736 is subtracted, instead of the quarter-rate convert.
// The argmax packs (order-preserving logit bits, ~row) into 64 bits and
// keeps the maximum with atomicMax: largest logit, lowest row on ties, NaN
// never chosen, -0 equal to +0, and row 0 when nothing beats -Inf.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spt_device.cuh"
#include "spt_internal.cuh"
#include "spt_ptx.cuh"

namespace spt {

namespace {

constexpr int kQ80Threads = 544;  // 16 consumer warps + 1 producer warp

// AVX2 reduction of the 32 chains held one per lane; valid in lane 0.
__device__ __forceinline__ float reduce_chains(float v, int lane) {
  const float v8 = __shfl_sync(0xffffffffu, v, (lane + 8) & 31);
  const float v16 = __shfl_sync(0xffffffffu, v, (lane + 16) & 31);
  const float v24 = __shfl_sync(0xffffffffu, v, (lane + 24) & 31);
  const float s = __fadd_rn(__fadd_rn(__fadd_rn(v, v8), v16), v24);  // lanes 0..7: s_l
  const float p = __fadd_rn(s, __shfl_sync(0xffffffffu, s, (lane + 4) & 31));   // lanes 0..3
  const float q = __fadd_rn(p, __shfl_sync(0xffffffffu, p, (lane + 1) & 31));   // lanes 0, 2
  return __fadd_rn(q, __shfl_sync(0xffffffffu, q, (lane + 2) & 31));          // lane 0
}

__device__ __forceinline__ unsigned long long argmax_key(float logit, int64_t row) {
  uint32_t bits = __float_as_uint(logit == 0.0f ? 0.0f : logit);  // -0 ties with +0
  bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);      // order-preserving
  return ((unsigned long long)bits << 32) | (unsigned long long)(0xffffffffu - (uint32_t)row);
}

struct Q80Launch {
  const uint8_t *w;          // packed row groups (q80_packed_bytes)
  int64_t rows;
  int input, row_bytes, blocks, rows_per_stage;
  const float *x;            // [input]
  float *y;                  // [rows] or null
  unsigned long long *best;  // argmax key
  int32_t *err;
};

// Warp roles: warps 0..15 consume (four groups of 4 taking the stages in
// turn, four rows per warp), warp 16 produces (its lane 0 issues the copies).
// Stage s is filled through full[s] (transaction bytes) and released through
// empty[s] (one arrival per consumer warp of the group that read it), so the
// copies of later stages run while earlier ones are computed.
constexpr int kQ80Stages = 4;
constexpr int kQ80Consumers = 16;
constexpr int kQ80Group = 4;              // consumer warps per stage (4 rows each)
constexpr int kQ80Groups = kQ80Consumers / kQ80Group;
constexpr int kQ80RowsPerCopy = 8;        // one bulk copy moves up to 8 rows (16-byte aligned)

__global__ void __launch_bounds__(kQ80Threads, 1) k_q80_gemv(const __grid_constant__ Q80Launch a) {
  extern __shared__ __align__(128) uint8_t q80_smem[];
  const int rps = a.rows_per_stage, rb = a.row_bytes, nb = a.blocks;
  const uint32_t stage_bytes = (uint32_t)((int64_t)rps * rb);
  float *xs = reinterpret_cast<float *>(q80_smem + (size_t)kQ80Stages * stage_bytes);
  float *wscale = xs + a.input;                                               // [16][nb][4]
  uint64_t *full = reinterpret_cast<uint64_t *>(wscale + (size_t)kQ80Consumers * 4 * nb);
  uint64_t *empty = full + kQ80Stages;
  unsigned long long *wbest = reinterpret_cast<unsigned long long *>(empty + kQ80Stages);  // [16]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n_chunks = (a.rows + rps - 1) / rps;
  if (tid == 0) {
    for (int s = 0; s < kQ80Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kQ80Group);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < a.input; i += blockDim.x) xs[i] = a.x[i];
  __syncthreads();
  unsigned long long best = 0ull;
  if (warp == kQ80Consumers) {
    // ---- producer ----
    if (lane == 0) {
      int it = 0;
      for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x, ++it) {
        const int s = it % kQ80Stages, use = it / kQ80Stages;
        if (use > 0 && !mbar_wait(&empty[s], (uint32_t)(use - 1) & 1u, a.err, 2)) break;
        const int64_t r0 = chunk * rps;
        // whole four-row groups: the last group's missing rows are zero padding
        const int nr = (int)(((a.rows - r0 < rps ? a.rows - r0 : rps) + 3) & ~3);
        uint32_t tx = 0;
        for (int p = 0; p < nr; p += kQ80RowsPerCopy)
          tx += (uint32_t)((int64_t)(min(kQ80RowsPerCopy, nr - p) * rb + 15) & ~15ll);
        mbar_expect_tx(&full[s], tx);
        uint8_t *dst = q80_smem + (size_t)s * stage_bytes;
        for (int p = 0; p < nr; p += kQ80RowsPerCopy) {
          // the last copy rounds up to 16 bytes: the matrix buffer is padded
          const uint32_t bytes = (uint32_t)((int64_t)(min(kQ80RowsPerCopy, nr - p) * rb + 15) & ~15ll);
          bulk_load(dst + (size_t)p * rb, a.w + (r0 + p) * rb, bytes, &full[s]);
        }
      }
      // if a wait gave up, copies may still be in flight: they land before
      // the CTA leaves (bounded wait for the last phase issued on each stage)
      for (int s = 0; s < kQ80Stages && s < it; ++s)
        mbar_wait_own(&full[s], (uint32_t)((it - 1 - s) / kQ80Stages) & 1u);
    }
  } else {
    // ---- consumers: group g takes stages it = g, g + 4, ...; each warp
    // runs four rows of the stage at once ----
    const int group = warp / kQ80Group, wi = warp % kQ80Group;
    float4 *sc = reinterpret_cast<float4 *>(wscale) + (size_t)warp * nb;  // [nb] x 4 rows
    int it = group;
    for (int64_t chunk = blockIdx.x + (int64_t)group * gridDim.x; chunk < n_chunks;
         chunk += (int64_t)kQ80Groups * gridDim.x, it += kQ80Groups) {
      const int s = it % kQ80Stages, use = it / kQ80Stages;
      if (!mbar_wait(&full[s], (uint32_t)use & 1u, a.err, 1)) break;
      const uint8_t *cb = q80_smem + (size_t)s * stage_bytes;
      const int64_t r0 = chunk * rps;
      const int nr = (int)(a.rows - r0 < rps ? a.rows - r0 : rps);
      for (int r = 4 * wi; r < nr; r += 4 * kQ80Group) {
        const int live = min(4, nr - r);  // rows past the end are padding, not written
        const uint8_t *gb = cb + (size_t)r * rb;  // this warp's row group
        for (int b = lane; b < nb; b += 32) {
          // float16 -> float32 is exact for every finite value and infinity
          // (quantFloat16Bits); a NaN scale gives a NaN either way
          const uint2 h = *reinterpret_cast<const uint2 *>(gb + 8 * b);
          sc[b] = make_float4(__half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu))),
                              __half2float(__ushort_as_half((unsigned short)(h.x >> 16))),
                              __half2float(__ushort_as_half((unsigned short)(h.y & 0xffffu))),
                              __half2float(__ushort_as_half((unsigned short)(h.y >> 16))));
        }
        __syncwarp();
        const uint32_t *qw = reinterpret_cast<const uint32_t *>(gb + 8 * nb) + lane;  // [nb][32] words
        // packed fp32 pairs (sm_100a f32x2, the compiler's own float2
        // operations): two independent IEEE round-to-nearest results each,
        // equal to the scalar ones
        float2 a01 = make_float2(0.0f, 0.0f), a23 = make_float2(0.0f, 0.0f);
        const float2 off = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll 5
        for (int b = 0; b < nb; ++b) {
          const float xv = xs[b * 32 + lane];
          const float4 sv = sc[b];
          // int8 -> float: (0x4B000000 | (byte ^ 0x80)) - 8388736, exact; byte k
          // of the word is row k's (sign-flipped) quant
          const uint32_t q = qw[b * 32];
          float2 w01 = make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7650)),
                                   __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7651)));
          float2 w23 = make_float2(__uint_as_float(__byte_perm(q, 0x4B000000u, 0x7652)),
                                   __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7653)));
          w01 = __fmul2_rn(__fadd2_rn(w01, off), make_float2(sv.x, sv.y));  // weight = int8 * scale (exact)
          w23 = __fmul2_rn(__fadd2_rn(w23, off), make_float2(sv.z, sv.w));
          const float2 xx = make_float2(xv, xv);
          a01 = __ffma2_rn(w01, xx, a01);
          a23 = __ffma2_rn(w23, xx, a23);
        }
        const float y[4] = {reduce_chains(a01.x, lane), reduce_chains(a01.y, lane), reduce_chains(a23.x, lane),
                            reduce_chains(a23.y, lane)};
        if (lane == 0) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (k >= live) break;
            if (a.y) a.y[r0 + r + k] = y[k];
            if (!isnan(y[k])) best = max(best, argmax_key(y[k], r0 + r + k));
          }
        }
        __syncwarp();  // the next rows' scales overwrite these
      }
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (lane == 0) wbest[warp] = best;
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kQ80Consumers; ++w) b = max(b, wbest[w]);
    if (b) atomicMax(a.best, b);
  }
}

// Upload-time repack, one thread per (row group, block): the group's four
// 34-byte blocks become 8 scale bytes at [block] and 32 words at [block][element]
// whose byte k is row k's quant ^ 0x80; rows past the end are zero.
__global__ void k_q80_repack(const uint8_t *__restrict__ raw, int64_t rows, int nb, uint8_t *__restrict__ out) {
  const int64_t groups = (rows + 3) / 4;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= groups * nb) return;
  const int64_t g = t / nb;
  const int b = (int)(t % nb);
  const int64_t rb = (int64_t)nb * 34;
  const uint8_t *src[4];
  bool has[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    has[k] = 4 * g + k < rows;
    src[k] = raw + (has[k] ? (4 * g + k) * rb + (int64_t)b * 34 : 0);
  }
  uint8_t *dst = out + g * 4 * rb;
  uint32_t sw[2] = {0u, 0u};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (has[k]) sw[k >> 1] |= ((uint32_t)src[k][0] | ((uint32_t)src[k][1] << 8)) << (16 * (k & 1));
  reinterpret_cast<uint2 *>(dst)[b] = make_uint2(sw[0], sw[1]);
  uint32_t *qw = reinterpret_cast<uint32_t *>(dst + 8 * nb) + (int64_t)b * 32;
  for (int c = 0; c < 32; ++c) {
    uint32_t w = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (has[k]) w |= (uint32_t)(src[k][2 + c] ^ 0x80u) << (8 * k);
    qw[c] = w;
  }
}

__global__ void k_q80_init(unsigned long long *best) {
  pdl_wait();
  pdl_trigger();
  *best = argmax_key(-INFINITY, 0);
}

__global__ void k_q80_finalize(const unsigned long long *best, int64_t *argmax, float *logit) {
  pdl_wait();
  pdl_trigger();
  const unsigned long long k = *best;
  const uint32_t hi = (uint32_t)(k >> 32);
  const uint32_t bits = (hi & 0x80000000u) ? (hi & 0x7fffffffu) : ~hi;
  if (argmax) *argmax = (int64_t)(0xffffffffu - (uint32_t)k);
  if (logit) *logit = __uint_as_float(bits);
}

}  // namespace

uint64_t q80_packed_bytes(int64_t rows, int input) {
  // whole four-row groups, + 64 bytes: the last copy rounds up to 16 bytes
  return (uint64_t)((rows + 3) / 4 * 4) * (uint64_t)(input / 32 * 34) + 64;
}

cudaError_t launch_q80_repack(const uint8_t *raw, int64_t rows, int input, uint8_t *packed, cudaStream_t stream) {
  const int nb = input / 32;
  const int64_t n = (rows + 3) / 4 * nb;
  if (n <= 0) return cudaSuccess;
  k_q80_repack<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(raw, rows, nb, packed);
  return cudaGetLastError();
}

size_t q80_smem_bytes(int input, int rps) {
  const int64_t rb = (int64_t)input / 32 * 34;
  return (size_t)((int64_t)kQ80Stages * rps * rb + (int64_t)input * 4 + (int64_t)kQ80Consumers * 4 * (input / 32) * 4 +
                  16 * kQ80Stages + 8 * kQ80Consumers);
}

int q80_rows_per_chunk(int input) {
  // rows per stage: a multiple of 8 (16-byte aligned copies), 16 when the
  // four-stage ring fits (the per-CTA maximum is 227 KB)
  for (int rps = 16; rps >= 8; rps -= 8)
    if (q80_smem_bytes(input, rps) <= 226 * 1024) return rps;
  return 0;
}

cudaError_t launch_q80(const uint8_t *w, int64_t rows, int input, const float *x, float *y,
                       unsigned long long *best, int64_t *argmax, float *logit, int32_t *err, int sm_count,
                       cudaStream_t stream) {
  const int rpc = q80_rows_per_chunk(input);
  if (rpc <= 0 || input % 32 != 0 || rows <= 0 || rows > 0xffffffffll) return cudaErrorInvalidValue;
  const size_t smem = q80_smem_bytes(input, rpc);
  cudaError_t e = opt_in_smem(k_q80_gemv, (int)smem);
  if (e != cudaSuccess) return e;
  Q80Launch a;
  a.w = w;
  a.rows = rows;
  a.input = input;
  a.row_bytes = input / 32 * 34;
  a.blocks = input / 32;
  a.rows_per_stage = rpc;
  a.x = x;
  a.y = y;
  a.best = best;
  a.err = err;
  const int64_t chunks = (rows + rpc - 1) / rpc;
  const int grid = (int)(chunks < sm_count ? chunks : sm_count);
  if ((e = launch_pdl(k_q80_init, dim3(1), dim3(1), 0, stream, best)) != cudaSuccess) return e;
  if ((e = launch_pdl(k_q80_gemv, dim3(grid), dim3(kQ80Threads), smem, stream, a)) != cudaSuccess) return e;
  return launch_pdl(k_q80_finalize, dim3(1), dim3(1), 0, stream, (const unsigned long long *)best, argmax, logit);
}

}  // namespace spt
