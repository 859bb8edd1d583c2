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
// The matrix (615 MB for GPT-OSS's 201,088 x 2,880 output head) streams
// through shared memory in chunks of rows_per_chunk rows, one bulk copy each,
// double-buffered; each chunk's block scales are decoded once into shared
// memory (the reference's float16 decode, NaN payloads included); each warp
// runs two rows at a time.  int8 -> float uses the exact magic-number form
// (0x4B000000 | (b ^ 0x80)) - 8388736 instead of the quarter-rate convert.
// The argmax packs (order-preserving logit bits, ~row) into 64 bits and
// keeps the maximum with atomicMax: largest logit, lowest row on ties, NaN
// never chosen, -0 equal to +0, and row 0 when nothing beats -Inf.
#include <cuda_runtime.h>
#include <stdint.h>

#include "spt_device.cuh"
#include "spt_internal.cuh"
#include "spt_ptx.cuh"

namespace spt {

namespace {

constexpr int kQ80Threads = 512;  // 16 warps, two rows each per chunk

// quantFloat16Bits (forward/quant_portable.go:20-35).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16, exponent = (h >> 10) & 31u, fraction = h & 1023u;
  uint32_t bits;
  if (exponent == 31u) {
    bits = sign | 0x7f800000u | fraction << 13;
  } else if (exponent != 0u) {
    bits = sign | (exponent + 112u) << 23 | fraction << 13;
  } else if (fraction == 0u) {
    bits = sign;
  } else {
    const uint32_t shift = (uint32_t)__clz(fraction) - 21u;
    bits = sign | (113u - shift) << 23 | ((fraction << shift) & 1023u) << 13;
  }
  return __uint_as_float(bits);
}

__device__ __forceinline__ float int8_to_f32(uint32_t byte) {
  return __fsub_rn(__uint_as_float(0x4B000000u | (byte ^ 0x80u)), 8388736.0f);
}

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
  const uint8_t *w;          // rows x row_bytes (+ at least 16 bytes of padding)
  int64_t rows;
  int input, row_bytes, blocks, rows_per_chunk;
  const float *x;            // [input]
  float *y;                  // [rows] or null
  unsigned long long *best;  // argmax key
  int32_t *err;
};

__global__ void __launch_bounds__(kQ80Threads, 1) k_q80_gemv(const __grid_constant__ Q80Launch a) {
  extern __shared__ __align__(128) uint8_t q80_smem[];
  const int rpc = a.rows_per_chunk, rb = a.row_bytes, nb = a.blocks;
  const uint32_t chunk_bytes = (uint32_t)((int64_t)rpc * rb);
  float *xs = reinterpret_cast<float *>(q80_smem + 2 * (size_t)chunk_bytes);
  float *scl = xs + a.input;                       // [rpc][nb]
  uint64_t *bar = reinterpret_cast<uint64_t *>(scl + (size_t)rpc * nb);  // [2]
  unsigned long long *wbest = reinterpret_cast<unsigned long long *>(bar + 2);  // [warps]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n_chunks = (a.rows + rpc - 1) / rpc;
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  auto issue = [&](int64_t chunk, int slot) {
    const int64_t r0 = chunk * rpc;
    const int64_t nr = a.rows - r0 < rpc ? a.rows - r0 : rpc;
    const uint32_t bytes = (uint32_t)((nr * rb + 15) & ~15ll);  // padding rows of the buffer cover the round-up
    mbar_expect_tx(&bar[slot], bytes);
    bulk_load(q80_smem + (size_t)slot * chunk_bytes, a.w + r0 * rb, bytes, &bar[slot]);
  };
  if (tid == 0) {
    if ((int64_t)blockIdx.x < n_chunks) issue(blockIdx.x, 0);
    if ((int64_t)blockIdx.x + gridDim.x < n_chunks) issue(blockIdx.x + gridDim.x, 1);
  }
  for (int i = tid; i < a.input; i += blockDim.x) xs[i] = a.x[i];
  unsigned long long best = 0ull;
  int it = 0;
  for (int64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x, ++it) {
    const int slot = it & 1;
    const uint32_t parity = (uint32_t)(it >> 1) & 1u;
    if (!mbar_wait(&bar[slot], parity, a.err, 1)) break;  // every thread waits: the buffer is shared
    const uint8_t *cb = q80_smem + (size_t)slot * chunk_bytes;
    const int64_t r0 = chunk * rpc;
    const int nr = (int)(a.rows - r0 < rpc ? a.rows - r0 : rpc);
    for (int i = tid; i < nr * nb; i += blockDim.x) {
      const int r = i / nb, b = i - r * nb;
      const uint8_t *blk = cb + (size_t)r * rb + (size_t)b * 34;
      scl[i] = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    }
    __syncthreads();
    for (int r = 2 * warp; r < nr; r += 2 * (blockDim.x >> 5)) {
      const bool two = r + 1 < nr;
      const uint8_t *q0 = cb + (size_t)r * rb + 2 + lane;
      const uint8_t *q1 = q0 + (two ? rb : 0);
      const float *s0 = scl + (size_t)r * nb;
      const float *s1 = s0 + (two ? nb : 0);
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 6
      for (int b = 0; b < nb; ++b) {
        const float xv = xs[b * 32 + lane];
        const float w0 = __fmul_rn(int8_to_f32(q0[b * 34]), s0[b]);
        const float w1 = __fmul_rn(int8_to_f32(q1[b * 34]), s1[b]);
        acc0 = fmaf(w0, xv, acc0);
        acc1 = fmaf(w1, xv, acc1);
      }
      const float y0 = reduce_chains(acc0, lane);
      const float y1 = reduce_chains(acc1, lane);
      if (lane == 0) {
        if (a.y) {
          a.y[r0 + r] = y0;
          if (two) a.y[r0 + r + 1] = y1;
        }
        if (!isnan(y0)) best = max(best, argmax_key(y0, r0 + r));
        if (two && !isnan(y1)) best = max(best, argmax_key(y1, r0 + r + 1));
      }
    }
    __syncthreads();  // buffer `slot` and the scales are free again
    if (tid == 0 && chunk + 2 * (int64_t)gridDim.x < n_chunks) issue(chunk + 2 * gridDim.x, slot);
  }
  if (lane == 0) wbest[warp] = best;
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = max(b, wbest[w]);
    if (b) atomicMax(a.best, b);
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

int q80_rows_per_chunk(int input) {
  const int64_t rb = (int64_t)input / 32 * 34;
  // two chunk buffers + x + the chunk's scales within ~200 KB; a multiple of 8
  // rows keeps every chunk start 16-byte aligned
  for (int rpc = 32; rpc >= 8; rpc -= 8) {
    const int64_t bytes = 2 * rpc * rb + (int64_t)input * 4 + (int64_t)rpc * (input / 32) * 4 + 16 + 8 * 32;
    if (bytes <= 200 * 1024) return rpc;
  }
  return 0;
}

size_t q80_smem_bytes(int input, int rpc) {
  const int64_t rb = (int64_t)input / 32 * 34;
  return (size_t)(2 * rpc * rb + (int64_t)input * 4 + (int64_t)rpc * (input / 32) * 4 + 16 +
                  8 * (kQ80Threads / 32));
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
  a.rows_per_chunk = rpc;
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
