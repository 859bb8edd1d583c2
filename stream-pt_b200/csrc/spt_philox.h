// spt_philox.h -- counter-based random numbers for the synthetic benchmark
// weights, identical on the host and the device.
//
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11): 10 rounds of two 32x32->64 multiplies with the
// published multipliers and Weyl key increments.  MXFP4 bytes are pure
// integer functions of (seed, layer, tensor, block), so a tensor generated on
// the device equals the host copy byte for byte.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define SPT_HD __host__ __device__ __forceinline__
#else
#define SPT_HD inline
#endif

namespace spt {

struct u32x4 {
  uint32_t x, y, z, w;
};

SPT_HD void mulhilo32(uint32_t a, uint32_t b, uint32_t *hi, uint32_t *lo) {
  uint64_t p = (uint64_t)a * (uint64_t)b;
  *hi = (uint32_t)(p >> 32);
  *lo = (uint32_t)p;
}

SPT_HD u32x4 philox4x32_10(u32x4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
  for (int round = 0; round < 10; ++round) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, ctr.x, &hi0, &lo0);
    mulhilo32(M1, ctr.z, &hi1, &lo1);
    u32x4 n;
    n.x = hi1 ^ ctr.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ ctr.w ^ k1;
    n.w = lo0;
    ctr = n;
    k0 += W0;
    k1 += W1;
  }
  return ctr;
}

// Tensor tags: (layer << 8) | kind.
enum SynthKind : uint32_t {
  kSynthGate = 0,
  kSynthUp = 1,
  kSynthDown = 2,
  kSynthRouter = 3,
  kSynthRouterBias = 4,
  kSynthGateBias = 5,
  kSynthUpBias = 6,
  kSynthDownBias = 7,
  kSynthZipfPerm = 8,
  kSynthNormWeight = 9,
};

SPT_HD uint32_t synth_tag(int64_t layer, uint32_t kind) {
  return ((uint32_t)layer << 8) | kind;
}

// One 17-byte GGUF MXFP4 block: byte 0 = E8M0 scale uniform in [lo, hi],
// bytes 1..16 = nibbles uniform over all 16 codes.  `block` is the block's
// linear index inside its tensor (expert-major, then row, then K).
SPT_HD void synth_mxfp4_block(uint64_t seed, uint32_t tag, uint64_t block, uint8_t lo,
                              uint8_t hi, uint8_t out[17]) {
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  u32x4 c = {(uint32_t)block, (uint32_t)(block >> 32), tag, 0u};
  u32x4 r = philox4x32_10(c, k0, k1);
  c.w = 1u;
  u32x4 s = philox4x32_10(c, k0, k1);
  uint32_t span = (uint32_t)hi - (uint32_t)lo + 1u;
  out[0] = (uint8_t)(lo + (uint32_t)(((uint64_t)s.x * span) >> 32));
  uint32_t words[4] = {r.x, r.y, r.z, r.w};
  for (int i = 0; i < 16; ++i) out[1 + i] = (uint8_t)(words[i >> 2] >> (8 * (i & 3)));
}

// Two uniform 32-bit words for element `index` of a float tensor.
SPT_HD void synth_uniform_pair(uint64_t seed, uint32_t tag, uint64_t index, uint32_t *a,
                               uint32_t *b) {
  u32x4 c = {(uint32_t)index, (uint32_t)(index >> 32), tag, 2u};
  u32x4 r = philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  *a = r.x;
  *b = r.y;
}

}  // namespace spt
