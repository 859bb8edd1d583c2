// spt_ptx.cuh -- small sm_100a PTX helpers shared by the kernels that stage
// data with bulk copies: mbarriers with a bounded wait, and the untiled bulk
// copy global -> shared memory.
#pragma once
#include <stdint.h>

namespace spt {
namespace {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~2^shift clock cycles (2^31: about a second
// at the B200's clock) and records `code` in err.  It also gives up at once
// when another role of the kernel has recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int32_t *err, int code, int shift = 31) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (*(volatile int32_t *)err != 0) return false;  // another role already gave up
      if (clock64() - t0 > (1ll << shift)) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// Bounded wait for work this thread started itself (copies or tensor-core
// operations in flight) on the way out after an error: unlike mbar_wait it
// does not stop when an error is recorded, only after ~2^shift clocks.
__device__ __forceinline__ bool mbar_wait_own(uint64_t *bar, uint32_t parity, int shift = 31) {
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0u && clock64() - t0 > (1ll << shift)) return false;
  }
}

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte asynchronous copy global -> shared memory (L2 only).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

}  // namespace
}  // namespace spt
