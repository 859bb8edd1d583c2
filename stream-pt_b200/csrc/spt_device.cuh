// spt_device.cuh -- device helpers shared by the CUDA-core and tensor-core
// kernels.
#pragma once
#include <cuda_runtime.h>
#include <math.h>

namespace spt {

// Go's builtin min/max on floats propagate NaN (forward/moe.go:67-68).
__device__ __forceinline__ float go_min(float a, float b) {
  return (isnan(a) || isnan(b)) ? __int_as_float(0x7fffffff) : (a < b ? a : b);
}
__device__ __forceinline__ float go_max(float a, float b) {
  return (isnan(a) || isnan(b)) ? __int_as_float(0x7fffffff) : (a > b ? a : b);
}

// gptOSSSwiGLU (forward/moe.go:66-70): f32 clamp, f32 -1.702*g, f64 exp
// rounded to f32, then g / (1+e) * (u+1) left to right.
__device__ __forceinline__ float swiglu_ref(float g, float u) {
  g = go_min(g, 7.0f);
  u = go_max(-7.0f, go_min(u, 7.0f));
  const float t = __fmul_rn(-1.702f, g);
  const float e = (float)exp((double)t);
  const float d = __fadd_rn(1.0f, e);
  return __fmul_rn(__fdiv_rn(g, d), __fadd_rn(u, 1.0f));
}

// The same activation with the fast float exponential and division
// intrinsics (relative error about 1e-6): for the tensor-core path, whose
// products already differ from the reference's by about 1e-4 of each block.
__device__ __forceinline__ float swiglu_f32(float g, float u) {
  g = go_min(g, 7.0f);
  u = go_max(-7.0f, go_min(u, 7.0f));
  const float e = __expf(-1.702f * g);
  return __fdividef(g, 1.0f + e) * (u + 1.0f);
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may begin while its predecessor is still
// running.  pdl_wait() returns once the predecessor grid has completed and
// its memory operations are visible (immediately when there is no such
// dependency); pdl_trigger() then lets the next kernel start launching.  Every
// forward-path kernel calls both, in that order, before touching global
// memory, so at most two consecutive kernels overlap and each reads only
// completed results.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace spt
