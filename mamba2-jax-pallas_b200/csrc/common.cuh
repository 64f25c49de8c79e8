// Shared device helpers for the SSD kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ssd_b200.h"

namespace ssd {

typedef __nv_bfloat16 bf16;

__device__ __forceinline__ float ld(const float* p) { return *p; }
__device__ __forceinline__ float ld(const bf16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st(float* p, float v) { *p = v; }
__device__ __forceinline__ void st(bf16* p, float v) { *p = __float2bfloat16_rn(v); }

// Read-only, streaming loads (data read once).
__device__ __forceinline__ float ldg(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ldg(const bf16* p) {
  return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(p)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Inclusive warp prefix sum.
__device__ __forceinline__ float warp_incl_scan(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    float t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// dt post-processing of chunk_cumsum_fwd.py:221-226: bias, thresholded softplus, clamp.
__device__ __forceinline__ float dt_process(float v, float bias, int softplus, float lo, float hi) {
  v += bias;
  if (softplus) v = (v <= 20.f) ? log1pf(expf(v)) : v;
  return fminf(fmaxf(v, lo), hi);
}

__device__ __forceinline__ float silu(float v) { return v / (1.f + expf(-v)); }

}  // namespace ssd
