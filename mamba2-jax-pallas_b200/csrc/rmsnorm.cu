// Gated RMSNorm over groups of the last axis (ops/rms_norm.py:15-92), the step after the
// SSD in a Mamba2 layer (modules/mamba2.py:401-406).
//
//   norm_before_gate:  out = x / sqrt(mean_g(x^2) + eps) * w * silu(z)
//   otherwise:         v = x * silu(z);  out = v / sqrt(mean_g(v^2) + eps) * w
//
// Pure HBM stream: x (and z) read once, out written once.  One warp owns one (row, group);
// in the layer the group is one SSD group's heads (H/G * P = 1024 values at the
// nemotron-h-8b shape), so a warp's whole group fits in registers: the fast kernel issues
// every 16-byte load of the group before reducing, then scales the registers and stores.
// Groups that are not a multiple of 256 values, or unaligned rows, take a two-pass kernel
// (the second pass re-reads the group from L1/L2).
#include "common.cuh"
#include "ssd_kernels.h"

namespace ssd {

namespace {

constexpr int RN_THREADS = 256;   // 8 warps = 8 groups per block
constexpr int RN_CHUNK = 8;       // values per lane per chunk (16 B of bf16, 32 B of f32)

struct RnArgs {
  int64_t units, ngroups, gs;
  int64_t xs, zs, os;
  float eps;
  int nbg;
  const void* x;
  const void* z;
  const void* w;
  void* out;
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[RN_CHUNK]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[2 * k] = __uint_as_float(u[k] << 16);
      v[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[RN_CHUNK]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      u[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 1 / sqrt(mean + eps), with IEEE sqrt and division: the reference divides x by the RMS
__device__ __forceinline__ float inv_rms(float sumsq, int64_t gs, float eps) {
  return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)gs), eps)));
}

// Fast path: NCH chunks of 8 values per lane, all loads issued before the reduction.
// Lane l owns values [(c*32 + l)*8, +8) of its group for c < NCH: a warp-wide chunk is 256
// contiguous values, so every load instruction of the warp is fully coalesced.
template <typename TX, typename TZ, typename TW, typename TO, int NCH, bool HAS_Z>
__global__ void __launch_bounds__(RN_THREADS) rmsnorm_cached_kernel(const RnArgs a) {
  const int64_t unit = (int64_t)blockIdx.x * (RN_THREADS / 32) + threadIdx.x / 32;
  if (unit >= a.units) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = unit / a.ngroups, g = unit - row * a.ngroups;
  const int64_t col0 = g * a.gs;
  const TX* xp = (const TX*)a.x + row * a.xs + col0;
  const TZ* zp = HAS_Z ? (const TZ*)a.z + row * a.zs + col0 : nullptr;
  float v[NCH][RN_CHUNK], zv[HAS_Z ? NCH : 1][RN_CHUNK];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t off = (int64_t)(c * 32 + lane) * RN_CHUNK;
    load8(xp + off, v[c]);
    if constexpr (HAS_Z) load8(zp + off, zv[c]);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int k = 0; k < RN_CHUNK; ++k) {
      if constexpr (HAS_Z) {
        zv[c][k] = silu(zv[c][k]);
        if (!a.nbg) { v[c][k] *= zv[c][k]; zv[c][k] = 1.f; }
      }
      ss = fmaf(v[c][k], v[c][k], ss);
    }
  }
  const float r = inv_rms(warp_sum(ss), a.gs, a.eps);
  const TW* wp = (const TW*)a.w + col0;
  TO* op = (TO*)a.out + row * a.os + col0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t off = (int64_t)(c * 32 + lane) * RN_CHUNK;
    float w[RN_CHUNK];
    load8(wp + off, w);
#pragma unroll
    for (int k = 0; k < RN_CHUNK; ++k) {
      float o = v[c][k] * r * w[k];
      if constexpr (HAS_Z) o *= zv[c][k];
      v[c][k] = o;
    }
    store8(op + off, v[c]);
  }
}

__device__ __forceinline__ float ld(const void* p, int dtype, int64_t i) {
  if (dtype == SSD_DTYPE_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
  return ((const float*)p)[i];
}

// General path: any group size and alignment; two passes over the group.
__global__ void __launch_bounds__(RN_THREADS) rmsnorm_generic_kernel(const RnArgs a, int xd, int zd,
                                                                     int wd, int od) {
  const int64_t unit = (int64_t)blockIdx.x * (RN_THREADS / 32) + threadIdx.x / 32;
  if (unit >= a.units) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = unit / a.ngroups, g = unit - row * a.ngroups;
  const int64_t col0 = g * a.gs;
  const int64_t xo = row * a.xs + col0, zo = row * a.zs + col0, oo = row * a.os + col0;
  const bool gate = a.z != nullptr;
  float ss = 0.f;
  for (int64_t i = lane; i < a.gs; i += 32) {
    float v = ld(a.x, xd, xo + i);
    if (gate && !a.nbg) v *= silu(ld(a.z, zd, zo + i));
    ss = fmaf(v, v, ss);
  }
  const float r = inv_rms(warp_sum(ss), a.gs, a.eps);
  for (int64_t i = lane; i < a.gs; i += 32) {
    float v = ld(a.x, xd, xo + i);
    float gz = gate ? silu(ld(a.z, zd, zo + i)) : 1.f;
    if (gate && !a.nbg) { v *= gz; gz = 1.f; }
    const float o = v * r * ld(a.w, wd, col0 + i) * gz;
    if (od == SSD_DTYPE_BF16) ((__nv_bfloat16*)a.out)[oo + i] = __float2bfloat16_rn(o);
    else ((float*)a.out)[oo + i] = o;
  }
}

template <typename TX, typename TZ, typename TW, typename TO, bool HAS_Z>
cudaError_t launch_cached(const RnArgs& a, int nch, dim3 grid, cudaStream_t st) {
  switch (nch) {
    case 1: rmsnorm_cached_kernel<TX, TZ, TW, TO, 1, HAS_Z><<<grid, RN_THREADS, 0, st>>>(a); break;
    case 2: rmsnorm_cached_kernel<TX, TZ, TW, TO, 2, HAS_Z><<<grid, RN_THREADS, 0, st>>>(a); break;
    case 4: rmsnorm_cached_kernel<TX, TZ, TW, TO, 4, HAS_Z><<<grid, RN_THREADS, 0, st>>>(a); break;
    default: rmsnorm_cached_kernel<TX, TZ, TW, TO, 8, HAS_Z><<<grid, RN_THREADS, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

template <typename TX, typename TW, typename TO>
cudaError_t dispatch_z(const RnArgs& a, int zd, int nch, dim3 grid, cudaStream_t st) {
  if (a.z == nullptr) return launch_cached<TX, float, TW, TO, false>(a, nch, grid, st);
  if (zd == SSD_DTYPE_BF16) return launch_cached<TX, __nv_bfloat16, TW, TO, true>(a, nch, grid, st);
  return launch_cached<TX, float, TW, TO, true>(a, nch, grid, st);
}

template <typename TX, typename TW>
cudaError_t dispatch_o(const RnArgs& a, int zd, int od, int nch, dim3 grid, cudaStream_t st) {
  if (od == SSD_DTYPE_BF16) return dispatch_z<TX, TW, __nv_bfloat16>(a, zd, nch, grid, st);
  return dispatch_z<TX, TW, float>(a, zd, nch, grid, st);
}

bool aligned16(const void* p, int64_t row_stride, int dtype) {
  const int64_t es = dtype == SSD_DTYPE_BF16 ? 2 : 4;
  return ((uintptr_t)p % 16 == 0) && ((row_stride * es) % 16 == 0);
}

}  // namespace

cudaError_t launch_rms_norm_gated(const ssd_rms_norm_params_t* p, cudaStream_t st) {
  RnArgs a;
  a.ngroups = p->hidden / p->group_size;
  a.units = p->rows * a.ngroups;
  a.gs = p->group_size;
  a.xs = p->x_stride_row; a.zs = p->z_stride_row; a.os = p->out_stride_row;
  a.eps = p->eps; a.nbg = p->norm_before_gate;
  a.x = p->x; a.z = p->z; a.w = p->weight; a.out = p->out;
  const dim3 grid((unsigned)((a.units + RN_THREADS / 32 - 1) / (RN_THREADS / 32)));
  const int64_t nch = a.gs / (32 * RN_CHUNK);
  const bool fast = a.gs % (32 * RN_CHUNK) == 0 && (nch == 1 || nch == 2 || nch == 4 || nch == 8) &&
                    aligned16(p->x, a.xs, p->x_dtype) && aligned16(p->out, a.os, p->out_dtype) &&
                    aligned16(p->weight, 0, p->weight_dtype) &&
                    (p->z == nullptr || aligned16(p->z, a.zs, p->z_dtype));
  if (!fast) {
    rmsnorm_generic_kernel<<<grid, RN_THREADS, 0, st>>>(a, p->x_dtype, p->z_dtype, p->weight_dtype,
                                                        p->out_dtype);
    return cudaGetLastError();
  }
  const int n = (int)nch;
  const bool xb = p->x_dtype == SSD_DTYPE_BF16, wb = p->weight_dtype == SSD_DTYPE_BF16;
  if (xb && wb) return dispatch_o<__nv_bfloat16, __nv_bfloat16>(a, p->z_dtype, p->out_dtype, n, grid, st);
  if (xb) return dispatch_o<__nv_bfloat16, float>(a, p->z_dtype, p->out_dtype, n, grid, st);
  if (wb) return dispatch_o<float, __nv_bfloat16>(a, p->z_dtype, p->out_dtype, n, grid, st);
  return dispatch_o<float, float>(a, p->z_dtype, p->out_dtype, n, grid, st);
}

}  // namespace ssd
