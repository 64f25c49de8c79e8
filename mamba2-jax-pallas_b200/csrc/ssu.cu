// Single-token decode step: selective_state_update (ops/selective_state_update.py:22-123).
//
//   dt' = softplus(dt + dt_bias)                 (jax.nn.softplus: log(1 + e^v))
//   state <- state * exp(dt' * A) + dt' * B * x  (in place)
//   out = sum_n state * C + D * x;  out *= silu(z)
//
// Pure HBM stream: the (b,H,P,N) f32 state is read once and written once.  One CTA
// per (batch, head); each warp owns rows p, each lane a 16-byte column slice, and
// R rows are loaded before any is used so every lane keeps R x 16 B in flight.
#include "common.cuh"
#include "ssd_kernels.h"

namespace ssd {

namespace {

constexpr int SSU_THREADS = 256;
constexpr int SSU_R = 8;

struct SsuArgs {
  int64_t H, P, G, N;
  int dt_ndim, A_ndim, D_ndim, bias_ndim, softplus;
  float* state;
  const void* x;
  const void* dt;
  const float* A;
  const void* B;
  const void* C;
  const float* D;
  const void* z;
  const float* dt_bias;
  float* out;
};

__device__ __forceinline__ float softplus_jax(float v) {
  return fmaxf(v, 0.f) + log1pf(expf(-fabsf(v)));
}

template <typename T, typename TDT, bool VEC>
__global__ void __launch_bounds__(SSU_THREADS) ssu_kernel(const SsuArgs a) {
  extern __shared__ float sm[];
  float* Bs = sm;
  float* Cs = sm + a.N;
  const int64_t bh = blockIdx.x;
  const int64_t bi = bh / a.H, h = bh % a.H;
  const int64_t g = h / (a.H / a.G);
  const T* Bp = (const T*)a.B + (bi * a.G + g) * a.N;
  const T* Cp = (const T*)a.C + (bi * a.G + g) * a.N;
  for (int n = threadIdx.x; n < a.N; n += SSU_THREADS) {
    Bs[n] = ldg(Bp + n);
    Cs[n] = ldg(Cp + n);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = SSU_THREADS / 32;
  float* S = a.state + bh * a.P * a.N;
  const float Ah = a.A_ndim == 1 ? a.A[h] : 0.f;
  for (int64_t p0 = (int64_t)warp * SSU_R; p0 < a.P; p0 += (int64_t)NW * SSU_R) {
    float dtv[SSU_R], xv[SSU_R], dAv[SSU_R], acc[SSU_R];
#pragma unroll
    for (int r = 0; r < SSU_R; ++r) {
      const int64_t p = min(p0 + r, a.P - 1);
      float d = a.dt_ndim == 2 ? ldg((const TDT*)a.dt + bh) : ldg((const TDT*)a.dt + bh * a.P + p);
      if (a.bias_ndim == 1) d += a.dt_bias[h];
      else if (a.bias_ndim == 2) d += a.dt_bias[h * a.P + p];
      if (a.softplus) d = softplus_jax(d);
      dtv[r] = d;
      xv[r] = ldg((const T*)a.x + bh * a.P + p);
      dAv[r] = expf(d * Ah);
      acc[r] = 0.f;
    }
    if (VEC) {
      const int64_t N4 = a.N >> 2;
      for (int64_t n4 = lane; n4 < N4; n4 += 32) {
        float4 s[SSU_R];
#pragma unroll
        for (int r = 0; r < SSU_R; ++r)
          if (p0 + r < a.P) s[r] = __ldcs(reinterpret_cast<const float4*>(S + (p0 + r) * a.N) + n4);
        const float4 bv = reinterpret_cast<const float4*>(Bs)[n4];
        const float4 cv = reinterpret_cast<const float4*>(Cs)[n4];
#pragma unroll
        for (int r = 0; r < SSU_R; ++r) {
          if (p0 + r >= a.P) continue;
          float4 da;
          if (a.A_ndim == 1) {
            da = make_float4(dAv[r], dAv[r], dAv[r], dAv[r]);
          } else {
            const float4 av = reinterpret_cast<const float4*>(a.A + (h * a.P + p0 + r) * a.N)[n4];
            da = make_float4(expf(dtv[r] * av.x), expf(dtv[r] * av.y), expf(dtv[r] * av.z), expf(dtv[r] * av.w));
          }
          const float dx = dtv[r] * xv[r];
          float4 o;
          o.x = s[r].x * da.x + dx * bv.x;
          o.y = s[r].y * da.y + dx * bv.y;
          o.z = s[r].z * da.z + dx * bv.z;
          o.w = s[r].w * da.w + dx * bv.w;
          __stcs(reinterpret_cast<float4*>(S + (p0 + r) * a.N) + n4, o);
          acc[r] += o.x * cv.x + o.y * cv.y + o.z * cv.z + o.w * cv.w;
        }
      }
    } else {
      for (int64_t n = lane; n < a.N; n += 32) {
#pragma unroll
        for (int r = 0; r < SSU_R; ++r) {
          if (p0 + r >= a.P) continue;
          float* sp = S + (p0 + r) * a.N + n;
          const float da = a.A_ndim == 1 ? dAv[r] : expf(dtv[r] * a.A[(h * a.P + p0 + r) * a.N + n]);
          const float o = *sp * da + dtv[r] * xv[r] * Bs[n];
          *sp = o;
          acc[r] += o * Cs[n];
        }
      }
    }
#pragma unroll
    for (int r = 0; r < SSU_R; ++r) {
      const float v = warp_sum(acc[r]);
      const int64_t p = p0 + r;
      if (lane == r && p < a.P) {
        float o = v;
        if (a.D_ndim == 1) o += a.D[h] * xv[r];
        else if (a.D_ndim == 2) o += a.D[h * a.P + p] * xv[r];
        if (a.z) o *= silu(ldg((const T*)a.z + bh * a.P + p));
        a.out[bh * a.P + p] = o;
      }
    }
  }
}


// Fast path for the common decode shapes (N % 128 == 0, P % 8 == 0, A / dt / D / dt_bias
// per head).  Each warp owns 8 state rows and issues every load it needs before any math:
// 8 x 16 B of state per lane (per 128 state columns), its slice of B and C, the 8 x values
// as one vector load and the head's dt.  No shared memory, no block barrier, ~64 registers,
// so several CTAs per SM keep enough bytes in flight to stream the state at HBM rate.
template <typename T, typename TDT, int NV>
__global__ void __launch_bounds__(SSU_THREADS) ssu_fast_kernel(const SsuArgs a) {
  const int64_t bh = blockIdx.x;
  const int64_t bi = bh / a.H, h = bh % a.H;
  const int64_t g = h / (a.H / a.G);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = SSU_THREADS / 32;
  const float Ah = a.A[h];
  const float bias = a.bias_ndim ? a.dt_bias[h] : 0.f;
  const float Dh = a.D_ndim ? a.D[h] : 0.f;
  float d = ldg((const TDT*)a.dt + bh) + bias;
  if (a.softplus) d = softplus_jax(d);
  const float dA = expf(d * Ah);
  float Bv[NV][4], Cv[NV][4];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int64_t n0 = (int64_t)(v * 32 + lane) * 4;
    const T* Bp = (const T*)a.B + (bi * a.G + g) * a.N + n0;
    const T* Cp = (const T*)a.C + (bi * a.G + g) * a.N + n0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      Bv[v][i] = ldg(Bp + i);
      Cv[v][i] = ldg(Cp + i);
    }
  }
  for (int64_t p0 = (int64_t)warp * 8; p0 < a.P; p0 += (int64_t)NW * 8) {
    float* S = a.state + (bh * a.P + p0) * a.N;
    float4 s[8][NV];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v) s[r][v] = __ldcs(reinterpret_cast<const float4*>(S + r * a.N) + v * 32 + lane);
    float xv[8], zv[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      xv[r] = ldg((const T*)a.x + bh * a.P + p0 + r);
      zv[r] = a.z ? ldg((const T*)a.z + bh * a.P + p0 + r) : 0.f;
    }
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float dx = d * xv[r];
      float t = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float4 o;
        o.x = fmaf(s[r][v].x, dA, dx * Bv[v][0]);
        o.y = fmaf(s[r][v].y, dA, dx * Bv[v][1]);
        o.z = fmaf(s[r][v].z, dA, dx * Bv[v][2]);
        o.w = fmaf(s[r][v].w, dA, dx * Bv[v][3]);
        __stcs(reinterpret_cast<float4*>(S + r * a.N) + v * 32 + lane, o);
        t += o.x * Cv[v][0] + o.y * Cv[v][1] + o.z * Cv[v][2] + o.w * Cv[v][3];
      }
      acc[r] = t;
    }
    // reduce the 8 row sums across the warp; lane r ends with row r's total
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] = warp_sum(acc[r]);
    if (lane < 8) {
      float o = acc[0], xo = xv[0], zo = zv[0];
#pragma unroll
      for (int r = 1; r < 8; ++r)
        if (lane == r) {
          o = acc[r];
          xo = xv[r];
          zo = zv[r];
        }
      o += Dh * xo;
      if (a.z) o *= silu(zo);
      a.out[bh * a.P + p0 + lane] = o;
    }
  }
}

template <typename T, typename TDT>
void ssu_launch_t(const SsuArgs& a, int64_t grid, bool vec, cudaStream_t st) {
  const size_t smem = 2 * a.N * sizeof(float);
  const bool fast = vec && a.A_ndim == 1 && a.dt_ndim == 2 && a.D_ndim <= 1 && a.bias_ndim <= 1 &&
                    a.P % 8 == 0 && (a.N == 128 || a.N == 256);
  if (fast) {
    if (a.N == 128) ssu_fast_kernel<T, TDT, 1><<<(unsigned)grid, SSU_THREADS, 0, st>>>(a);
    else ssu_fast_kernel<T, TDT, 2><<<(unsigned)grid, SSU_THREADS, 0, st>>>(a);
  } else if (vec)
    ssu_kernel<T, TDT, true><<<(unsigned)grid, SSU_THREADS, smem, st>>>(a);
  else
    ssu_kernel<T, TDT, false><<<(unsigned)grid, SSU_THREADS, smem, st>>>(a);
}

}  // namespace

cudaError_t launch_ssu(const ssu_params_t* p, cudaStream_t st) {
  SsuArgs a;
  a.H = p->nheads; a.P = p->headdim; a.G = p->ngroups; a.N = p->dstate;
  a.dt_ndim = p->dt_ndim; a.A_ndim = p->A_ndim; a.D_ndim = p->D_ndim;
  a.bias_ndim = p->dt_bias ? p->dt_bias_ndim : 0; a.softplus = p->dt_softplus;
  a.state = p->state; a.x = p->x; a.dt = p->dt; a.A = p->A; a.B = p->B; a.C = p->C;
  a.D = p->D_ndim ? p->D : nullptr; a.z = p->z; a.dt_bias = p->dt_bias; a.out = p->out;
  const bool vec = (a.N % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.state) & 15) == 0) &&
                   (a.A_ndim == 1 || (reinterpret_cast<uintptr_t>(a.A) & 15) == 0);
  const int64_t grid = p->batch * p->nheads;
  if (p->dtype == SSD_DTYPE_BF16) {
    if (p->dt_dtype == SSD_DTYPE_BF16) ssu_launch_t<bf16, bf16>(a, grid, vec, st);
    else ssu_launch_t<bf16, float>(a, grid, vec, st);
  } else {
    if (p->dt_dtype == SSD_DTYPE_BF16) ssu_launch_t<float, bf16>(a, grid, vec, st);
    else ssu_launch_t<float, float>(a, grid, vec, st);
  }
  return cudaGetLastError();
}

}  // namespace ssd
