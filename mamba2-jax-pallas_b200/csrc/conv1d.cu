// Causal depthwise conv1d over time (causal_conv1d.py:18-85) and its decode step
// (causal_conv1d.py:88-139).
//
//   xm[b,d,t]  = x[b,d,t] * keep[b,t]       keep = seq_idx constant on [t, t+width-1]
//   out[b,d,t] = act(bias[d] + sum_j w[d,j] xm[b,d,t-(width-1)+j])   (xm = 0 before t = 0)
//
// keep restates _mask_sequence_boundaries (causal_conv1d.py:143-193): x[t] is zeroed when
// any of positions t+1 .. t+width-1 (below seqlen) holds a different id than the position
// before it, i.e. unless seq_idx is constant on [t, min(t+width-1, L-1)].
//
// Pure HBM stream: every input is read once and every output written once.  The layer's
// activations are channels-last ((b, L, dim) with the conv over L), so the main kernel
// walks a run of tokens per thread with 16 bytes of adjacent channels per load (coalesced
// across the warp), keeps the last width-1 inputs in registers and has the run's keep mask
// in shared memory.  Other layouts take a one-thread-per-output kernel.
#include "common.cuh"
#include "ptx_sm100.cuh"
#include "ssd_kernels.h"

namespace ssd {

namespace {

constexpr int CL_THREADS = 128;
constexpr int CL_RUN = 16;      // tokens per thread, all loaded up front
constexpr int GEN_THREADS = 256;
constexpr int MAX_WIDTH = 8;

struct ConvArgs {
  int64_t dim, L;
  int64_t xb, xd, xt, ob, od, ot;   // element strides
  int width, silu;
  const void* x;
  const void* w;
  const void* bias;
  int w_bf16, b_bf16;       // weight / bias stored as bf16 (else f32)
  const int32_t* seq;
  void* out;
};

__device__ __forceinline__ float act(float v, int silu_on) { return silu_on ? silu(v) : v; }

// silu(v) = v sigmoid(v) = 0.5 v (1 + tanh(v / 2)), with one tanh.approx
__device__ __forceinline__ float silu_tanh(float v) {
  const float h = 0.5f * v;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

// keep[t] for one batch row: seq constant on [t, min(t + width - 1, L - 1)]
__device__ __forceinline__ float keep_at(const int32_t* seq_row, int64_t t, int64_t L, int width) {
  if (seq_row == nullptr) return 1.f;
  const int32_t s0 = seq_row[t];
  for (int j = 1; j < width; ++j) {
    if (t + j >= L) break;
    if (seq_row[t + j] != s0) return 0.f;
  }
  return 1.f;
}

template <typename TO, int V>
__device__ __forceinline__ void store_vec(TO* p, const float (&v)[V]) {
  if constexpr (sizeof(TO) == 4) {
#pragma unroll
    for (int k = 0; k < V; k += 4)
      *reinterpret_cast<float4*>(p + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < V; k += 8) {
      uint32_t u[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[k + 2 * i], v[k + 2 * i + 1]);
        u[i] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(p + k) = make_uint4(u[0], u[1], u[2], u[3]);
    }
  }
}

// Scalar weight / bias element as f32 (bf16 or f32 storage).
__device__ __forceinline__ float wld(const void* p, int is_bf16, int64_t i) {
  return is_bf16 ? __bfloat162float(__ldg(reinterpret_cast<const bf16*>(p) + i))
                 : __ldg(reinterpret_cast<const float*>(p) + i);
}

// N contiguous weights as f32, 4 per load (8 bytes of bf16 or 16 bytes of f32); N % 4 == 0
// and the start 8- (bf16) or 16-byte (f32) aligned.
template <int N>
__device__ __forceinline__ void wld_vec(const void* p, int is_bf16, int64_t off, float (&v)[N]) {
  if (is_bf16) {
    const uint2* q = reinterpret_cast<const uint2*>(reinterpret_cast<const bf16*>(p) + off);
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const uint2 u = __ldg(q + i);
      v[4 * i] = __uint_as_float(u.x << 16); v[4 * i + 1] = __uint_as_float(u.x & 0xffff0000u);
      v[4 * i + 2] = __uint_as_float(u.y << 16); v[4 * i + 3] = __uint_as_float(u.y & 0xffff0000u);
    }
  } else {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + off);
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 t = __ldg(q + i);
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
  }
}

// 16 bytes of x as V floats
template <typename T, int V>
__device__ __forceinline__ void unpack_vec(const uint4 q, float (&v)[V]) {
  if constexpr (sizeof(T) == 4) {
    v[0] = __uint_as_float(q.x); v[1] = __uint_as_float(q.y);
    v[2] = __uint_as_float(q.z); v[3] = __uint_as_float(q.w);
  } else {
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[2 * k] = __uint_as_float(u[k] << 16);
      v[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
}

// Channels-last: x and out have unit channel stride.  Thread = V adjacent channels (16
// bytes of x) over CL_RUN tokens; grid (channel blocks, token runs, batch).  Every load of
// the run (CL_RUN + W - 1 tokens of 16 bytes) is issued before the first output is
// computed, so a thread has ~300 bytes in flight; the runs are short so that the grid is
// several waves deep (the c2 layer: 2560 blocks) and its last wave is a small share.
template <typename T, typename TO, int W>
__global__ void __launch_bounds__(CL_THREADS) conv1d_cl_kernel(const ConvArgs a) {
  constexpr int V = 16 / sizeof(T);
  constexpr int NL = CL_RUN + W - 1;
  __shared__ float keep[NL];
  const int64_t bi = blockIdx.z;
  const int64_t t0 = (int64_t)blockIdx.y * CL_RUN;
  const int64_t nt = min((int64_t)CL_RUN, a.L - t0);
  const int32_t* seq_row = a.seq ? a.seq + bi * a.L : nullptr;
  // keep for tokens t0-(W-1) .. t0+nt-1 (0 before the sequence start: causal zero padding)
  for (int i = threadIdx.x; i < NL; i += CL_THREADS) {
    const int64_t t = t0 - (W - 1) + i;
    keep[i] = (t < 0 || i >= nt + W - 1) ? 0.f : keep_at(seq_row, t, a.L, W);
  }
  const int64_t c0 = ((int64_t)blockIdx.x * CL_THREADS + threadIdx.x) * V;
  const bool active = c0 < a.dim;
  const T* xp = (const T*)a.x + bi * a.xb + (active ? c0 : 0);
  uint4 raw[NL];
#pragma unroll
  for (int i = 0; i < NL; ++i) {
    // clamped, unconditional loads (a conditional load would wait at its merge)
    const int64_t t = min(max(t0 - (W - 1) + i, (int64_t)0), a.L - 1);
    raw[i] = __ldg(reinterpret_cast<const uint4*>(xp + t * a.xt));
  }
  // this thread's V*W weights and V biases are contiguous: 16-byte loads (scalar loads at
  // a 4*W-float lane stride cost one L1 wavefront per lane and saturated L1)
  float w[V][W], bias[V];
  {
    const int64_t cw = active ? c0 : 0;
    float wf[V * W];
    wld_vec<V * W>(a.w, a.w_bf16, cw * W, wf);
#pragma unroll
    for (int k = 0; k < V; ++k)
#pragma unroll
      for (int j = 0; j < W; ++j) w[k][j] = wf[k * W + j];
    float bf[V];
    if (a.bias) {
      wld_vec<V>(a.bias, a.b_bf16, cw, bf);
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k) bf[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < V; ++k) bias[k] = bf[k];
  }
  __syncthreads();
  if (!active) return;
  TO* op = (TO*)a.out + bi * a.ob + c0;
  // window of the W-1 masked inputs before the current token
  float win[W > 1 ? W - 1 : 1][V];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) {
    float v[V];
    unpack_vec<T, V>(raw[j], v);
#pragma unroll
    for (int k = 0; k < V; ++k) win[j][k] = t0 - (W - 1) + j < 0 ? 0.f : v[k] * keep[j];
  }
#pragma unroll
  for (int i = 0; i < CL_RUN; ++i) {
    if (i >= nt) break;
    const float kc = keep[i + W - 1];
    float xv[V], o[V];
    unpack_vec<T, V>(raw[i + W - 1], xv);
    // channel pairs on the packed f32x2 units (each lane of fma.rn.f32x2 rounds as fmaf
    // does, so the sums equal the scalar form bit for bit)
#pragma unroll
    for (int k = 0; k < V; k += 2) {
      const float2 xc = ptx::mul2(make_float2(xv[k], xv[k + 1]), make_float2(kc, kc));
      float2 acc = make_float2(bias[k], bias[k + 1]);
#pragma unroll
      for (int j = 0; j < W - 1; ++j)
        acc = ptx::fma2(make_float2(w[k][j], w[k + 1][j]), make_float2(win[j][k], win[j][k + 1]), acc);
      acc = ptx::fma2(make_float2(w[k][W - 1], w[k + 1][W - 1]), xc, acc);
      if constexpr (sizeof(TO) == 2) {
        // bf16 out: SiLU by one tanh.approx (relative error about 2^-11, well inside the
        // output's rounding); f32 out keeps the exact form
        o[k] = a.silu ? silu_tanh(acc.x) : acc.x;
        o[k + 1] = a.silu ? silu_tanh(acc.y) : acc.y;
      } else {
        o[k] = act(acc.x, a.silu);
        o[k + 1] = act(acc.y, a.silu);
      }
#pragma unroll
      for (int j = 0; j + 1 < W - 1; ++j) {
        win[j][k] = win[j + 1][k];
        win[j][k + 1] = win[j + 1][k + 1];
      }
      if (W > 1) {
        win[W > 1 ? W - 2 : 0][k] = xc.x;
        win[W > 1 ? W - 2 : 0][k + 1] = xc.y;
      }
    }
    store_vec<TO, V>(op + (t0 + i) * a.ot, o);
  }
}

// Any strides: one thread per output element.
template <typename T, typename TO>
__global__ void __launch_bounds__(GEN_THREADS) conv1d_generic_kernel(const ConvArgs a, int64_t total) {
  const int64_t idx = (int64_t)blockIdx.x * GEN_THREADS + threadIdx.x;
  if (idx >= total) return;
  const int64_t t = idx % a.L, d = (idx / a.L) % a.dim, bi = idx / (a.L * a.dim);
  const int32_t* seq_row = a.seq ? a.seq + bi * a.L : nullptr;
  const T* xp = (const T*)a.x + bi * a.xb + d * a.xd;
  float acc = a.bias ? wld(a.bias, a.b_bf16, d) : 0.f;
  for (int j = 0; j < a.width; ++j) {
    const int64_t s = t - (a.width - 1) + j;
    if (s < 0) continue;
    acc = fmaf(wld(a.w, a.w_bf16, d * a.width + j), ldg(xp + s * a.xt) * keep_at(seq_row, s, a.L, a.width), acc);
  }
  st((TO*)a.out + bi * a.ob + d * a.od + t * a.ot, act(acc, a.silu));
}

struct UpdArgs {
  int64_t batch, dim, sb, sd;
  int width, silu;
  const void* x;
  void* state;
  const void* w;
  const void* bias;
  int w_bf16, b_bf16;
  void* out;
};

template <typename TX, typename TS, typename TO>
__global__ void __launch_bounds__(GEN_THREADS) conv1d_update_kernel(const UpdArgs a) {
  const int64_t idx = (int64_t)blockIdx.x * GEN_THREADS + threadIdx.x;
  if (idx >= a.batch * a.dim) return;
  const int64_t bi = idx / a.dim, d = idx % a.dim;
  TS* s = (TS*)a.state + bi * a.sb + d * a.sd;
  float v[MAX_WIDTH];
#pragma unroll
  for (int j = 0; j < MAX_WIDTH; ++j)
    if (j + 1 < a.width) v[j] = ld(s + j + 1);
  {
    // the new input as the state stores it (the output reads the stored values)
    TS xs;
    st(&xs, ldg((const TX*)a.x + idx));
    v[a.width - 1 < MAX_WIDTH ? a.width - 1 : 0] = ld(&xs);
  }
  float acc = a.bias ? wld(a.bias, a.b_bf16, d) : 0.f;
#pragma unroll
  for (int j = 0; j < MAX_WIDTH; ++j) {
    if (j < a.width) {
      st(s + j, v[j]);
      acc = fmaf(wld(a.w, a.w_bf16, d * a.width + j), v[j], acc);
    }
  }
  st((TO*)a.out + idx, act(acc, a.silu));
}

template <typename T, typename TO>
cudaError_t launch_cl(const ConvArgs& a, int64_t batch, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const dim3 grid((unsigned)((a.dim / V + CL_THREADS - 1) / CL_THREADS), (unsigned)((a.L + CL_RUN - 1) / CL_RUN),
                  (unsigned)batch);
  switch (a.width) {
    case 1: conv1d_cl_kernel<T, TO, 1><<<grid, CL_THREADS, 0, st>>>(a); break;
    case 2: conv1d_cl_kernel<T, TO, 2><<<grid, CL_THREADS, 0, st>>>(a); break;
    case 3: conv1d_cl_kernel<T, TO, 3><<<grid, CL_THREADS, 0, st>>>(a); break;
    case 4: conv1d_cl_kernel<T, TO, 4><<<grid, CL_THREADS, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T, typename TO>
cudaError_t launch_conv_typed(const ConvArgs& a, int64_t batch, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  // the vector store writes 16 bytes of bf16 at a time: f32 in, bf16 out is not vectorised
  if constexpr (sizeof(TO) == 4 || V % 8 == 0) {
    const bool cl = a.xd == 1 && a.od == 1 && a.width <= 4 && a.dim % V == 0 &&
                    (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.bias) & 15) == 0 &&
                    a.xb % V == 0 && a.xt % V == 0 && a.ob % V == 0 && a.ot % V == 0;
    if (cl) return launch_cl<T, TO>(a, batch, st);
  }
  const int64_t total = batch * a.dim * a.L;
  conv1d_generic_kernel<T, TO><<<(unsigned)((total + GEN_THREADS - 1) / GEN_THREADS), GEN_THREADS, 0, st>>>(a, total);
  return cudaGetLastError();
}

}  // namespace

// The channels-last kernel takes widths 1-4 (Mamba2's d_conv is 4); wider kernels, odd
// strides and unaligned pointers run the one-thread-per-output kernel.
cudaError_t launch_conv1d(const ssd_conv1d_params_t* p, cudaStream_t st) {
  ConvArgs a;
  a.dim = p->dim; a.L = p->seqlen;
  a.xb = p->x_stride_b; a.xd = p->x_stride_d; a.xt = p->x_stride_t;
  a.ob = p->out_stride_b; a.od = p->out_stride_d; a.ot = p->out_stride_t;
  a.width = p->width; a.silu = p->silu != 0;
  a.x = p->x; a.w = p->weight; a.bias = p->bias; a.seq = p->seq_idx; a.out = p->out;
  a.w_bf16 = p->weight_dtype == SSD_DTYPE_BF16; a.b_bf16 = p->bias_dtype == SSD_DTYPE_BF16;
  const bool xf = p->dtype == SSD_DTYPE_F32, of = p->out_dtype == SSD_DTYPE_F32;
  if (xf && of) return launch_conv_typed<float, float>(a, p->batch, st);
  if (xf) return launch_conv_typed<float, bf16>(a, p->batch, st);
  if (of) return launch_conv_typed<bf16, float>(a, p->batch, st);
  return launch_conv_typed<bf16, bf16>(a, p->batch, st);
}

cudaError_t launch_conv1d_update(const ssd_conv1d_update_params_t* p, cudaStream_t st) {
  UpdArgs a;
  a.batch = p->batch; a.dim = p->dim; a.sb = p->state_stride_b; a.sd = p->state_stride_d;
  a.width = p->width; a.silu = p->silu != 0;
  a.x = p->x_new; a.state = p->conv_state; a.w = p->weight; a.bias = p->bias; a.out = p->out;
  a.w_bf16 = p->weight_dtype == SSD_DTYPE_BF16; a.b_bf16 = p->bias_dtype == SSD_DTYPE_BF16;
  const unsigned grid = (unsigned)((p->batch * p->dim + GEN_THREADS - 1) / GEN_THREADS);
  const int code = (p->x_dtype == SSD_DTYPE_F32 ? 4 : 0) + (p->state_dtype == SSD_DTYPE_F32 ? 2 : 0) +
                   (p->out_dtype == SSD_DTYPE_F32 ? 1 : 0);
  switch (code) {
    case 0: conv1d_update_kernel<bf16, bf16, bf16><<<grid, GEN_THREADS, 0, st>>>(a); break;
    case 1: conv1d_update_kernel<bf16, bf16, float><<<grid, GEN_THREADS, 0, st>>>(a); break;
    case 2: conv1d_update_kernel<bf16, float, bf16><<<grid, GEN_THREADS, 0, st>>>(a); break;
    case 3: conv1d_update_kernel<bf16, float, float><<<grid, GEN_THREADS, 0, st>>>(a); break;
    case 4: conv1d_update_kernel<float, bf16, bf16><<<grid, GEN_THREADS, 0, st>>>(a); break;
    case 5: conv1d_update_kernel<float, bf16, float><<<grid, GEN_THREADS, 0, st>>>(a); break;
    case 6: conv1d_update_kernel<float, float, bf16><<<grid, GEN_THREADS, 0, st>>>(a); break;
    default: conv1d_update_kernel<float, float, float><<<grid, GEN_THREADS, 0, st>>>(a); break;
  }
  return cudaGetLastError();
}

}  // namespace ssd
