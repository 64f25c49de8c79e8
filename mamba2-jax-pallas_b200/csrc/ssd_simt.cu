// CUDA-core (fp32 FFMA) kernels for the five SSD forward stages and the varlen states.
//
// These are the exact-fp32 path (fp32 inputs need rel-L2 <= 1e-4, which a single
// bf16/tf32 tensor-core pass cannot give) and the per-stage entry points of the
// C ABI.  Every stage reads the reference layouts directly; there is no
// pre-transposition pass.  Tiles are 64x64 outputs per 256-thread CTA with a
// 32-deep K slice staged in shared memory.
#include "common.cuh"
#include "ssd_kernels.h"

namespace ssd {

constexpr int TM = 64, TN = 64, TK = 32, NT = 256, PADW = TM + 1;

// ---------------------------------------------------------------------------
// Stage 1: chunk_cumsum (chunk_cumsum_fwd.py:194-235; ssd_naive.py:66-68 order:
// dA = dt*A, then an inclusive scan inside the chunk).  One warp per (batch, head, chunk):
// lane l owns positions [l*per, (l+1)*per) (per = Q/32 <= 8), loads them all at once, scans
// them serially and adds the warp's exclusive prefix.  grid ceil(b*H*nc / 8), 256 threads.
// ---------------------------------------------------------------------------
template <typename TDT>
__global__ void __launch_bounds__(NT) chunk_cumsum_kernel(
    const TDT* __restrict__ dt, const float* __restrict__ A, const float* __restrict__ dt_bias,
    int softplus, float lo, float hi, int L, int H, int Q, int nc, int64_t nwarps,
    float* __restrict__ dA_cs, float* __restrict__ dt_out) {
  const int64_t wid = (int64_t)blockIdx.x * (NT / 32) + (threadIdx.x >> 5);
  if (wid >= nwarps) return;
  const int lane = threadIdx.x & 31;
  const int c = wid % nc;
  const int h = (wid / nc) % H;
  const int bi = wid / ((int64_t)nc * H);
  const int per = Q / 32;
  const float bias = dt_bias ? dt_bias[h] : 0.f;
  const float a = A[h];
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t pos = (int64_t)c * Q + lane * per + j;
    v[j] = (j < per && pos < L) ? ldg(dt + ((int64_t)bi * L + pos) * H + h) : 0.f;
  }
  float loc[8];
  float run = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t pos = (int64_t)c * Q + lane * per + j;
    v[j] = (j < per && pos < L) ? dt_process(v[j], bias, softplus, lo, hi) : 0.f;
    run += v[j] * a;
    loc[j] = run;
  }
  const float excl = warp_incl_scan(run) - run;
  const int64_t base = (((int64_t)bi * H + h) * nc + c) * Q + lane * per;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j < per) {
      dA_cs[base + j] = loc[j] + excl;
      dt_out[base + j] = v[j];
    }
}

// ---------------------------------------------------------------------------
// Stage 2: chunk_state (ssd_naive.py:77-128 + seq_idx rule chunk_state_fwd.py:246-269)
// states[b,c,h,p,n] = sum_k x[k,p] * exp(dA_last - dA_k) * dt_k * B[k,n]
// grid (b*nc*H, ceil(P/64), ceil(N/64)).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) chunk_state_kernel(
    const T* __restrict__ x, const T* __restrict__ Bm, const float* __restrict__ dt,
    const float* __restrict__ dA, const int32_t* __restrict__ seq_idx,
    int L, int H, int P, int G, int N, int Q, int nc, float* __restrict__ states) {
  __shared__ float xs[TK][PADW];
  __shared__ float bs[TK][PADW];
  __shared__ float scale[256];
  const int64_t bch = blockIdx.x;
  const int h = bch % H;
  const int c = (bch / H) % nc;
  const int bi = bch / ((int64_t)H * nc);
  const int g = h / (H / G);
  const int p0 = blockIdx.y * TM, n0 = blockIdx.z * TN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t rowbase = (int64_t)bi * L + (int64_t)c * Q;   // first token of the chunk
  const float* dAc = dA + (((int64_t)bi * H + h) * nc + c) * Q;
  const float* dtc = dt + (((int64_t)bi * H + h) * nc + c) * Q;
  const float dlast = dAc[Q - 1];
  int last_seq = 0;
  if (seq_idx) {
    const int64_t e = min((int64_t)(c + 1) * Q, (int64_t)L) - 1;
    last_seq = seq_idx[(int64_t)bi * L + e];
  }
  for (int k = tid; k < Q; k += NT) {
    const int64_t pos = (int64_t)c * Q + k;
    float sc = expf(dlast - dAc[k]) * dtc[k];
    if (seq_idx) {
      const int sk = pos < L ? seq_idx[(int64_t)bi * L + pos] : -1;
      if (!(last_seq >= 0 && sk == last_seq)) sc = 0.f;
    }
    scale[k] = sc;
  }
  float acc[4][4] = {};
  __syncthreads();
  for (int k0 = 0; k0 < Q; k0 += TK) {
    for (int e = tid; e < TK * TM; e += NT) {
      const int kk = e / TM, i = e % TM;
      const int64_t pos = (int64_t)c * Q + k0 + kk;
      float xv = 0.f, bv = 0.f;
      if (pos < L) {
        if (p0 + i < P) xv = ldg(x + ((rowbase + k0 + kk) * H + h) * P + p0 + i) * scale[k0 + kk];
        if (n0 + i < N) bv = ldg(Bm + ((rowbase + k0 + kk) * G + g) * N + n0 + i);
      }
      xs[kk][i] = xv;
      bs[kk][i] = bv;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* outp = states + ((((int64_t)bi * nc + c) * H + h) * P) * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = p0 + ty * 4 + i;
    if (p >= P) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n < N) outp[(int64_t)p * N + n] = acc[i][j];
    }
  }
}

// ---------------------------------------------------------------------------
// Stage 3: state_passing (tests/test_state_passing_and_bmm.py:92-138 loop form;
// seq_idx resets state_passing_fwd.py:208-225).  grid (ceil(dim/(4*256)), b*H).
// ---------------------------------------------------------------------------
template <typename TO>
__global__ void __launch_bounds__(NT) state_passing_kernel(
    const float* states, const float* __restrict__ dA_chunk, int64_t stride_bh, int64_t stride_c,
    const float* __restrict__ init, const int32_t* __restrict__ seq_idx, int nc, int H,
    int64_t dim, int64_t L, int Q, TO* out, float* __restrict__ final_states) {
  const int64_t bh = blockIdx.y;
  const int bi = bh / H, h = bh % H;
  const int64_t d0 = ((int64_t)blockIdx.x * NT + threadIdx.x) * 4;
  if (d0 >= dim) return;
  const int cnt = (int)min((int64_t)4, dim - d0);
  float run[4] = {0.f, 0.f, 0.f, 0.f};
  if (init)
    for (int j = 0; j < cnt; ++j) run[j] = init[bh * dim + d0 + j];
  int prev_seq = 0;
  const float* dAp = dA_chunk + bh * stride_bh;
  // Eight chunks' states and decays are loaded before any of them is written back: out may
  // alias states, but the write of chunk c only replaces what was read for chunk c.
  constexpr int DEPTH = 8;
  for (int c0 = 0; c0 < nc; c0 += DEPTH) {
    float s[DEPTH][4], scale[DEPTH];
#pragma unroll
    for (int q = 0; q < DEPTH; ++q) {
      const int c = c0 + q;
      if (c >= nc) break;
      const int64_t off = (((int64_t)bi * nc + c) * H + h) * dim + d0;
      if (cnt == 4 && ((off & 3) == 0)) {
        const float4 v = *reinterpret_cast<const float4*>(states + off);
        s[q][0] = v.x; s[q][1] = v.y; s[q][2] = v.z; s[q][3] = v.w;
      } else {
        for (int j = 0; j < 4; ++j) s[q][j] = j < cnt ? states[off + j] : 0.f;
      }
      scale[q] = dAp[c * stride_c];
    }
#pragma unroll
    for (int q = 0; q < DEPTH; ++q) {
      const int c = c0 + q;
      if (c >= nc) break;
      const int64_t off = (((int64_t)bi * nc + c) * H + h) * dim + d0;
      float sc = expf(scale[q]);
      if (seq_idx) {
        const int64_t e = min((int64_t)(c + 1) * Q, L) - 1;
        const int cur = seq_idx[(int64_t)bi * L + e];
        if (cur != prev_seq) sc = 0.f;
        prev_seq = cur;
      }
      for (int j = 0; j < cnt; ++j) {
        st(out + off + j, run[j]);
        run[j] = sc * run[j] + s[q][j];
      }
    }
  }
  if (final_states)
    for (int j = 0; j < cnt; ++j) final_states[bh * dim + d0 + j] = run[j];
}

// ---------------------------------------------------------------------------
// Stage 4: bmm_chunk (ssd_naive.py:189-216; masks bmm_chunk_fwd.py:348-372).
// grid (b*nc*G, ceil(Q/64), ceil(Q/64)).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NT) bmm_chunk_kernel(
    const T* __restrict__ a, const T* __restrict__ b, const int32_t* __restrict__ seq_idx,
    int causal, int L, int G, int K, int Q, int nc, float* __restrict__ out) {
  __shared__ float as[TK][PADW];
  __shared__ float bs[TK][PADW];
  const int64_t bcg = blockIdx.x;
  const int g = bcg % G;
  const int c = (bcg / G) % nc;
  const int bi = bcg / ((int64_t)G * nc);
  const int m0 = blockIdx.y * TM, n0 = blockIdx.z * TN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t rowbase = (int64_t)bi * L + (int64_t)c * Q;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int e = tid; e < TK * TM; e += NT) {
      const int i = e / TK, kk = e % TK;
      const int64_t pa = (int64_t)c * Q + m0 + i, pb = (int64_t)c * Q + n0 + i;
      float av = 0.f, bv = 0.f;
      if (k0 + kk < K) {
        if (m0 + i < Q && pa < L) av = ldg(a + ((rowbase + m0 + i) * G + g) * K + k0 + kk);
        if (n0 + i < Q && pb < L) bv = ldg(b + ((rowbase + n0 + i) * G + g) * K + k0 + kk);
      }
      as[kk][i] = av;
      bs[kk][i] = bv;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < TK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* o = out + ((((int64_t)bi * nc + c) * G + g) * Q) * Q;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= Q) continue;
    const int64_t pm = (int64_t)c * Q + m;
    const int sm = seq_idx ? (pm < L ? seq_idx[(int64_t)bi * L + pm] : -1) : 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= Q) continue;
      float v = acc[i][j];
      if (causal && n > m) v = 0.f;
      if (seq_idx) {
        const int64_t pn = (int64_t)c * Q + n;
        const int sn = pn < L ? seq_idx[(int64_t)bi * L + pn] : -1;
        if (sm != sn) v = 0.f;
      }
      o[(int64_t)m * Q + n] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Stage 5: chunk_scan (ssd_naive.py:223-318; seq_idx rules
// tests/test_chunk_scan_and_varlen.py:133-255).  Decay is exp(dA_m - dA_k) from the
// difference (never the factored exp(dA_m)*exp(-dA_k)).
// grid (b*nc*H, ceil(Q/64), ceil(P/64)).
// ---------------------------------------------------------------------------
template <typename T, typename TS>
__global__ void __launch_bounds__(NT) chunk_scan_kernel(
    const float* __restrict__ cb, const T* __restrict__ x, const float* __restrict__ dt,
    const float* __restrict__ dA, const T* __restrict__ Cm, const TS* __restrict__ states,
    const float* __restrict__ D, int D_ndim, const T* __restrict__ z,
    const int32_t* __restrict__ seq_idx, int L, int H, int P, int G, int N, int Q, int nc,
    float* __restrict__ out, float* __restrict__ out_x) {
  __shared__ float as[TK][PADW];
  __shared__ float bs[TK][PADW];
  __shared__ float dAk[256], dtk[256];
  __shared__ int seqk[256];
  __shared__ float sdec[TM];
  const int64_t bch = blockIdx.x;
  const int h = bch % H;
  const int c = (bch / H) % nc;
  const int bi = bch / ((int64_t)H * nc);
  const int g = h / (H / G);
  const int m0 = blockIdx.y * TM, p0 = blockIdx.z * TN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t rowbase = (int64_t)bi * L + (int64_t)c * Q;
  const float* dAc = dA + (((int64_t)bi * H + h) * nc + c) * Q;
  const float* dtc = dt + (((int64_t)bi * H + h) * nc + c) * Q;
  int prev_seq = 0;
  if (seq_idx && c > 0) prev_seq = seq_idx[(int64_t)bi * L + (int64_t)c * Q - 1];
  for (int k = tid; k < Q; k += NT) {
    const int64_t pos = (int64_t)c * Q + k;
    dAk[k] = dAc[k];
    dtk[k] = dtc[k];
    seqk[k] = seq_idx ? (pos < L ? seq_idx[(int64_t)bi * L + pos] : -1) : 0;
  }
  __syncthreads();
  if (tid < TM) {
    const int m = m0 + tid;
    float v = 0.f;
    if (m < Q) {
      v = expf(dAk[m]);
      if (seq_idx && seqk[m] != prev_seq) v = 0.f;
    }
    sdec[tid] = v;
  }
  float acc[4][4] = {};
  const int kend = min(Q, m0 + TM);
  const float* cbt = cb + ((((int64_t)bi * nc + c) * G + g) * Q) * Q;
  // intra-chunk: sum_{k<=m} CB[m,k] exp(dA_m - dA_k) dt_k x[k,p]
  for (int k0 = 0; k0 < kend; k0 += TK) {
    __syncthreads();
    for (int e = tid; e < TK * TM; e += NT) {
      const int i = e / TK, kk = e % TK;
      const int m = m0 + i, k = k0 + kk;
      float v = 0.f;
      if (m < Q && k < Q && k <= m && seqk[k] == seqk[m])
        v = cbt[(int64_t)m * Q + k] * expf(dAk[m] - dAk[k]) * dtk[k];
      as[kk][i] = v;
    }
    for (int e = tid; e < TK * TN; e += NT) {
      const int kk = e / TN, j = e % TN;
      const int64_t pos = (int64_t)c * Q + k0 + kk;
      float v = 0.f;
      if (k0 + kk < Q && pos < L && p0 + j < P) v = ldg(x + ((rowbase + k0 + kk) * H + h) * P + p0 + j);
      bs[kk][j] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < TK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
  // inter-chunk: exp(dA_m) * mask_m * sum_n C[m,n] state[p,n]
  const TS* stp = states + ((((int64_t)bi * nc + c) * H + h) * P) * N;
  for (int n0 = 0; n0 < N; n0 += TK) {
    __syncthreads();
    for (int e = tid; e < TK * TM; e += NT) {
      const int i = e / TK, kk = e % TK;
      const int64_t pos = (int64_t)c * Q + m0 + i;
      float v = 0.f;
      if (m0 + i < Q && pos < L && n0 + kk < N)
        v = ldg(Cm + ((rowbase + m0 + i) * G + g) * N + n0 + kk) * sdec[i];
      as[kk][i] = v;
    }
    for (int e = tid; e < TK * TN; e += NT) {
      const int j = e / TK, kk = e % TK;
      float v = 0.f;
      if (p0 + j < P && n0 + kk < N) v = ldg(stp + (int64_t)(p0 + j) * N + n0 + kk);
      bs[kk][j] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < TK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
  // epilogue: D skip, z gate (ssd_naive.py:304-318)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    const int64_t pos = (int64_t)c * Q + m;
    if (m >= Q || pos >= L) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = p0 + tx + 16 * j;
      if (p >= P) continue;
      const int64_t idx = ((rowbase + m) * H + h) * P + p;
      float v = acc[i][j];
      if (D_ndim) v += ldg(x + idx) * (D_ndim == 1 ? D[h] : D[(int64_t)h * P + p]);
      if (z) {
        if (out_x) out_x[idx] = v;
        v *= silu(ldg(z + idx));
      }
      out[idx] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Varlen final states (chunk_state_fwd.py:448-597; test ref
// tests/test_chunk_scan_and_varlen.py:504-589).  grid (S*H, ceil(P/64), ceil(N/64)).
// ---------------------------------------------------------------------------
template <typename T, typename TS>
__global__ void __launch_bounds__(NT) chunk_state_varlen_kernel(
    const T* __restrict__ Bm, const T* __restrict__ x, const float* __restrict__ dt,
    const float* __restrict__ dA, const int32_t* __restrict__ cu, const TS* __restrict__ cs,
    int64_t T_total, int H, int P, int G, int N, int Q, int nc, float* __restrict__ out) {
  __shared__ float xs[TK][PADW];
  __shared__ float bs[TK][PADW];
  __shared__ float scale[256];
  const int s = blockIdx.x / H, h = blockIdx.x % H;
  const int g = h / (H / G);
  const int p0 = blockIdx.y * TM, n0 = blockIdx.z * TN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t start = cu[s], end = cu[s + 1];
  const int lc = (int)((end - 1) / Q);
  const int64_t c0 = (int64_t)lc * Q;
  const int sic = (int)max(start - c0, (int64_t)0);
  const int lv = (int)(end - c0 - 1);
  const float* dAc = dA + ((int64_t)h * nc + lc) * Q;
  const float* dtc = dt + ((int64_t)h * nc + lc) * Q;
  const float dlast = dAc[lv];
  for (int k = tid; k < Q; k += NT)
    scale[k] = (k >= sic && k <= lv) ? expf(dlast - dAc[k]) * dtc[k] : 0.f;
  float acc[4][4] = {};
  __syncthreads();
  const int kend = lv + 1;
  for (int k0 = sic & ~(TK - 1); k0 < kend; k0 += TK) {
    for (int e = tid; e < TK * TM; e += NT) {
      const int kk = e / TM, i = e % TM;
      const int64_t pos = c0 + k0 + kk;
      float xv = 0.f, bv = 0.f;
      if (k0 + kk < Q && pos < T_total) {
        if (p0 + i < P) xv = ldg(x + (pos * H + h) * P + p0 + i) * scale[k0 + kk];
        if (n0 + i < N) bv = ldg(Bm + (pos * G + g) * N + n0 + i);
      }
      xs[kk][i] = xv;
      bs[kk][i] = bv;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  const bool has_prev = start < c0;
  const float cscale = expf(dlast);
  const TS* csp = cs + (((int64_t)lc * H + h) * P) * N;
  float* o = out + (((int64_t)s * H + h) * P) * N;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = p0 + ty * 4 + i;
    if (p >= P) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (has_prev) v += ld(csp + (int64_t)p * N + n) * cscale;
      o[(int64_t)p * N + n] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
static inline unsigned cdiv(int64_t a, int64_t b) { return (unsigned)((a + b - 1) / b); }

cudaError_t launch_chunk_cumsum(const void* dt, int dt_dtype, const float* A, const float* dt_bias,
                                int softplus, float lo, float hi, int64_t b, int64_t L, int64_t H,
                                int64_t Q, float* dA_cs, float* dt_out, cudaStream_t st) {
  const int nc = (int)((L + Q - 1) / Q);
  const int64_t nw = b * H * nc;
  const unsigned grid = cdiv(nw, NT / 32);
  if (dt_dtype == SSD_DTYPE_BF16)
    chunk_cumsum_kernel<bf16><<<grid, NT, 0, st>>>((const bf16*)dt, A, dt_bias, softplus, lo, hi, (int)L, (int)H,
                                                   (int)Q, nc, nw, dA_cs, dt_out);
  else
    chunk_cumsum_kernel<float><<<grid, NT, 0, st>>>((const float*)dt, A, dt_bias, softplus, lo, hi, (int)L, (int)H,
                                                    (int)Q, nc, nw, dA_cs, dt_out);
  return cudaGetLastError();
}

cudaError_t launch_chunk_state(const void* x, const void* B, int dtype, const float* dt,
                               const float* dA, const int32_t* seq_idx, int64_t b, int64_t L,
                               int64_t H, int64_t P, int64_t G, int64_t N, int64_t Q,
                               float* states, cudaStream_t st) {
  const int nc = (int)((L + Q - 1) / Q);
  dim3 grid((unsigned)(b * nc * H), cdiv(P, TM), cdiv(N, TN));
  if (dtype == SSD_DTYPE_BF16)
    chunk_state_kernel<bf16><<<grid, NT, 0, st>>>((const bf16*)x, (const bf16*)B, dt, dA, seq_idx,
                                                  (int)L, (int)H, (int)P, (int)G, (int)N, (int)Q, nc, states);
  else
    chunk_state_kernel<float><<<grid, NT, 0, st>>>((const float*)x, (const float*)B, dt, dA, seq_idx,
                                                   (int)L, (int)H, (int)P, (int)G, (int)N, (int)Q, nc, states);
  return cudaGetLastError();
}

cudaError_t launch_state_passing(const float* states, const float* dA_chunk, int64_t stride_bh,
                                 int64_t stride_c, const float* init, const int32_t* seq_idx,
                                 int64_t b, int64_t nc, int64_t H, int64_t dim, int64_t L,
                                 int64_t Q, void* out, int out_dtype, float* final_states,
                                 cudaStream_t st) {
  dim3 grid(cdiv(dim, 4 * NT), (unsigned)(b * H));
  if (out_dtype == SSD_DTYPE_BF16)
    state_passing_kernel<bf16><<<grid, NT, 0, st>>>(states, dA_chunk, stride_bh, stride_c, init, seq_idx,
                                                    (int)nc, (int)H, dim, L, (int)Q, (bf16*)out, final_states);
  else
    state_passing_kernel<float><<<grid, NT, 0, st>>>(states, dA_chunk, stride_bh, stride_c, init, seq_idx,
                                                     (int)nc, (int)H, dim, L, (int)Q, (float*)out, final_states);
  return cudaGetLastError();
}

cudaError_t launch_bmm_chunk(const void* a, const void* b, int dtype, const int32_t* seq_idx,
                             int causal, int64_t batch, int64_t L, int64_t G, int64_t K,
                             int64_t Q, float* out, cudaStream_t st) {
  const int nc = (int)((L + Q - 1) / Q);
  dim3 grid((unsigned)(batch * nc * G), cdiv(Q, TM), cdiv(Q, TN));
  if (dtype == SSD_DTYPE_BF16)
    bmm_chunk_kernel<bf16><<<grid, NT, 0, st>>>((const bf16*)a, (const bf16*)b, seq_idx, causal,
                                                (int)L, (int)G, (int)K, (int)Q, nc, out);
  else
    bmm_chunk_kernel<float><<<grid, NT, 0, st>>>((const float*)a, (const float*)b, seq_idx, causal,
                                                 (int)L, (int)G, (int)K, (int)Q, nc, out);
  return cudaGetLastError();
}

template <typename T, typename TS>
static void chunk_scan_dispatch(dim3 grid, cudaStream_t st, const float* cb, const void* x,
                                const float* dt, const float* dA, const void* C, const void* states,
                                const float* D, int D_ndim, const void* z, const int32_t* seq_idx,
                                int64_t L, int64_t H, int64_t P, int64_t G, int64_t N, int64_t Q,
                                int nc, float* out, float* out_x) {
  chunk_scan_kernel<T, TS><<<grid, NT, 0, st>>>(cb, (const T*)x, dt, dA, (const T*)C, (const TS*)states,
                                                D, D_ndim, (const T*)z, seq_idx, (int)L, (int)H, (int)P,
                                                (int)G, (int)N, (int)Q, nc, out, out_x);
}

cudaError_t launch_chunk_scan(const float* cb, const void* x, int dtype, const float* dt,
                              const float* dA, const void* C, const void* states, int states_dtype,
                              const float* D, int D_ndim, const void* z, const int32_t* seq_idx,
                              int64_t b, int64_t L, int64_t H, int64_t P, int64_t G, int64_t N,
                              int64_t Q, float* out, float* out_x, cudaStream_t st) {
  const int nc = (int)((L + Q - 1) / Q);
  dim3 grid((unsigned)(b * nc * H), cdiv(Q, TM), cdiv(P, TN));
  if (dtype == SSD_DTYPE_BF16) {
    if (states_dtype == SSD_DTYPE_BF16)
      chunk_scan_dispatch<bf16, bf16>(grid, st, cb, x, dt, dA, C, states, D, D_ndim, z, seq_idx, L, H, P, G, N, Q, nc, out, out_x);
    else
      chunk_scan_dispatch<bf16, float>(grid, st, cb, x, dt, dA, C, states, D, D_ndim, z, seq_idx, L, H, P, G, N, Q, nc, out, out_x);
  } else {
    if (states_dtype == SSD_DTYPE_BF16)
      chunk_scan_dispatch<float, bf16>(grid, st, cb, x, dt, dA, C, states, D, D_ndim, z, seq_idx, L, H, P, G, N, Q, nc, out, out_x);
    else
      chunk_scan_dispatch<float, float>(grid, st, cb, x, dt, dA, C, states, D, D_ndim, z, seq_idx, L, H, P, G, N, Q, nc, out, out_x);
  }
  return cudaGetLastError();
}

cudaError_t launch_chunk_state_varlen(const void* B, const void* x, int dtype, const float* dt,
                                      const float* dA, const int32_t* cu, int S, const void* cs,
                                      int states_dtype, int64_t T_total, int64_t H, int64_t P,
                                      int64_t G, int64_t N, int64_t Q, float* out, cudaStream_t st) {
  const int nc = (int)((T_total + Q - 1) / Q);
  dim3 grid((unsigned)(S * H), cdiv(P, TM), cdiv(N, TN));
#define VARLEN_LAUNCH(T, TS)                                                                   \
  chunk_state_varlen_kernel<T, TS><<<grid, NT, 0, st>>>((const T*)B, (const T*)x, dt, dA, cu, \
                                                        (const TS*)cs, T_total, (int)H, (int)P, \
                                                        (int)G, (int)N, (int)Q, nc, out)
  if (dtype == SSD_DTYPE_BF16) {
    if (states_dtype == SSD_DTYPE_BF16) VARLEN_LAUNCH(bf16, bf16); else VARLEN_LAUNCH(bf16, float);
  } else {
    if (states_dtype == SSD_DTYPE_BF16) VARLEN_LAUNCH(float, bf16); else VARLEN_LAUNCH(float, float);
  }
#undef VARLEN_LAUNCH
  return cudaGetLastError();
}

}  // namespace ssd
