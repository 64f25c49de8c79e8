// Sequence-parallel decay fix-up.  A rank that ran its token segment from a zero state adds
// the contribution of the state S entering the segment (received from the ranks before it):
//
//   out[b,t,h,:] += exp(dA(t)) * (C[b,t,g(h),:] . S[b,h,:,:]^T) * (silu(z[b,t,h,:]) if z)
//       for t < carried_len[b] (the tokens of the sequence carried into the segment),
//   final[b,h]   += exp(dA(L-1)) * S[b,h]   if carried_len[b] == L (the carried sequence
//       reaches the segment's end), else final is unchanged (a reset zeroes the decay),
//
// with dA(t) the segment-wide cumulative sum of dt*A: the chunk totals of the chunks before
// t's chunk plus the within-chunk cumsum (the (b,H,nc,Q) layout of chunk_cumsum_fwd.py:288).
// This is the inter-chunk term of chunk_scan_fwd.py:108-232 with the received state in
// place of the zero initial state; the z gate is linear in y, so it applies to the added
// term alone.
//
// One CTA per (64-token tile, head, batch row).  C^T (N x 64) and S^T (N x P) are staged in
// shared memory as f32 with n as the row, so each thread's 4x4 output tile reads two
// 16-byte vectors per n.  The extra x-block of the grid does the final-state update.
#include "common.cuh"
#include "ssd_kernels.h"

namespace ssd {

namespace {

constexpr int FX_THREADS = 256;
constexpr int FX_TOK = 64;

struct FxArgs {
  int64_t L, H, P, G, N, Q, nc;
  const void* C;
  const void* z;
  const float* dA;
  const float* S;
  const int32_t* carried;
  float* out;
  float* final_states;
};

template <typename T>
__global__ void __launch_bounds__(FX_THREADS) sp_fixup_kernel(const FxArgs a) {
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  const int64_t bi = blockIdx.z, h = blockIdx.y;
  const int64_t ntiles = (a.L + FX_TOK - 1) / FX_TOK;
  const int64_t clen = a.carried ? min((int64_t)a.carried[bi], a.L) : a.L;
  const float* dAh = a.dA + (bi * a.H + h) * a.nc * a.Q;
  const float* Sh = a.S + (bi * a.H + h) * a.P * a.N;
  const int tid = threadIdx.x;

  if (blockIdx.x == ntiles) {   // final state: += exp(total decay) * S when carried to the end
    if (a.final_states == nullptr || clen < a.L) return;
    float part = 0.f;
    for (int64_t c = tid; c < a.nc; c += FX_THREADS) part += dAh[c * a.Q + a.Q - 1];
    __shared__ float red[FX_THREADS / 32];
    part = warp_sum(part);
    if ((tid & 31) == 0) red[tid >> 5] = part;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < FX_THREADS / 32; ++w) tot += red[w];
    const float dec = __expf(tot);
    float* fh = a.final_states + (bi * a.H + h) * a.P * a.N;
    for (int64_t i = tid; i < a.P * a.N; i += FX_THREADS) fh[i] = fmaf(dec, Sh[i], fh[i]);
    return;
  }

  const int64_t t0 = (int64_t)blockIdx.x * FX_TOK;
  if (t0 >= clen) return;
  const int64_t nt = min((int64_t)FX_TOK, clen - t0);
  const int64_t g = h / (a.H / a.G);
  float* Ct = sm;                       // [N][FX_TOK]
  float* St = sm + a.N * FX_TOK;        // [N][P]
  float* dg = St + a.N * a.P;           // [FX_TOK] exp(dA(t))
  float* base = dg + FX_TOK;            // [1] sum of chunk totals before t0's chunk

  // chunk totals before t0's chunk (warp 0), then per-token decays
  if (tid < 32) {
    const int64_t c0 = t0 / a.Q;
    float part = 0.f;
    for (int64_t c = tid; c < c0; c += 32) part += dAh[c * a.Q + a.Q - 1];
    part = warp_sum(part);
    if (tid == 0) base[0] = part;
  }
  // S^T and C^T into shared memory (global reads coalesced along n)
  for (int64_t i = tid; i < a.P * a.N; i += FX_THREADS) {
    const int64_t p = i / a.N, n = i - p * a.N;
    St[n * a.P + p] = Sh[i];
  }
  const T* Cb = (const T*)a.C + (bi * a.L * a.G + g) * a.N;
  for (int64_t i = tid; i < FX_TOK * a.N; i += FX_THREADS) {
    const int64_t k = i / a.N, n = i - k * a.N;
    Ct[n * FX_TOK + k] = k < nt ? ldg(Cb + (t0 + k) * a.G * a.N + n) : 0.f;
  }
  __syncthreads();
  if (tid == 0) {
    float run = base[0];
    int64_t cprev = t0 / a.Q;
    for (int k = 0; k < FX_TOK; ++k) {
      const int64_t t = t0 + k;
      if (t >= t0 + nt) { dg[k] = 0.f; continue; }
      const int64_t c = t / a.Q;
      for (; cprev < c; ++cprev) run += dAh[cprev * a.Q + a.Q - 1];
      dg[k] = __expf(run + dAh[c * a.Q + (t - c * a.Q)]);
    }
  }
  __syncthreads();

  const int np4 = (int)(a.P / 4);
  for (int tile = tid; tile < (FX_TOK / 4) * np4; tile += FX_THREADS) {
    const int tq = tile / np4, tp = tile - tq * np4;
    float acc[4][4] = {};
    for (int64_t n = 0; n < a.N; ++n) {
      const float4 cv = *reinterpret_cast<const float4*>(Ct + n * FX_TOK + 4 * tq);
      const float4 sv = *reinterpret_cast<const float4*>(St + n * a.P + 4 * tp);
      const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(cc[i], ss[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = 4 * tq + i;
      if (k >= nt) break;
      const int64_t row = ((bi * a.L + t0 + k) * a.H + h) * a.P + 4 * tp;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float f = dg[k] * acc[i][j];
        if (a.z) f *= silu(ldg((const T*)a.z + row + j));
        a.out[row + j] += f;
      }
    }
  }
}

}  // namespace

size_t sp_fixup_smem_bytes(int64_t P, int64_t N) {
  return (size_t)(N * FX_TOK + N * P + FX_TOK + 4) * sizeof(float);
}

cudaError_t launch_sp_fixup(const ssd_sp_fixup_params_t* p, cudaStream_t st) {
  FxArgs a;
  a.L = p->seqlen; a.H = p->nheads; a.P = p->headdim; a.G = p->ngroups; a.N = p->dstate;
  a.Q = p->chunk_size; a.nc = (a.L + a.Q - 1) / a.Q;
  a.C = p->C; a.z = p->z; a.dA = p->dA_cumsum; a.S = p->state_in; a.carried = p->carried_len;
  a.out = p->out; a.final_states = p->final_states;
  const size_t smem = sp_fixup_smem_bytes(a.P, a.N);
  const dim3 grid((unsigned)((a.L + FX_TOK - 1) / FX_TOK + 1), (unsigned)a.H, (unsigned)p->batch);
  cudaError_t e;
  if (p->dtype == SSD_DTYPE_BF16) {
    e = cudaFuncSetAttribute(sp_fixup_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sp_fixup_kernel<bf16><<<grid, FX_THREADS, smem, st>>>(a);
  } else {
    e = cudaFuncSetAttribute(sp_fixup_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    sp_fixup_kernel<float><<<grid, FX_THREADS, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace ssd
