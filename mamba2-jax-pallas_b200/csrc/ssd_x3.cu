// Tensor-core (tcgen05) chunk_state, bmm_chunk and chunk_scan for fp32 inputs.
//
// fp32 operands are split into two bf16 terms, v = hi + lo with hi = bf16(v) and
// lo = bf16(v - hi) (v - hi is exact in fp32), and every product is taken as
// hi*hi + hi*lo + lo*hi with fp32 accumulation in TMEM: the "bf16x3" scheme of Henry,
// Tang and Heinecke, "Leveraging the bfloat16 Artificial Intelligence Datatype For
// Higher-Precision Computations" (ARITH 2019).  The dropped lo*lo term and the rounding of
// lo are each below 2^-16 of the product, so a stage's relative error is about 1e-5, inside
// the fp32 bound of rel-L2 1e-4, while the operands take half the shared memory of a
// three-term tf32 split and the MMAs run at the bf16 rate.
//
// Every kernel is one 256-thread CTA per 128-row output tile.  The K loop runs over 64-wide
// blocks through a two-stage shared-memory ring: all threads load a block with plain
// coalesced loads (which also transposes the operands whose K dimension is strided in
// HBM), split it into hi/lo bf16 tiles in the 128-byte-swizzled K-major layout, and one
// thread issues 3 x (block K / 16) MMAs and commits them to the stage's mbarrier, which the
// refill of that stage two blocks later waits on.  The epilogue reads the accumulator from
// TMEM (warp w: lanes 32(w%4).., column half w/4) and applies the stage's masks, skip term
// and gate in fp32.  Same layouts, masks and outputs as the CUDA-core stages in
// ssd_simt.cu; the reference stages are kernels/{chunk_state_fwd,bmm_chunk_fwd,
// chunk_scan_fwd}.py.
#include <mutex>

#include "common.cuh"
#include "ptx_sm100.cuh"
#include "ssd_x3.h"

namespace ssd {
namespace x3 {

constexpr int NTH = 256;
constexpr int KB = 64;                             // K elements per block (one 128-byte swizzle row)
constexpr long long TIMEOUT_CYCLES = 4000000000LL;  // about 2 s at the boost clock

// Bounded wait on an mbarrier phase; a wait that gives up records 0x100|id in the status
// word (when there is one) and returns false.  The caller carries on: every wait is bounded,
// so the launch ends either way, and the status word tells the host its output is incomplete.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, unsigned* status, int id) {
  const long long t0 = clock64();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > TIMEOUT_CYCLES) {
      if (status) atomicCAS(status, 0u, (unsigned)(0x100 | id));
      return false;
    }
  }
  return true;
}

// 8 consecutive-K fp32 values -> the hi and lo bf16 16-byte chunks (row r, chunk j) of a
// 128-byte-swizzled K-major tile.
__device__ __forceinline__ void put8(uint8_t* hi, uint8_t* lo, int r, int j, const float (&v)[8]) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    const float2 af = __bfloat1622float2(a);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i] - af.x, v[2 * i + 1] - af.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&a);
    l[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  const uint32_t off = ptx::sw128_off((uint32_t)r, (uint32_t)j);
  *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float comp(const float4& f, int e) { return e == 0 ? f.x : e == 1 ? f.y : e == 2 ? f.z : f.w; }

// Shared state of one CTA: the mbarriers of the two stages and the TMEM base address.
struct Ctl {
  uint64_t bar[2];
  uint32_t tmem;
  uint32_t pad;
};

__device__ __forceinline__ uint32_t tmem_cols(int n) {
  uint32_t c = 32;
  while ((int)c < n) c <<= 1;
  return c;
}

__device__ __forceinline__ void setup(Ctl* ctl, uint32_t ncols) {
  if (threadIdx.x == 0) {
    ptx::mbar_init(&ctl->bar[0], 1);
    ptx::mbar_init(&ctl->bar[1], 1);
    ptx::fence_mbar_init();
  }
  if (threadIdx.x < 32) {
    ptx::tmem_alloc(&ctl->tmem, ncols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
}

__device__ __forceinline__ void teardown(Ctl* ctl, uint32_t ncols) {
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(ctl->tmem, ncols);
  }
}

// Issue the 3 x ksteps MMAs of one K block (thread 0 only) and commit them to `bar`.
__device__ __forceinline__ void issue_block(uint32_t d, uint32_t idesc, const uint8_t* a_hi, const uint8_t* a_lo,
                                            const uint8_t* b_hi, const uint8_t* b_lo, int ksteps, bool first,
                                            uint64_t* bar) {
  ptx::tc_fence_after();
  const uint32_t ah = ptx::smem_u32(a_hi), al = ptx::smem_u32(a_lo), bh = ptx::smem_u32(b_hi),
                 bl = ptx::smem_u32(b_lo);
  for (int kk = 0; kk < ksteps; ++kk) {
    const uint32_t o = 32u * kk;
    ptx::mma_f16(d, ptx::sdesc_sw128(ah + o, 16, 1024), ptx::sdesc_sw128(bh + o, 16, 1024), idesc,
                 (first && kk == 0) ? 0u : 1u);
    ptx::mma_f16(d, ptx::sdesc_sw128(ah + o, 16, 1024), ptx::sdesc_sw128(bl + o, 16, 1024), idesc, 1u);
    ptx::mma_f16(d, ptx::sdesc_sw128(al + o, 16, 1024), ptx::sdesc_sw128(bh + o, 16, 1024), idesc, 1u);
  }
  ptx::mma_commit(bar);
}

// The K loop shared by the three kernels.  Stage s holds [A hi | A lo | B hi | B lo] with
// RA and RB rows.  ld(blk, regs) issues the global loads of block blk into registers,
// st(blk, regs, a_hi, a_lo, b_hi, b_lo) splits and stores them; the loads of block blk+1 are
// issued right after block blk is published, so they are in flight while its MMAs run and
// while the other CTA on the SM converts.  ksteps(blk) gives the block's K/16.  Returns
// after the last block's MMAs completed (or a wait gave up).
template <typename Regs, typename Ld, typename St, typename Steps>
__device__ __forceinline__ void k_loop(uint8_t* smem, Ctl* ctl, int RA, int RB, int nblk, uint32_t idesc,
                                       unsigned* status, Ld&& ld, St&& st, Steps&& ksteps) {
  const uint32_t stage_bytes = (uint32_t)(RA + RB) * 256u;
  Regs regs;
  if (nblk > 0) ld(0, regs);
  for (int it = 0; it < nblk; ++it) {
    const int s = it & 1;
    if (it >= 2) wait_phase(&ctl->bar[s], ((it - 2) >> 1) & 1, status, 1);
    uint8_t* a_hi = smem + s * stage_bytes;
    uint8_t* a_lo = a_hi + RA * 128;
    uint8_t* b_hi = a_lo + RA * 128;
    uint8_t* b_lo = b_hi + RB * 128;
    st(it, regs, a_hi, a_lo, b_hi, b_lo);
    ptx::fence_proxy_async_smem();
    __syncthreads();
    if (it + 1 < nblk) ld(it + 1, regs);
    if (threadIdx.x == 0) issue_block(ctl->tmem, idesc, a_hi, a_lo, b_hi, b_lo, ksteps(it), it == 0, &ctl->bar[s]);
  }
  if (nblk > 0) wait_phase(&ctl->bar[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, status, 2);
  ptx::tc_fence_after();
}

// Tile loaders.  A unit is (row r, 16-byte chunk j) of a K-major operand tile: 8 consecutive
// K values of one row.  "Natural" tiles have the K run contiguous in HBM (two float4 per
// unit, eight threads per 256-byte row).  "Transposed" tiles have their rows contiguous in
// HBM and K strided: a thread loads 8 float4 at K = 8j..8j+7 covering rows 4q..4q+3, which
// are the 8 values of 4 units (consecutive threads take consecutive q, so a warp reads 512
// contiguous bytes per K).  Addresses are clamped into the tensor; what a clamped load
// brings in is finite and is zeroed or never read (masks at conversion, MMA K extent).
__device__ __forceinline__ uint8_t* aligned_smem(uint8_t* raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------
// bmm_chunk: out[b,c,g,m,s] = sum_k a[m,k] b[s,k] (ssd_naive.py:189-216), zero where
// causal and s > m, or where seq_idx differs between rows m and s (bmm_chunk_fwd.py:348-372).
// grid (b*nc*G, ceil(Q/128), ceil(Q/128)); M = 128 rows m, N = up to 128 columns s, K = K.
// With causal, tiles wholly above the diagonal only write their zeros.
// ---------------------------------------------------------------------------
struct BmmRegs {
  float4 a[8], b[8];
};

__global__ void __launch_bounds__(NTH, 1) x3_bmm_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                         const int32_t* __restrict__ seq_idx, int causal, int L,
                                                         int G, int K, int Q, int nc, float* __restrict__ out,
                                                         unsigned* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  __shared__ Ctl ctl;
  __shared__ int seqs[256];
  const int64_t bcg = blockIdx.x;
  const int g = bcg % G;
  const int c = (bcg / G) % nc;
  const int bi = bcg / ((int64_t)G * nc);
  const int m0 = blockIdx.y * 128, n0 = blockIdx.z * 128;
  const int NC = min(128, Q - n0);   // columns of this tile (a multiple of 32)
  const int64_t rowbase = (int64_t)bi * L + (int64_t)c * Q;
  const int mlast = (int)min((int64_t)Q, (int64_t)L - (int64_t)c * Q) - 1;   // last row inside the sequence
  const int tid = threadIdx.x, w = tid >> 5, lg = w & 3, half = w >> 2;
  const int m = m0 + 32 * lg + (tid & 31);
  float* o = out + ((((int64_t)bi * nc + c) * G + g) * Q) * Q + (int64_t)m * Q + n0;
  const int cw = NC / 2;
  if (causal && n0 > m0 + 127) {
    if (m < Q)
      for (int s0 = half * cw; s0 < (half + 1) * cw; s0 += 4) *reinterpret_cast<float4*>(o + s0) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  for (int s = tid; s < Q; s += NTH) {
    const int64_t pos = (int64_t)c * Q + s;
    seqs[s] = seq_idx ? (pos < L ? seq_idx[(int64_t)bi * L + pos] : -1) : 0;
  }
  setup(&ctl, 128);
  const int nblk = (K + KB - 1) / KB;
  k_loop<BmmRegs>(
      smem, &ctl, 128, 128, nblk, ptx::idesc_bf16_f32(128, NC, 0, 0), status,
      [&](int blk, BmmRegs& R) {
        const int k0 = blk * KB;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int u = q * NTH + tid, r = u >> 3, k = min(k0 + 8 * (u & 7), K - 8);
          const float* pa = a + ((rowbase + min(m0 + r, mlast)) * G + g) * K + k;
          R.a[2 * q] = ldg4(pa);
          R.a[2 * q + 1] = ldg4(pa + 4);
          if (r < NC) {
            const float* pb = b + ((rowbase + min(n0 + r, mlast)) * G + g) * K + k;
            R.b[2 * q] = ldg4(pb);
            R.b[2 * q + 1] = ldg4(pb + 4);
          }
        }
      },
      [&](int, const BmmRegs& R, uint8_t* ah, uint8_t* al, uint8_t* bh, uint8_t* bl) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int u = q * NTH + tid, r = u >> 3, j = u & 7;
          float v[8];
          const bool va = m0 + r <= mlast;
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = va ? comp(R.a[2 * q + i / 4], i & 3) : 0.f;
          put8(ah, al, r, j, v);
          if (r < NC) {
            const bool vb = n0 + r <= mlast;
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = vb ? comp(R.b[2 * q + i / 4], i & 3) : 0.f;
            put8(bh, bl, r, j, v);
          }
        }
      },
      [&](int blk) { return (min(K - blk * KB, KB) + 15) / 16; });
  const int sm = m < Q ? seqs[m] : 0;
  for (int s0 = half * cw; s0 < (half + 1) * cw; s0 += 16) {
    float v[16];
    ptx::tmem_ld16(ctl.tmem + ((uint32_t)(32 * lg) << 16) + s0, v);
    ptx::tmem_ld_wait();
    if (m < Q) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int s = n0 + s0 + i;
        if ((causal && s > m) || (seq_idx && seqs[s] != sm)) v[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(o + s0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  }
  teardown(&ctl, 128);
}

// ---------------------------------------------------------------------------
// chunk_state: states[b,c,h,p,n] = sum_k B[k,n] exp(dA_last - dA_k) dt_k x[k,p]
// (ssd_naive.py:77-128), tokens outside the last token's sequence masked
// (chunk_state_fwd.py:246-269).  grid (b*nc*H, ceil(N/128)); M = 128 state rows n,
// N = P = 32 * PU columns p, K = Q tokens.  Both operands are transposed tiles.
// ---------------------------------------------------------------------------
template <int PU>
struct CsRegs {
  float4 a[8], b[PU >= 8 ? 16 : 8];
};

template <int PU>
__global__ void __launch_bounds__(NTH, PU <= 2 ? 2 : 1) x3_chunk_state_kernel(
    const float* __restrict__ x, const float* __restrict__ Bm, const float* __restrict__ dt,
    const float* __restrict__ dA, const int32_t* __restrict__ seq_idx, int L, int H, int G, int N, int Q,
    int nc, float* __restrict__ states, unsigned* status) {
  constexpr int P = 32 * PU, QG = P / 4, TB = PU >= 8 ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  __shared__ Ctl ctl;
  __shared__ float scale[256];
  const int64_t bch = blockIdx.x;
  const int h = bch % H;
  const int c = (bch / H) % nc;
  const int bi = bch / ((int64_t)H * nc);
  const int g = h / (H / G);
  const int n0 = blockIdx.y * 128;
  const int tid = threadIdx.x;
  const int64_t rowbase = (int64_t)bi * L + (int64_t)c * Q;
  const int klast = (int)min((int64_t)Q, (int64_t)L - (int64_t)c * Q) - 1;
  const float* dAc = dA + (((int64_t)bi * H + h) * nc + c) * Q;
  const float* dtc = dt + (((int64_t)bi * H + h) * nc + c) * Q;
  const float dlast = dAc[Q - 1];
  int last_seq = 0;
  if (seq_idx) last_seq = seq_idx[(int64_t)bi * L + min((int64_t)(c + 1) * Q, (int64_t)L) - 1];
  for (int k = tid; k < 256; k += NTH) {
    const int64_t pos = (int64_t)c * Q + k;
    float sc = (k < Q && pos < L) ? expf(dlast - dAc[k]) * dtc[k] : 0.f;
    if (seq_idx && sc != 0.f) {
      const int sk = seq_idx[(int64_t)bi * L + pos];
      if (!(last_seq >= 0 && sk == last_seq)) sc = 0.f;
    }
    scale[k] = sc;
  }
  constexpr uint32_t ncols = P < 32 ? 32 : P;
  setup(&ctl, ncols);
  const int nblk = (Q + KB - 1) / KB;
  const int an = min(n0 + 4 * (tid & 31), N - 4), aj = tid >> 5;
  k_loop<CsRegs<PU>>(
      smem, &ctl, 128, P, nblk, ptx::idesc_bf16_f32(128, P, 0, 0), status,
      [&](int blk, CsRegs<PU>& R) {
        const int k0 = blk * KB;
#pragma unroll
        for (int i = 0; i < 8; ++i) R.a[i] = ldg4(Bm + ((rowbase + min(k0 + 8 * aj + i, klast)) * G + g) * N + an);
#pragma unroll
        for (int t = 0; t < TB; ++t) {
          const int pr = t * NTH + tid;
          if (pr < 2 * P) {
            const int q = pr % QG, j = pr / QG;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              R.b[8 * t + i] = ldg4(x + ((rowbase + min(k0 + 8 * j + i, klast)) * H + h) * P + 4 * q);
          }
        }
      },
      [&](int blk, const CsRegs<PU>& R, uint8_t* ah, uint8_t* al, uint8_t* bh, uint8_t* bl) {
        const int k0 = blk * KB;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = comp(R.a[i], e);
          put8(ah, al, 4 * (tid & 31) + e, aj, v);
        }
#pragma unroll
        for (int t = 0; t < TB; ++t) {
          const int pr = t * NTH + tid;
          if (pr < 2 * P) {
            const int q = pr % QG, j = pr / QG;
            float sc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) sc[i] = scale[k0 + 8 * j + i];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float v[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] = comp(R.b[8 * t + i], e) * sc[i];
              put8(bh, bl, 4 * q + e, j, v);
            }
          }
        }
      },
      [&](int blk) { return (min(Q - blk * KB, KB) + 15) / 16; });
  const int w = tid >> 5, lg = w & 3, half = w >> 2;
  const int n = n0 + 32 * lg + (tid & 31);
  float* o = states + ((((int64_t)bi * nc + c) * H + h) * P) * N + n;
  constexpr int cw = P / 2;
#pragma unroll
  for (int p0 = 0; p0 < cw; p0 += 16) {
    float v[16];
    ptx::tmem_ld16(ctl.tmem + ((uint32_t)(32 * lg) << 16) + half * cw + p0, v);
    ptx::tmem_ld_wait();
    if (n < N) {
#pragma unroll
      for (int i = 0; i < 16; ++i) o[(int64_t)(half * cw + p0 + i) * N] = v[i];
    }
  }
  teardown(&ctl, ncols);
}

// ---------------------------------------------------------------------------
// chunk_scan: out[m,p] = sum_{k<=m} CB[m,k] exp(dA_m - dA_k) dt_k x[k,p]
//                      + exp(dA_m) sum_n C[m,n] state[p,n]  (+ D x, * silu(z))
// (ssd_naive.py:223-318; seq_idx rules tests/test_chunk_scan_and_varlen.py:133-255).
// grid (b*nc*H, ceil(Q/128)); M = 128 rows m, N = P = 32 * PU columns p; the K loop runs
// over the causal token blocks k < min(Q, m0 + 128) (A = masked, decayed CB, natural;
// B = x, transposed) and then the state blocks n < N (A = C scaled by exp(dA_m), natural;
// B = the state, natural), all into one accumulator.
// ---------------------------------------------------------------------------
template <int PU>
struct ScRegs {
  float4 a[8], b[PU >= 8 ? 16 : 8];
};

template <int PU>
__global__ void __launch_bounds__(NTH, PU <= 2 ? 2 : 1) x3_chunk_scan_kernel(
    const float* __restrict__ cb, const float* __restrict__ x, const float* __restrict__ dt,
    const float* __restrict__ dA, const float* __restrict__ Cm, const float* __restrict__ states,
    const float* __restrict__ D, int D_ndim, const float* __restrict__ z, const int32_t* __restrict__ seq_idx,
    int L, int H, int G, int N, int Q, int nc, float* __restrict__ out, float* __restrict__ out_x,
    unsigned* status) {
  constexpr int P = 32 * PU, QG = P / 4, TB = PU >= 8 ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = aligned_smem(smem_raw);
  __shared__ Ctl ctl;
  __shared__ __align__(16) float dAk[256];
  __shared__ __align__(16) float dtk[256];
  __shared__ __align__(16) int seqk[256];
  __shared__ float sdec[128];
  const int64_t bch = blockIdx.x;
  const int h = bch % H;
  const int c = (bch / H) % nc;
  const int bi = bch / ((int64_t)H * nc);
  const int g = h / (H / G);
  const int m0 = blockIdx.y * 128;
  const int tid = threadIdx.x;
  const int64_t rowbase = (int64_t)bi * L + (int64_t)c * Q;
  const int mlast = (int)min((int64_t)Q, (int64_t)L - (int64_t)c * Q) - 1;
  const float* dAc = dA + (((int64_t)bi * H + h) * nc + c) * Q;
  const float* dtc = dt + (((int64_t)bi * H + h) * nc + c) * Q;
  int prev_seq = 0;
  if (seq_idx && c > 0) prev_seq = seq_idx[(int64_t)bi * L + (int64_t)c * Q - 1];
  for (int k = tid; k < Q; k += NTH) {
    const int64_t pos = (int64_t)c * Q + k;
    dAk[k] = dAc[k];
    dtk[k] = dtc[k];
    seqk[k] = seq_idx ? (pos < L ? seq_idx[(int64_t)bi * L + pos] : -1) : 0;
  }
  __syncthreads();
  if (tid < 128) {
    const int m = m0 + tid;
    float v = 0.f;
    if (m <= mlast) {
      v = expf(dAk[m]);
      if (seq_idx && seqk[m] != prev_seq) v = 0.f;
    }
    sdec[tid] = v;
  }
  constexpr uint32_t ncols = P < 32 ? 32 : P;
  setup(&ctl, ncols);   // its barrier also publishes sdec
  const int kend = min(Q, m0 + 128);
  const int nintra = (kend + KB - 1) / KB, nblk = nintra + (N + KB - 1) / KB;
  const float* cbt = cb + ((((int64_t)bi * nc + c) * G + g) * Q) * Q;
  const float* stp = states + ((((int64_t)bi * nc + c) * H + h) * P) * N;
  k_loop<ScRegs<PU>>(
      smem, &ctl, 128, P, nblk, ptx::idesc_bf16_f32(128, P, 0, 0), status,
      [&](int blk, ScRegs<PU>& R) {
        if (blk < nintra) {
          const int k0 = blk * KB;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int u = q * NTH + tid, m = m0 + (u >> 3), k = k0 + 8 * (u & 7);
            if (m < Q && k <= m) {
              R.a[2 * q] = ldg4(cbt + (int64_t)m * Q + k);
              R.a[2 * q + 1] = ldg4(cbt + (int64_t)m * Q + k + 4);
            }
          }
#pragma unroll
          for (int t = 0; t < TB; ++t) {
            const int pr = t * NTH + tid;
            if (pr < 2 * P) {
              const int q = pr % QG, j = pr / QG;
#pragma unroll
              for (int i = 0; i < 8; ++i)
                R.b[8 * t + i] = ldg4(x + ((rowbase + min(k0 + 8 * j + i, mlast)) * H + h) * P + 4 * q);
            }
          }
        } else {
          const int n0 = (blk - nintra) * KB;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int u = q * NTH + tid, n = min(n0 + 8 * (u & 7), N - 8);
            const float* pc = Cm + ((rowbase + min(m0 + (u >> 3), mlast)) * G + g) * N + n;
            R.a[2 * q] = ldg4(pc);
            R.a[2 * q + 1] = ldg4(pc + 4);
          }
#pragma unroll
          for (int q = 0; q < PU; ++q) {
            const int u = q * NTH + tid, n = min(n0 + 8 * (u & 7), N - 8);
            const float* ps = stp + (int64_t)(u >> 3) * N + n;
            R.b[2 * q] = ldg4(ps);
            R.b[2 * q + 1] = ldg4(ps + 4);
          }
        }
      },
      [&](int blk, const ScRegs<PU>& R, uint8_t* ah, uint8_t* al, uint8_t* bh, uint8_t* bl) {
        if (blk < nintra) {
          const int k0 = blk * KB;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int u = q * NTH + tid, r = u >> 3, j = u & 7, m = m0 + r, k = k0 + 8 * j;
            float v[8];
            if (m < Q && k <= m) {
              // the unit's 8 columns' dA, dt (and seq ids) as 16-byte shared loads
              const float dm = dAk[m];
              const float4 a0 = *reinterpret_cast<const float4*>(dAk + k), a1 = *reinterpret_cast<const float4*>(dAk + k + 4);
              const float4 t0 = *reinterpret_cast<const float4*>(dtk + k), t1 = *reinterpret_cast<const float4*>(dtk + k + 4);
              bool keep[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) keep[i] = k + i <= m;
              if (seq_idx) {
                const int sm = seqk[m];
                const int4 s0 = *reinterpret_cast<const int4*>(seqk + k), s1 = *reinterpret_cast<const int4*>(seqk + k + 4);
                keep[0] &= s0.x == sm; keep[1] &= s0.y == sm; keep[2] &= s0.z == sm; keep[3] &= s0.w == sm;
                keep[4] &= s1.x == sm; keep[5] &= s1.y == sm; keep[6] &= s1.z == sm; keep[7] &= s1.w == sm;
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float ak = comp(i < 4 ? a0 : a1, i & 3), tk = comp(i < 4 ? t0 : t1, i & 3);
                v[i] = keep[i] ? comp(R.a[2 * q + i / 4], i & 3) * expf(dm - ak) * tk : 0.f;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) v[i] = 0.f;
            }
            put8(ah, al, r, j, v);
          }
#pragma unroll
          for (int t = 0; t < TB; ++t) {
            const int pr = t * NTH + tid;
            if (pr < 2 * P) {
              const int q = pr % QG, j = pr / QG;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = comp(R.b[8 * t + i], e);
                put8(bh, bl, 4 * q + e, j, v);
              }
            }
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int u = q * NTH + tid, r = u >> 3;
            const float sd = sdec[r];
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = comp(R.a[2 * q + i / 4], i & 3) * sd;
            put8(ah, al, r, u & 7, v);
          }
#pragma unroll
          for (int q = 0; q < PU; ++q) {
            const int u = q * NTH + tid;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = comp(R.b[2 * q + i / 4], i & 3);
            put8(bh, bl, u >> 3, u & 7, v);
          }
        }
      },
      [&](int blk) {
        return blk < nintra ? (min(kend - blk * KB, KB) + 15) / 16 : (min(N - (blk - nintra) * KB, KB) + 15) / 16;
      });
  const int w = tid >> 5, lg = w & 3, half = w >> 2;
  const int m = m0 + 32 * lg + (tid & 31);
  const bool row_ok = m <= mlast;
  const int64_t rowoff = ((rowbase + m) * H + h) * P;
  constexpr int cw = P / 2;
#pragma unroll
  for (int pp = 0; pp < cw; pp += 16) {
    const int p0 = half * cw + pp;
    float v[16];
    ptx::tmem_ld16(ctl.tmem + ((uint32_t)(32 * lg) << 16) + p0, v);
    ptx::tmem_ld_wait();
    if (!row_ok) continue;
    if (D_ndim) {
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 xv = ldg4(x + rowoff + p0 + i);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          v[i + e] += comp(xv, e) * (D_ndim == 1 ? D[h] : D[(int64_t)h * P + p0 + i + e]);
      }
    }
    if (z) {
      if (out_x)
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(out_x + rowoff + p0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 zv = ldg4(z + rowoff + p0 + i);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[i + e] *= silu(comp(zv, e));
      }
    }
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      *reinterpret_cast<float4*>(out + rowoff + p0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  }
  teardown(&ctl, ncols);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
inline bool al16(const void* p) { return !(reinterpret_cast<uintptr_t>(p) & 15); }

inline size_t smem_bytes(int RA, int RB) { return (size_t)(RA + RB) * 256 * 2 + 1024; }

// Dynamic shared memory opt-in, per device and kernel (the attribute belongs to the current
// device's context).
template <typename K>
bool ensure_attr(K kern, int kid, size_t bytes) {
  constexpr int kMaxDev = 64, kKernels = 9;
  static std::mutex mu;
  static size_t done[kMaxDev][kKernels] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < kMaxDev && done[dev][kid] >= bytes) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) return false;
  if (dev >= 0 && dev < kMaxDev) done[dev][kid] = bytes;
  return true;
}

// headdim -> the kernel instance index (P = 32, 64, 128, 256), or -1.
inline int p_index(int64_t P) { return P == 32 ? 0 : P == 64 ? 1 : P == 128 ? 2 : P == 256 ? 3 : -1; }

}  // namespace x3

bool x3_bmm_supported(const void* a, const void* b, int dtype, int64_t K, int64_t Q) {
  return dtype == SSD_DTYPE_F32 && K % 16 == 0 && Q % 32 == 0 && Q <= 256 && x3::al16(a) && x3::al16(b);
}

bool x3_chunk_state_supported(const void* x, const void* B, int dtype, int64_t P, int64_t N, int64_t Q) {
  return dtype == SSD_DTYPE_F32 && x3::p_index(P) >= 0 && N % 4 == 0 && N >= 4 && Q % 32 == 0 && Q <= 256 &&
         x3::al16(x) && x3::al16(B);
}

bool x3_chunk_scan_supported(const void* x, const void* C, const void* z, const float* cb, const void* states,
                             int dtype, int states_dtype, int64_t P, int64_t N, int64_t Q, const float* out,
                             const float* out_x) {
  return dtype == SSD_DTYPE_F32 && states_dtype == SSD_DTYPE_F32 && x3::p_index(P) >= 0 && N % 16 == 0 &&
         Q % 32 == 0 && Q <= 256 && x3::al16(x) && x3::al16(C) && x3::al16(cb) && x3::al16(states) &&
         x3::al16(out) && (!z || x3::al16(z)) && (!out_x || x3::al16(out_x));
}

static inline unsigned cdiv_u(int64_t a, int64_t b) { return (unsigned)((a + b - 1) / b); }

cudaError_t launch_x3_bmm(const float* a, const float* b, const int32_t* seq_idx, int causal, int64_t batch,
                          int64_t L, int64_t G, int64_t K, int64_t Q, float* out, unsigned* status,
                          cudaStream_t st) {
  const int nc = (int)((L + Q - 1) / Q);
  const size_t smem = x3::smem_bytes(128, 128);
  if (!x3::ensure_attr(x3::x3_bmm_kernel, 0, smem)) return cudaErrorInvalidConfiguration;
  x3::x3_bmm_kernel<<<dim3((unsigned)(batch * nc * G), cdiv_u(Q, 128), cdiv_u(Q, 128)), x3::NTH, smem, st>>>(
      a, b, seq_idx, causal, (int)L, (int)G, (int)K, (int)Q, nc, out, status);
  return cudaGetLastError();
}

cudaError_t launch_x3_chunk_state(const float* x, const float* B, const float* dt, const float* dA,
                                  const int32_t* seq_idx, int64_t b, int64_t L, int64_t H, int64_t P, int64_t G,
                                  int64_t N, int64_t Q, float* states, unsigned* status, cudaStream_t st) {
  using Kern = void (*)(const float*, const float*, const float*, const float*, const int32_t*, int, int, int, int,
                        int, int, float*, unsigned*);
  static const Kern kerns[4] = {x3::x3_chunk_state_kernel<1>, x3::x3_chunk_state_kernel<2>,
                                x3::x3_chunk_state_kernel<4>, x3::x3_chunk_state_kernel<8>};
  const int pi = x3::p_index(P);
  if (pi < 0) return cudaErrorInvalidValue;
  const int nc = (int)((L + Q - 1) / Q);
  const size_t smem = x3::smem_bytes(128, (int)P);
  if (!x3::ensure_attr(kerns[pi], 1 + pi, smem)) return cudaErrorInvalidConfiguration;
  kerns[pi]<<<dim3((unsigned)(b * nc * H), cdiv_u(N, 128)), x3::NTH, smem, st>>>(
      x, B, dt, dA, seq_idx, (int)L, (int)H, (int)G, (int)N, (int)Q, nc, states, status);
  return cudaGetLastError();
}

cudaError_t launch_x3_chunk_scan(const float* cb, const float* x, const float* dt, const float* dA, const float* C,
                                 const float* states, const float* D, int D_ndim, const float* z,
                                 const int32_t* seq_idx, int64_t b, int64_t L, int64_t H, int64_t P, int64_t G,
                                 int64_t N, int64_t Q, float* out, float* out_x, unsigned* status,
                                 cudaStream_t st) {
  using Kern = void (*)(const float*, const float*, const float*, const float*, const float*, const float*,
                        const float*, int, const float*, const int32_t*, int, int, int, int, int, int, float*,
                        float*, unsigned*);
  static const Kern kerns[4] = {x3::x3_chunk_scan_kernel<1>, x3::x3_chunk_scan_kernel<2>,
                                x3::x3_chunk_scan_kernel<4>, x3::x3_chunk_scan_kernel<8>};
  const int pi = x3::p_index(P);
  if (pi < 0) return cudaErrorInvalidValue;
  const int nc = (int)((L + Q - 1) / Q);
  const size_t smem = x3::smem_bytes(128, (int)P);
  if (!x3::ensure_attr(kerns[pi], 5 + pi, smem)) return cudaErrorInvalidConfiguration;
  kerns[pi]<<<dim3((unsigned)(b * nc * H), cdiv_u(Q, 128)), x3::NTH, smem, st>>>(
      cb, x, dt, dA, C, states, D, D_ndim, z, seq_idx, (int)L, (int)H, (int)G, (int)N, (int)Q, nc, out, out_x,
      status);
  return cudaGetLastError();
}

}  // namespace ssd
