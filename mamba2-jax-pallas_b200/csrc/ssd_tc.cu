// Fused tcgen05 SSD forward for bf16 inputs (sm_100a).
//
// One CTA owns one (batch, head) and walks the sequence in internal chunks of 128
// tokens, carrying the running state S (N x P, f32) in the epilogue threads' registers.
// Nothing but the inputs, the outputs and the final state touches HBM: no chunk states,
// no CB matrix, no dA arrays.  The result does not depend on the internal chunk size
// (the reference's chunk_size only sets its own tiling; the seq_idx rules of
// chunk_state_fwd.py:246-269, state_passing_fwd.py:208-225 and chunk_scan_fwd.py:294-322
// compose to per-sequence semantics at any chunking), so every chunk_size maps here.
//
// Per chunk c (t = token in chunk, m = output row, n = state dim, p = head dim):
//   MMA1  CB[m][t]  = C[m][:] . B[t][:]                 (M=128, N=128, K=N)   TMEM
//   E2    S[m][t]   = CB[m][t] exp(dA_m - dA_t) dt_t    (t <= m, same seq)    -> smem bf16
//   MMA2  Y[m][p]   = S[m][:] . x[:][p]                 (M=128, N=64,  K=128) TMEM
//   MMA3  Yi[m][p]  = C[m][:] . S_c[p][:]               (M=128, N=64,  K=N)   TMEM
//   E1    xs[t][p]  = x[t][p] exp(dA_last - dA_t) dt_t  (chunk-end seq only)  -> smem bf16
//   MMA_L Lt[n][p]  = B[:][n] . xs[:][p]                (M=N,   N=64,  K=128) TMEM
//   E3    S_{c+1}   = keep_c exp(dA_last) S_c + Lt      (TMEM, f32)           -> smem bf16
//   E4    out[m][p] = Y + exp(dA_m) [seq_m == prev] Yi + D x ; * silu(z)
// Decay factors are always formed from differences of the in-chunk cumulative sums
// (never exp(dA_m) * exp(-dA_t)), as ssd_naive.py:264-268 does.
//
// Warp roles: warps 0-3 build scores and scaled x (chunk row r = TMEM lane r), warps 4-7
// update the state and write the output (they run one phase behind), warp 8 is the TMA
// producer, warp 9 issues the MMAs.  The running state lives in TMEM (f32).  Every mbarrier wait is bounded; on timeout the CTA
// records SSD_ERR_TIMEOUT in the status word, drains its async work and exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "ptx_sm100.cuh"
#include "ssd_tc.h"

namespace ssd {
namespace {

constexpr int QI = 128;       // internal chunk (tokens)
constexpr int PT = 64;        // head dim handled by the kernel
constexpr int NT_ = 128;      // state dim handled by the kernel
constexpr int NTHREADS = 320;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_CB = 0, COL_Y = 128, COL_YI = 192, COL_L = 256, COL_ST = 320;

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t SZ_C = QI * NT_ * 2;          // 32 KB  (two 64-wide swizzled boxes)
constexpr uint32_t SZ_X = QI * PT * 2;           // 16 KB
constexpr uint32_t SZ_STAGE = 2 * SZ_C + SZ_X;   // C, B, x
constexpr uint32_t OFF_STAGE = 0;
constexpr uint32_t OFF_S = 2 * SZ_STAGE;         // scores, 32 KB (two K-blocks)
constexpr uint32_t OFF_XS = OFF_S + QI * QI * 2; // 16 KB
constexpr uint32_t OFF_ST = OFF_XS + SZ_X;       // state bf16 [n][p], 16 KB
constexpr uint32_t OFF_MISC = OFF_ST + NT_ * PT * 2;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 2048 + 1024;

enum Bar { FULL0, FULL1, EMPTY0, EMPTY1, B_CB, CB_FREE, B_YI, ST_FULL, XS_FULL, B_L, L_FREE, S_FULL, B_Y, Y_FREE,
           DRAIN, NBARS };

struct Misc {
  uint64_t bar[NBARS];
  float dA[QI];
  float dt[QI];
  int seq[QI];
  float red[4];
  float red_o[4];
  float dA_last_o;
  int end_seq_o;
  uint32_t tmem_base;
  volatile int abort;
};
static_assert(sizeof(Misc) <= 2048, "misc area");

struct TcArgs {
  CUtensorMap tm_x, tm_b, tm_c;
  int L, H, G, nci;
  int dt_bf16, softplus, D_ndim;
  float lo, hi;
  const void* dt;
  const float* A;
  const float* dt_bias;
  const float* D;
  const bf16* x;
  const bf16* z;
  const float* init;
  const int32_t* seq_idx;
  float* out;
  float* out_x;
  float* final_states;
  unsigned* status;
};

constexpr unsigned TIMEOUT_NS = 2000000000u;  // 2 s; a normal launch takes well under 1 ms

// Bounded wait.  Returns false (after flagging the CTA and the status word) on timeout or
// when another role of this CTA already gave up.
__device__ __forceinline__ bool wait_bar(Misc* m, int id, uint32_t parity, unsigned* status) {
  if (ptx::mbar_try_wait(&m->bar[id], parity)) return true;
  const uint64_t t0 = ptx::globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ptx::mbar_try_wait(&m->bar[id], parity)) return true;
    if (m->abort) return false;
    if (ptx::globaltimer() - t0 > TIMEOUT_NS) {
      m->abort = 1;
      atomicCAS(status, 0u, (unsigned)(0x100 | id));
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// ---------------------------------------------------------------------------
// producer (warp 8, lane 0): C, B, x tiles of each chunk into a 2-stage ring
// ---------------------------------------------------------------------------
__device__ void producer(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h, int g) {
  const uint32_t bytes = SZ_STAGE;
  int c = 0;
  for (; c < a.nci; ++c) {
    const int s = c & 1;
    if (c >= 2 && !wait_bar(m, EMPTY0 + s, ((c >> 1) - 1) & 1, a.status)) break;
    uint8_t* st = sm + OFF_STAGE + s * SZ_STAGE;
    uint64_t* full = &m->bar[FULL0 + s];
    ptx::mbar_arrive_expect_tx(full, bytes);
    const int t0 = c * QI;
    ptx::tma_load_3d(st, &a.tm_c, full, g * NT_, t0, bi);
    ptx::tma_load_3d(st + SZ_C / 2, &a.tm_c, full, g * NT_ + 64, t0, bi);
    ptx::tma_load_3d(st + SZ_C, &a.tm_b, full, g * NT_, t0, bi);
    ptx::tma_load_3d(st + SZ_C + SZ_C / 2, &a.tm_b, full, g * NT_ + 64, t0, bi);
    ptx::tma_load_3d(st + 2 * SZ_C, &a.tm_x, full, h * PT, t0, bi);
  }
  // drain: never leave the CTA with bulk copies still landing in its shared memory
  for (int k = (c >= 2 ? c - 2 : 0); k < c; ++k) {
    const int s = k & 1;
    const uint64_t t0 = ptx::globaltimer();
    while (!ptx::mbar_try_wait(&m->bar[FULL0 + s], (k >> 1) & 1) && ptx::globaltimer() - t0 < TIMEOUT_NS) {
    }
  }
}

// ---------------------------------------------------------------------------
// MMA issuer (warp 9, lane 0)
// ---------------------------------------------------------------------------
__device__ void mma_issuer(const TcArgs& a, uint8_t* sm, Misc* m) {
  const uint32_t tmem = m->tmem_base;
  const uint32_t base = ptx::smem_u32(sm);
  constexpr uint32_t ID_CB = ptx::idesc_bf16_f32(128, 128, 0, 0);
  constexpr uint32_t ID_YI = ptx::idesc_bf16_f32(128, 64, 0, 1);
  constexpr uint32_t ID_L = ptx::idesc_bf16_f32(128, 64, 1, 1);
  constexpr uint32_t ID_Y = ptx::idesc_bf16_f32(128, 64, 0, 1);
  bool ok = true;
  for (int c = 0; c < a.nci && ok; ++c) {
    const int s = c & 1;
    const uint32_t st = base + OFF_STAGE + s * SZ_STAGE;
    const uint32_t sC = st, sB = st + SZ_C, sX = st + 2 * SZ_C;
    // MMA1: CB = C . B^T (both K-major: row = token, K = state dim in two 64-wide boxes)
    if (!(ok = wait_bar(m, FULL0 + s, (c >> 1) & 1, a.status))) break;
    if (c > 0 && !(ok = wait_bar(m, CB_FREE, (c - 1) & 1, a.status))) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < NT_ / 16; ++i) {
      const uint32_t off = (i >> 2) * (SZ_C / 2) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_CB, ptx::sdesc_sw128(sC + off, 16, 1024), ptx::sdesc_sw128(sB + off, 16, 1024),
                   ID_CB, i > 0);
    }
    ptx::mma_commit(&m->bar[B_CB]);
    // MMA3: Yi = C . S_c^T   (B operand = state [n][p], MN-major)
    if (!(ok = wait_bar(m, ST_FULL, c & 1, a.status))) break;
    if (c > 0 && !(ok = wait_bar(m, Y_FREE, (c - 1) & 1, a.status))) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < NT_ / 16; ++i) {
      const uint32_t offa = (i >> 2) * (SZ_C / 2) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_YI, ptx::sdesc_sw128(sC + offa, 16, 1024),
                   ptx::sdesc_sw128(base + OFF_ST + i * 2048, 8192, 1024), ID_YI, i > 0);
    }
    ptx::mma_commit(&m->bar[B_YI]);
    // MMA_L: Lt = B^T . xs   (A = B tile read MN-major, B = xs [t][p] MN-major)
    if (!(ok = wait_bar(m, XS_FULL, c & 1, a.status))) break;
    if (c > 0 && !(ok = wait_bar(m, L_FREE, (c - 1) & 1, a.status))) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < QI / 16; ++i) {
      ptx::mma_f16(tmem + COL_L, ptx::sdesc_sw128(sB + i * 2048, SZ_C / 2, 1024),
                   ptx::sdesc_sw128(base + OFF_XS + i * 2048, 8192, 1024), ID_L, i > 0);
    }
    ptx::mma_commit(&m->bar[B_L]);
    // MMA2: Y = S . x   (A = scores K-major, B = x [t][p] MN-major)
    if (!(ok = wait_bar(m, S_FULL, c & 1, a.status))) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < QI / 16; ++i) {
      const uint32_t offa = (i >> 2) * (QI * 128) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_Y, ptx::sdesc_sw128(base + OFF_S + offa, 16, 1024),
                   ptx::sdesc_sw128(sX + i * 2048, 8192, 1024), ID_Y, i > 0);
    }
    ptx::mma_commit(&m->bar[B_Y]);
    ptx::mma_commit(&m->bar[EMPTY0 + s]);
  }
  // drain: wait (bounded) until every issued MMA has completed
  ptx::mma_commit(&m->bar[DRAIN]);
  const uint64_t t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(&m->bar[DRAIN], 0) && ptx::globaltimer() - t0 < TIMEOUT_NS) {
  }
}

// ---------------------------------------------------------------------------
// helpers shared by the two worker warpgroups
// ---------------------------------------------------------------------------
struct ChunkDt {
  float raw;
  int seq;
};

__device__ __forceinline__ ChunkDt load_dt(const TcArgs& a, int bi, int h, int c, int r) {
  ChunkDt d{0.f, -1};
  const int64_t pos = (int64_t)c * QI + r;
  if (c < a.nci && pos < a.L) {
    const int64_t di = ((int64_t)bi * a.L + pos) * a.H + h;
    d.raw = a.dt_bf16 ? __bfloat162float(((const bf16*)a.dt)[di]) : ((const float*)a.dt)[di];
    d.seq = a.seq_idx ? a.seq_idx[(int64_t)bi * a.L + pos] : 0;
  }
  return d;
}

// 16-byte words of a bf16 row, scaled by `s`, repacked.
__device__ __forceinline__ uint4 scale_row16(uint4 w, float s) {
  uint4 o;
  float2 f;
  f = unpack_bf16(w.x); o.x = pack_bf16(f.x * s, f.y * s);
  f = unpack_bf16(w.y); o.y = pack_bf16(f.x * s, f.y * s);
  f = unpack_bf16(w.z); o.z = pack_bf16(f.x * s, f.y * s);
  f = unpack_bf16(w.w); o.w = pack_bf16(f.x * s, f.y * s);
  return o;
}

__device__ __forceinline__ void set_word(uint4 (&o)[4], int w, uint32_t v) {
  if ((w & 3) == 0) o[w >> 2].x = v;
  else if ((w & 3) == 1) o[w >> 2].y = v;
  else if ((w & 3) == 2) o[w >> 2].z = v;
  else o[w >> 2].w = v;
}

// ---------------------------------------------------------------------------
// score worker (warps 0-3): dt/dA of the chunk, xs = x * scale, S = CB o decay
// ---------------------------------------------------------------------------
__device__ void score_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h) {
  const int r = threadIdx.x;  // 0..127
  const int q = r >> 5, lane = r & 31;
  const uint32_t tmem = m->tmem_base + ((uint32_t)(q * 32) << 16);
  const float Ah = a.A[h];
  const float bias = a.dt_bias ? a.dt_bias[h] : 0.f;
  // decays factor as exp(dA_r - dA_R) * exp(dA_R - dA_t) with both exponents <= 0 when
  // the cumulative sum is non-increasing (A <= 0, dt >= 0); otherwise every element is
  // formed directly.
  const bool factor = (Ah <= 0.f) && (a.lo >= 0.f);
  const bool has_seq = a.seq_idx != nullptr;
  uint8_t* S_sm = sm + OFF_S;
  uint8_t* xs_sm = sm + OFF_XS;
  ChunkDt nxt = load_dt(a, bi, h, 0, r);
  for (int c = 0; c < a.nci; ++c) {
    const int s = c & 1;
    const int64_t t0 = (int64_t)c * QI;
    const ChunkDt cur = nxt;
    nxt = load_dt(a, bi, h, c + 1, r);
    const float dtv = (t0 + r < a.L) ? dt_process(cur.raw, bias, a.softplus, a.lo, a.hi) : 0.f;
    const int seqv = cur.seq;
    float cs = warp_incl_scan(dtv * Ah);
    if (lane == 31) m->red[q] = cs;
    ptx::named_bar_sync(1, 128);
    for (int w = 0; w < q; ++w) cs += m->red[w];
    const float dA = cs;
    m->dA[r] = dA;
    m->dt[r] = dtv;
    m->seq[r] = seqv;
    ptx::named_bar_sync(1, 128);
    const float dA_last = m->dA[QI - 1];
    const int last_valid = (int)min((int64_t)QI - 1, (int64_t)a.L - 1 - t0);
    const int end_seq = m->seq[last_valid];
    const float scale = (end_seq >= 0 && seqv == end_seq) ? __expf(dA_last - dA) * dtv : 0.f;

    // ---- E1: xs = x * scale ------------------------------------------------------
    if (!wait_bar(m, FULL0 + s, (c >> 1) & 1, a.status)) return;
    if (c > 0 && !wait_bar(m, B_L, (c - 1) & 1, a.status)) return;   // MMA_L(c-1) done with xs
    const uint8_t* x_sm = sm + OFF_STAGE + s * SZ_STAGE + 2 * SZ_C;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 w = *reinterpret_cast<const uint4*>(x_sm + ptx::sw128_off(r, j));
      *reinterpret_cast<uint4*>(xs_sm + ptx::sw128_off(r, j)) = scale_row16(w, scale);
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      ptx::mbar_arrive(&m->bar[XS_FULL]);
      ptx::mbar_arrive(&m->bar[EMPTY0 + s]);
    }

    // ---- E2: S[r][t] = CB[r][t] exp(dA_r - dA_t) dt_t  (t <= r, same sequence) ------
    if (!wait_bar(m, B_CB, c & 1, a.status)) return;
    if (c > 0 && !wait_bar(m, B_Y, (c - 1) & 1, a.status)) return;   // MMA2(c-1) done with S
    ptx::tc_fence_after();
    const float dA_R = m->dA[q * 32];
    const float u = __expf(dA - dA_R);
#pragma unroll 1
    for (int k32 = 0; k32 < 4; ++k32) {
      uint4 o[4];
      if (k32 < q && factor) {
        const int tl = k32 * 32 + lane;
        const float vl = __expf(dA_R - m->dA[tl]) * m->dt[tl];
        const int sl = m->seq[tl];
        float v[32];
        ptx::tmem_ld32(tmem + COL_CB + k32 * 32, v);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float s0 = v[i] * u * __shfl_sync(0xffffffffu, vl, i);
          float s1 = v[i + 1] * u * __shfl_sync(0xffffffffu, vl, i + 1);
          if (has_seq) {
            if (__shfl_sync(0xffffffffu, sl, i) != seqv) s0 = 0.f;
            if (__shfl_sync(0xffffffffu, sl, i + 1) != seqv) s1 = 0.f;
          }
          set_word(o, i >> 1, pack_bf16(s0, s1));
        }
      } else if (k32 <= q) {
        float v[32];
        ptx::tmem_ld32(tmem + COL_CB + k32 * 32, v);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int t = k32 * 32 + i;
          const bool ok0 = t <= r && (!has_seq || m->seq[t] == seqv);
          const bool ok1 = t + 1 <= r && (!has_seq || m->seq[t + 1] == seqv);
          const float s0 = ok0 ? v[i] * __expf(dA - m->dA[t]) * m->dt[t] : 0.f;
          const float s1 = ok1 ? v[i + 1] * __expf(dA - m->dA[t + 1]) * m->dt[t + 1] : 0.f;
          set_word(o, i >> 1, pack_bf16(s0, s1));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = make_uint4(0, 0, 0, 0);
      }
      const int kb = k32 >> 1;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(S_sm + kb * (QI * 128) + ptx::sw128_off(r, (k32 & 1) * 4 + j)) = o[j];
    }
    ptx::tc_fence_before();
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      ptx::mbar_arrive(&m->bar[CB_FREE]);
      ptx::mbar_arrive(&m->bar[S_FULL]);
    }
  }
}

// ---------------------------------------------------------------------------
// output worker (warps 4-7): state update in TMEM and the output epilogue
// ---------------------------------------------------------------------------
__device__ void out_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h) {
  const int r = threadIdx.x - 128;  // 0..127
  const int q = r >> 5, lane = r & 31;
  const uint32_t tmem = m->tmem_base + ((uint32_t)(q * 32) << 16);
  const int64_t L = a.L, H = a.H;
  const float Ah = a.A[h];
  const float bias = a.dt_bias ? a.dt_bias[h] : 0.f;
  const float D1 = a.D_ndim == 1 ? a.D[h] : 0.f;
  uint8_t* st_sm = sm + OFF_ST;
  const int64_t bh = (int64_t)bi * H + h;

  // state row n = r as bf16 into the MMA3 operand buffer ([n][p], 128B swizzled rows)
  auto publish_state = [&](const float (&lo)[32], const float (&hi)[32]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float* v = j < 4 ? lo + 8 * j : hi + 8 * (j - 4);
      uint4 w;
      w.x = pack_bf16(v[0], v[1]);
      w.y = pack_bf16(v[2], v[3]);
      w.z = pack_bf16(v[4], v[5]);
      w.w = pack_bf16(v[6], v[7]);
      *reinterpret_cast<uint4*>(st_sm + ptx::sw128_off(r, j)) = w;
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&m->bar[ST_FULL]);
  };
  {
    float lo[32], hi[32];
#pragma unroll
    for (int p = 0; p < 32; ++p) {
      lo[p] = a.init ? a.init[(bh * PT + p) * NT_ + r] : 0.f;
      hi[p] = a.init ? a.init[(bh * PT + 32 + p) * NT_ + r] : 0.f;
    }
    ptx::tmem_st32(tmem + COL_ST, lo);
    ptx::tmem_st32(tmem + COL_ST + 32, hi);
    ptx::tmem_st_wait();
    publish_state(lo, hi);
  }

  int prev_end = 0;
  ChunkDt nxt = load_dt(a, bi, h, 0, r);
  for (int c = 0; c < a.nci; ++c) {
    const int s = c & 1;
    const int64_t t0 = (int64_t)c * QI;
    const int64_t pos = t0 + r;
    const bool valid = pos < L;
    const int64_t o0 = (((int64_t)bi * L + (valid ? pos : 0)) * H + h) * PT;
    // z row of this chunk: issued now, used at the end of the chunk
    uint4 zr[8];
    if (a.z && valid) {
#pragma unroll
      for (int j = 0; j < 8; ++j) zr[j] = __ldg(reinterpret_cast<const uint4*>(a.z + o0) + j);
    }
    const ChunkDt cur = nxt;
    nxt = load_dt(a, bi, h, c + 1, r);
    const float dtv = valid ? dt_process(cur.raw, bias, a.softplus, a.lo, a.hi) : 0.f;
    float cs = warp_incl_scan(dtv * Ah);
    if (lane == 31) m->red_o[q] = cs;
    const int last_valid = (int)min((int64_t)QI - 1, L - 1 - t0);
    if (r == last_valid) m->end_seq_o = cur.seq;
    ptx::named_bar_sync(2, 128);
    for (int w = 0; w < q; ++w) cs += m->red_o[w];
    const float dA = cs;
    const float dA_last = m->red_o[0] + m->red_o[1] + m->red_o[2] + m->red_o[3];
    const int end_seq = m->end_seq_o;
    ptx::named_bar_sync(2, 128);
    const bool keep = end_seq == prev_end;
    const float sdec = (cur.seq == prev_end) ? __expf(dA) : 0.f;   // prev chunk's end seq
    prev_end = end_seq;
    const float decay = keep ? __expf(dA_last) : 0.f;

    // x row for the D term (copied out so the stage can be recycled)
    if (!wait_bar(m, FULL0 + s, (c >> 1) & 1, a.status)) return;
    uint4 xr[8];
    const uint8_t* x_sm = sm + OFF_STAGE + s * SZ_STAGE + 2 * SZ_C;
#pragma unroll
    for (int j = 0; j < 8; ++j) xr[j] = *reinterpret_cast<const uint4*>(x_sm + ptx::sw128_off(r, j));
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&m->bar[EMPTY0 + s]);

    // ---- E3: S_{c+1} = decay * S_c + Lt  (TMEM), bf16 copy for the next MMA3 ----------
    if (!wait_bar(m, B_L, c & 1, a.status)) return;
    ptx::tc_fence_after();
    float lo[32], hi[32], v[32];
    ptx::tmem_ld32(tmem + COL_L, v);
    ptx::tmem_ld32(tmem + COL_ST, lo);
    ptx::tmem_ld_wait();
#pragma unroll
    for (int p = 0; p < 32; ++p) lo[p] = decay * lo[p] + v[p];
    ptx::tmem_ld32(tmem + COL_L + 32, v);
    ptx::tmem_ld32(tmem + COL_ST + 32, hi);
    ptx::tmem_ld_wait();
#pragma unroll
    for (int p = 0; p < 32; ++p) hi[p] = decay * hi[p] + v[p];
    ptx::tmem_st32(tmem + COL_ST, lo);
    ptx::tmem_st32(tmem + COL_ST + 32, hi);
    ptx::tmem_st_wait();
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&m->bar[L_FREE]);
    if (!wait_bar(m, B_YI, c & 1, a.status)) return;   // MMA3(c) done reading S_c
    if (c + 1 < a.nci) publish_state(lo, hi);
    if (c + 1 == a.nci && a.final_states) {
#pragma unroll
      for (int p = 0; p < 32; ++p) {
        a.final_states[(bh * PT + p) * NT_ + r] = lo[p];
        a.final_states[(bh * PT + 32 + p) * NT_ + r] = hi[p];
      }
    }

    // ---- E4: out = Y + sdec * Yi + D x; z gate ------------------------------------------
    if (!wait_bar(m, B_Y, c & 1, a.status)) return;
    ptx::tc_fence_after();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float y[32];
      ptx::tmem_ld32(tmem + COL_Y + 32 * half, y);
      ptx::tmem_ld32(tmem + COL_YI + 32 * half, v);
      ptx::tmem_ld_wait();
#pragma unroll
      for (int p = 0; p < 32; ++p) y[p] += sdec * v[p];
      if (half == 1) {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&m->bar[Y_FREE]);
      }
      if (!valid) continue;
      if (a.D_ndim) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 w4 = xr[4 * half + j];
          const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16(wv[k]);
            const int p = 8 * j + 2 * k;
            const float d0 = a.D_ndim == 1 ? D1 : a.D[(int64_t)h * PT + 32 * half + p];
            const float d1 = a.D_ndim == 1 ? D1 : a.D[(int64_t)h * PT + 32 * half + p + 1];
            y[p] += d0 * f.x;
            y[p + 1] += d1 * f.y;
          }
        }
      }
      if (a.z) {
        if (a.out_x) {
#pragma unroll
          for (int p = 0; p < 32; p += 4)
            *reinterpret_cast<float4*>(a.out_x + o0 + 32 * half + p) = make_float4(y[p], y[p + 1], y[p + 2], y[p + 3]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 w4 = zr[4 * half + j];
          const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16(wv[k]);
            y[8 * j + 2 * k] *= silu(f.x);
            y[8 * j + 2 * k + 1] *= silu(f.y);
          }
        }
      }
#pragma unroll
      for (int p = 0; p < 32; p += 4)
        __stcs(reinterpret_cast<float4*>(a.out + o0 + 32 * half + p), make_float4(y[p], y[p + 1], y[p + 2], y[p + 3]));
    }
  }
}

__global__ void __launch_bounds__(NTHREADS, 1) ssd_fused_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Misc* m = reinterpret_cast<Misc*>(sm + OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bi = bh / a.H, h = bh % a.H;
  const int g = h / (a.H / a.G);

  if (threadIdx.x == 0) {
    ptx::mbar_init(&m->bar[FULL0], 1);
    ptx::mbar_init(&m->bar[FULL1], 1);
    ptx::mbar_init(&m->bar[EMPTY0], 9);   // MMA commit + 4 score warps + 4 output warps
    ptx::mbar_init(&m->bar[EMPTY1], 9);
    ptx::mbar_init(&m->bar[B_CB], 1);
    ptx::mbar_init(&m->bar[CB_FREE], 4);
    ptx::mbar_init(&m->bar[B_YI], 1);
    ptx::mbar_init(&m->bar[ST_FULL], 4);
    ptx::mbar_init(&m->bar[XS_FULL], 4);
    ptx::mbar_init(&m->bar[B_L], 1);
    ptx::mbar_init(&m->bar[L_FREE], 4);
    ptx::mbar_init(&m->bar[S_FULL], 4);
    ptx::mbar_init(&m->bar[B_Y], 1);
    ptx::mbar_init(&m->bar[Y_FREE], 4);
    ptx::mbar_init(&m->bar[DRAIN], 1);
    m->abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    ptx::prefetch_tmap(&a.tm_x);
    ptx::prefetch_tmap(&a.tm_b);
    ptx::prefetch_tmap(&a.tm_c);
  }
  if (warp == 9) {
    ptx::tmem_alloc(&m->tmem_base, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  if (warp < 4) {
    score_worker(a, sm, m, bi, h);
  } else if (warp < 8) {
    out_worker(a, sm, m, bi, h);
  } else if (warp == 8) {
    if (lane == 0) producer(a, sm, m, bi, h, g);
  } else {
    if (lane == 0) mma_issuer(a, sm, m);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(m->tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D bf16 map over (inner = cols, rows = L, batch) with a 64 x 128 x 1 box, 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t L, uint64_t b) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {cols, L, b};
  cuuint64_t strides[2] = {cols * 2, cols * L * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)QI, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool tc_supported(const ssd_fwd_params_t* p) {
  if (p->dtype != SSD_DTYPE_BF16 || p->headdim != PT || p->dstate != NT_) return false;
  if (p->dA_cumsum || p->dt_out || p->varlen_states) return false;
  if (p->batch * p->nheads > 0x7fffffff) return false;
  const uintptr_t al = 15;
  if ((reinterpret_cast<uintptr_t>(p->x) | reinterpret_cast<uintptr_t>(p->B) | reinterpret_cast<uintptr_t>(p->C) |
       reinterpret_cast<uintptr_t>(p->out) | reinterpret_cast<uintptr_t>(p->z) |
       reinterpret_cast<uintptr_t>(p->out_x)) & al)
    return false;
  return encode_fn() != nullptr;
}

size_t tc_workspace_bytes(const ssd_fwd_params_t* p) { return tc_supported(p) ? 256 : 0; }

int tc_num_launches(const ssd_fwd_params_t*) { return 1; }

int tc_combined_fwd(const ssd_fwd_params_t* p, void* workspace, cudaStream_t st) {
  TcArgs a;
  memset(&a, 0, sizeof(a));
  const int64_t b = p->batch, L = p->seqlen, H = p->nheads, G = p->ngroups;
  if (!make_map(&a.tm_x, p->x, (uint64_t)H * PT, L, b) || !make_map(&a.tm_b, p->B, (uint64_t)G * NT_, L, b) ||
      !make_map(&a.tm_c, p->C, (uint64_t)G * NT_, L, b))
    return SSD_ERR_CUDA;
  a.L = (int)L; a.H = (int)H; a.G = (int)G; a.nci = (int)((L + QI - 1) / QI);
  a.dt_bf16 = p->dt_dtype == SSD_DTYPE_BF16; a.softplus = p->dt_softplus; a.D_ndim = p->D ? p->D_ndim : 0;
  a.lo = p->dt_min; a.hi = p->dt_max;
  a.dt = p->dt; a.A = p->A; a.dt_bias = p->dt_bias; a.D = p->D;
  a.x = (const bf16*)p->x; a.z = (const bf16*)p->z; a.init = p->initial_states; a.seq_idx = p->seq_idx;
  a.out = p->out; a.out_x = p->z ? p->out_x : nullptr; a.final_states = p->final_states;
  a.status = (unsigned*)workspace;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(ssd_fused_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
        cudaSuccess)
      return SSD_ERR_CUDA;
    attr = true;
  }
  if (cudaMemsetAsync(workspace, 0, 4, st) != cudaSuccess) return SSD_ERR_CUDA;
  ssd_fused_tc_kernel<<<(unsigned)(b * H), NTHREADS, SMEM_BYTES, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? SSD_OK : SSD_ERR_CUDA;
}

}  // namespace ssd
