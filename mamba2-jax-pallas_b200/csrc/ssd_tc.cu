// Fused tcgen05 SSD forward for bf16 inputs (sm_100a).
//
// One CTA owns one (batch, head) and walks the sequence in internal chunks of 128 tokens.
// Nothing but the inputs, the outputs and the final state touches HBM: no chunk states,
// no CB matrix, no dA arrays.  The result does not depend on the internal chunk size
// (the reference's chunk_size only sets its own tiling; the seq_idx rules of
// chunk_state_fwd.py:246-269, state_passing_fwd.py:208-225 and chunk_scan_fwd.py:294-322
// compose to per-sequence semantics at any chunking), so every chunk_size maps here.
//
// Per chunk c (t = token in chunk, m = output row, n = state dim, p = head dim):
//   MMA1  CB[m][t]  = C[m][:] . B[t][:]                 (M=128, N=128, K=N)   TMEM
//   E2    S[m][t]   = CB[m][t] exp(dA_m - dA_t) dt_t    (t <= m, same seq)    -> smem bf16
//   MMA2  Y[m][p]   = S[m][:] . x[:][p]                 (M=128, N=64,  K=128) TMEM (2 bufs)
//   MMA3  Yi[m][p]  = C[m][:] . S_c[p][:]               (M=128, N=64,  K=N)   TMEM (2 bufs)
//   E1    xs[t][p]  = x[t][p] exp(dA_last - dA_t) dt_t  (chunk-end seq only)  -> smem bf16
//   MMA_L St[n][p] += B[:][n] . xs[:][p]                (M=N,   N=64,  K=128) TMEM state
//   E3    S_{c+1}   = St (already keep_c exp(dA_last_c) S_c + L_c);  bf16 -> smem for MMA3,
//                     St <- keep_{c+1} exp(dA_last_{c+1}) S_{c+1} for the next MMA_L
//   E4    out[m][p] = Y + exp(dA_m) [seq_m == prev] Yi + D x ; * silu(z)
// Decay factors are always formed from differences of the in-chunk cumulative sums
// (never exp(dA_m) * exp(-dA_t)), as ssd_naive.py:264-268 does.
//
// The only serial dependence between chunks is the state: E3(c) -> MMA3/MMA_L(c+1) ->
// E3(c+1).  Everything else is pipelined around it by warp role:
//   warps 0-3  (S0) dt/dA of the chunk, half of xs and of the score blocks
//   warps 4-7  (S1) the other halves
//   warps 8-11 (T)  state recurrence E3
//   warps 12-15(O)  output epilogue E4 (one chunk behind, double-buffered Y/Yi)
//   warp 16 TMA producer, warp 17 MMA issuer.
// Warp w reads TMEM lanes 32*(w%4)..+31, i.e. chunk rows of its quadrant.
// Every mbarrier wait is bounded; on timeout the CTA records SSD_ERR_TIMEOUT in the status
// word, drains its async work and exits.
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
constexpr int NTHREADS = 576;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_CB = 0, COL_Y0 = 128, COL_YI0 = 192, COL_ST = 384;  // Y/Yi buffer b at +128*b

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t SZ_C = QI * NT_ * 2;          // 32 KB  (two 64-wide swizzled boxes)
constexpr uint32_t SZ_X = QI * PT * 2;           // 16 KB
constexpr uint32_t SZ_STAGE = 2 * SZ_C + SZ_X;   // C, B, x
constexpr uint32_t OFF_STAGE = 0;
constexpr uint32_t OFF_S = 2 * SZ_STAGE;         // scores, 32 KB (two K-blocks)
constexpr uint32_t OFF_XS = OFF_S + QI * QI * 2; // 16 KB
constexpr uint32_t OFF_ST = OFF_XS + SZ_X;       // state bf16 [n][p], 16 KB
constexpr uint32_t OFF_MISC = OFF_ST + NT_ * PT * 2;
constexpr uint32_t MISC_BYTES = 2560;
constexpr uint32_t SMEM_BYTES = OFF_MISC + MISC_BYTES;   // bytes used from the 1024-aligned base
constexpr uint32_t SMEM_LAUNCH_BYTES = 232448;            // per-CTA maximum; the rest is alignment slack

enum Bar { FULL0, FULL1, EMPTY0, EMPTY1, B_CB, CB_FREE, XS_FULL, S_FULL, ST_READY, B_L, B_Y0, B_Y1, Y_FREE0,
           Y_FREE1, DRAIN, NBARS };

// arrivals per phase
constexpr uint32_t EMPTY_COUNT = 1 + 8 + 4;   // MMA commit, S0+S1 warps (xs), O warps (D x)

struct Misc {
  uint64_t bar[NBARS];
  float dA[2][QI];      // per-chunk cumulative dt*A, double-buffered by chunk parity
  float dt[2][QI];      // processed dt
  float red_s[4];
  float red_t[2][4];
  int end_t[2];
  float red_o[2][4];
  int end_o[2];
  uint32_t tmem_base;
  volatile int abort;
};
static_assert(sizeof(Misc) <= MISC_BYTES, "misc area");

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
// producer (warp 16, lane 0): C, B, x tiles of each chunk into a 2-stage ring
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
// MMA issuer (warp 17, lane 0)
// ---------------------------------------------------------------------------
__device__ void mma_issuer(const TcArgs& a, uint8_t* sm, Misc* m) {
  const uint32_t tmem = m->tmem_base;
  const uint32_t base = ptx::smem_u32(sm);
  constexpr uint32_t ID_CB = ptx::idesc_bf16_f32(128, 128, 0, 0);
  constexpr uint32_t ID_YI = ptx::idesc_bf16_f32(128, 64, 0, 1);
  constexpr uint32_t ID_L = ptx::idesc_bf16_f32(128, 64, 1, 1);
  constexpr uint32_t ID_Y = ptx::idesc_bf16_f32(128, 64, 0, 1);
  for (int c = 0; c < a.nci; ++c) {
    const int s = c & 1, yb = c & 1;
    const uint32_t st = base + OFF_STAGE + s * SZ_STAGE;
    const uint32_t sC = st, sB = st + SZ_C, sX = st + 2 * SZ_C;
    // MMA1: CB = C . B^T (both K-major: row = token, K = state dim in two 64-wide boxes)
    if (!wait_bar(m, FULL0 + s, (c >> 1) & 1, a.status)) break;
    if (c > 0 && !wait_bar(m, CB_FREE, (c - 1) & 1, a.status)) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < NT_ / 16; ++i) {
      const uint32_t off = (i >> 2) * (SZ_C / 2) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_CB, ptx::sdesc_sw128(sC + off, 16, 1024), ptx::sdesc_sw128(sB + off, 16, 1024),
                   ID_CB, i > 0);
    }
    ptx::mma_commit(&m->bar[B_CB]);
    // MMA3: Yi[yb] = C . S_c^T   (B operand = bf16 state [n][p], MN-major)
    if (!wait_bar(m, ST_READY, c & 1, a.status)) break;
    if (c >= 2 && !wait_bar(m, Y_FREE0 + yb, ((c - 2) >> 1) & 1, a.status)) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < NT_ / 16; ++i) {
      const uint32_t offa = (i >> 2) * (SZ_C / 2) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_YI0 + 128 * yb, ptx::sdesc_sw128(sC + offa, 16, 1024),
                   ptx::sdesc_sw128(base + OFF_ST + i * 2048, 8192, 1024), ID_YI, i > 0);
    }
    // MMA_L: St += B^T . xs  onto the pre-scaled state (A = B tile MN-major, B = xs MN-major)
    if (!wait_bar(m, XS_FULL, c & 1, a.status)) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < QI / 16; ++i) {
      ptx::mma_f16(tmem + COL_ST, ptx::sdesc_sw128(sB + i * 2048, SZ_C / 2, 1024),
                   ptx::sdesc_sw128(base + OFF_XS + i * 2048, 8192, 1024), ID_L, 1);
    }
    ptx::mma_commit(&m->bar[B_L]);   // state S_{c+1} complete; MMA3(c) done with the bf16 state
    // MMA2: Y[yb] = S . x   (A = scores K-major, B = x [t][p] MN-major)
    if (!wait_bar(m, S_FULL, c & 1, a.status)) break;
    ptx::tc_fence_after();
#pragma unroll
    for (int i = 0; i < QI / 16; ++i) {
      const uint32_t offa = (i >> 2) * (QI * 128) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_Y0 + 128 * yb, ptx::sdesc_sw128(base + OFF_S + offa, 16, 1024),
                   ptx::sdesc_sw128(sX + i * 2048, 8192, 1024), ID_Y, i > 0);
    }
    ptx::mma_commit(&m->bar[B_Y0 + yb]);
    ptx::mma_commit(&m->bar[EMPTY0 + s]);
  }
  // drain: wait (bounded) until every issued MMA has completed
  ptx::mma_commit(&m->bar[DRAIN]);
  const uint64_t t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(&m->bar[DRAIN], 0) && ptx::globaltimer() - t0 < TIMEOUT_NS) {
  }
}

// ---------------------------------------------------------------------------
// helpers shared by the worker warpgroups
// ---------------------------------------------------------------------------
struct ChunkDt {
  float raw;
  int seq;
};

// Raw dt and seq id of chunk row r (seq -1 past the end of the sequence or the chunks).
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

__device__ __forceinline__ int seq_at(const TcArgs& a, int bi, int64_t pos) {
  return (pos < a.L) ? a.seq_idx[(int64_t)bi * a.L + pos] : -1;
}

// Chunk-level values every role needs: dA_last (sum of dt*A over the chunk) and the seq id
// at the chunk's last valid position.  One reduction through `red`/`endv` + one named
// barrier; the caller double-buffers the slots by chunk parity.
__device__ __forceinline__ void chunk_totals(float v, int seqv, int r, int last_valid, float* red, int* endv,
                                             int bar_id, float& total, int& end_seq) {
  const float w = warp_sum(v);
  if ((r & 31) == 0) red[r >> 5] = w;
  if (r == last_valid) *endv = seqv;
  ptx::named_bar_sync(bar_id, 128);
  total = red[0] + red[1] + red[2] + red[3];
  end_seq = *endv;
}

// 16-byte word of 8 bf16, scaled by `s`, repacked.
__device__ __forceinline__ uint4 scale_row16(uint4 w, float s) {
  uint4 o;
  float2 f;
  f = unpack_bf16(w.x); o.x = pack_bf16(f.x * s, f.y * s);
  f = unpack_bf16(w.y); o.y = pack_bf16(f.x * s, f.y * s);
  f = unpack_bf16(w.z); o.z = pack_bf16(f.x * s, f.y * s);
  f = unpack_bf16(w.w); o.w = pack_bf16(f.x * s, f.y * s);
  return o;
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
}

// ---------------------------------------------------------------------------
// score workers S0 (warps 0-3, half 0) and S1 (warps 4-7, half 1).
// S0 computes the chunk's processed dt and cumulative dA into shared memory; both
// halves then build xs columns [32*half, 32*half+32) and score column blocks
// {half, half+2} of their rows, which balances the causal triangle (quadrant q has
// q+1 non-zero 32-column blocks) to at most two blocks per warp.
// Loops stay rolled (8-column steps) to keep the per-chunk code small.
// ---------------------------------------------------------------------------
__device__ void score_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h, int half) {
  const int r = threadIdx.x & 127;
  const int q = r >> 5, lane = r & 31;
  const uint32_t tmem = m->tmem_base + ((uint32_t)(q * 32) << 16);
  const float Ah = a.A[h];
  const float bias = a.dt_bias ? a.dt_bias[h] : 0.f;
  // Below the diagonal block the decay factors as exp(dA_r - dA_R) * exp(dA_R - dA_t)
  // (R = first row of the warp's block) with both exponents <= 0 when the cumulative
  // sum is non-increasing (A <= 0, dt >= 0); otherwise every element is formed directly.
  const bool factor = (Ah <= 0.f) && (a.lo >= 0.f);
  const bool has_seq = a.seq_idx != nullptr;
  uint8_t* S_sm = sm + OFF_S;
  uint8_t* xs_sm = sm + OFF_XS;
  ChunkDt nxt = half == 0 ? load_dt(a, bi, h, 0, r) : ChunkDt{0.f, 0};
#pragma unroll 1
  for (int c = 0; c < a.nci; ++c) {
    const int s = c & 1, buf = c & 1;
    const int64_t t0 = (int64_t)c * QI;
    const bool valid = t0 + r < a.L;
    if (half == 0) {
      const ChunkDt cur = nxt;
      nxt = load_dt(a, bi, h, c + 1, r);
      const float dtv = valid ? dt_process(cur.raw, bias, a.softplus, a.lo, a.hi) : 0.f;
      float cs = warp_incl_scan(dtv * Ah);
      if (lane == 31) m->red_s[q] = cs;
      ptx::named_bar_sync(1, 128);
      for (int w = 0; w < q; ++w) cs += m->red_s[w];
      m->dA[buf][r] = cs;
      m->dt[buf][r] = dtv;
    }
    ptx::named_bar_sync(3, 256);
    const float dA = m->dA[buf][r];
    const float dtv = m->dt[buf][r];
    const float dA_last = m->dA[buf][QI - 1];
    const int last_valid = (int)min((int64_t)QI - 1, (int64_t)a.L - 1 - t0);
    int seqv = valid ? 0 : -1, end_seq = 0, sl0 = 0, sl1 = 0;
    if (has_seq) {
      seqv = seq_at(a, bi, t0 + r);
      end_seq = seq_at(a, bi, t0 + last_valid);
      sl0 = seq_at(a, bi, t0 + half * 32 + lane);
      sl1 = seq_at(a, bi, t0 + (half + 2) * 32 + lane);
    }
    const float scale = (end_seq >= 0 && seqv == end_seq) ? __expf(dA_last - dA) * dtv : 0.f;

    // ---- E1: xs = x * scale (this half's 4 16-byte words of row r) -----------------
    if (!wait_bar(m, FULL0 + s, (c >> 1) & 1, a.status)) return;
    if (c > 0 && !wait_bar(m, B_L, (c - 1) & 1, a.status)) return;   // MMA_L(c-1) done with xs
    const uint8_t* x_sm = sm + OFF_STAGE + s * SZ_STAGE + 2 * SZ_C;
#pragma unroll 1
    for (int j = 4 * half; j < 4 * half + 4; ++j) {
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
    if (c > 0 && !wait_bar(m, B_Y0 + ((c - 1) & 1), ((c - 1) >> 1) & 1, a.status)) return;  // MMA2(c-1) done with S
    ptx::tc_fence_after();
    const float dA_R = m->dA[buf][q * 32];
    const float u = __expf(dA - dA_R);
#pragma unroll 1
    for (int kk = 0; kk < 2; ++kk) {
      const int k32 = half + 2 * kk;
      uint8_t* Srow = S_sm + (k32 >> 1) * (QI * 128);
      const int j0 = (k32 & 1) * 4;
      if (k32 > q) {
#pragma unroll 1
        for (int sub = 0; sub < 4; ++sub)
          *reinterpret_cast<uint4*>(Srow + ptx::sw128_off(r, j0 + sub)) = make_uint4(0, 0, 0, 0);
        continue;
      }
      const int tl = k32 * 32 + lane;
      const float dAl = m->dA[buf][tl];
      const float dtl = m->dt[buf][tl];
      const int sl = kk == 0 ? sl0 : sl1;
      const bool fac = factor && k32 < q;
      const bool diag = k32 == q;
      const float vl = fac ? __expf(dA_R - dAl) * dtl : 0.f;
#pragma unroll 1
      for (int sub = 0; sub < 4; ++sub) {
        float v[8];
        ptx::tmem_ld8(tmem + COL_CB + k32 * 32 + sub * 8, v);
        ptx::tmem_ld_wait();
        if (fac) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int src = sub * 8 + i;
            float w = u * __shfl_sync(0xffffffffu, vl, src);
            if (has_seq && __shfl_sync(0xffffffffu, sl, src) != seqv) w = 0.f;
            v[i] *= w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int src = sub * 8 + i;
            const float dAt = __shfl_sync(0xffffffffu, dAl, src);
            const float dtt = __shfl_sync(0xffffffffu, dtl, src);
            bool ok = !diag || src <= lane;
            if (has_seq) ok = ok && (__shfl_sync(0xffffffffu, sl, src) == seqv);
            v[i] = v[i] * __expf(ok ? dA - dAt : -INFINITY) * dtt;
          }
        }
        *reinterpret_cast<uint4*>(Srow + ptx::sw128_off(r, j0 + sub)) = pack8(v);
      }
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
// state worker T (warps 8-11): the inter-chunk recurrence.  Thread r owns state row
// n = r (TMEM lane r, 64 f32 columns).  MMA_L(c) accumulates L_c onto the pre-scaled
// state keep_c exp(dA_last_c) S_c, so after B_L(c) the columns hold S_{c+1}.
// ---------------------------------------------------------------------------
__device__ void state_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h) {
  const int r = threadIdx.x & 127;
  const int q = r >> 5, lane = r & 31;
  const uint32_t tmem = m->tmem_base + ((uint32_t)(q * 32) << 16) + COL_ST;
  const float Ah = a.A[h];
  const float bias = a.dt_bias ? a.dt_bias[h] : 0.f;
  uint8_t* st_sm = sm + OFF_ST;
  const int64_t bh = (int64_t)bi * a.H + h;
  int prev_end = 0;
  // decay applied to S_c before L_c is added (0 at a sequence reset, ssd rule A9)
  auto chunk_decay = [&](int cc, const ChunkDt& cur) -> float {
    const int64_t t0 = (int64_t)cc * QI;
    const bool valid = t0 + r < a.L;
    const float dtv = valid ? dt_process(cur.raw, bias, a.softplus, a.lo, a.hi) : 0.f;
    const int last_valid = (int)min((int64_t)QI - 1, (int64_t)a.L - 1 - t0);
    float total;
    int end_seq;
    chunk_totals(dtv * Ah, cur.seq, r, last_valid, m->red_t[cc & 1], &m->end_t[cc & 1], 4, total, end_seq);
    const bool keep = end_seq == prev_end;
    prev_end = end_seq;
    return keep ? __expf(total) : 0.f;
  };
  ChunkDt nxt = load_dt(a, bi, h, 0, r);
  float decay = chunk_decay(0, nxt);
  nxt = load_dt(a, bi, h, 1, r);
  // S_0 = initial state (or 0): bf16 operand for MMA3(0), pre-scaled f32 for MMA_L(0)
#pragma unroll 1
  for (int j = 0; j < 8; ++j) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = a.init ? a.init[(bh * PT + 8 * j + i) * NT_ + r] : 0.f;
    *reinterpret_cast<uint4*>(st_sm + ptx::sw128_off(r, j)) = pack8(v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] *= decay;
    ptx::tmem_st8(tmem + 8 * j, v);
  }
  ptx::tmem_st_wait();
  ptx::tc_fence_before();
  ptx::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(&m->bar[ST_READY]);

#pragma unroll 1
  for (int c = 0; c < a.nci; ++c) {
    const bool more = c + 1 < a.nci;
    if (more) {
      decay = chunk_decay(c + 1, nxt);
      nxt = load_dt(a, bi, h, c + 2, r);
    }
    if (!wait_bar(m, B_L, c & 1, a.status)) return;
    ptx::tc_fence_after();
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
      float v[8];
      ptx::tmem_ld8(tmem + 8 * j, v);
      ptx::tmem_ld_wait();
      if (more) {
        *reinterpret_cast<uint4*>(st_sm + ptx::sw128_off(r, j)) = pack8(v);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] *= decay;
        ptx::tmem_st8(tmem + 8 * j, v);
      } else if (a.final_states) {
#pragma unroll
        for (int i = 0; i < 8; ++i) a.final_states[(bh * PT + 8 * j + i) * NT_ + r] = v[i];
      }
    }
    if (more) {
      ptx::tmem_st_wait();
      ptx::tc_fence_before();
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&m->bar[ST_READY]);
    }
  }
}

// ---------------------------------------------------------------------------
// output worker O (warps 12-15): out[m][p] = Y + sdec_m Yi + D x, z gate; one chunk
// behind the MMAs thanks to the double-buffered Y/Yi accumulators.
// ---------------------------------------------------------------------------
__device__ void out_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h) {
  const int r = threadIdx.x & 127;
  const int q = r >> 5, lane = r & 31;
  const uint32_t tmem = m->tmem_base + ((uint32_t)(q * 32) << 16);
  const int64_t L = a.L, H = a.H;
  const float Ah = a.A[h];
  const float bias = a.dt_bias ? a.dt_bias[h] : 0.f;
  const float D1 = a.D_ndim == 1 ? a.D[h] : 0.f;
  int prev_end = 0;
  ChunkDt nxt = load_dt(a, bi, h, 0, r);
#pragma unroll 1
  for (int c = 0; c < a.nci; ++c) {
    const int s = c & 1, yb = c & 1;
    const int64_t t0 = (int64_t)c * QI;
    const int64_t pos = t0 + r;
    const bool valid = pos < L;
    const int64_t o0 = (((int64_t)bi * L + (valid ? pos : 0)) * H + h) * PT;
    const ChunkDt cur = nxt;
    nxt = load_dt(a, bi, h, c + 1, r);
    const float dtv = valid ? dt_process(cur.raw, bias, a.softplus, a.lo, a.hi) : 0.f;
    float cs = warp_incl_scan(dtv * Ah);
    if (lane == 31) m->red_o[c & 1][q] = cs;
    const int last_valid = (int)min((int64_t)QI - 1, L - 1 - t0);
    if (r == last_valid) m->end_o[c & 1] = cur.seq;
    ptx::named_bar_sync(2, 128);
    for (int w = 0; w < q; ++w) cs += m->red_o[c & 1][w];
    const int end_seq = m->end_o[c & 1];
    const float sdec = (cur.seq == prev_end) ? __expf(cs) : 0.f;   // rows continuing the previous chunk's sequence
    prev_end = end_seq;

    if (!wait_bar(m, B_Y0 + yb, (c >> 1) & 1, a.status)) return;
    ptx::tc_fence_after();
    const uint8_t* x_sm = sm + OFF_STAGE + s * SZ_STAGE + 2 * SZ_C;
    const bool zon = a.z != nullptr && valid;
    const uint4* zp = reinterpret_cast<const uint4*>(a.z + o0);
    uint4 zn = make_uint4(0, 0, 0, 0);
    if (zon) zn = __ldg(zp);
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
      float y[8], yi[8];
      ptx::tmem_ld8(tmem + COL_Y0 + 128 * yb + 8 * j, y);
      ptx::tmem_ld8(tmem + COL_YI0 + 128 * yb + 8 * j, yi);
      const uint4 zc = zn;
      if (zon && j < 7) zn = __ldg(zp + j + 1);
      const uint4 xw = *reinterpret_cast<const uint4*>(x_sm + ptx::sw128_off(r, j));
      ptx::tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] += sdec * yi[i];
      if (a.D_ndim) {
        const uint32_t wv[4] = {xw.x, xw.y, xw.z, xw.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16(wv[k]);
          const int p = 8 * j + 2 * k;
          y[2 * k] += (a.D_ndim == 1 ? D1 : a.D[(int64_t)h * PT + p]) * f.x;
          y[2 * k + 1] += (a.D_ndim == 1 ? D1 : a.D[(int64_t)h * PT + p + 1]) * f.y;
        }
      }
      if (valid) {
        if (a.z) {
          if (a.out_x) {
            *reinterpret_cast<float4*>(a.out_x + o0 + 8 * j) = make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4*>(a.out_x + o0 + 8 * j + 4) = make_float4(y[4], y[5], y[6], y[7]);
          }
          const uint32_t wv[4] = {zc.x, zc.y, zc.z, zc.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = unpack_bf16(wv[k]);
            y[2 * k] *= silu(f.x);
            y[2 * k + 1] *= silu(f.y);
          }
        }
        __stcs(reinterpret_cast<float4*>(a.out + o0 + 8 * j), make_float4(y[0], y[1], y[2], y[3]));
        __stcs(reinterpret_cast<float4*>(a.out + o0 + 8 * j + 4), make_float4(y[4], y[5], y[6], y[7]));
      }
    }
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      ptx::mbar_arrive(&m->bar[Y_FREE0 + yb]);
      ptx::mbar_arrive(&m->bar[EMPTY0 + s]);
    }
  }
}

__global__ void __launch_bounds__(NTHREADS, 1) ssd_fused_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
  uint8_t* sm = reinterpret_cast<uint8_t*>((raw + 1023) & ~uintptr_t(1023));
  if (sm - smem_raw > (ptrdiff_t)(SMEM_LAUNCH_BYTES - SMEM_BYTES)) {
    // the dynamic shared window is not aligned enough for the swizzled tiles: report, do nothing
    if (threadIdx.x == 0) atomicCAS(a.status, 0u, 0x200u);
    return;
  }
  Misc* m = reinterpret_cast<Misc*>(sm + OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bi = bh / a.H, h = bh % a.H;
  const int g = h / (a.H / a.G);

  if (threadIdx.x == 0) {
    ptx::mbar_init(&m->bar[FULL0], 1);
    ptx::mbar_init(&m->bar[FULL1], 1);
    ptx::mbar_init(&m->bar[EMPTY0], EMPTY_COUNT);
    ptx::mbar_init(&m->bar[EMPTY1], EMPTY_COUNT);
    ptx::mbar_init(&m->bar[B_CB], 1);
    ptx::mbar_init(&m->bar[CB_FREE], 8);
    ptx::mbar_init(&m->bar[XS_FULL], 8);
    ptx::mbar_init(&m->bar[S_FULL], 8);
    ptx::mbar_init(&m->bar[ST_READY], 4);
    ptx::mbar_init(&m->bar[B_L], 1);
    ptx::mbar_init(&m->bar[B_Y0], 1);
    ptx::mbar_init(&m->bar[B_Y1], 1);
    ptx::mbar_init(&m->bar[Y_FREE0], 4);
    ptx::mbar_init(&m->bar[Y_FREE1], 4);
    ptx::mbar_init(&m->bar[DRAIN], 1);
    m->abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 16 && lane == 0) {
    ptx::prefetch_tmap(&a.tm_x);
    ptx::prefetch_tmap(&a.tm_b);
    ptx::prefetch_tmap(&a.tm_c);
  }
  if (warp == 17) {
    ptx::tmem_alloc(&m->tmem_base, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  if (warp < 8) {
    score_worker(a, sm, m, bi, h, warp >> 2);
  } else if (warp < 12) {
    state_worker(a, sm, m, bi, h);
  } else if (warp < 16) {
    out_worker(a, sm, m, bi, h);
  } else if (warp == 16) {
    if (lane == 0) producer(a, sm, m, bi, h, g);
  } else {
    if (lane == 0) mma_issuer(a, sm, m);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 17) {
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
    if (cudaFuncSetAttribute(ssd_fused_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LAUNCH_BYTES) !=
        cudaSuccess)
      return SSD_ERR_CUDA;
    attr = true;
  }
  if (cudaMemsetAsync(workspace, 0, 4, st) != cudaSuccess) return SSD_ERR_CUDA;
  ssd_fused_tc_kernel<<<(unsigned)(b * H), NTHREADS, SMEM_LAUNCH_BYTES, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? SSD_OK : SSD_ERR_CUDA;
}

}  // namespace ssd
