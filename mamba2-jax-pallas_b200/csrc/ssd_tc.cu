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
//   E2    S[m][t]   = CB[m][t] exp(dA_m - dA_t) dt_t    (t <= m, same seq)    -> TMEM bf16
//         S[m][m]  += D                                 (the skip term D x rides on MMA2)
//   MMA2  Y[m][p]   = S[m][:] . x[:][p]                 (M=128, N=64,  K=128) TMEM
//   MMA3  Yi[m][p]  = C[m][:] . S_c[p][:]               (M=128, N=64,  K=N)   TMEM (2 bufs at N=128)
//   E1    xs[t][p]  = x[t][p] exp(dA_last - dA_t) dt_t  (chunk-end seq only)  -> smem bf16
//   MMA_L Lt[n][p]  = B[:][n] . xs[:][p]                (M=N,   N=64,  K=128) TMEM
//   E3    S_{c+1}   = keep_c exp(dA_last_c) S_c + Lt    (TMEM f32)  -> bf16 smem for MMA3
//   E4    out[m][p] = Y + exp(dA_m) [seq_m == prev] Yi ; * silu(z)
// Decay factors come from differences of the in-chunk cumulative sums, as in
// ssd_naive.py:264-268, never from exp(dA_m) * exp(-dA_t) over a whole chunk.  Within one
// 32-token column block k they factor as exp(dA_m - dA_{32k}) * exp(dA_{32k} - dA_t) when
// dA is non-increasing and the block's range is at most 60 (both factors then stay in
// float range); other blocks are formed element by element.
//
// The only serial dependence between chunks is the state: E3(c) -> MMA3(c+1) -> E3(c+1).
// Everything else is pipelined around it by warp role (16 warps, so every SM sub-partition
// holds 4 warps and each thread may use 128 registers):
//   warp 0      MMA issuer B (lane 0): MMA3, MMA_L (the state chain)
//   warp 1      MMA issuer A (lane 0): MMA1, MMA2; owns the TMEM allocation (512 columns)
//   warp 2      TMA producer (lane 0)
//   warp 3      dA producer (lane 0): the chunk's cumulative dA and decay factors, computed
//               by the dt pre-pass, bulk-copied into shared memory
//   warps 4-7   SA: xs columns 0-31, score column blocks 0 and 2 of each row quadrant
//   warps 8-11  SB: xs columns 32-63, score column blocks 1 and 3
//   warps 12-15 T: the state recurrence E3 and the output epilogue E4 of the previous chunk
//               (staged in shared memory, written by TMA bulk stores)
// MMA_L accumulates the chunk's state contribution L_c in its own TMEM columns, so xs and
// MMA_L do not wait for the state chain.  The bf16 scores go back into TMEM (over the CB
// columns already read) and MMA2 takes them from there as its A operand.  Warp w reads TMEM lanes 32*(w%4)..+31, i.e. chunk
// rows of its quadrant; TMEM reads are issued 32 columns at a time with one wait, since
// each round trip is expensive.
// Every mbarrier wait is bounded; on timeout the CTA records SSD_ERR_TIMEOUT in the status
// word, drains its async work and exits.
#include <cuda.h>
#include <cstdio>
#include <cstdlib>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "ptx_sm100.cuh"
#include "ssd_kernels.h"
#include "ssd_tc.h"

namespace ssd {
namespace {

constexpr int QI = 128;       // internal chunk (tokens)
constexpr int PT = 64;        // head dim handled by the kernel
constexpr int NTHREADS = 512;
// Single-lane roles of warps 0-3.  Warp w issues on SM sub-partition w % 4, which it shares
// with the score and state warps of row quadrant w % 4; quadrant 3 has the most score work
// (four 32-column blocks against one in quadrant 0), so the lightest role sits on 3 and
// the state chain's MMA issuer on 0.
constexpr int W_ISSUE_B = 0, W_ISSUE_A = 1, W_PRODUCER = 2, W_DA = 3;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t MISC_BYTES = 2624;
constexpr uint32_t SMEM_LAUNCH_BYTES = 232448;            // per-CTA maximum; the rest is alignment slack
// TMEM columns: CB / bf16 scores, two buffers (b at 128*b) | Y buffers | Yi buffers (64 each) |
// f32 state (64 per 128-row half of the state dim).  MMA_L accumulates straight onto the
// state after T has scaled it by the chunk decay, so the state update needs no column of
// its own and the CB region can be double-buffered.
constexpr uint32_t COL_CB0 = 0, COL_Y0 = 256;
// Yi buffers at N = 128 (Y gets the other of three 64-column slots).  Two Yi buffers let
// the output of c-1 follow the state copy of c, but MMA2(c) must then wait for it: slower
// on long single sequences, faster on many short CTAs.  Default one.
#ifndef SSD_TC_YI_BUFS
#define SSD_TC_YI_BUFS 1
#endif

// Layout for state dim NT (128 or 256).  C and B stream through a 2-stage ring in 128-column
// halves (one half per stage), x through its own ring.  Shared memory (from a 1024-aligned
// base): CB ring | x ring | scores 32 KB | xs 16 KB | bf16 state [n][p] | misc.
template <int NT>
struct Geo {
  static constexpr int NH = NT / 128;               // 128-column halves of the state dim
  static constexpr int XST = NH == 1 ? 2 : 1;       // x buffers
  static constexpr int YIB = NH == 1 ? SSD_TC_YI_BUFS : 1;   // Yi accumulator buffers
  static constexpr int YB = NH == 1 ? 3 - YIB : 1;           // Y accumulator buffers
  static constexpr uint32_t COL_YI0 = COL_Y0 + 64 * YB;
  static constexpr uint32_t SZ_H = QI * 128 * 2;    // one half of C or B: 32 KB (two 64-col boxes)
  static constexpr uint32_t SZ_CBST = 2 * SZ_H;     // ring stage: C half + B half
  static constexpr uint32_t SZ_X = QI * PT * 2;     // 16 KB
  static constexpr uint32_t OFF_CB = 0;
  static constexpr uint32_t OFF_X = 2 * SZ_CBST;
  static constexpr uint32_t OFF_S = OFF_X + XST * SZ_X;
  static constexpr uint32_t OFF_XS = OFF_S + QI * QI * 2;
  static constexpr uint32_t OFF_ST = OFF_XS + SZ_X;
  static constexpr uint32_t OFF_MISC = OFF_ST + NT * PT * 2;
  static constexpr uint32_t SMEM_BYTES = OFF_MISC + MISC_BYTES;
  static constexpr uint32_t COL_ST = COL_YI0 + 64 * YIB;
  static_assert(SMEM_BYTES <= SMEM_LAUNCH_BYTES, "shared memory");
  static_assert(COL_ST + 64 * NH <= TMEM_COLS, "tensor memory");
};

// Barriers.  Every barrier that a role can reach again for a later chunk before another role
// has consumed the current phase is per buffer (B_CB, CB_FREE, S_FULL_*, B_YI, YI_FREE), so
// no waiter can see a phase parity two phases late.
enum Bar { CB_FULL0, CB_FULL1, CB_EMPTY0, CB_EMPTY1, X_FULL0, X_FULL1, X_EMPTY0, X_EMPTY1, B_CB0, B_CB1,
           CB_FREE0, CB_FREE1, XS_FULL, S_FULL_A0, S_FULL_A1, S_FULL_B0, S_FULL_B1,
           ST_READY, SCALED, B_L, XS_FREE, B_Y0, B_Y1, B_YI0, B_YI1, Y_FREE0, Y_FREE1, YI_FREE0, YI_FREE1, DA_READY0, DA_READY1, DA_FREE0,
           DA_FREE1, OUT_READ, STAGED, DRAIN, NBARS };

// arrivals per phase
constexpr uint32_t X_EMPTY_COUNT = 1 + 4 + 4;   // MMA2 commit, SA and SB warps (their halves of xs)
constexpr uint32_t DA_FREE_COUNT = 12;        // SA, SB and T warps done with a chunk's dA/dt arrays

struct Misc {
  float dA[2][QI];      // per-chunk cumulative dt*A, double-buffered by chunk parity
  // Per token t of 32-token block k: w_t = exp(dA_{32k} - dA_t) dt_t when block k is
  // factored (block_factored), else the processed dt_t.
  float dt[2][QI];
  float Dh;             // skip coefficient of the head (0 without D)
  uint64_t bar[NBARS];
  uint32_t tmem_base;
  int nci;              // chunks of this CTA's walk (from the schedule when there is one)
  volatile int abort;
};
static_assert(sizeof(Misc) <= MISC_BYTES, "misc area");

struct TcArgs {
  CUtensorMap tm_x, tm_b, tm_c, tm_out;
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
  float* varlen_states;        // (num_seqs, H, P, N) or null
  const float* dtprep;         // per (b, h, chunk): dA[128] then w[128], from tc_dt_prep_kernel
  int prep_cap;                // chunk slots per (b, h) in dtprep
  const int* sched_n;          // chunk count written by the schedule kernel, or null
  const int2* sched;           // {t0, varlen slot or -1} per chunk, entry nci = {L, -1}
  unsigned* status;
  long long test_wait_cycles;  // > 0: test mode, see the start of ssd_fused_tc_kernel
  int seg_k;                   // rows per batch row when the sequence is split (1: no split)
  int rows;                    // batch rows of the walk (b * seg_k)
  int num_seqs;                // varlen states: sequences
  int sched_cap;               // varlen: schedule entries (without the sentinel)
  const float* seg_state;      // split: L_j of every segment but the last, (b*seg_k, H, P, N)
  const float* seg_tot;        // split: total dA of each segment, (b*seg_k, H)
  unsigned long long* trace;   // debug phase timestamps (CTA 0, SSD_TC_TRACE=1), or null
};

// Debug trace: globaltimer at phase boundaries of CTA 0, slot [role][chunk][phase].  Compiled
// in only with -DSSD_TC_DEBUG_TRACE (and then enabled at run time by SSD_TC_TRACE=1).
#ifdef SSD_TC_DEBUG_TRACE
#define TRACE(role, c, ph)                                                                       \
  do {                                                                                           \
    if (a.trace && blockIdx.x == 0 && (threadIdx.x & 31) == 0 && (c) < 64)                      \
      a.trace[((role) * 64 + (c)) * 16 + (ph)] = ptx::globaltimer();                             \
  } while (0)
#else
#define TRACE(role, c, ph) \
  do {                     \
  } while (0)
#endif

// Wait bound in SM clock cycles: about 2 s at the B200's 1.97 GHz boost clock, where a
// normal launch takes well under 1 ms.  The cycle counter is cheap to read, the global
// timer is not.
constexpr long long TIMEOUT_CYCLES = 4000000000LL;

// SSD_DEBUG builds (build.py --debug, libssd_b200_debug.so) check every global index the
// fused kernel computes against its tensor's extent; an index out of range is not accessed
// and the status word records 0x300 | site (ssd_status_decode reports it).  Release builds
// compile the checks away.
#ifdef SSD_DEBUG
__device__ __noinline__ bool dbg_fail(unsigned* status, int site) {
  atomicCAS(status, 0u, 0x300u | (unsigned)site);
  return false;
}
#define DBG_IN(idx, n, site) \
  (((int64_t)(idx) >= 0 && (int64_t)(idx) < (int64_t)(n)) ? true : dbg_fail(a.status, (site)))
#else
#define DBG_IN(idx, n, site) true
#endif

// Bounded wait.  Returns false (after flagging the CTA and the status word) on timeout or
// when another role of this CTA already gave up.  One probe is inlined; the spin loop is
// a single out-of-line copy, so the many wait sites add little to the hot code (which
// otherwise outgrows the instruction cache).
__device__ __noinline__ bool wait_bar_slow(Misc* m, int id, uint32_t parity, unsigned* status) {
  const long long t0 = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (ptx::mbar_try_wait(&m->bar[id], parity)) return true;
    }
    if (m->abort) return false;
    if (clock64() - t0 > TIMEOUT_CYCLES) {
      m->abort = 1;
      atomicCAS(status, 0u, (unsigned)(0x100 | id));
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bar(Misc* m, int id, uint32_t parity, unsigned* status) {
  if (ptx::mbar_try_wait(&m->bar[id], parity)) return true;
  return wait_bar_slow(m, id, parity, status);
}

// silu(v) = v sigmoid(v) = 0.5 v (1 + tanh(v / 2)): one tanh.approx (relative error about
// 2^-11) instead of an exponential and a reciprocal.  Used for the z gate of the bf16-input
// epilogue, whose tolerance is far wider; the fp32 pipeline keeps the exact form.
__device__ __forceinline__ float silu_tanh(float v) {
  const float h = 0.5f * v;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// Tokens [t0, t0 + n) of chunk c.  Without a schedule the chunks tile the sequence in 128s;
// with one (varlen states) every packed sequence is tiled from its own start, so each
// sequence ends at a chunk end and its final state is the running state after that chunk.
struct Span {
  int t0, n, vslot;   // vslot: index of the sequence this chunk ends, or -1
};
__device__ __forceinline__ Span span_at(const TcArgs& a, int c) {
  Span s;
  if (a.sched) {
    const bool ok = DBG_IN(c + 1, a.sched_cap + 1, 1);
    const int2 e = ok ? a.sched[c] : make_int2(0, -1);
    s.t0 = e.x;
    s.vslot = e.y;
    s.n = (ok ? a.sched[c + 1].x : e.x) - e.x;
  } else {
    s.t0 = c * QI;
    s.n = min(QI, a.L - s.t0);
    s.vslot = -1;
  }
  return s;
}

// ---------------------------------------------------------------------------
// producer (warp 2, lane 0): per chunk, the C and B columns of the head's group in
// 128-column halves through a 2-stage ring, and the chunk's x tile through its own ring
// ---------------------------------------------------------------------------
template <int NT>
__device__ void producer(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h, int g) {
  using G_ = Geo<NT>;
  int k = 0, c = 0;
  bool ok = true;
  const int nci = m->nci;
  for (; c < nci && ok; ++c) {
    const int t0 = span_at(a, c).t0;
    TRACE(6, c, 0);
    for (int hh = 0; hh < G_::NH; ++hh, ++k) {
      const int s = k & 1;
      if (k >= 2 && !(ok = wait_bar(m, CB_EMPTY0 + s, ((k >> 1) - 1) & 1, a.status))) break;
      uint8_t* st = sm + G_::OFF_CB + s * G_::SZ_CBST;
      uint64_t* full = &m->bar[CB_FULL0 + s];
      ptx::mbar_arrive_expect_tx(full, G_::SZ_CBST);
      const int col = g * NT + hh * 128;
      ptx::tma_load_3d(st, &a.tm_c, full, col, t0, bi);
      ptx::tma_load_3d(st + G_::SZ_H / 2, &a.tm_c, full, col + 64, t0, bi);
      ptx::tma_load_3d(st + G_::SZ_H, &a.tm_b, full, col, t0, bi);
      ptx::tma_load_3d(st + G_::SZ_H + G_::SZ_H / 2, &a.tm_b, full, col + 64, t0, bi);
    }
    if (!ok) break;
    const int xb = c % G_::XST;
    if (c >= G_::XST && !(ok = wait_bar(m, X_EMPTY0 + xb, ((c / G_::XST) - 1) & 1, a.status))) break;
    ptx::mbar_arrive_expect_tx(&m->bar[X_FULL0 + xb], G_::SZ_X);
    ptx::tma_load_3d(sm + G_::OFF_X + xb * G_::SZ_X, &a.tm_x, &m->bar[X_FULL0 + xb], h * PT, t0, bi);
    TRACE(6, c, 1);
  }
  // drain: never leave the CTA with bulk copies still landing in its shared memory
  const long long t0 = clock64();
  for (int kk = (k >= 2 ? k - 2 : 0); kk < k; ++kk)
    while (!ptx::mbar_try_wait(&m->bar[CB_FULL0 + (kk & 1)], (kk >> 1) & 1) && clock64() - t0 < TIMEOUT_CYCLES) {
    }
  for (int cc = (c >= G_::XST ? c - G_::XST : 0); cc < c; ++cc)
    while (!ptx::mbar_try_wait(&m->bar[X_FULL0 + cc % G_::XST], (cc / G_::XST) & 1) &&
           clock64() - t0 < TIMEOUT_CYCLES) {
    }
}

// ---------------------------------------------------------------------------
// dA producer (warp 3, lane 0): each chunk's dA and w arrays (from the dt pre-pass) into the
// shared arrays of its parity, as soon as the readers of chunk c-2 have released them.
// Kept apart from the C/B/x producer so neither waits on the other's consumers.
// ---------------------------------------------------------------------------
__device__ void da_producer(const TcArgs& a, Misc* m, int bi, int h) {
  const int nci = m->nci;
  int c = 0;
  for (; c < nci; ++c) {
    const int buf = c & 1;
    if (c >= 2 && !wait_bar(m, DA_FREE0 + buf, ((c >> 1) - 1) & 1, a.status)) break;
    const int64_t si = (((int64_t)bi * a.H + h) * a.prep_cap + c) * (2 * QI);
    if (!DBG_IN(si + 2 * QI - 1, (int64_t)a.rows * a.H * a.prep_cap * 2 * QI, 2)) break;
    const float* src = a.dtprep + si;
    ptx::mbar_arrive_expect_tx(&m->bar[DA_READY0 + buf], 2 * QI * 4);
    ptx::bulk_load(m->dA[buf], src, QI * 4, &m->bar[DA_READY0 + buf]);
    ptx::bulk_load(m->dt[buf], src + QI, QI * 4, &m->bar[DA_READY0 + buf]);
  }
  // drain: never leave the CTA with bulk copies still landing in its shared memory
  const long long t0 = clock64();
  for (int cc = (c >= 2 ? c - 2 : 0); cc < c; ++cc)
    while (!ptx::mbar_try_wait(&m->bar[DA_READY0 + (cc & 1)], (cc >> 1) & 1) && clock64() - t0 < TIMEOUT_CYCLES) {
    }
}

// ---------------------------------------------------------------------------
// MMA issuers.  The four MMAs of a chunk have different inputs, and a single issuer in a
// fixed order would queue the state chain (MMA3, MMA_L) behind the score pipeline.  So two
// threads issue, each in chunk order with blocking waits:
//   A (warp 1, lane 0)  MMA1(c)  CB = C.B^T   into CB buffer c%2, after C,B(c) and E2(c-2)
//                       MMA2(c)  Y = S.x      after the scores of c (in that CB buffer), x(c)
//                                             and the output of c-1
//   B (warp 0, lane 0)  MMA3(c)  Yi = C.S_c^T after C(c), the bf16 state S_c, a free Yi buffer
//                       MMA_L(c) S += B^T.xs  onto the state T has scaled by the chunk decay
// With one chunk of C/B per ring stage (N=128), A issues MMA1(c+1) before MMA2(c), so the
// scores of chunk c+1 can start as soon as those of c are done.  MMA2(c) and MMA1(c+2) share
// TMEM columns and come from thread A, whose tcgen05.mma execute in issue order.  The C/B
// ring stage takes one commit from each thread.
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ bool issue_mma1(const TcArgs& a, uint8_t* sm, Misc* m, int c) {
  using G_ = Geo<NT>;
  constexpr uint32_t ID_CB = ptx::idesc_bf16_f32(128, 128, 0, 0);
  const uint32_t tmem = m->tmem_base, base = ptx::smem_u32(sm);
  const int cb = c & 1;
  for (int hh = 0; hh < G_::NH; ++hh) {
    const int k = c * G_::NH + hh;
    if (!wait_bar(m, CB_FULL0 + (k & 1), (k >> 1) & 1, a.status)) return false;
    // E2(c-2) done with this CB buffer (MMA2(c-2) was issued earlier by this thread)
    if (hh == 0 && c >= 2 && !wait_bar(m, CB_FREE0 + cb, ((c >> 1) - 1) & 1, a.status)) return false;
    ptx::tc_fence_after();
    const uint32_t sC = base + G_::OFF_CB + (k & 1) * G_::SZ_CBST, sB = sC + G_::SZ_H;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t off = (i >> 2) * (G_::SZ_H / 2) + (i & 3) * 32;
      ptx::mma_f16(tmem + COL_CB0 + 128 * cb, ptx::sdesc_sw128(sC + off, 16, 1024),
                   ptx::sdesc_sw128(sB + off, 16, 1024), ID_CB, (hh > 0 || i > 0) ? 1u : 0u);
    }
  }
  ptx::mma_commit(&m->bar[B_CB0 + cb]);
  for (int hh = 0; hh < G_::NH; ++hh) ptx::mma_commit(&m->bar[CB_EMPTY0 + ((c * G_::NH + hh) & 1)]);
  TRACE(4, c, 1);
  return true;
}

template <int NT>
__device__ __forceinline__ bool issue_mma2(const TcArgs& a, uint8_t* sm, Misc* m, int c) {
  using G_ = Geo<NT>;
  constexpr uint32_t ID_Y = ptx::idesc_bf16_f32(128, 64, 0, 1);
  const uint32_t tmem = m->tmem_base, base = ptx::smem_u32(sm);
  const int cb = c & 1, xb = c % G_::XST, yb = c % G_::YB;
  if (!wait_bar(m, S_FULL_A0 + cb, (c >> 1) & 1, a.status)) return false;
  if (!wait_bar(m, X_FULL0 + xb, (c / G_::XST) & 1, a.status)) return false;
  // the output of c-YB has read this Y buffer
  if (c >= G_::YB && !wait_bar(m, Y_FREE0 + yb, ((c / G_::YB) - 1) & 1, a.status)) return false;
  TRACE(4, c, 4);
  ptx::tc_fence_after();
  const uint32_t sX = base + G_::OFF_X + xb * G_::SZ_X;
  // A = bf16 scores in TMEM (tokens 32k..32k+31 in the first 16 columns of CB block k),
  // B = x [t][p] MN-major.  K-steps of score blocks 0, 1 first, then those of 2, 3.
#pragma unroll
  for (int i = 0; i < QI / 16; ++i) {
    if (i == QI / 32) {
      if (!wait_bar(m, S_FULL_B0 + cb, (c >> 1) & 1, a.status)) return false;
      TRACE(4, c, 8);
      ptx::tc_fence_after();
    }
    ptx::mma_f16_ts(tmem + COL_Y0 + 64 * yb, tmem + COL_CB0 + 128 * cb + 32 * (i >> 1) + 8 * (i & 1),
                    ptx::sdesc_sw128(sX + i * 2048, 8192, 1024), ID_Y, i > 0 ? 1u : 0u);
  }
  ptx::mma_commit(&m->bar[X_EMPTY0 + xb]);
  ptx::mma_commit(&m->bar[B_Y0 + yb]);
  TRACE(4, c, 5);
  return true;
}

template <int NT>
__device__ void mma_issuer_a(const TcArgs& a, uint8_t* sm, Misc* m) {
  using G_ = Geo<NT>;
  const int nci = m->nci;
  if (G_::NH == 1) {
    if (nci > 0 && !issue_mma1<NT>(a, sm, m, 0)) goto drain;
    for (int c = 0; c < nci; ++c) {
      if (c + 1 < nci && !issue_mma1<NT>(a, sm, m, c + 1)) goto drain;
      if (!issue_mma2<NT>(a, sm, m, c)) goto drain;
    }
  } else {
    // the ring holds one chunk: C/B(c+1) arrive only after chunk c's MMAs, so MMA2(c) first
    for (int c = 0; c < nci; ++c) {
      if (!issue_mma1<NT>(a, sm, m, c)) goto drain;
      if (!issue_mma2<NT>(a, sm, m, c)) goto drain;
    }
  }
drain:
  // wait (bounded) until every MMA this thread issued has completed
  ptx::mma_commit(&m->bar[DRAIN]);
  const long long t0 = clock64();
  while (!ptx::mbar_try_wait(&m->bar[DRAIN], 0) && clock64() - t0 < TIMEOUT_CYCLES) {
  }
}

template <int NT>
__device__ void mma_issuer_b(const TcArgs& a, uint8_t* sm, Misc* m) {
  using G_ = Geo<NT>;
  const uint32_t tmem = m->tmem_base;
  const uint32_t base = ptx::smem_u32(sm);
  constexpr uint32_t ID_YI = ptx::idesc_bf16_f32(128, 64, 0, 1);
  constexpr uint32_t ID_L = ptx::idesc_bf16_f32(128, 64, 1, 1);
  const int nci = m->nci;
  for (int c = 0; c < nci; ++c) {
    for (int hh = 0; hh < G_::NH; ++hh) {
      const int k = c * G_::NH + hh;
      if (!wait_bar(m, CB_FULL0 + (k & 1), (k >> 1) & 1, a.status)) goto drain;
    }
    // MMA_L first: it does not wait for the previous output
    // MMA_L: S_{c+1} = (scaled S_c) + B^T . xs, one 128-row half of the state dim per stage
    if (!wait_bar(m, XS_FULL, c & 1, a.status)) goto drain;
    if (!wait_bar(m, SCALED, c & 1, a.status)) goto drain;
    ptx::tc_fence_after();
    for (int hh = 0; hh < G_::NH; ++hh) {
      const uint32_t sB = base + G_::OFF_CB + ((c * G_::NH + hh) & 1) * G_::SZ_CBST + G_::SZ_H;
#pragma unroll
      for (int i = 0; i < QI / 16; ++i)
        ptx::mma_f16(tmem + G_::COL_ST + 64 * hh, ptx::sdesc_sw128(sB + i * 2048, G_::SZ_H / 2, 1024),
                     ptx::sdesc_sw128(base + G_::OFF_XS + i * 2048, 8192, 1024), ID_L, 1u);
    }
    ptx::mma_commit(&m->bar[XS_FREE]);   // MMA_L(c) done with xs
    TRACE(4, c, 3);
    // MMA3: Yi = C . S_c^T (B operand = bf16 state [n][p], MN-major)
    if (!wait_bar(m, ST_READY, c & 1, a.status)) goto drain;
    // the output of c-YIB has read this Yi buffer
    if (c >= G_::YIB && !wait_bar(m, YI_FREE0 + c % G_::YIB, ((c / G_::YIB) - 1) & 1, a.status)) goto drain;
    ptx::tc_fence_after();
    for (int hh = 0; hh < G_::NH; ++hh) {
      const uint32_t sC = base + G_::OFF_CB + ((c * G_::NH + hh) & 1) * G_::SZ_CBST;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t offa = (i >> 2) * (G_::SZ_H / 2) + (i & 3) * 32;
        ptx::mma_f16(tmem + G_::COL_YI0 + 64 * (c % G_::YIB), ptx::sdesc_sw128(sC + offa, 16, 1024),
                     ptx::sdesc_sw128(base + G_::OFF_ST + hh * (128 * 128) + i * 2048, 8192, 1024), ID_YI,
                     (hh > 0 || i > 0) ? 1u : 0u);
      }
    }
    ptx::mma_commit(&m->bar[B_YI0 + c % G_::YIB]);
    TRACE(4, c, 2);
    ptx::mma_commit(&m->bar[B_L]);   // S_{c+1} ready; MMA3(c) done with the bf16 state
    for (int hh = 0; hh < G_::NH; ++hh) ptx::mma_commit(&m->bar[CB_EMPTY0 + ((c * G_::NH + hh) & 1)]);
  }
drain:
  ptx::mma_commit(&m->bar[DRAIN]);
  const long long t0 = clock64();
  while (!ptx::mbar_try_wait(&m->bar[DRAIN], 0) && clock64() - t0 < TIMEOUT_CYCLES) {
  }
}

// ---------------------------------------------------------------------------
// helpers shared by the worker warpgroups
// ---------------------------------------------------------------------------
// Raw dt of chunk row r, loaded unconditionally from a clamped (always valid) address: the
// caller masks rows past the chunk's end when it uses the value.  A conditional load here
// would be merged with its fallback value at once, and the merge waits for the load (a
// few microseconds under this kernel's memory traffic), defeating the prefetch.
template <bool DT_BF16>
__device__ __forceinline__ float load_dt(const TcArgs& a, int bi, int h, int nci, int c, int r) {
  const Span sp = span_at(a, min(c, nci - 1));
  const int64_t di = ((int64_t)bi * a.L + sp.t0 + min(r, sp.n - 1)) * a.H + h;
  if (DT_BF16) return __bfloat162float(__ldg((const bf16*)a.dt + di));
  return __ldg((const float*)a.dt + di);
}

__device__ __forceinline__ int seq_at(const TcArgs& a, int bi, int64_t pos) {
  return (pos < a.L && DBG_IN((int64_t)bi * a.L + pos, (int64_t)a.rows * a.L, 3)) ? a.seq_idx[(int64_t)bi * a.L + pos]
                                                                               : -1;
}

// 16-byte word of 8 bf16, scaled by `s`, repacked.
__device__ __forceinline__ uint4 scale_row16(uint4 w, float s) {
  uint4 o;
  float2 f;
  const float2 ss = make_float2(s, s);
  f = ptx::mul2(unpack_bf16(w.x), ss); o.x = pack_bf16(f.x, f.y);
  f = ptx::mul2(unpack_bf16(w.y), ss); o.y = pack_bf16(f.x, f.y);
  f = ptx::mul2(unpack_bf16(w.z), ss); o.z = pack_bf16(f.x, f.y);
  f = ptx::mul2(unpack_bf16(w.w), ss); o.w = pack_bf16(f.x, f.y);
  return o;
}

// ---------------------------------------------------------------------------
// dt pre-pass (its own launch, before the fused kernel): for every (batch, head, chunk) the
// processed dt (bias, softplus, clamp; chunk_cumsum_fwd.py:221-231), the in-chunk cumulative
// dA = cumsum(dt * A) and the decay column factors w, 1 KB per chunk.  The fused kernel's
// producer bulk-copies each chunk's 1 KB into shared memory, so no warp of that kernel
// waits on these scattered loads (several microseconds each under its memory traffic).
// Decay factors per 32-token block k: exp(dA_m - dA_t) = exp(dA_m - dA_{32k}) * w_t with
// w_t = exp(dA_{32k} - dA_t) dt_t.  With dA non-increasing (A <= 0, dt >= 0) the first
// factor is <= 1 for m >= 32k and w_t <= exp(block range); blocks whose range exceeds 60
// (or every block when dA may increase) store dt_t and are formed element by element.
// ---------------------------------------------------------------------------
constexpr float FAC_RANGE = 60.f;

__device__ __forceinline__ bool block_factored(bool factor, const float* dA, int k) {
  return factor && (dA[32 * k] - dA[32 * k + 31] <= FAC_RANGE);
}

template <bool DT_BF16>
__global__ void __launch_bounds__(128) tc_dt_prep_kernel(const __grid_constant__ TcArgs a, float* __restrict__ out) {
  const int c = blockIdx.x, bi = blockIdx.y;
  const int nci = a.sched_n ? *a.sched_n : a.nci;
  const int h = blockIdx.z * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (c >= nci || h >= a.H) return;
  const Span sp = span_at(a, c);
  const float Ah = a.A[h];
  const float bias = a.dt_bias ? a.dt_bias[h] : 0.f;
  const bool factor = (Ah <= 0.f) && (a.lo >= 0.f);   // dA non-increasing
  float d[4], run = 0.f, cs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * lane + i;
    float raw = 0.f;
    if (r < sp.n) {
      const int64_t di = ((int64_t)bi * a.L + sp.t0 + r) * a.H + h;
      raw = DT_BF16 ? __bfloat162float(((const bf16*)a.dt)[di]) : ((const float*)a.dt)[di];
    }
    d[i] = r < sp.n ? dt_process(raw, bias, a.softplus, a.lo, a.hi) : 0.f;
    run += d[i] * Ah;
    cs[i] = run;
  }
  const float excl = warp_incl_scan(run) - run;
  float dAv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) dAv[i] = cs[i] + excl;
  const float dAs = __shfl_sync(0xffffffffu, dAv[0], lane & ~7);
  const float dAe = __shfl_sync(0xffffffffu, dAv[3], lane | 7);
  const bool fk = factor && (dAs - dAe <= FAC_RANGE);
  float w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = fk ? __expf(dAs - dAv[i]) * d[i] : d[i];
  float* o = out + (((int64_t)bi * a.H + h) * a.prep_cap + c) * (2 * QI);
  reinterpret_cast<float4*>(o)[lane] = make_float4(dAv[0], dAv[1], dAv[2], dAv[3]);
  reinterpret_cast<float4*>(o + QI)[lane] = make_float4(w[0], w[1], w[2], w[3]);
}

// Output epilogue of chunk c (run by T): out = Y + sdec Yi, z gate (Y holds D x).  Row r is
// staged as f32 in the (free) score buffer as two 128B-swizzled [128][32] boxes and
// written by one TMA bulk store per box, so global writes are full lines.  The inner
// loops carry no data-dependent branches (each costs tens of cycles when unrolled).
template <int NT, bool HAS_Z>
__device__ bool output_chunk(const TcArgs& a, uint8_t* sm, Misc* m, uint32_t tmem, int bi, int h, int c, int r,
                             float sdec) {
  using G_ = Geo<NT>;
  const int yb = c % G_::YB, yib = c % G_::YIB;
  const int lane = r & 31;
  const Span sp = span_at(a, c);
  const int64_t pos = (int64_t)sp.t0 + r;
  const bool valid = r < sp.n;
  const int64_t o0 = (((int64_t)bi * a.L + (valid ? pos : sp.t0)) * a.H + h) * PT;
  float* const out_x = a.out_x;
  // z of this row, loaded unconditionally (rows past the chunk read a valid row and are
  // never stored) and issued before the waits so its latency overlaps them
  uint4 zq[8];
  if (HAS_Z) {
    const bool zok = DBG_IN(o0 + PT - 1, (int64_t)a.rows * a.L * a.H * PT, 4);
    const uint4* const zp = reinterpret_cast<const uint4*>(a.z + (zok ? o0 : 0));
#pragma unroll
    for (int k = 0; k < 8; ++k) zq[k] = __ldg(zp + k);
  }
  if (!wait_bar(m, B_Y0 + yb, (c / G_::YB) & 1, a.status)) return false;
  if (!wait_bar(m, B_YI0 + yib, (c / G_::YIB) & 1, a.status)) return false;
  if ((r >> 5) == 0 || (r >> 5) == 3) TRACE(2 + ((r >> 5) == 3), c + 1, 8);
  ptx::tc_fence_after();
  // the previous chunk's bulk store must have read the staging buffer (long done by now)
  if (c > 0) {
    if (r == 0) {
      ptx::bulk_wait_read();
      ptx::mbar_arrive(&m->bar[OUT_READ]);
    }
    if (!wait_bar(m, OUT_READ, (c - 1) & 1, a.status)) return false;
  }
  uint8_t* stage = sm + G_::OFF_S;
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float y[32], yi[32];
    ptx::tmem_ld32(tmem + COL_Y0 + 64 * yb + 32 * half, y);
    ptx::tmem_ld32(tmem + G_::COL_YI0 + 64 * yib + 32 * half, yi);
    uint32_t zw[16];
    if (HAS_Z) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 w = half == 0 ? zq[k] : zq[4 + k];
        zw[4 * k] = w.x; zw[4 * k + 1] = w.y; zw[4 * k + 2] = w.z; zw[4 * k + 3] = w.w;
      }
    }
    ptx::tmem_ld_wait();
#pragma unroll
    for (int k = 0; k < 32; k += 2) {   // Y already holds D x (diagonal)
      const float2 o = ptx::fma2(make_float2(sdec, sdec), make_float2(yi[k], yi[k + 1]), make_float2(y[k], y[k + 1]));
      y[k] = o.x;
      y[k + 1] = o.y;
    }
    if (HAS_Z) {
      if (out_x != nullptr && valid && DBG_IN(o0 + PT - 1, (int64_t)a.rows * a.L * a.H * PT, 5)) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(out_x + o0 + 32 * half + i) = make_float4(y[i], y[i + 1], y[i + 2], y[i + 3]);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float2 f = unpack_bf16(zw[k]);
        y[2 * k] *= silu_tanh(f.x);
        y[2 * k + 1] *= silu_tanh(f.y);
      }
    }
    uint8_t* box = stage + half * (QI * 128);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      *reinterpret_cast<float4*>(box + ptx::sw128_off(r, k)) =
          make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
  }
  ptx::tc_fence_before();
  ptx::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    ptx::mbar_arrive(&m->bar[Y_FREE0 + yb]);
    ptx::mbar_arrive(&m->bar[YI_FREE0 + yib]);
    ptx::mbar_arrive(&m->bar[STAGED]);
  }
  if ((r >> 5) == 0 || (r >> 5) == 3) TRACE(2 + ((r >> 5) == 3), c + 1, 9);
  if (r == 0) {
    // all 128 rows staged: one bulk store per 32-column box
    if (!wait_bar(m, STAGED, c & 1, a.status)) return false;
    ptx::tma_store_3d(&a.tm_out, stage, h * PT, sp.t0, bi);
    ptx::tma_store_3d(&a.tm_out, stage + QI * 128, h * PT + 32, sp.t0, bi);
    ptx::bulk_commit();
    // A short chunk followed by more tokens (a packed sequence ending) also stored rows of
    // the next chunk, which that chunk stores again: let this store land first.
    if (sp.n < QI && sp.t0 + QI < a.L) ptx::bulk_wait_all();
  }
  if ((r >> 5) == 0 || (r >> 5) == 3) TRACE(2 + ((r >> 5) == 3), c + 1, 10);
  return true;
}

// One 32-column block of scores for row r (v holds CB[r][t], t = block start + i, on
// entry; packed bf16 pairs on exit).  Factored blocks: decay u_r * w_t, w read from shared
// memory (the same address in every lane), two packed f32x2 products per column pair.

// A block below the diagonal without sequence masks: every column counts.
__device__ __forceinline__ void score_block_full(const float (&v)[32], uint32_t (&pk)[16], float u, const float* wc) {
  const float2 uu = make_float2(u, u);
#pragma unroll
  for (int i4 = 0; i4 < 8; ++i4) {
    const float4 w4 = *reinterpret_cast<const float4*>(wc + 4 * i4);
    const float2 p0 = ptx::mul2(make_float2(v[4 * i4], v[4 * i4 + 1]), ptx::mul2(uu, make_float2(w4.x, w4.y)));
    const float2 p1 = ptx::mul2(make_float2(v[4 * i4 + 2], v[4 * i4 + 3]), ptx::mul2(uu, make_float2(w4.z, w4.w)));
    pk[2 * i4] = pack_bf16(p0.x, p0.y);
    pk[2 * i4 + 1] = pack_bf16(p1.x, p1.y);
  }
}

// Masked: columns i > lim are zero (lim = lane on the diagonal block, 31 below it), and
// with HAS_SEQ so are columns of another sequence; column dcol (the diagonal) adds dg.
template <bool HAS_SEQ>
__device__ __forceinline__ void score_block_fac(const float (&v)[32], uint32_t (&pk)[16], float u, const float* wc,
                                                int lim, int sl, int seqv, int dcol, float dg) {
  const float2 uu = make_float2(u, u);
#pragma unroll
  for (int i4 = 0; i4 < 8; ++i4) {
    const float4 w4 = *reinterpret_cast<const float4*>(wc + 4 * i4);
    const float2 p0 = ptx::mul2(make_float2(v[4 * i4], v[4 * i4 + 1]), ptx::mul2(uu, make_float2(w4.x, w4.y)));
    const float2 p1 = ptx::mul2(make_float2(v[4 * i4 + 2], v[4 * i4 + 3]), ptx::mul2(uu, make_float2(w4.z, w4.w)));
    const float pv[4] = {p0.x, p0.y, p1.x, p1.y};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * i4 + j;
      bool ok = i <= lim;
      if (HAS_SEQ) {
        // every lane takes part in the shuffle (a short-circuited __shfl_sync would diverge)
        const int st = __shfl_sync(0xffffffffu, sl, i);
        ok = ok && (st == seqv);
      }
      o[j] = (ok ? pv[j] : 0.f) + (i == dcol ? dg : 0.f);
    }
    pk[2 * i4] = pack_bf16(o[0], o[1]);
    pk[2 * i4 + 1] = pack_bf16(o[2], o[3]);
  }
}

// Blocks that do not factor (dA may increase, or its range in the block exceeds 60, as for
// heads with large |A| dt): exp(dA_r - dA_t) dt_t per element.
template <bool HAS_SEQ>
__device__ __forceinline__ void score_block_exact(const float (&v)[32], uint32_t (&pk)[16], float dA, const float* dAc,
                                                  const float* dtc, int lim, int sl, int seqv, int dcol, float dg) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float o[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      bool ok = i + j <= lim;
      if (HAS_SEQ) {
        const int st = __shfl_sync(0xffffffffu, sl, i + j);   // all lanes shuffle, then combine
        ok = ok && (st == seqv);
      }
      o[j] = v[i + j] * __expf(ok ? dA - dAc[i + j] : -INFINITY) * dtc[i + j] + (i + j == dcol ? dg : 0.f);
    }
    pk[i / 2] = pack_bf16(o[0], o[1]);
  }
}

// ---------------------------------------------------------------------------
// score workers SA (warps 4-7, half 0) and SB (warps 8-11, half 1).  Both build score
// column blocks {half, half+2} of the rows of their quadrant (quadrant q has q+1 non-zero
// blocks, so no warp does more than two).  Each also builds half of xs first.
// ---------------------------------------------------------------------------
template <int NT, bool HAS_SEQ, bool HAS_Z>
__device__ void score_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h, int half) {
  const int r = threadIdx.x & 127;
  const int q = r >> 5, lane = r & 31;
  const uint32_t tmem = m->tmem_base + ((uint32_t)(q * 32) << 16);
  constexpr bool has_seq = HAS_SEQ;
  const bool factor = (a.A[h] <= 0.f) && (a.lo >= 0.f);   // dA non-increasing
  const float dg = m->Dh;
  using G_ = Geo<NT>;
  uint8_t* xs_sm = sm + G_::OFF_XS;
  const int nci = m->nci;
#pragma unroll 1
  for (int c = 0; c < nci; ++c) {
    const int buf = c & 1, xb = c % G_::XST;
    const Span sp = span_at(a, c);
    const int64_t t0 = sp.t0;
    const int trole = 2 * half + (q == 3);
    (void)trole;
    if (q == 0 || q == 3) TRACE(trole, c, 0);
    int seqv = (r < sp.n) ? 0 : -1, end_seq = 0, sl0 = 0, sl1 = 0;
    const int last_valid = sp.n - 1;
    if (has_seq) {
      seqv = (r < sp.n) ? seq_at(a, bi, t0 + r) : -1;
      end_seq = seq_at(a, bi, t0 + last_valid);
      sl0 = seq_at(a, bi, t0 + half * 32 + lane);
      sl1 = seq_at(a, bi, t0 + (half + 2) * 32 + lane);
    }
    if (!wait_bar(m, DA_READY0 + buf, (c >> 1) & 1, a.status)) return;
    const float dA = m->dA[buf][r];
    if (q == 0 || q == 3) TRACE(trole, c, 2);

    {
      // ---- E1: xs[r] = x[r] * exp(dA_last - dA_r) dt_r  (chunk-end sequence only) -----
      // SA writes head-dim columns 0-31, SB columns 32-63
      // exp(dA_last - dA_r) dt_r, from w_r = exp(dA_{32q} - dA_r) dt_r in a factored block
      const bool fq = block_factored(factor, m->dA[buf], q);
      const float e1 = __expf(m->dA[buf][QI - 1] - (fq ? m->dA[buf][32 * q] : dA)) * m->dt[buf][r];
      const float scale = (end_seq >= 0 && seqv == end_seq) ? e1 : 0.f;
      if (!wait_bar(m, X_FULL0 + xb, (c / G_::XST) & 1, a.status)) return;
      if (c > 0 && !wait_bar(m, XS_FREE, (c - 1) & 1, a.status)) return;   // MMA_L(c-1) done with xs
      if (q == 0 || q == 3) TRACE(trole, c, 3);
      const uint8_t* x_sm = sm + G_::OFF_X + xb * G_::SZ_X;
#pragma unroll
      for (int k = 4 * half; k < 4 * half + 4; ++k)
        *reinterpret_cast<uint4*>(xs_sm + ptx::sw128_off(r, k)) =
            scale_row16(*reinterpret_cast<const uint4*>(x_sm + ptx::sw128_off(r, k)), scale);
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&m->bar[XS_FULL]);
      if (q == 0 || q == 3) TRACE(trole, c, 8);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&m->bar[X_EMPTY0 + xb]);
      if (q == 0 || q == 3) TRACE(trole, c, 4);
    }

    // ---- E2: S[r][t] = CB[r][t] exp(dA_r - dA_t) dt_t  (t <= r, same sequence) ------
    const int cb = c & 1;
    if (!wait_bar(m, B_CB0 + cb, (c >> 1) & 1, a.status)) return;
    if (q == 0 || q == 3) TRACE(trole, c, 6);
    ptx::tc_fence_after();
#pragma unroll 1
    for (int kk = 0; kk < 2; ++kk) {
      const int k32 = half + 2 * kk;
      // bf16 scores of this block replace the first 16 of its 32 CB columns (read first)
      const uint32_t tS = tmem + COL_CB0 + 128 * cb + k32 * 32;
      if (k32 > q) {
        // above the diagonal: zero scores
        const uint32_t zero[16] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
        ptx::tmem_st16(tS, zero);
      } else {
        const int sl = kk == 0 ? sl0 : sl1;
        const bool fac = block_factored(factor, m->dA[buf], k32);
        const int lim = k32 == q ? lane : 31;
        const float* dAc = m->dA[buf] + k32 * 32;
        const float* wc = m->dt[buf] + k32 * 32;
        float v[32];
        uint32_t pk[16];
        ptx::tmem_ld32(tS, v);   // one TMEM round trip per block
        ptx::tmem_ld_wait();
        if (q == 0 || q == 3) TRACE(trole, c, 11 + 2 * kk);
        // the skip term D x rides on the diagonal: S[r][r] += D
        const int dcol = k32 == q ? lane : -1;
        if (fac && !HAS_SEQ && k32 < q) score_block_full(v, pk, __expf(dA - dAc[0]), wc);
        else if (fac) score_block_fac<HAS_SEQ>(v, pk, __expf(dA - dAc[0]), wc, lim, sl, seqv, dcol, dg);
        else score_block_exact<HAS_SEQ>(v, pk, dA, dAc, wc, lim, sl, seqv, dcol, dg);
        ptx::tmem_st16(tS, pk);
        if (q == 0 || q == 3) TRACE(trole, c, 12 + 2 * kk);
      }
      if (kk == 0) {
        // blocks 0 and 1 (SA, SB) of this quadrant are in TMEM: MMA2 may start on them
        ptx::tmem_st_wait();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&m->bar[S_FULL_A0 + cb]);
      }
    }
    ptx::tmem_st_wait();
    ptx::tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      ptx::mbar_arrive(&m->bar[CB_FREE0 + cb]);
      ptx::mbar_arrive(&m->bar[S_FULL_B0 + cb]);
      ptx::mbar_arrive(&m->bar[DA_FREE0 + buf]);
    }
    if (q == 0 || q == 3) TRACE(trole, c, 7);
    if (q == 1 || q == 2) TRACE(7, c, 2 * half + (q == 2));
  }
}


// ---------------------------------------------------------------------------
// state worker T (warps 12-15).  S_{c+1} = decay_c S_c + B^T xs_c, with the product added
// by MMA_L(c) onto the state T has already scaled in TMEM.  Per chunk c, once MMA_L(c) is
// done: read S_{c+1}, write its bf16 copy for MMA3(c+1) (and the varlen / final state),
// store decay_{c+1} S_{c+1} back for MMA_L(c+1); the output epilogue of c-1 runs before
// (one Yi buffer) or after (two) that copy.  Thread r owns state rows
// n = r + 128*hh (TMEM lane r, 64 f32 columns per 128-row half).  decay_c is 0 when the
// chunk-end sequence id changes (state_passing_fwd.py:208-225; the id before the first
// chunk counts as 0).
// ---------------------------------------------------------------------------
template <int NT, bool HAS_SEQ>
__device__ __forceinline__ bool chunk_decay(const TcArgs& a, Misc* m, int bi, int c, int r, int& prev_end,
                                            float& decay, float& sdec) {
  const int buf = c & 1, lane = r & 31;
  const Span sp = span_at(a, c);
  const int end_seq = HAS_SEQ ? seq_at(a, bi, (int64_t)sp.t0 + sp.n - 1) : 0;
  // row r continues the previous chunk's sequence: it reads the passed state (rule A9)
  bool cont = r < sp.n;
  if (HAS_SEQ) {
    const int sr = seq_at(a, bi, (int64_t)sp.t0 + r);
    const int sp0 = c == 0 ? 0 : seq_at(a, bi, (int64_t)sp.t0 - 1);
    cont = cont && sr == sp0;
  }
  if (!wait_bar(m, DA_READY0 + buf, (c >> 1) & 1, a.status)) return false;
  const float dA_last = m->dA[buf][QI - 1];
  sdec = cont ? __expf(m->dA[buf][r]) : 0.f;
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(&m->bar[DA_FREE0 + buf]);
  decay = (end_seq == prev_end) ? __expf(dA_last) : 0.f;
  prev_end = end_seq;
  return true;
}

template <int NT, bool HAS_SEQ, bool HAS_Z>
__device__ void state_worker(const TcArgs& a, uint8_t* sm, Misc* m, int bi, int h) {
  using G_ = Geo<NT>;
  const int r = threadIdx.x & 127;
  const int q = r >> 5, lane = r & 31;
  const uint32_t tl = m->tmem_base + ((uint32_t)(q * 32) << 16);
  uint8_t* st_sm = sm + G_::OFF_ST;
  // with a split sequence, row bi is segment bi % seg_k of batch row bi / seg_k: only the
  // last segment's state is a final state
  const int64_t ib = bi / a.seg_k, fbh = ib * a.H + h;
  const int jseg = bi % a.seg_k;
  float* const fin = (jseg == a.seg_k - 1) ? a.final_states : nullptr;
  const int nci = m->nci;
  if (nci <= 0) return;
  int prev_end = 0;
  float decay, sd_cur, sd_next = 0.f, sd_prev = 0.f;   // per-row inter-chunk factors of c, c+1, c-1
  if (!chunk_decay<NT, HAS_SEQ>(a, m, bi, 0, r, prev_end, decay, sd_cur)) return;
  // S_0 = initial state (or 0): bf16 operand for MMA3(0); decay_0 S_0 in TMEM for MMA_L(0)
#pragma unroll 1
  for (int seg = 0; seg < 2 * G_::NH; ++seg) {
    const int hh = seg >> 1, half = seg & 1;
    const int n = hh * 128 + r;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    // S_j = sum_{l<j} exp(total dA of segments l+1..j-1) L_l + exp(total dA of 0..j-1) S_init
    // (segment j = bi % seg_k of batch row bi / seg_k; without a split j = 0, S_0 = S_init)
    float sdA = 0.f;
    // the segment-state pass may still be running (this kernel is its programmatic
    // dependent): wait for its results before the first read
    if (jseg > 0 && seg == 0) ptx::griddep_wait();
    for (int l = jseg - 1; l >= 0; --l) {
      const int64_t lr = (ib * a.seg_k + l) * a.H + h;
      if (!DBG_IN(lr * PT * NT + (int64_t)(32 * half + 31) * NT + n, (int64_t)a.rows * a.H * PT * NT, 6)) break;
      const float coef = __expf(sdA);
      const float* Ll = a.seg_state + lr * PT * NT + n;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaf(coef, __ldcg(Ll + (32 * half + i) * NT), v[i]);
      sdA += __ldcg(a.seg_tot + lr);
    }
    if (a.init && DBG_IN(((ib * a.H + h) * PT + 32 * half + 31) * NT + n, (int64_t)(a.rows / a.seg_k) * a.H * PT * NT, 7)) {
      const float coef = __expf(sdA);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaf(coef, a.init[((ib * a.H + h) * PT + 32 * half + i) * NT + n], v[i]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(st_sm + ptx::sw128_off(n, 4 * half + j)) =
          make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                     pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= decay;
    ptx::tmem_st32(tl + G_::COL_ST + 64 * hh + 32 * half, v);
  }
  ptx::tmem_st_wait();
  ptx::tc_fence_before();
  ptx::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    ptx::mbar_arrive(&m->bar[ST_READY]);
    ptx::mbar_arrive(&m->bar[SCALED]);
  }

#pragma unroll 1
  for (int c = 0; c < nci; ++c) {
    const bool more = c + 1 < nci;
    // this chunk ends packed sequence sp.vslot: the state after it is that sequence's
    // final state (chunk_state_fwd.py:448-597 computes the same per sequence)
    const Span sp = span_at(a, c);
    float* const vdst = (sp.vslot >= 0 && DBG_IN(sp.vslot, a.num_seqs, 8))
                            ? a.varlen_states + ((int64_t)sp.vslot * a.H + h) * PT * NT : nullptr;
    TRACE(5, c, 0);
    if (more && !chunk_decay<NT, HAS_SEQ>(a, m, bi, c + 1, r, prev_end, decay, sd_next)) return;
    // With one Yi buffer MMA3(c) writes Yi after the output of c-1 has read it, so that
    // output comes first; with two it follows the state copy, overlapping MMA3/MMA_L(c+1).
    if (G_::YIB == 1 && c > 0 && !output_chunk<NT, HAS_Z>(a, sm, m, tl, bi, h, c - 1, r, sd_prev)) return;
    if (!wait_bar(m, B_L, c & 1, a.status)) return;   // S_{c+1} ready, MMA3(c) done with the copy of S_c
    TRACE(5, c, 1);
    ptx::tc_fence_after();
#pragma unroll 1
    for (int seg = 0; seg < 2 * G_::NH; ++seg) {
      const int hh = seg >> 1, half = seg & 1;
      const int n = hh * 128 + r;
      float sv[32];
      ptx::tmem_ld32(tl + G_::COL_ST + 64 * hh + 32 * half, sv);
      ptx::tmem_ld_wait();
      if (vdst != nullptr) {
#pragma unroll
        for (int i = 0; i < 32; ++i) vdst[(32 * half + i) * NT + n] = sv[i];
      }
      if (more) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(st_sm + ptx::sw128_off(n, 4 * half + j)) =
              make_uint4(pack_bf16(sv[8 * j], sv[8 * j + 1]), pack_bf16(sv[8 * j + 2], sv[8 * j + 3]),
                         pack_bf16(sv[8 * j + 4], sv[8 * j + 5]), pack_bf16(sv[8 * j + 6], sv[8 * j + 7]));
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 d2 = ptx::mul2(make_float2(sv[i], sv[i + 1]), make_float2(decay, decay));
          sv[i] = d2.x;
          sv[i + 1] = d2.y;
        }
        ptx::tmem_st32(tl + G_::COL_ST + 64 * hh + 32 * half, sv);
      } else if (fin && DBG_IN((fbh * PT + 32 * half + 31) * NT + n, (int64_t)(a.rows / a.seg_k) * a.H * PT * NT, 9)) {
#pragma unroll
        for (int i = 0; i < 32; ++i) fin[(fbh * PT + 32 * half + i) * NT + n] = sv[i];
      }
    }
    if (more) {
      ptx::tmem_st_wait();
      ptx::tc_fence_before();
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(&m->bar[ST_READY]);
        ptx::mbar_arrive(&m->bar[SCALED]);
      }
    }
    TRACE(5, c, 2);
    if (G_::YIB == 2 && c > 0 && !output_chunk<NT, HAS_Z>(a, sm, m, tl, bi, h, c - 1, r, sd_prev)) return;
    sd_prev = sd_cur;
    sd_cur = sd_next;
  }
  if (!output_chunk<NT, HAS_Z>(a, sm, m, tl, bi, h, nci - 1, r, sd_prev)) return;
  if (r == 0) ptx::bulk_wait_all();   // every bulk store of this CTA has landed
}

template <int NT, bool HAS_SEQ, bool HAS_Z>
__global__ void __launch_bounds__(NTHREADS, 1) ssd_fused_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // Align by pointer arithmetic on the shared array itself (not through an integer cast)
  // so that every access below stays a shared-space load/store.
  uint8_t* sm = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);
  using G_ = Geo<NT>;
  if (sm - smem_raw > (ptrdiff_t)(SMEM_LAUNCH_BYTES - G_::SMEM_BYTES)) {
    // the dynamic shared window is not aligned enough for the swizzled tiles: report, do nothing
    if (threadIdx.x == 0) atomicCAS(a.status, 0u, 0x200u);
    return;
  }
  Misc* m = reinterpret_cast<Misc*>(sm + G_::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bi = bh / a.H, h = bh % a.H;
  const int g = h / (a.H / a.G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NBARS; ++i) ptx::mbar_init(&m->bar[i], 1);   // single arrivals, then the counted ones:
    ptx::mbar_init(&m->bar[CB_EMPTY0], 2);   // one commit from each MMA issuer
    ptx::mbar_init(&m->bar[CB_EMPTY1], 2);
    ptx::mbar_init(&m->bar[X_EMPTY0], X_EMPTY_COUNT);
    ptx::mbar_init(&m->bar[X_EMPTY1], X_EMPTY_COUNT);
    ptx::mbar_init(&m->bar[CB_FREE0], 8);    // SA and SB done with the CB buffer
    ptx::mbar_init(&m->bar[CB_FREE1], 8);
    ptx::mbar_init(&m->bar[XS_FULL], 8);     // SA and SB: their halves of xs
    ptx::mbar_init(&m->bar[S_FULL_A0], 8);   // SA and SB: score blocks 0, 1
    ptx::mbar_init(&m->bar[S_FULL_A1], 8);
    ptx::mbar_init(&m->bar[S_FULL_B0], 8);   // SA and SB: score blocks 2, 3
    ptx::mbar_init(&m->bar[S_FULL_B1], 8);
    ptx::mbar_init(&m->bar[ST_READY], 4);    // T: bf16 state copy for MMA3
    ptx::mbar_init(&m->bar[SCALED], 4);      // T: TMEM state scaled by the chunk decay
    ptx::mbar_init(&m->bar[Y_FREE0], 4);     // T: output read Y
    ptx::mbar_init(&m->bar[Y_FREE1], 4);
    ptx::mbar_init(&m->bar[YI_FREE0], 4);    // T: output read Yi
    ptx::mbar_init(&m->bar[YI_FREE1], 4);
    ptx::mbar_init(&m->bar[DA_FREE0], DA_FREE_COUNT);
    ptx::mbar_init(&m->bar[DA_FREE1], DA_FREE_COUNT);
    ptx::mbar_init(&m->bar[STAGED], 4);
    ptx::mbar_init(&m->bar[DRAIN], 2);
    m->abort = 0;
    m->nci = a.sched_n ? *a.sched_n : a.nci;
    ptx::fence_mbar_init();
  }
#ifdef SSD_TC_DEBUG_TRACE
  if (a.trace && threadIdx.x == 0 && blockIdx.x < 2048) {
    a.trace[8 * 64 * 16 + 3 * blockIdx.x] = ptx::globaltimer();
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    a.trace[8 * 64 * 16 + 3 * blockIdx.x + 2] = smid;
  }
#endif
  if (threadIdx.x == 0) m->Dh = a.D_ndim == 1 ? a.D[h] : 0.f;
  if (warp == W_PRODUCER && lane == 0) {
    ptx::prefetch_tmap(&a.tm_x);
    ptx::prefetch_tmap(&a.tm_b);
    ptx::prefetch_tmap(&a.tm_c);
    ptx::prefetch_tmap(&a.tm_out);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&m->tmem_base, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();

  if (a.test_wait_cycles > 0) {
    // Test mode (SSD_FLAG_TEST_WAIT_TIMEOUT): a bounded wait on a barrier that nothing
    // arrives on yet (DRAIN, before any role has run) runs out, the status word records it
    // and the CTA skips its work.  It exercises the timeout report with no copy or MMA in
    // flight.
    if (threadIdx.x == 0) {
      const long long t0 = clock64();
      bool ok = false;
      while (!(ok = ptx::mbar_try_wait(&m->bar[DRAIN], 0)) && clock64() - t0 < a.test_wait_cycles) {
      }
      if (!ok) {
        m->abort = 1;
        atomicCAS(a.status, 0u, (unsigned)(0x100 | DRAIN));
      }
    }
    __syncthreads();
  }
  if (m->abort) {
    // nothing issued: fall through to the TMEM release
  } else if (warp == W_PRODUCER) {
    if (lane == 0) producer<NT>(a, sm, m, bi, h, g);
  } else if (warp == W_ISSUE_A) {
    if (lane == 0) mma_issuer_a<NT>(a, sm, m);
  } else if (warp == W_DA) {
    if (lane == 0) da_producer(a, m, bi, h);
  } else if (warp == W_ISSUE_B) {
    if (lane == 0) mma_issuer_b<NT>(a, sm, m);
  } else if (warp < 12) {
    score_worker<NT, HAS_SEQ, HAS_Z>(a, sm, m, bi, h, (warp - 4) >> 2);
  } else {
    state_worker<NT, HAS_SEQ, HAS_Z>(a, sm, m, bi, h);
  }
  ptx::tc_fence_before();
  __syncthreads();
#ifdef SSD_TC_DEBUG_TRACE
  if (a.trace && threadIdx.x == 0 && blockIdx.x < 2048) a.trace[8 * 64 * 16 + 3 * blockIdx.x + 1] = ptx::globaltimer();
#endif
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(m->tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Chunk schedule for varlen states (one block of 1024 threads).  Segment j of the packed
// row is [p_j, p_{j+1}) with p_0 = 0, p_{k+1} = cu[k] (k = 0..S, clamped to [0, L] and made
// non-decreasing) and p_{S+2} = L; segment k+1 is packed sequence k.  Each segment is cut
// into 128-token chunks from its own start; the last chunk of sequence k carries slot k.
// Empty sequences get a zero state (as chunk_state_fwd.py's varlen path yields for them).
// Writes the chunk count to hdr[0] and at most `cap` entries plus the {L, -1} sentinel.
// ---------------------------------------------------------------------------
constexpr int SCHED_THREADS = 1024;

__global__ void __launch_bounds__(SCHED_THREADS) tc_schedule_kernel(const int32_t* __restrict__ cu, int S, int L,
                                                                    int cap, int* __restrict__ hdr,
                                                                    int2* __restrict__ sched, float* vstates,
                                                                    int64_t vstride) {
  __shared__ int wred[32];
  __shared__ int carry_max, carry_cnt, nempty;
  __shared__ int empty_list[SCHED_THREADS];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const unsigned full = 0xffffffffu;
  if (tid == 0) {
    carry_max = 0;
    carry_cnt = 0;
  }
  const int nseg = S + 2;
  for (int base = 0; base < nseg; base += SCHED_THREADS) {
    if (tid == 0) nempty = 0;
    __syncthreads();
    const int j = base + tid;
    const int cmax = carry_max, ccnt = carry_cnt;
    int e = 0;
    if (j <= S) e = min(max(cu[j], 0), L);
    else if (j == S + 1) e = L;
    // inclusive max-scan of the segment ends -> non-decreasing ends
    int v = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(full, v, o);
      if (lane >= o) v = max(v, t);
    }
    if (lane == 31) wred[w] = v;
    __syncthreads();
    if (w == 0) {
      int t = wred[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(full, t, o);
        if (lane >= o) t = max(t, u);
      }
      wred[lane] = t;
    }
    __syncthreads();
    const int before = max(cmax, w > 0 ? wred[w - 1] : 0);   // end of the segment before this warp
    const int pend = max(v, before);
    int pstart = __shfl_up_sync(full, pend, 1);
    if (lane == 0) pstart = before;
    const int tile_max = max(cmax, wred[31]);
    __syncthreads();
    const int len = j < nseg ? pend - pstart : 0;
    const int nch = (len + QI - 1) / QI;
    // exclusive sum-scan of the chunk counts
    int c = nch;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(full, c, o);
      if (lane >= o) c += t;
    }
    if (lane == 31) wred[w] = c;
    __syncthreads();
    if (w == 0) {
      int t = wred[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(full, t, o);
        if (lane >= o) t += u;
      }
      wred[lane] = t;
    }
    __syncthreads();
    const int off = ccnt + (w > 0 ? wred[w - 1] : 0) + c - nch;
    const bool is_seq = j >= 1 && j <= S;
    for (int i = 0; i < nch; ++i)
      if (off + i < cap) sched[off + i] = make_int2(pstart + QI * i, (is_seq && i == nch - 1) ? j - 1 : -1);
    if (is_seq && len == 0) empty_list[atomicAdd(&nempty, 1)] = j - 1;
    const int tile_cnt = wred[31];
    __syncthreads();
    if (tid == 0) {
      carry_max = tile_max;
      carry_cnt = ccnt + tile_cnt;
    }
    const int ne = nempty;
    if (vstates != nullptr)
      for (int k = 0; k < ne; ++k) {
        float* dst = vstates + (int64_t)empty_list[k] * vstride;
        for (int64_t i = tid; i < vstride; i += SCHED_THREADS) dst[i] = 0.f;
      }
    __syncthreads();
  }
  if (tid == 0) {
    const int n = min(carry_cnt, cap);
    hdr[0] = n;
    sched[n] = make_int2(L, -1);
  }
}

// ---------------------------------------------------------------------------
// Sequence split (few heads per GPU, e.g. one head-sharded rank of a layer).  The fused
// kernel walks one head's chunks serially, so b*H CTAs well below the SM count leave most of
// the GPU idle.  The sequence of each batch row is then cut into seg_k chunk-aligned
// segments, run as seg_k rows of a (b*seg_k, L/seg_k) view of the same memory.  Segment j
// needs the state S_j entering it:
//   tc_segstate_kernel  per (row, head) of every segment but the last: the segment's state
//                       from a zero start, L_j = sum_t exp(dA_end - dA_t) dt_t B_t^T x_t
//                       (one tcgen05 accumulation over the segment's tokens; each token's
//                       x row is scaled in shared memory), and its total dA
// and the fused kernel's state warps start segment j from
//   S_j = sum_{l<j} exp(total dA of segments l+1..j-1) L_l + exp(total dA of 0..j-1) S_init.  Only the state recurrence
// crosses segments (state_passing_fwd.py:108-151 restated over segments), so outputs and
// the final state equal the unsplit walk up to rounding.
// ---------------------------------------------------------------------------
struct SegArgs {
  CUtensorMap tm_x, tm_b;
  int H, G, k, nc;              // heads, groups, segments per row, chunks per segment
  int rows;                     // b * k
  float lo;                     // dt clamp minimum (the decays factor when it is >= 0)
  const float* A;
  const float* dtprep;          // pre-pass output of the (b*k, L/k) view
  float* seg_state;             // (b*k, H, P, N): L_j
  float* seg_tot;               // (b*k, H): total dA of segment j
  unsigned* status;
};

template <int NT>
struct SegGeo {
  static constexpr int STAGES = NT == 256 ? 2 : 4;        // B + x tiles of that many chunks in flight
  static constexpr uint32_t SZ_B = QI * NT * 2;         // B tile of one chunk
  static constexpr uint32_t SZ_X = QI * PT * 2;         // x tile
  static constexpr uint32_t SZ_STAGE = SZ_B + SZ_X;
  static constexpr uint32_t OFF_XS = STAGES * SZ_STAGE;   // two xs buffers
  static constexpr uint32_t BYTES = OFF_XS + 2 * SZ_X;
  static constexpr uint32_t TCOLS = NT == 256 ? 128 : 64;
};

__device__ __forceinline__ bool seg_wait(uint64_t* bar, uint32_t parity, unsigned* status, int id) {
  const long long t0 = clock64();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > TIMEOUT_CYCLES) {
      if (status) atomicCAS(status, 0u, (unsigned)(0x100 | id));
      return false;
    }
  }
  return true;
}

// What row r of chunk c needs from the pre-pass output: dA_last - ref and w_r.
struct SegRow {
  float e, w;
};
__device__ __forceinline__ SegRow seg_row(const float* dA, bool factor, int r) {
  const int q = r >> 5;
  const float last = dA[QI - 1], d0 = dA[32 * q], d31 = dA[32 * q + 31], dr = dA[r];
  const bool fq = factor && (d0 - d31 <= FAC_RANGE);   // block_factored on the same values
  return {last - (fq ? d0 : dr), dA[QI + r]};
}

template <int NT>
__device__ __forceinline__ void seg_load(const SegArgs& a, uint8_t* st, uint64_t* bar, int g, int h, int c, int row) {
  using G_ = SegGeo<NT>;
  ptx::mbar_arrive_expect_tx(bar, G_::SZ_STAGE);
  for (int hh = 0; hh < NT / 64; ++hh) ptx::tma_load_3d(st + hh * (QI * 128), &a.tm_b, bar, g * NT + 64 * hh, c * QI, row);
  ptx::tma_load_3d(st + G_::SZ_B, &a.tm_x, bar, h * PT, c * QI, row);
}

template <int NT>
__global__ void __launch_bounds__(128, 1) tc_segstate_kernel(const __grid_constant__ SegArgs a) {
  using G_ = SegGeo<NT>;
  constexpr int ST = G_::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full[ST], done[2], fin;
  __shared__ uint32_t tbase;
  __shared__ float tots[64];
  __shared__ volatile int bad;
  const int r = threadIdx.x, warp = r >> 5;
  // block -> (batch row, segment j < k-1, head)
  const int per = (a.k - 1) * a.H;
  const int b0 = blockIdx.x / per, rem = blockIdx.x % per;
  const int j = rem / a.H, h = rem % a.H;
  const int row = b0 * a.k + j, g = h / (a.H / a.G);
  const int nc = a.nc;
  const float* prep = a.dtprep + ((int64_t)row * a.H + h) * nc * (2 * QI);
  if (r == 0) {
    for (int i = 0; i < ST; ++i) ptx::mbar_init(&full[i], 1);
    ptx::mbar_init(&done[0], 1);
    ptx::mbar_init(&done[1], 1);
    ptx::mbar_init(&fin, 1);
    bad = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    ptx::tmem_alloc(&tbase, G_::TCOLS);
    ptx::tmem_relinquish();
  }
  // chunk totals of the segment (dA of each chunk's last token), for the suffix decays
  for (int c = r; c < nc; c += 128) tots[c] = prep[(int64_t)c * 2 * QI + QI - 1];
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  // the fused kernel may start now: its CTAs read this pass's results only after waiting
  ptx::griddep_launch_dependents();
  if (r == 0)
    for (int c = 0; c < nc && c < ST; ++c) seg_load<NT>(a, sm + c * G_::SZ_STAGE, &full[c], g, h, c, row);
  const bool factor = (a.A[h] <= 0.f) && (a.lo >= 0.f);
  float suffix = 0.f;
  for (int c = 0; c < nc; ++c) suffix += tots[c];   // total dA of the segment
  const float total = suffix;
  constexpr uint32_t ID_L = ptx::idesc_bf16_f32(128, 64, 1, 1);
  SegRow nxt = seg_row(prep, factor, r);            // chunk 0's factors, then one chunk ahead
  for (int c = 0; c < nc; ++c) {
    suffix -= tots[c];                               // dA of the chunks after c
    const int s = c % ST;
    const SegRow cur = nxt;
    if (c + 1 < nc) nxt = seg_row(prep + (int64_t)(c + 1) * 2 * QI, factor, r);
    // exp(dA_end - dA_r) dt_r = exp(suffix + dA_last - ref) w_r
    const float scale = __expf(suffix + cur.e) * cur.w;
    // xs buffer c % 2 is free once MMA(c-2) is done; the tiles of chunk c have landed
    if (c >= 2 && !seg_wait(&done[c & 1], ((c >> 1) - 1) & 1, a.status, 1)) bad = 1;
    if (!seg_wait(&full[s], (c / ST) & 1, a.status, 2)) bad = 1;
    __syncthreads();   // every thread sees the same `bad` (the waits above are bounded)
    if (bad) break;
    const uint8_t* xt = sm + s * G_::SZ_STAGE + G_::SZ_B;
    uint8_t* xs = sm + G_::OFF_XS + (c & 1) * G_::SZ_X;
    uint4 w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = *reinterpret_cast<const uint4*>(xt + ptx::sw128_off(r, k));
#pragma unroll
    for (int k = 0; k < 8; ++k) *reinterpret_cast<uint4*>(xs + ptx::sw128_off(r, k)) = scale_row16(w[k], scale);
    ptx::fence_proxy_async_smem();
    __syncthreads();
    if (r == 0) {
      ptx::tc_fence_after();
      const uint32_t base = ptx::smem_u32(sm);
      for (int hh = 0; hh < NT / 128; ++hh) {
        const uint32_t sB = base + s * G_::SZ_STAGE + hh * (QI * 256);
#pragma unroll
        for (int i = 0; i < QI / 16; ++i)
          ptx::mma_f16(tbase + 64 * hh, ptx::sdesc_sw128(sB + i * 2048, QI * 128, 1024),
                       ptx::sdesc_sw128(base + G_::OFF_XS + (c & 1) * G_::SZ_X + i * 2048, 8192, 1024), ID_L,
                       (c > 0 || i > 0) ? 1u : 0u);
      }
      ptx::mma_commit(&done[c & 1]);
      // refill the stage of chunk c-1 (its MMA was issued an iteration ago) with chunk c-1+ST
      const int cr = c - 1 + ST;
      if (c >= 1 && cr < nc) {
        if (!seg_wait(&done[(c - 1) & 1], ((c - 1) >> 1) & 1, a.status, 3)) bad = 1;
        else seg_load<NT>(a, sm + ((c - 1) % ST) * G_::SZ_STAGE, &full[(c - 1) % ST], g, h, cr, row);
      }
    }
  }
  if (r == 0) ptx::mma_commit(&fin);
  const bool ok = seg_wait(&fin, 0, a.status, 4) && !bad;
  ptx::tc_fence_after();
  if (ok) {
    // L_j[p][n] for n = lane + 32 warp + 128 hh (TMEM lane n), p = column
    float* dst = a.seg_state + ((int64_t)row * a.H + h) * PT * NT;
    for (int hh = 0; hh < NT / 128; ++hh) {
      for (int half = 0; half < 2; ++half) {
        float v[32];
        ptx::tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + 64 * hh + 32 * half, v);
        ptx::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[(int64_t)(32 * half + i) * NT + 128 * hh + r] = v[i];
      }
    }
    if (r == 0) a.seg_tot[(int64_t)row * a.H + h] = total;
  }
  // do not leave with copies still landing in shared memory: the last load of every stage
  if (r == 0) {
    for (int st = 0; st < ST && st < nc; ++st) {
      const int last = st + ((nc - 1 - st) / ST) * ST;   // last chunk loaded into stage st
      seg_wait(&full[st], (last / ST) & 1, a.status, 5);
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, G_::TCOLS);
  }
}


// ---------------------------------------------------------------------------
// Sequence-parallel decay fix-up on the tensor cores (bf16 C, P = 64, N = 128 or 256).
// For every token t of the carried sequence, out[t] += exp(dA(t)) (C_t . S^T) (silu(z_t)),
// the inter-chunk term of chunk_scan_fwd.py:108-232 with the received state S: per
// 128-token tile one tcgen05 product Y = C_tile . S^T (M = 128 tokens, N = 64, K = dstate;
// A = the C tile by TMA, B = S as bf16 [n][p] in shared memory, as the fused kernel's MMA3),
// then each thread adds its token's row.  dA(t) is the segment-wide cumulative dt*A: the
// chunk totals before t's chunk plus the within-chunk value, from the (b, H, nc, Q)
// chunk_cumsum output.  The extra x-block updates the final state.
// ---------------------------------------------------------------------------
struct FixArgs {
  CUtensorMap tm_c;
  int64_t L, H, G, Q, nc;
  const float* dA;
  const float* S;
  const int32_t* carried;
  const bf16* z;
  float* out;
  float* final_states;
  unsigned* status;
};

template <int NT>
__global__ void __launch_bounds__(128) tc_sp_fixup_kernel(const __grid_constant__ FixArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (ptx::smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr uint32_t SZ_C = QI * NT * 2, OFF_ST = SZ_C;
  __shared__ uint64_t full, done;
  __shared__ uint32_t tbase;
  __shared__ float base_dA;
  const int r = threadIdx.x, warp = r >> 5, lane = r & 31;
  const int64_t bi = blockIdx.z, h = blockIdx.y;
  const int64_t ntiles = (a.L + QI - 1) / QI;
  const int64_t clen = a.carried ? min((int64_t)a.carried[bi], a.L) : a.L;
  const float* dAh = a.dA + (bi * a.H + h) * a.nc * a.Q;
  const float* Sh = a.S + (bi * a.H + h) * PT * NT;
  if (blockIdx.x == ntiles) {   // final state: += exp(total dA) S when the carried sequence reaches the end
    if (a.final_states == nullptr || clen < a.L) return;
    float part = 0.f;
    for (int64_t c = r; c < a.nc; c += 128) part += dAh[c * a.Q + a.Q - 1];
    __shared__ float red[4];
    part = warp_sum(part);
    if (lane == 0) red[warp] = part;
    __syncthreads();
    const float dec = __expf(red[0] + red[1] + red[2] + red[3]);
    float* fh = a.final_states + (bi * a.H + h) * PT * NT;
    for (int64_t i = r; i < PT * NT; i += 128) fh[i] = fmaf(dec, Sh[i], fh[i]);
    return;
  }
  const int64_t t0 = (int64_t)blockIdx.x * QI;
  if (t0 >= clen) return;
  const int g = (int)(h / (a.H / a.G));
  if (r == 0) {
    ptx::mbar_init(&full, 1);
    ptx::mbar_init(&done, 1);
    ptx::fence_mbar_init();
    ptx::mbar_arrive_expect_tx(&full, SZ_C);
    for (int j = 0; j < NT / 64; ++j) ptx::tma_load_3d(sm + j * (QI * 128), &a.tm_c, &full, g * NT + 64 * j, (int)t0, (int)bi);
  }
  if (warp == 0) {
    ptx::tmem_alloc(&tbase, 64);
    ptx::tmem_relinquish();
    // chunk totals before t0's chunk
    const int64_t c0 = t0 / a.Q;
    float part = 0.f;
    for (int64_t c = lane; c < c0; c += 32) part += dAh[c * a.Q + a.Q - 1];
    part = warp_sum(part);
    if (lane == 0) base_dA = part;
  }
  // S as bf16 [n][p] (128-byte rows, swizzled): thread r owns rows n = r + 128 hh
  uint8_t* st_sm = sm + OFF_ST;
  for (int hh = 0; hh < NT / 128; ++hh) {
    const int n = hh * 128 + r;
    for (int half = 0; half < 2; ++half) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = Sh[(int64_t)(32 * half + i) * NT + n];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(st_sm + ptx::sw128_off(n, 4 * half + j)) =
            make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                       pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
    }
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  bool ok = true;
  if (r == 0) {
    if (seg_wait(&full, 0, a.status, 6)) {
      constexpr uint32_t ID = ptx::idesc_bf16_f32(128, 64, 0, 1);
      const uint32_t base = ptx::smem_u32(sm);
      for (int hh = 0; hh < NT / 128; ++hh) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t offa = hh * (QI * 256) + (i >> 2) * (QI * 128) + (i & 3) * 32;
          ptx::mma_f16(tbase, ptx::sdesc_sw128(base + offa, 16, 1024),
                       ptx::sdesc_sw128(base + OFF_ST + hh * (128 * 128) + i * 2048, 8192, 1024), ID,
                       (hh > 0 || i > 0) ? 1u : 0u);
        }
      }
    }
    ptx::mma_commit(&done);
  }
  // this thread's token: its decay while the MMA runs
  const int64_t t = t0 + r;
  float dg = 0.f;
  if (t < clen) {
    const int64_t c = t / a.Q;
    float run = base_dA;
    for (int64_t cc = t0 / a.Q; cc < c; ++cc) run += dAh[cc * a.Q + a.Q - 1];
    dg = __expf(run + dAh[c * a.Q + (t - c * a.Q)]);
  }
  ok = seg_wait(&done, 0, a.status, 7);
  ptx::tc_fence_after();
  if (ok) {
    for (int half = 0; half < 2; ++half) {
      float y[32];
      ptx::tmem_ld32(tbase + ((uint32_t)(warp * 32) << 16) + 32 * half, y);
      ptx::tmem_ld_wait();
      if (t < clen) {
        const int64_t row = ((bi * a.L + t) * a.H + h) * PT + 32 * half;
        float4* o = reinterpret_cast<float4*>(a.out + row);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float4 v = o[k];
          float f[4] = {dg * y[4 * k], dg * y[4 * k + 1], dg * y[4 * k + 2], dg * y[4 * k + 3]};
          if (a.z) {
#pragma unroll
            for (int e = 0; e < 4; ++e) f[e] *= silu(__bfloat162float(a.z[row + 4 * k + e]));
          }
          v.x += f[0]; v.y += f[1]; v.z += f[2]; v.w += f[3];
          o[k] = v;
        }
      }
    }
  } else if (r == 0) {
    seg_wait(&full, 0, a.status, 8);   // never leave with the copy still landing
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, 64);
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

// 3-D map over (inner = cols, rows = L, batch) with a (128 bytes) x 128 x 1 box, 128B swizzle:
// bf16 boxes are 64 columns wide, f32 boxes 32.
bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t L, uint64_t b, bool f32 = false) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const uint64_t es_bytes = f32 ? 4 : 2;
  cuuint64_t dims[3] = {cols, L, b};
  cuuint64_t strides[2] = {cols * es_bytes, cols * L * es_bytes};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es_bytes), (cuuint32_t)QI, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base),
            dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool tc_supported(const ssd_fwd_params_t* p) {
  if (p->dtype != SSD_DTYPE_BF16 || p->headdim != PT || (p->dstate != 128 && p->dstate != 256)) return false;
  if (p->dA_cumsum || p->dt_out) return false;
  // the skip term rides on the diagonal of the scores, which holds one D per head
  if (p->D && p->D_ndim == 2) return false;
  // varlen states come from the per-sequence chunk schedule, which needs the seq_idx masks
  // inside the chunks it still shares with other sequences' rows.  With initial states the
  // reference's varlen result depends on its chunking (the first sequence sees the initial
  // state only if it crosses a chunk boundary, chunk_state_fwd.py:448-597), so those
  // calls stay on the stage pipeline, which follows it exactly.
  if (p->varlen_states &&
      (!p->seq_idx || !p->cu_seqlens || p->num_seqs <= 0 || p->batch != 1 || p->initial_states))
    return false;
  if (p->batch * p->nheads > 0x7fffffff) return false;
  const uintptr_t al = 15;
  if ((reinterpret_cast<uintptr_t>(p->x) | reinterpret_cast<uintptr_t>(p->B) | reinterpret_cast<uintptr_t>(p->C) |
       reinterpret_cast<uintptr_t>(p->out) | reinterpret_cast<uintptr_t>(p->z) |
       reinterpret_cast<uintptr_t>(p->out_x)) & al)
    return false;
  return encode_fn() != nullptr;
}

bool trace_enabled() {
#ifndef SSD_TC_DEBUG_TRACE
  return false;
#endif
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("SSD_TC_TRACE");
    on = (e && e[0] == '1') ? 1 : 0;
  }
  return on == 1;
}

// Workspace (the status word is separate, owned by the caller): with varlen states the
// chunk schedule (an 8-byte header, then cap + 1 int2 entries); the dt pre-pass output; with
// SSD_TC_TRACE=1 a 64 KB phase trace.
int64_t sched_cap(const ssd_fwd_params_t* p) { return (p->seqlen + QI - 1) / QI + p->num_seqs + 2; }
size_t sched_bytes(const ssd_fwd_params_t* p) {
  return p->varlen_states ? (size_t)(8 + 8 * (sched_cap(p) + 1) + 255) / 256 * 256 : 0;
}

// Segments per batch row of the sequence split (1: none).  Used when few (batch, head)
// walks would leave most SMs idle: no packed sequences (the segment states then compose by
// plain decays), chunk-aligned segments of at least two and at most 64 chunks.
int seg_split(const ssd_fwd_params_t* p) {
  if (p->seq_idx || p->varlen_states || p->seqlen % QI) return 1;
  const int64_t bh = p->batch * p->nheads, nci = p->seqlen / QI;
  // SSD_TC_SEGMENTS=k (tuning experiments only) forces the segment count
  static const int forced = [] {
    const char* e = getenv("SSD_TC_SEGMENTS");
    return e ? atoi(e) : 0;
  }();
  if (forced == 0 && bh >= 96) return 1;
  int k = forced > 0 ? (int)std::min<int64_t>(forced, nci / 2) : (int)std::min<int64_t>(148 / bh, nci / 2);
  while (k > 1 && (nci % k || nci / k > 64)) --k;
  return std::max(k, 1);
}

// dt pre-pass output: 1 KB per (batch, head, chunk slot).
int64_t prep_cap(const ssd_fwd_params_t* p) {
  return p->varlen_states ? sched_cap(p) : (p->seqlen + QI - 1) / QI / seg_split(p);
}
size_t prep_bytes(const ssd_fwd_params_t* p) {
  return (size_t)p->batch * seg_split(p) * p->nheads * prep_cap(p) * 2 * QI * 4;
}
// sequence split: L_j (b*k, H, P, N) f32, then the segment totals (b*k, H)
size_t seg_bytes(const ssd_fwd_params_t* p) {
  const int k = seg_split(p);
  if (k == 1) return 0;
  const size_t rows = (size_t)p->batch * k * p->nheads;
  return rows * PT * p->dstate * 4 + (rows * 4 + 255) / 256 * 256;
}

size_t tc_workspace_bytes(const ssd_fwd_params_t* p) {
  return tc_supported(p) ? sched_bytes(p) + prep_bytes(p) + seg_bytes(p) + (trace_enabled() ? 8 * 64 * 16 * 8 + 65536 : 0)
                         : 0;
}

int tc_num_launches(const ssd_fwd_params_t* p) { return p->varlen_states ? 3 : seg_split(p) > 1 ? 3 : 2; }

// Dynamic shared memory opt-in, per device and kernel variant (the attribute belongs to the
// current device's context, so a process that drives several GPUs sets it on each).
bool ensure_smem_attr(void (*kern)(TcArgs), int kid) {
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static uint8_t done[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < kMaxDev && (done[dev] >> kid & 1)) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LAUNCH_BYTES) != cudaSuccess)
    return false;
  if (dev >= 0 && dev < kMaxDev) done[dev] |= (uint8_t)(1u << kid);
  return true;
}

bool tc_sp_fixup_supported(const ssd_sp_fixup_params_t* p) {
  return p->dtype == SSD_DTYPE_BF16 && p->headdim == PT && (p->dstate == 128 || p->dstate == 256) &&
         !(reinterpret_cast<uintptr_t>(p->C) & 15) && !(reinterpret_cast<uintptr_t>(p->out) & 15) &&
         p->batch * p->nheads <= 65535 && p->seqlen < 0x7fffffff && encode_fn() != nullptr;
}

int tc_sp_fixup(const ssd_sp_fixup_params_t* p, cudaStream_t st) {
  FixArgs a;
  memset(&a, 0, sizeof(a));
  if (!make_map(&a.tm_c, p->C, (uint64_t)p->ngroups * p->dstate, p->seqlen, p->batch)) {
    set_last_error("cuTensorMapEncodeTiled failed for C");
    return SSD_ERR_CUDA;
  }
  a.L = p->seqlen; a.H = p->nheads; a.G = p->ngroups; a.Q = p->chunk_size;
  a.nc = (p->seqlen + p->chunk_size - 1) / p->chunk_size;
  a.dA = p->dA_cumsum; a.S = p->state_in; a.carried = p->carried_len; a.z = (const bf16*)p->z;
  a.out = p->out; a.final_states = p->final_states;
  a.status = nullptr;   // no workspace: a wait that gives up leaves that tile's tokens without the update
  const dim3 grid((unsigned)((p->seqlen + QI - 1) / QI + 1), (unsigned)p->nheads, (unsigned)p->batch);
  if (p->dstate == 256) {
    const uint32_t bytes = QI * 256 * 2 + 256 * PT * 2 + 1024;
    cudaFuncSetAttribute(tc_sp_fixup_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    tc_sp_fixup_kernel<256><<<grid, 128, bytes, st>>>(a);
  } else {
    const uint32_t bytes = QI * 128 * 2 + 128 * PT * 2 + 1024;
    cudaFuncSetAttribute(tc_sp_fixup_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    tc_sp_fixup_kernel<128><<<grid, 128, bytes, st>>>(a);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return SSD_ERR_CUDA;
  }
  return SSD_OK;
}

int tc_combined_fwd(const ssd_fwd_params_t* p, unsigned* status, void* workspace, cudaStream_t st) {
  TcArgs a;
  memset(&a, 0, sizeof(a));
  // with a sequence split the walk runs on the (b*k, L/k) view of the same memory
  const int k = seg_split(p);
  const int64_t b = p->batch * k, L = p->seqlen / k, H = p->nheads, G = p->ngroups;
  if (!make_map(&a.tm_x, p->x, (uint64_t)H * PT, L, b) || !make_map(&a.tm_b, p->B, (uint64_t)G * p->dstate, L, b) ||
      !make_map(&a.tm_c, p->C, (uint64_t)G * p->dstate, L, b) ||
      !make_map(&a.tm_out, p->out, (uint64_t)H * PT, L, b, true)) {
    set_last_error("cuTensorMapEncodeTiled failed for x/B/C/out");
    return SSD_ERR_CUDA;
  }
  a.L = (int)L; a.H = (int)H; a.G = (int)G; a.nci = (int)((L + QI - 1) / QI);
  a.dt_bf16 = p->dt_dtype == SSD_DTYPE_BF16; a.softplus = p->dt_softplus; a.D_ndim = p->D ? p->D_ndim : 0;
  a.lo = p->dt_min; a.hi = p->dt_max;
  a.dt = p->dt; a.A = p->A; a.dt_bias = p->dt_bias; a.D = p->D;
  a.x = (const bf16*)p->x; a.z = (const bf16*)p->z; a.init = p->initial_states; a.seq_idx = p->seq_idx;
  a.out = p->out; a.out_x = p->z ? p->out_x : nullptr; a.final_states = p->final_states;
  a.varlen_states = p->varlen_states;
  a.status = status;
  a.test_wait_cycles = (p->flags & SSD_FLAG_TEST_WAIT_TIMEOUT) ? 20000 : 0;
  float* prep_out = (float*)((char*)workspace + sched_bytes(p));
  a.dtprep = prep_out;
  a.prep_cap = (int)prep_cap(p);
  a.seg_k = k;
  a.rows = (int)b;
  a.num_seqs = p->num_seqs;
  a.sched_cap = p->varlen_states ? (int)sched_cap(p) : 0;
  a.trace = trace_enabled() ? (unsigned long long*)((char*)workspace + sched_bytes(p) + prep_bytes(p) + seg_bytes(p))
                            : nullptr;
  typedef void (*KernelFn)(TcArgs);
  static const KernelFn kernels[8] = {
      ssd_fused_tc_kernel<128, false, false>, ssd_fused_tc_kernel<128, false, true>,
      ssd_fused_tc_kernel<128, true, false>,  ssd_fused_tc_kernel<128, true, true>,
      ssd_fused_tc_kernel<256, false, false>, ssd_fused_tc_kernel<256, false, true>,
      ssd_fused_tc_kernel<256, true, false>,  ssd_fused_tc_kernel<256, true, true>};
  const int kid = (p->dstate == 256 ? 4 : 0) + (p->seq_idx ? 2 : 0) + (p->z ? 1 : 0);
  const KernelFn kern = kernels[kid];
  if (!ensure_smem_attr(kern, kid)) {
    set_last_error("cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed");
    return SSD_ERR_CUDA;
  }
  if (p->varlen_states) {
    const int64_t cap = sched_cap(p);
    if (cap > 0x3fffffff) {
      set_last_error("varlen chunk schedule too long");
      return SSD_ERR_UNSUPPORTED;
    }
    int* hdr = (int*)workspace;
    int2* sched = (int2*)((char*)workspace + 8);
    tc_schedule_kernel<<<1, SCHED_THREADS, 0, st>>>(p->cu_seqlens, p->num_seqs, (int)L, (int)cap, hdr, sched,
                                                    p->varlen_states, H * PT * p->dstate);
    a.sched_n = hdr;
    a.sched = sched;
  }
  {
    const dim3 grid((unsigned)a.prep_cap, (unsigned)b, (unsigned)((H + 3) / 4));
    if (a.dt_bf16) tc_dt_prep_kernel<true><<<grid, 128, 0, st>>>(a, prep_out);
    else tc_dt_prep_kernel<false><<<grid, 128, 0, st>>>(a, prep_out);
  }
  if (k > 1) {
    SegArgs sa;
    memset(&sa, 0, sizeof(sa));
    sa.tm_x = a.tm_x;
    sa.tm_b = a.tm_b;
    sa.H = (int)H; sa.G = (int)G; sa.k = k; sa.nc = (int)(L / QI); sa.rows = (int)b; sa.lo = p->dt_min;
    sa.A = p->A; sa.dtprep = prep_out; sa.status = status;
    const size_t rows = (size_t)b * H, pn = (size_t)PT * p->dstate;
    float* seg_state = (float*)((char*)workspace + sched_bytes(p) + prep_bytes(p));
    sa.seg_state = seg_state;
    sa.seg_tot = seg_state + rows * pn;
    const unsigned nblk = (unsigned)(p->batch * (k - 1) * H);
    if (p->dstate == 256) {
      const uint32_t bytes = SegGeo<256>::BYTES + 1024;
      cudaFuncSetAttribute(tc_segstate_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      tc_segstate_kernel<256><<<nblk, 128, bytes, st>>>(sa);
    } else {
      const uint32_t bytes = SegGeo<128>::BYTES + 1024;
      cudaFuncSetAttribute(tc_segstate_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      tc_segstate_kernel<128><<<nblk, 128, bytes, st>>>(sa);
    }
    a.seg_state = seg_state;
    a.seg_tot = sa.seg_tot;
  }
  if (k > 1) {
    // a programmatic dependent of the segment-state pass: its prologue, loads and
    // intra-chunk work overlap that pass; the state warps wait for its results
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)(b * H));
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = SMEM_LAUNCH_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, a);
  } else {
    kern<<<(unsigned)(b * H), NTHREADS, SMEM_LAUNCH_BYTES, st>>>(a);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[160];
    snprintf(msg, sizeof(msg), "ssd_fused_tc_kernel launch: %s", cudaGetErrorString(e));
    set_last_error(msg);
    return SSD_ERR_CUDA;
  }
  return SSD_OK;
}

}  // namespace ssd
