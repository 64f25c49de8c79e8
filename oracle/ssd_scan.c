/*
 * ssd_scan.c -- float64 token-by-token recurrence of the Mamba2 SSD layer (C, OpenMP).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for full-size parity tests.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the product path
 * never does.  Built by oracle/build_scan.py into oracle/_build/libssd_scan.so.
 *
 * It computes the same function as the reference's chunked forward
 * (src/mamba2_jax/ops/ssd_naive.py:325-397, kernels/ssd_combined.py:46-203) through the
 * recurrence that the chunked form factorises, one token at a time:
 *
 *   dt'   = clamp(softplus?(dt + dt_bias), dt_min, dt_max)       (chunk_cumsum_fwd.py:221-231,
 *                                                                  softplus with threshold 20)
 *   S     = exp(dt' A) S + dt' x B^T                              (S is P x N per head)
 *   y     = S C + D x ;  out = y * silu(z)                         (chunk_scan_fwd.py)
 *
 * Packed sequences (seq_idx): S restarts from zero at a token whose id differs from the
 * previous token's; the initial state feeds the tokens before the first change only when
 * their id is 0 (the rules of chunk_state_fwd.py:246-269, state_passing_fwd.py:208-225 and
 * chunk_scan_fwd.py:294-322 compose to this at any chunk size).  The final state is S after
 * the last token; varlen states (cu_seqlens, batch 1) are S after the last token of each
 * sequence, zero for an empty one.  Padded positions never enter (the kernel path's rule).
 *
 * Cost is O(b L H P N) with no chunk-quadratic term, so full BASELINE sizes finish in
 * seconds on a many-core host.  Heads [h0, h1) only are computed (outputs of other heads
 * are left untouched), so callers can check a subset.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct ssd_scan_args {
  int64_t b, L, H, P, G, N;
  int64_t h0, h1;             /* head range */
  const float* x;             /* (b,L,H,P) */
  const float* dt;            /* (b,L,H) */
  const float* A;             /* (H,) */
  const float* B;             /* (b,L,G,N) */
  const float* C;             /* (b,L,G,N) */
  const float* D;             /* (H,) or (H,P) or NULL */
  int32_t D_ndim;
  int32_t dt_softplus;
  const float* z;             /* (b,L,H,P) or NULL */
  const float* dt_bias;       /* (H,) or NULL */
  double dt_min, dt_max;
  const float* init;          /* (b,H,P,N) or NULL */
  const int32_t* seq_idx;     /* (b,L) or NULL */
  const int32_t* cu_seqlens;  /* (num_seqs+1,) or NULL; batch 1 */
  int64_t num_seqs;
  double* out;                /* (b,L,H,P) */
  double* final_states;       /* (b,H,P,N) or NULL */
  double* varlen_states;      /* (num_seqs,H,P,N) or NULL */
} ssd_scan_args_t;

static double proc_dt(double v, double bias, int sp, double lo, double hi) {
  v += bias;
  if (sp) v = v <= 20.0 ? log1p(exp(v)) : v;
  if (v < lo) v = lo;
  if (v > hi) v = hi;
  return v;
}

int ssd_scan_f64(const ssd_scan_args_t* a) {
  const int64_t b = a->b, L = a->L, H = a->H, P = a->P, G = a->G, N = a->N;
  if (b <= 0 || L <= 0 || H <= 0 || P <= 0 || G <= 0 || N <= 0 || H % G) return 1;
  if (a->h0 < 0 || a->h1 > H || a->h0 >= a->h1) return 1;
  const int64_t r = H / G, nh = a->h1 - a->h0;
  /* varlen: the sequence that ends at token t (or -1) */
  int64_t* end_of = NULL;
  if (a->varlen_states && a->cu_seqlens) {
    if (b != 1) return 1;
    end_of = (int64_t*)malloc(sizeof(int64_t) * L);
    if (!end_of) return 2;
    for (int64_t t = 0; t < L; ++t) end_of[t] = -1;
    for (int64_t k = 0; k < a->num_seqs; ++k) {
      int64_t s = a->cu_seqlens[k], e = a->cu_seqlens[k + 1];
      if (s < 0) s = 0;
      if (e > L) e = L;
      if (e > s) end_of[e - 1] = k;
      else
        for (int64_t h = a->h0; h < a->h1; ++h)
          memset(a->varlen_states + ((k * H + h) * P) * N, 0, sizeof(double) * P * N);
    }
  }
  int err = 0;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t bh = 0; bh < b * nh; ++bh) {
    const int64_t bi = bh / nh, h = a->h0 + bh % nh, g = h / r;
    double* S = (double*)malloc(sizeof(double) * P * N);
    double* xs = (double*)malloc(sizeof(double) * P);
    double* bb = (double*)malloc(sizeof(double) * N);
    double* cc = (double*)malloc(sizeof(double) * N);
    if (!S || !xs || !bb || !cc) {
#pragma omp atomic write
      err = 2;
      free(S); free(xs); free(bb); free(cc);
      continue;
    }
    const double Ah = a->A[h], bias = a->dt_bias ? a->dt_bias[h] : 0.0;
    const int start0 = !a->seq_idx || a->seq_idx[bi * L] == 0;
    for (int64_t i = 0; i < P * N; ++i)
      S[i] = (a->init && start0) ? (double)a->init[((bi * H + h) * P) * N + i] : 0.0;
    for (int64_t t = 0; t < L; ++t) {
      if (a->seq_idx && t > 0 && a->seq_idx[bi * L + t] != a->seq_idx[bi * L + t - 1])
        memset(S, 0, sizeof(double) * P * N);
      const double d = proc_dt(a->dt[(bi * L + t) * H + h], bias, a->dt_softplus, a->dt_min, a->dt_max);
      const double dec = exp(d * Ah);
      const float* xp = a->x + ((bi * L + t) * H + h) * P;
      const float* Bp = a->B + ((bi * L + t) * G + g) * N;
      const float* Cp = a->C + ((bi * L + t) * G + g) * N;
      for (int64_t p = 0; p < P; ++p) xs[p] = d * (double)xp[p];
      for (int64_t n = 0; n < N; ++n) {
        bb[n] = Bp[n];
        cc[n] = Cp[n];
      }
      double* o = a->out + ((bi * L + t) * H + h) * P;
      for (int64_t p = 0; p < P; ++p) {
        double* Sp = S + p * N;
        const double xv = xs[p];
        double acc = 0.0;
        for (int64_t n = 0; n < N; ++n) {
          Sp[n] = dec * Sp[n] + xv * bb[n];
          acc += Sp[n] * cc[n];
        }
        if (a->D) acc += (a->D_ndim == 2 ? (double)a->D[h * P + p] : (double)a->D[h]) * (double)xp[p];
        if (a->z) {
          const double zv = a->z[((bi * L + t) * H + h) * P + p];
          acc *= zv / (1.0 + exp(-zv));
        }
        o[p] = acc;
      }
      if (end_of && end_of[t] >= 0)
        memcpy(a->varlen_states + ((end_of[t] * H + h) * P) * N, S, sizeof(double) * P * N);
    }
    if (a->final_states) memcpy(a->final_states + ((bi * H + h) * P) * N, S, sizeof(double) * P * N);
    free(S); free(xs); free(bb); free(cc);
  }
  free(end_of);
  return err;
}
