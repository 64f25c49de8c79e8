/*
 * ssd_b200.h — C ABI of the B200 (sm_100a) Mamba2 SSD forward and decode-step kernels.
 *
 * This is the drop-in boundary.  Each entry point replaces one function of the
 * reference's hot path (AlexG1105/mamba2-jax-pallas, cited as path:line below) and is
 * what a jax.ffi handler, a ctypes binding or a C++ caller binds.
 *
 * Conventions (all entry points):
 *   - Plain device pointers; every tensor is dense row-major ("contiguous") in the
 *     documented layout.  Dims use the reference's names: b=batch, L=seqlen,
 *     H=nheads, P=headdim, G=ngroups, N=dstate, Q=chunk_size, nc=ceil(L/Q).
 *     Head h reads group h / (H/G).
 *   - Input tensors x, B, C, z (and dt, separately) are SSD_DTYPE_F32 or
 *     SSD_DTYPE_BF16; A, D, dt_bias, initial_states and every output are float32.
 *   - Work is enqueued on `stream`; nothing blocks the host and nothing allocates
 *     device memory.  Scratch memory, where needed, is caller-provided
 *     (`workspace`, size from the matching *_workspace_bytes()).
 *   - The return value is an ssd_status_t; on failure ssd_last_error() returns a
 *     thread-local message.  Shape/pointer errors are reported before any launch.
 *   - Calls on one stream are ordered; concurrent calls on different streams must
 *     not share output or workspace buffers.
 */
#ifndef SSD_B200_H_
#define SSD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSD_B200_ABI_VERSION 2

typedef enum ssd_status {
  SSD_OK = 0,
  SSD_ERR_INVALID_ARG = 1,   /* bad shape, null pointer, inconsistent dims */
  SSD_ERR_UNSUPPORTED = 2,   /* valid but not implemented (e.g. dtype combination) */
  SSD_ERR_ALIGNMENT = 3,     /* pointer not aligned as the kernel requires */
  SSD_ERR_WORKSPACE = 4,     /* workspace null or too small */
  SSD_ERR_CUDA = 5,          /* a CUDA launch or runtime call failed */
  SSD_ERR_TIMEOUT = 6        /* a bounded inter-CTA wait gave up (device status word) */
} ssd_status_t;

typedef enum ssd_dtype {
  SSD_DTYPE_F32 = 0,
  SSD_DTYPE_BF16 = 1
} ssd_dtype_t;

/* Opaque CUDA stream (cudaStream_t); 0 = legacy default stream. */
typedef void* ssd_stream_t;

/* Parameters of the combined forward.  Optional pointers may be NULL. */
typedef struct ssd_fwd_params {
  int64_t batch, seqlen, nheads, headdim, ngroups, dstate, chunk_size;
  int32_t dtype;          /* ssd_dtype_t of x, B, C, z */
  int32_t dt_dtype;       /* ssd_dtype_t of dt */
  int32_t dt_softplus;    /* nonzero: dt <- (dt <= 20 ? log1p(exp(dt)) : dt) after bias */
  int32_t D_ndim;         /* 0: no D, 1: D is (H,), 2: D is (H,P) */
  float dt_min, dt_max;   /* clamp applied after softplus (use +INFINITY for no max) */
  int32_t num_seqs;       /* entries of cu_seqlens minus one (varlen states only) */
  int32_t flags;          /* SSD_FLAG_* */
  /* inputs */
  const void* x;          /* (b,L,H,P) */
  const void* dt;         /* (b,L,H) */
  const float* A;         /* (H,) */
  const void* B;          /* (b,L,G,N) */
  const void* C;          /* (b,L,G,N) */
  const float* D;         /* (H,) or (H,P) */
  const void* z;          /* (b,L,H,P) gate: out *= z*sigmoid(z) */
  const float* dt_bias;   /* (H,) */
  const float* initial_states; /* (b,H,P,N) */
  const int32_t* seq_idx;      /* (b,L) packed-sequence ids */
  const int32_t* cu_seqlens;   /* (num_seqs+1,), requires batch == 1 */
  /* outputs */
  float* out;             /* (b,L,H,P), required */
  float* out_x;           /* (b,L,H,P) pre-gate output (only with z) */
  float* final_states;    /* (b,H,P,N) */
  float* varlen_states;   /* (num_seqs,H,P,N), requires cu_seqlens */
  float* dA_cumsum;       /* optional copy-out of stage-1 results, (b,H,nc,Q) */
  float* dt_out;          /* (b,H,nc,Q) */
} ssd_fwd_params_t;

/* flags */
#define SSD_FLAG_FORCE_SIMT   1  /* use the staged pipeline on the CUDA cores only (exact
                                    fp32 FFMA stages), for any input dtype */
#define SSD_FLAG_ROUND_STATES 2  /* round passed chunk states to the input dtype before
                                    chunk_scan, as ssd_combined.py:140 does */
#define SSD_FLAG_BF16_MMA     4  /* fp32 inputs: round x, B, C (and z) to bf16 into the
                                    workspace and run the tensor-core pipeline, as the
                                    reference's Pallas kernels do for fp32 inputs (bf16 MMA
                                    operands, fp32 accumulation); without it fp32 inputs run
                                    the staged pipeline with split-bf16 tensor-core stages
                                    (relative error about 1e-5) */
#define SSD_FLAG_TEST_WAIT_TIMEOUT 8  /* test only: every CTA of the fused tensor-core kernel
                                    first runs a short bounded wait on a barrier that nothing
                                    arrives on, so the wait gives up, the status word records
                                    SSD_ERR_TIMEOUT and the launch does no work (checks the
                                    timeout report without faulting anything) */

/* Bytes of device workspace ssd_combined_fwd needs for these params; 0 when the params are
 * invalid (ssd_combined_fwd then reports why).  The first 4 bytes of every workspace are the
 * device status word (see ssd_status_copy_async). */
size_t ssd_combined_workspace_bytes(const ssd_fwd_params_t* p);

/* Enqueue on `stream` a copy of the device status word of the ssd_combined_fwd call that
 * used `workspace` (its first 4 bytes) to `dst` (host-pinned or device memory).  The word is
 * 0 after a complete launch; a bounded wait inside the fused kernel that gave up (a hang
 * that was cut short) sets it.  Pass the value, once the stream reached the copy, to
 * ssd_status_decode.  No reference counterpart: the reference's kernels have no bounded
 * waits (its failure handling is the Python fallback of src/mamba2_jax/modules/mamba2.py:59-74). */
int ssd_status_copy_async(const void* workspace, uint32_t* dst, ssd_stream_t stream);

/* SSD_OK for a zero status word, else the status it records (SSD_ERR_TIMEOUT for a bounded
 * wait that gave up, SSD_ERR_ALIGNMENT for an unusable shared-memory window), with a
 * description in ssd_last_error().  No reference counterpart (see above). */
int ssd_status_decode(uint32_t word);

/* 1 if ssd_combined_fwd runs the fused tcgen05 pipeline (bf16 MMA operands) for these
 * params, else 0: the staged five-launch pipeline, whose chunk_state, bmm_chunk and
 * chunk_scan run on the tensor cores with split-bf16 operands for fp32 inputs of a
 * supported shape (ssd_set_fp32_stage_path) and on the CUDA cores otherwise.  No reference
 * counterpart: introspection for callers that size graphs or report which path ran. */
int ssd_combined_uses_tensor_cores(const ssd_fwd_params_t* p);

/* Number of kernel launches one ssd_combined_fwd call enqueues for these params.
 * No reference counterpart (introspection). */
int ssd_combined_num_launches(const ssd_fwd_params_t* p);

/* Combined SSD forward.
 * Replaces mamba_chunk_scan_combined_fwd (src/mamba2_jax/kernels/ssd_combined.py:46-203)
 * and, as its fallback target, mamba_chunk_scan_combined_naive
 * (src/mamba2_jax/ops/ssd_naive.py:325-397). */
int ssd_combined_fwd(const ssd_fwd_params_t* p, void* workspace, size_t workspace_bytes,
                     ssd_stream_t stream);

/* Size of the static scratch ssd_combined_fwd_noalloc uses on each GPU (16 MiB). */
#define SSD_NOALLOC_SCRATCH_BYTES (16 << 20)

/* Combined SSD forward for callers that cannot allocate device memory (no workspace slot,
 * or cudaMalloc not allowed where they run).  No counterpart in the reference: it is
 * ssd_combined_fwd with its scratch in a library-owned static device array of
 * SSD_NOALLOC_SCRATCH_BYTES per GPU, reserved once this code is loaded on that GPU (at the
 * latest by the first call there) and held until process exit.
 * Returns SSD_ERR_WORKSPACE when ssd_combined_workspace_bytes(p) exceeds that size.
 * The first call on a device resolves the array's address (cudaGetSymbolAddress); make it
 * before any stream capture.  All calls on a device share the array, so calls that overlap
 * on the GPU race; calls ordered on one stream are safe.  Allocates nothing. */
int ssd_combined_fwd_noalloc(const ssd_fwd_params_t* p, ssd_stream_t stream);

/* Stage 1.  Replaces chunk_cumsum_fwd (src/mamba2_jax/kernels/chunk_cumsum_fwd.py:288-302,
 * :194-235).  dt (b,L,H) -> dA_cumsum, dt_out (b,H,nc,Q) float32.  Padded tail
 * positions (>= L) get dt_out = 0, as the kernel path does (:228-231). */
int ssd_chunk_cumsum_fwd(const void* dt, int32_t dt_dtype, const float* A, const float* dt_bias,
                         int32_t dt_softplus, float dt_min, float dt_max,
                         int64_t batch, int64_t seqlen, int64_t nheads, int64_t chunk_size,
                         float* dA_cumsum, float* dt_out, ssd_stream_t stream);

/* Stage 2.  Replaces chunk_state_fwd (src/mamba2_jax/kernels/chunk_state_fwd.py:424-441,
 * preprocess :194-304).  states (b,nc,H,P,N) float32. */
int ssd_chunk_state_fwd(const void* x, const void* B, int32_t dtype,
                        const float* dt_out, const float* dA_cumsum, const int32_t* seq_idx,
                        int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                        int64_t ngroups, int64_t dstate, int64_t chunk_size,
                        float* states, ssd_stream_t stream);

/* Stage 3.  Replaces state_passing_fwd (src/mamba2_jax/kernels/state_passing_fwd.py:348-363,
 * :158-341).  states (b,nc,H,dim) float32; dA_chunk_cumsum is read at
 * dA_chunk[(bi*H + h)*stride_bh + c*stride_c] (for a (b,H,nc) array: stride_bh = nc,
 * stride_c = 1).  out (b,nc,H,dim) in out_dtype (may alias states), final (b,H,dim) f32.
 * seq_idx (b,seqlen) needs chunk_size. */
int ssd_state_passing_fwd(const float* states, const float* dA_chunk, int64_t stride_bh,
                          int64_t stride_c, const float* initial_states, const int32_t* seq_idx,
                          int64_t batch, int64_t nchunks, int64_t nheads, int64_t dim,
                          int64_t seqlen, int64_t chunk_size,
                          void* out, int32_t out_dtype, float* final_states,
                          ssd_stream_t stream);

/* Stage 4.  Replaces bmm_chunk_fwd (src/mamba2_jax/kernels/bmm_chunk_fwd.py:381-400,
 * :293-374).  out[b,c,g,m,n] = sum_k a[b,cQ+m,g,k] * b[b,cQ+n,g,k], (b,nc,G,Q,Q) f32;
 * seq_idx mask and optional causal (lower-triangular) mask. */
int ssd_bmm_chunk_fwd(const void* a, const void* b, int32_t dtype, const int32_t* seq_idx,
                      int32_t causal, int64_t batch, int64_t seqlen, int64_t ngroups,
                      int64_t k, int64_t chunk_size, float* out, ssd_stream_t stream);

/* Stage 5.  Replaces chunk_scan_fwd (src/mamba2_jax/kernels/chunk_scan_fwd.py:579-600,
 * :482-572).  cb (b,nc,G,Q,Q) f32; states = passed states (b,nc,H,P,N) in states_dtype.
 * out / out_x (b,L,H,P) f32. */
int ssd_chunk_scan_fwd(const float* cb, const void* x, int32_t dtype, const float* dt_out,
                       const float* dA_cumsum, const void* C, const void* states,
                       int32_t states_dtype, const float* D, int32_t D_ndim, const void* z,
                       const int32_t* seq_idx,
                       int64_t batch, int64_t seqlen, int64_t nheads, int64_t headdim,
                       int64_t ngroups, int64_t dstate, int64_t chunk_size,
                       float* out, float* out_x, ssd_stream_t stream);

/* Varlen final states.  Replaces chunk_state_varlen_mosaic
 * (src/mamba2_jax/kernels/chunk_state_fwd.py:448-597).  B (T,G,N), x (T,H,P) in dtype;
 * dt_out, dA_cumsum (H,nc,Q); chunk_states = passed states (nc,H,P,N) in states_dtype;
 * out (num_seqs,H,P,N) f32. */
int ssd_chunk_state_varlen_fwd(const void* B, const void* x, int32_t dtype,
                               const float* dt_out, const float* dA_cumsum,
                               const int32_t* cu_seqlens, int32_t num_seqs,
                               const void* chunk_states, int32_t states_dtype,
                               int64_t total_seqlen, int64_t nheads, int64_t headdim,
                               int64_t ngroups, int64_t dstate, int64_t chunk_size,
                               float* out, ssd_stream_t stream);

/* Parameters of the single-token decode step. */
typedef struct ssu_params {
  int64_t batch, nheads, headdim, ngroups, dstate;
  int32_t dtype;          /* ssd_dtype_t of x, z, B, C */
  int32_t dt_dtype;       /* ssd_dtype_t of dt */
  int32_t dt_ndim;        /* 2: dt (b,H); 3: dt (b,H,P) */
  int32_t A_ndim;         /* 1: A (H,); 3: A (H,P,N) */
  int32_t D_ndim;         /* 0, 1 (H,) or 2 (H,P) */
  int32_t dt_bias_ndim;   /* 0, 1 (H,) or 2 (H,P) */
  int32_t dt_softplus;    /* nonzero: dt <- log(1 + exp(dt)) after bias */
  int32_t reserved;
  float* state;           /* (b,H,P,N) f32, updated IN PLACE */
  const void* x;          /* (b,H,P) */
  const void* dt;
  const float* A;
  const void* B;          /* (b,G,N) */
  const void* C;          /* (b,G,N) */
  const float* D;
  const void* z;          /* (b,H,P) or NULL */
  const float* dt_bias;
  float* out;             /* (b,H,P) f32 */
} ssu_params_t;

/* Decode step.  Replaces selective_state_update
 * (src/mamba2_jax/ops/selective_state_update.py:22-123); the state is updated in place
 * instead of returned as a new array. */
int ssd_selective_state_update(const ssu_params_t* p, ssd_stream_t stream);

/* Causal depthwise conv1d over time (the step before the SSD in a Mamba2 layer).
 * x and out are logically (batch, dim, seqlen), addressed by element strides, so the
 * channels-last (batch, seqlen, dim) activations of the layer are read without a copy.
 * out[b,d,t] = act(bias[d] + sum_j weight[d,j] * xm[b,d,t-(width-1)+j]) with xm = 0
 * before t = 0, act = SiLU or identity.  With seq_idx, xm[b,d,t] = x[b,d,t] unless one of
 * positions t+1 .. t+width-1 (inside the sequence) starts a new sequence id, in which case
 * it is 0: the masking of causal_conv1d.py:143-193, which also drops those inputs from
 * the outputs of their own sequence.  Arithmetic is f32; out is rounded once. */
typedef struct ssd_conv1d_params {
  int64_t batch, dim, seqlen;
  int64_t x_stride_b, x_stride_d, x_stride_t;       /* element strides of x */
  int64_t out_stride_b, out_stride_d, out_stride_t; /* element strides of out */
  int32_t width;          /* kernel_size, 1 .. 8 */
  int32_t dtype;          /* ssd_dtype_t of x */
  int32_t out_dtype;      /* ssd_dtype_t of out */
  int32_t silu;           /* nonzero: activation "silu" */
  const void* x;
  const void* weight;     /* (dim, width) contiguous, f32 or bf16 (weight_dtype) */
  const void* bias;       /* (dim,) f32 or bf16 (bias_dtype), or NULL */
  const int32_t* seq_idx; /* (batch, seqlen) contiguous, or NULL */
  void* out;              /* must not overlap x */
  int32_t weight_dtype;   /* ssd_dtype_t of weight (0 = f32) */
  int32_t bias_dtype;     /* ssd_dtype_t of bias (0 = f32) */
} ssd_conv1d_params_t;

/* Replaces causal_conv1d (src/mamba2_jax/ops/causal_conv1d.py:18-85). */
int ssd_causal_conv1d_fwd(const ssd_conv1d_params_t* p, ssd_stream_t stream);

/* One decode step of the conv: conv_state (batch, dim, width), width contiguous, is shifted
 * left by one with x_new (batch, dim) written into its last slot, IN PLACE; then
 * out[b,d] = act(bias[d] + sum_j weight[d,j] * conv_state[b,d,j]). */
typedef struct ssd_conv1d_update_params {
  int64_t batch, dim;
  int64_t state_stride_b, state_stride_d;  /* element strides of conv_state (width: 1) */
  int32_t width;          /* 1 .. 8 */
  int32_t x_dtype;        /* ssd_dtype_t of x_new */
  int32_t state_dtype;    /* ssd_dtype_t of conv_state */
  int32_t out_dtype;      /* ssd_dtype_t of out */
  int32_t silu;
  int32_t reserved;
  const void* x_new;      /* (batch, dim) contiguous */
  void* conv_state;
  const void* weight;     /* (dim, width) contiguous, f32 or bf16 (weight_dtype) */
  const void* bias;       /* (dim,) f32 or bf16 (bias_dtype), or NULL */
  void* out;              /* (batch, dim) contiguous */
  int32_t weight_dtype;   /* ssd_dtype_t of weight (0 = f32) */
  int32_t bias_dtype;     /* ssd_dtype_t of bias (0 = f32) */
} ssd_conv1d_update_params_t;

/* Replaces causal_conv1d_update (src/mamba2_jax/ops/causal_conv1d.py:88-139); the state
 * is updated in place instead of returned as a new array. */
int ssd_causal_conv1d_update(const ssd_conv1d_update_params_t* p, ssd_stream_t stream);

/* Gated RMSNorm over groups of the last axis (the step after the SSD in a Mamba2 layer).
 * x, z and out are logically (rows, hidden): the last axis is contiguous, rows are addressed
 * by an element stride.  For each row and each group of group_size values (hidden must be a
 * multiple of group_size):
 *   norm_before_gate != 0:  out = x / sqrt(mean(x^2) + eps) * weight * silu(z)
 *   norm_before_gate == 0:  v = x * silu(z); out = v / sqrt(mean(v^2) + eps) * weight
 * z may be NULL (no gate).  Arithmetic is f32 (IEEE sqrt and division); out is rounded once. */
typedef struct ssd_rms_norm_params {
  int64_t rows, hidden, group_size;
  int64_t x_stride_row, z_stride_row, out_stride_row;  /* element strides between rows */
  int32_t x_dtype, z_dtype, weight_dtype, out_dtype;   /* ssd_dtype_t each */
  int32_t norm_before_gate;
  float eps;
  const void* x;
  const void* z;          /* or NULL */
  const void* weight;     /* (hidden,) contiguous */
  void* out;              /* must not partially overlap x or z (out == x is allowed) */
} ssd_rms_norm_params_t;

/* Replaces rms_norm_gated (src/mamba2_jax/ops/rms_norm.py:15-92), called by the Mamba2
 * mixer at src/mamba2_jax/modules/mamba2.py:401-406 with group_size = d_ssm / ngroups. */
int ssd_rms_norm_gated(const ssd_rms_norm_params_t* p, ssd_stream_t stream);

/* Sequence-parallel decay fix-up.  A rank that ran its token segment (b, L) of a longer
 * sequence from a zero initial state adds the state S entering the segment, received from
 * the ranks before it, in place:
 *   out[b,t,h,:] += exp(dA(t)) * (C[b,t,g,:] . S[b,h,:,:]^T) * silu(z[b,t,h,:])  (z optional)
 *     for t < carried_len[b] (the tokens of the sequence carried into the segment; NULL
 *     means all L tokens),
 *   final_states[b,h] += exp(dA(L-1)) * S[b,h]   when carried_len[b] >= L (optional),
 * where dA(t) is the segment-wide cumulative sum of dt*A, read from the segment's
 * chunk_cumsum output (b,H,nc,Q).  headdim must be a multiple of 4. */
typedef struct ssd_sp_fixup_params {
  int64_t batch, seqlen, nheads, headdim, ngroups, dstate, chunk_size;
  int32_t dtype;              /* ssd_dtype_t of C and z */
  int32_t reserved;
  const void* C;              /* (b,L,G,N) */
  const void* z;              /* (b,L,H,P) or NULL */
  const float* dA_cumsum;     /* (b,H,nc,Q) within-chunk cumsum of dt*A */
  const float* state_in;      /* (b,H,P,N) */
  const int32_t* carried_len; /* (b,) or NULL */
  float* out;                 /* (b,L,H,P), updated in place */
  float* final_states;        /* (b,H,P,N), updated in place, or NULL */
} ssd_sp_fixup_params_t;

/* The decay fix-up of the optional sequence-parallel mode.  The reference has no
 * sequence parallelism; this applies the state-passing recurrence of
 * src/mamba2_jax/kernels/state_passing_fwd.py:108-151 and the inter-chunk term of
 * src/mamba2_jax/kernels/chunk_scan_fwd.py:108-232 across a segment boundary. */
int ssd_sp_state_fixup(const ssd_sp_fixup_params_t* p, ssd_stream_t stream);

/* Thread-local description of the last failure on this host thread ("" if none). */
const char* ssd_last_error(void);

/* SSD_B200_ABI_VERSION of the loaded library. */
int ssd_abi_version(void);

/* Process-wide choice of the kernels behind chunk_state, bmm_chunk and chunk_scan for fp32
 * inputs, in ssd_combined_fwd's staged pipeline and in the three stage entry points:
 * 0 (default) = tcgen05 MMAs on split-bf16 operands (hi + lo, three products each, fp32
 * accumulation) where the shape allows (headdim a multiple of 32 up to 256, dstate a
 * multiple of 16, 16-byte aligned rows), 1 = fp32 FFMA on the CUDA cores.  Returns the
 * previous choice, or -1 (and ssd_last_error says why) for any other value.  No reference counterpart (its stages are
 * Pallas kernels with one operand precision). */
int ssd_set_fp32_stage_path(int32_t path);

#ifdef __cplusplus
}
#endif

#endif /* SSD_B200_H_ */
