// C ABI entry points (include/ssd_b200.h): argument validation, workspace carving and
// stage orchestration.  No entry point allocates device memory or blocks the host.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "ssd_kernels.h"
#include "ssd_tc.h"
#include "ssd_x3.h"
#include <atomic>

namespace {
using ssd::bf16;

thread_local char g_err[512] = "";

// Stage kernels for fp32 inputs: 0 = tensor cores (split-bf16) where the shape allows,
// 1 = CUDA cores always (ssd_set_fp32_stage_path).
std::atomic<int> g_fp32_stage_path{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return SSD_OK;
  return fail(SSD_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

bool dtype_ok(int d) { return d == SSD_DTYPE_F32 || d == SSD_DTYPE_BF16; }

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Every workspace starts with this region: the device status word (first 4 bytes), cleared
// on the stream by each ssd_combined_fwd call and set by a bounded wait that gives up.
constexpr size_t STATUS_BYTES = 256;

int check_dims(int64_t b, int64_t L, int64_t H, int64_t P, int64_t G, int64_t N, int64_t Q) {
  if (b <= 0 || L <= 0 || H <= 0 || P <= 0 || G <= 0 || N <= 0 || Q <= 0)
    return fail(SSD_ERR_INVALID_ARG, "dims must be positive (b=%lld L=%lld H=%lld P=%lld G=%lld N=%lld Q=%lld)",
                (long long)b, (long long)L, (long long)H, (long long)P, (long long)G, (long long)N, (long long)Q);
  if (H % G != 0) return fail(SSD_ERR_INVALID_ARG, "nheads (%lld) must be a multiple of ngroups (%lld)", (long long)H, (long long)G);
  if (Q % 32 != 0 || Q > 256)
    return fail(SSD_ERR_UNSUPPORTED, "chunk_size %lld unsupported (need a multiple of 32, <= 256)", (long long)Q);
  return SSD_OK;
}

struct Workspace {
  size_t dA, dt, states, passed_lp, cb, total;
};

Workspace plan_ws(const ssd_fwd_params_t* p) {
  const int64_t nc = (p->seqlen + p->chunk_size - 1) / p->chunk_size;
  const size_t cs = (size_t)p->batch * p->nheads * nc * p->chunk_size * sizeof(float);
  const size_t st = (size_t)p->batch * nc * p->nheads * p->headdim * p->dstate * sizeof(float);
  const size_t cb = (size_t)p->batch * nc * p->ngroups * p->chunk_size * p->chunk_size * sizeof(float);
  Workspace w;
  size_t off = STATUS_BYTES;   // the status word leads every workspace
  w.dA = off; off += align256(cs);
  w.dt = off; off += align256(cs);
  w.states = off; off += align256(st);
  w.passed_lp = off;
  if ((p->flags & SSD_FLAG_ROUND_STATES) && p->dtype == SSD_DTYPE_BF16) off += align256(st / 2);
  w.cb = off; off += align256(cb);
  w.total = off;
  return w;
}

int validate_fwd(const ssd_fwd_params_t* p) {
  if (!p) return fail(SSD_ERR_INVALID_ARG, "params is NULL");
  int s = check_dims(p->batch, p->seqlen, p->nheads, p->headdim, p->ngroups, p->dstate, p->chunk_size);
  if (s) return s;
  if (!dtype_ok(p->dtype) || !dtype_ok(p->dt_dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (!p->x || !p->dt || !p->A || !p->B || !p->C || !p->out)
    return fail(SSD_ERR_INVALID_ARG, "x, dt, A, B, C and out are required");
  if (p->D_ndim < 0 || p->D_ndim > 2 || (p->D_ndim && !p->D)) return fail(SSD_ERR_INVALID_ARG, "bad D_ndim / D");
  if (p->out_x && !p->z) return fail(SSD_ERR_INVALID_ARG, "out_x requires z");
  if (p->varlen_states) {
    if (!p->cu_seqlens || p->num_seqs <= 0) return fail(SSD_ERR_INVALID_ARG, "varlen_states requires cu_seqlens and num_seqs > 0");
    if (p->batch != 1) return fail(SSD_ERR_INVALID_ARG, "cu_seqlens for varlen states is only supported with batch=1");
  }
  if (std::isnan(p->dt_min) || std::isnan(p->dt_max) || p->dt_min > p->dt_max)
    return fail(SSD_ERR_INVALID_ARG, "bad dt_limit");
  return SSD_OK;
}

// fp32 -> bf16 copies of x, B, C (and z) for SSD_FLAG_BF16_MMA: one launch, blockIdx.y picks
// the tensor, each thread converts 4 consecutive elements per step.
struct ConvJob {
  const float* src[4];
  bf16* dst[4];
  int64_t n[4];
};

__global__ void __launch_bounds__(256) to_bf16_kernel(const __grid_constant__ ConvJob j) {
  const int t = blockIdx.y;
  const float* __restrict__ src = j.src[t];
  bf16* __restrict__ dst = j.dst[t];
  const int64_t n = j.n[t];
  if (!src) return;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 4;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 4 <= n && ((reinterpret_cast<uintptr_t>(src + i) & 15) == 0)) {
      const float4 v = *reinterpret_cast<const float4*>(src + i);
      __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
      reinterpret_cast<__nv_bfloat162*>(dst + i)[0] = a;
      reinterpret_cast<__nv_bfloat162*>(dst + i)[1] = b;
    } else {
      for (int64_t k = i; k < i + 4 && k < n; ++k) dst[k] = __float2bfloat16_rn(src[k]);
    }
  }
}

// SSD_FLAG_BF16_MMA: the bf16 copies sit at the head of the workspace (256-byte aligned
// each); `q` is the params with the inputs redirected there and dtype bf16.
struct Bf16Plan {
  bool on;
  ssd_fwd_params_t q;
  size_t off_x, off_b, off_c, off_z, bytes;
};

Bf16Plan plan_bf16(const ssd_fwd_params_t* p, const void* workspace) {
  Bf16Plan r;
  memset(&r, 0, sizeof(r));
  if (!(p->flags & SSD_FLAG_BF16_MMA) || p->dtype != SSD_DTYPE_F32 || (p->flags & SSD_FLAG_FORCE_SIMT)) return r;
  const size_t nx = (size_t)p->batch * p->seqlen * p->nheads * p->headdim;
  const size_t nb = (size_t)p->batch * p->seqlen * p->ngroups * p->dstate;
  size_t off = STATUS_BYTES;
  r.off_x = off; off += align256(nx * 2);
  r.off_b = off; off += align256(nb * 2);
  r.off_c = off; off += align256(nb * 2);
  r.off_z = off; if (p->z) off += align256(nx * 2);
  r.bytes = off;
  r.q = *p;
  r.q.dtype = SSD_DTYPE_BF16;
  r.q.flags &= ~SSD_FLAG_BF16_MMA;
  // for sizing without a workspace, any 256-aligned address stands in
  const char* base = workspace ? (const char*)workspace : reinterpret_cast<const char*>(uintptr_t(256));
  r.q.x = base + r.off_x;
  r.q.B = base + r.off_b;
  r.q.C = base + r.off_c;
  r.q.z = p->z ? base + r.off_z : nullptr;
  r.on = ssd::tc_supported(&r.q);
  return r;
}

}  // namespace

namespace ssd {
void set_last_error(const char* msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }
}  // namespace ssd

extern "C" {

const char* ssd_last_error(void) { return g_err; }

int ssd_abi_version(void) { return SSD_B200_ABI_VERSION; }

int ssd_set_fp32_stage_path(int32_t path) {
  g_err[0] = 0;
  if (path != 0 && path != 1) {
    fail(SSD_ERR_INVALID_ARG, "path must be 0 (tensor cores) or 1 (CUDA cores)");
    return -1;
  }
  return g_fp32_stage_path.exchange(path);
}

size_t ssd_combined_workspace_bytes(const ssd_fwd_params_t* p) {
  if (!p) return 0;
  {
    char keep[sizeof(g_err)];   // sizing is a query: leave the last error as it was
    memcpy(keep, g_err, sizeof(g_err));
    const int s = validate_fwd(p);
    memcpy(g_err, keep, sizeof(g_err));
    if (s) return 0;
  }
  const Bf16Plan bp = plan_bf16(p, nullptr);
  if (bp.on) return bp.bytes + ssd::tc_workspace_bytes(&bp.q);
  const size_t tc = STATUS_BYTES + ssd::tc_workspace_bytes(p);
  const size_t simt = plan_ws(p).total;
  return tc > simt ? tc : simt;
}

int ssd_status_copy_async(const void* workspace, uint32_t* dst, ssd_stream_t stream) {
  g_err[0] = 0;
  if (!workspace || !dst) return fail(SSD_ERR_INVALID_ARG, "workspace and dst are required");
  return cuda_status(cudaMemcpyAsync(dst, workspace, sizeof(uint32_t), cudaMemcpyDefault, (cudaStream_t)stream),
                     "cudaMemcpyAsync of the status word");
}

int ssd_status_decode(uint32_t word) {
  g_err[0] = 0;
  if (word == 0) return SSD_OK;
  if ((word & ~0xffu) == 0x100u)
    return fail(SSD_ERR_TIMEOUT, "a bounded wait of the fused kernel gave up (barrier %u); the launch's outputs "
                "are incomplete", word & 0xffu);
  if ((word & ~0xffu) == 0x300u)
    return fail(SSD_ERR_INVALID_ARG, "debug build: the fused kernel computed an out-of-range index (site %u) and "
                "skipped that access", word & 0xffu);
  if (word == 0x200u)
    return fail(SSD_ERR_ALIGNMENT, "the fused kernel's dynamic shared memory window was not 1024-byte alignable; "
                "the launch did no work");
  return fail(SSD_ERR_CUDA, "unknown device status word 0x%x", word);
}

int ssd_combined_uses_tensor_cores(const ssd_fwd_params_t* p) {
  if (!p || validate_fwd(p) != SSD_OK || (p->flags & SSD_FLAG_FORCE_SIMT)) return 0;
  return (plan_bf16(p, nullptr).on || ssd::tc_supported(p)) ? 1 : 0;
}

int ssd_combined_num_launches(const ssd_fwd_params_t* p) {
  if (!p || validate_fwd(p) != SSD_OK) return 0;
  const Bf16Plan bp = plan_bf16(p, nullptr);
  if (bp.on) return 1 + ssd::tc_num_launches(&bp.q);
  if (ssd_combined_uses_tensor_cores(p)) return ssd::tc_num_launches(p);
  return 5 + (p->varlen_states ? 1 : 0);
}

int ssd_combined_fwd(const ssd_fwd_params_t* p, void* workspace, size_t workspace_bytes,
                     ssd_stream_t stream_) {
  g_err[0] = 0;
  int s = validate_fwd(p);
  if (s) return s;
  cudaStream_t st = (cudaStream_t)stream_;
  const size_t need = ssd_combined_workspace_bytes(p);
  if (!workspace || workspace_bytes < need)
    return fail(SSD_ERR_WORKSPACE, "workspace of %zu bytes required, %zu given", need, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(SSD_ERR_ALIGNMENT, "workspace must be 256-byte aligned");
  unsigned* status = (unsigned*)workspace;
  if ((s = cuda_status(cudaMemsetAsync(status, 0, sizeof(unsigned), st), "cudaMemsetAsync of the status word")))
    return s;

  // fp32 inputs with bf16 MMA operands: convert, then the tensor-core pipeline
  const Bf16Plan bp = plan_bf16(p, workspace);
  if (bp.on) {
    char* ws = (char*)workspace;
    ConvJob j;
    memset(&j, 0, sizeof(j));
    const int64_t nx = p->batch * p->seqlen * p->nheads * p->headdim;
    const int64_t nb = p->batch * p->seqlen * p->ngroups * p->dstate;
    j.src[0] = (const float*)p->x; j.dst[0] = (bf16*)(ws + bp.off_x); j.n[0] = nx;
    j.src[1] = (const float*)p->B; j.dst[1] = (bf16*)(ws + bp.off_b); j.n[1] = nb;
    j.src[2] = (const float*)p->C; j.dst[2] = (bf16*)(ws + bp.off_c); j.n[2] = nb;
    if (p->z) { j.src[3] = (const float*)p->z; j.dst[3] = (bf16*)(ws + bp.off_z); j.n[3] = nx; }
    const int64_t most = nx > nb ? nx : nb;
    const unsigned gx = (unsigned)std::min<int64_t>((most / 4 + 255) / 256, 4 * 148);
    to_bf16_kernel<<<dim3(gx, 4), 256, 0, st>>>(j);
    if ((s = cuda_status(cudaGetLastError(), "to_bf16_kernel"))) return s;
    return ssd::tc_combined_fwd(&bp.q, status, ws + bp.bytes, st);
  }

  // Tensor-core pipeline for bf16 inputs when the shape is one it covers.
  if (!(p->flags & SSD_FLAG_FORCE_SIMT) && ssd::tc_supported(p)) {
    return ssd::tc_combined_fwd(p, status, (char*)workspace + STATUS_BYTES, st);
  }

  const Workspace w = plan_ws(p);
  char* ws = (char*)workspace;
  const int64_t b = p->batch, L = p->seqlen, H = p->nheads, P = p->headdim, G = p->ngroups,
                N = p->dstate, Q = p->chunk_size, nc = (L + Q - 1) / Q;
  float* dA = p->dA_cumsum ? p->dA_cumsum : (float*)(ws + w.dA);
  float* dt = p->dt_out ? p->dt_out : (float*)(ws + w.dt);
  float* states = (float*)(ws + w.states);
  float* cb = (float*)(ws + w.cb);
  const bool lp = (p->flags & SSD_FLAG_ROUND_STATES) && p->dtype == SSD_DTYPE_BF16;
  void* passed = lp ? (void*)(ws + w.passed_lp) : (void*)states;
  const int passed_dtype = lp ? SSD_DTYPE_BF16 : SSD_DTYPE_F32;

  if ((s = cuda_status(ssd::launch_chunk_cumsum(p->dt, p->dt_dtype, p->A, p->dt_bias, p->dt_softplus,
                                                p->dt_min, p->dt_max, b, L, H, Q, dA, dt, st), "chunk_cumsum")))
    return s;
  const bool x3 = !(p->flags & SSD_FLAG_FORCE_SIMT) && g_fp32_stage_path.load() == 0;
  if (x3 && ssd::x3_chunk_state_supported(p->x, p->B, p->dtype, P, N, Q))
    s = cuda_status(ssd::launch_x3_chunk_state((const float*)p->x, (const float*)p->B, dt, dA, p->seq_idx, b, L, H,
                                               P, G, N, Q, states, status, st), "x3_chunk_state");
  else
    s = cuda_status(ssd::launch_chunk_state(p->x, p->B, p->dtype, dt, dA, p->seq_idx, b, L, H, P, G, N, Q,
                                            states, st), "chunk_state");
  if (s) return s;
  if ((s = cuda_status(ssd::launch_state_passing(states, dA + (Q - 1), nc * Q, Q, p->initial_states, p->seq_idx,
                                                 b, nc, H, P * N, L, Q, passed, passed_dtype,
                                                 p->final_states, st), "state_passing")))
    return s;
  if (x3 && ssd::x3_bmm_supported(p->C, p->B, p->dtype, N, Q))
    // causal: chunk_scan reads CB only at k <= m, so tiles above the diagonal need no MMAs
    s = cuda_status(ssd::launch_x3_bmm((const float*)p->C, (const float*)p->B, p->seq_idx, 1, b, L, G, N, Q, cb,
                                       status, st), "x3_bmm_chunk");
  else
    s = cuda_status(ssd::launch_bmm_chunk(p->C, p->B, p->dtype, p->seq_idx, 0, b, L, G, N, Q, cb, st), "bmm_chunk");
  if (s) return s;
  if (x3 && ssd::x3_chunk_scan_supported(p->x, p->C, p->z, cb, passed, p->dtype, passed_dtype, P, N, Q, p->out,
                                         p->out_x))
    s = cuda_status(ssd::launch_x3_chunk_scan(cb, (const float*)p->x, dt, dA, (const float*)p->C,
                                              (const float*)passed, p->D, p->D_ndim, (const float*)p->z,
                                              p->seq_idx, b, L, H, P, G, N, Q, p->out, p->out_x, status, st),
                    "x3_chunk_scan");
  else
    s = cuda_status(ssd::launch_chunk_scan(cb, p->x, p->dtype, dt, dA, p->C, passed, passed_dtype, p->D, p->D_ndim,
                                           p->z, p->seq_idx, b, L, H, P, G, N, Q, p->out, p->out_x, st),
                    "chunk_scan");
  if (s) return s;
  if (p->varlen_states) {
    if ((s = cuda_status(ssd::launch_chunk_state_varlen(p->B, p->x, p->dtype, dt, dA, p->cu_seqlens, p->num_seqs,
                                                        passed, passed_dtype, L, H, P, G, N, Q,
                                                        p->varlen_states, st), "chunk_state_varlen")))
      return s;
  }
  return SSD_OK;
}

int ssd_chunk_cumsum_fwd(const void* dt, int32_t dt_dtype, const float* A, const float* dt_bias,
                         int32_t dt_softplus, float dt_min, float dt_max, int64_t batch, int64_t seqlen,
                         int64_t nheads, int64_t chunk_size, float* dA_cumsum, float* dt_out,
                         ssd_stream_t stream) {
  g_err[0] = 0;
  int s = check_dims(batch, seqlen, nheads, 1, 1, 1, chunk_size);
  if (s) return s;
  if (!dt || !A || !dA_cumsum || !dt_out) return fail(SSD_ERR_INVALID_ARG, "null pointer");
  if (!dtype_ok(dt_dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  return cuda_status(ssd::launch_chunk_cumsum(dt, dt_dtype, A, dt_bias, dt_softplus, dt_min, dt_max, batch,
                                              seqlen, nheads, chunk_size, dA_cumsum, dt_out,
                                              (cudaStream_t)stream), "chunk_cumsum");
}

int ssd_chunk_state_fwd(const void* x, const void* B, int32_t dtype, const float* dt_out,
                        const float* dA_cumsum, const int32_t* seq_idx, int64_t batch, int64_t seqlen,
                        int64_t nheads, int64_t headdim, int64_t ngroups, int64_t dstate,
                        int64_t chunk_size, float* states, ssd_stream_t stream) {
  g_err[0] = 0;
  int s = check_dims(batch, seqlen, nheads, headdim, ngroups, dstate, chunk_size);
  if (s) return s;
  if (!x || !B || !dt_out || !dA_cumsum || !states) return fail(SSD_ERR_INVALID_ARG, "null pointer");
  if (!dtype_ok(dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (g_fp32_stage_path.load() == 0 && ssd::x3_chunk_state_supported(x, B, dtype, headdim, dstate, chunk_size))
    return cuda_status(ssd::launch_x3_chunk_state((const float*)x, (const float*)B, dt_out, dA_cumsum, seq_idx, batch,
                                                  seqlen, nheads, headdim, ngroups, dstate, chunk_size, states,
                                                  nullptr, (cudaStream_t)stream), "x3_chunk_state");
  return cuda_status(ssd::launch_chunk_state(x, B, dtype, dt_out, dA_cumsum, seq_idx, batch, seqlen, nheads,
                                             headdim, ngroups, dstate, chunk_size, states,
                                             (cudaStream_t)stream), "chunk_state");
}

int ssd_state_passing_fwd(const float* states, const float* dA_chunk, int64_t stride_bh, int64_t stride_c,
                          const float* initial_states, const int32_t* seq_idx, int64_t batch,
                          int64_t nchunks, int64_t nheads, int64_t dim, int64_t seqlen, int64_t chunk_size,
                          void* out, int32_t out_dtype, float* final_states, ssd_stream_t stream) {
  g_err[0] = 0;
  if (batch <= 0 || nchunks <= 0 || nheads <= 0 || dim <= 0)
    return fail(SSD_ERR_INVALID_ARG, "dims must be positive");
  if (!states || !dA_chunk || !out) return fail(SSD_ERR_INVALID_ARG, "null pointer");
  if (!dtype_ok(out_dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (seq_idx) {
    if (chunk_size <= 0 || seqlen <= 0) return fail(SSD_ERR_INVALID_ARG, "seq_idx requires chunk_size and seqlen");
    if ((seqlen + chunk_size - 1) / chunk_size != nchunks)
      return fail(SSD_ERR_INVALID_ARG, "ceil(seqlen/chunk_size) != nchunks");
  }
  if (out_dtype != SSD_DTYPE_F32 && (const void*)out == (const void*)states)
    return fail(SSD_ERR_INVALID_ARG, "out may alias states only for float32 output");
  return cuda_status(ssd::launch_state_passing(states, dA_chunk, stride_bh, stride_c, initial_states, seq_idx,
                                               batch, nchunks, nheads, dim, seqlen, chunk_size, out, out_dtype,
                                               final_states, (cudaStream_t)stream), "state_passing");
}

int ssd_bmm_chunk_fwd(const void* a, const void* b, int32_t dtype, const int32_t* seq_idx, int32_t causal,
                      int64_t batch, int64_t seqlen, int64_t ngroups, int64_t k, int64_t chunk_size,
                      float* out, ssd_stream_t stream) {
  g_err[0] = 0;
  int s = check_dims(batch, seqlen, ngroups, 1, ngroups, k, chunk_size);
  if (s) return s;
  if (!a || !b || !out) return fail(SSD_ERR_INVALID_ARG, "null pointer");
  if (!dtype_ok(dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (g_fp32_stage_path.load() == 0 && ssd::x3_bmm_supported(a, b, dtype, k, chunk_size))
    return cuda_status(ssd::launch_x3_bmm((const float*)a, (const float*)b, seq_idx, causal, batch, seqlen, ngroups,
                                          k, chunk_size, out, nullptr, (cudaStream_t)stream), "x3_bmm_chunk");
  return cuda_status(ssd::launch_bmm_chunk(a, b, dtype, seq_idx, causal, batch, seqlen, ngroups, k, chunk_size,
                                           out, (cudaStream_t)stream), "bmm_chunk");
}

int ssd_chunk_scan_fwd(const float* cb, const void* x, int32_t dtype, const float* dt_out,
                       const float* dA_cumsum, const void* C, const void* states, int32_t states_dtype,
                       const float* D, int32_t D_ndim, const void* z, const int32_t* seq_idx, int64_t batch,
                       int64_t seqlen, int64_t nheads, int64_t headdim, int64_t ngroups, int64_t dstate,
                       int64_t chunk_size, float* out, float* out_x, ssd_stream_t stream) {
  g_err[0] = 0;
  int s = check_dims(batch, seqlen, nheads, headdim, ngroups, dstate, chunk_size);
  if (s) return s;
  if (!cb || !x || !dt_out || !dA_cumsum || !C || !states || !out) return fail(SSD_ERR_INVALID_ARG, "null pointer");
  if (!dtype_ok(dtype) || !dtype_ok(states_dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (D_ndim < 0 || D_ndim > 2 || (D_ndim && !D)) return fail(SSD_ERR_INVALID_ARG, "bad D_ndim / D");
  if (out_x && !z) return fail(SSD_ERR_INVALID_ARG, "out_x requires z");
  if (g_fp32_stage_path.load() == 0 &&
      ssd::x3_chunk_scan_supported(x, C, z, cb, states, dtype, states_dtype, headdim, dstate, chunk_size, out, out_x))
    return cuda_status(ssd::launch_x3_chunk_scan(cb, (const float*)x, dt_out, dA_cumsum, (const float*)C,
                                                 (const float*)states, D, D_ndim, (const float*)z, seq_idx, batch,
                                                 seqlen, nheads, headdim, ngroups, dstate, chunk_size, out, out_x,
                                                 nullptr, (cudaStream_t)stream), "x3_chunk_scan");
  return cuda_status(ssd::launch_chunk_scan(cb, x, dtype, dt_out, dA_cumsum, C, states, states_dtype, D, D_ndim,
                                            z, seq_idx, batch, seqlen, nheads, headdim, ngroups, dstate,
                                            chunk_size, out, out_x, (cudaStream_t)stream), "chunk_scan");
}

int ssd_chunk_state_varlen_fwd(const void* B, const void* x, int32_t dtype, const float* dt_out,
                               const float* dA_cumsum, const int32_t* cu_seqlens, int32_t num_seqs,
                               const void* chunk_states, int32_t states_dtype, int64_t total_seqlen,
                               int64_t nheads, int64_t headdim, int64_t ngroups, int64_t dstate,
                               int64_t chunk_size, float* out, ssd_stream_t stream) {
  g_err[0] = 0;
  int s = check_dims(1, total_seqlen, nheads, headdim, ngroups, dstate, chunk_size);
  if (s) return s;
  if (num_seqs <= 0) return fail(SSD_ERR_INVALID_ARG, "num_seqs must be positive");
  if (!B || !x || !dt_out || !dA_cumsum || !cu_seqlens || !chunk_states || !out)
    return fail(SSD_ERR_INVALID_ARG, "null pointer");
  if (!dtype_ok(dtype) || !dtype_ok(states_dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  return cuda_status(ssd::launch_chunk_state_varlen(B, x, dtype, dt_out, dA_cumsum, cu_seqlens, num_seqs,
                                                    chunk_states, states_dtype, total_seqlen, nheads, headdim,
                                                    ngroups, dstate, chunk_size, out, (cudaStream_t)stream),
                     "chunk_state_varlen");
}

int ssd_selective_state_update(const ssu_params_t* p, ssd_stream_t stream) {
  g_err[0] = 0;
  if (!p) return fail(SSD_ERR_INVALID_ARG, "params is NULL");
  if (p->batch <= 0 || p->nheads <= 0 || p->headdim <= 0 || p->ngroups <= 0 || p->dstate <= 0)
    return fail(SSD_ERR_INVALID_ARG, "dims must be positive");
  if (p->nheads % p->ngroups) return fail(SSD_ERR_INVALID_ARG, "nheads must be a multiple of ngroups");
  if (!dtype_ok(p->dtype) || !dtype_ok(p->dt_dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (!p->state || !p->x || !p->dt || !p->A || !p->B || !p->C || !p->out)
    return fail(SSD_ERR_INVALID_ARG, "state, x, dt, A, B, C and out are required");
  if (p->dt_ndim != 2 && p->dt_ndim != 3) return fail(SSD_ERR_INVALID_ARG, "dt_ndim must be 2 or 3");
  if (p->A_ndim != 1 && p->A_ndim != 3) return fail(SSD_ERR_INVALID_ARG, "A_ndim must be 1 or 3");
  if (p->D_ndim < 0 || p->D_ndim > 2 || (p->D_ndim && !p->D)) return fail(SSD_ERR_INVALID_ARG, "bad D_ndim / D");
  if (p->dt_bias && (p->dt_bias_ndim < 1 || p->dt_bias_ndim > 2)) return fail(SSD_ERR_INVALID_ARG, "bad dt_bias_ndim");
  if (p->dstate > 8192) return fail(SSD_ERR_UNSUPPORTED, "dstate > 8192 unsupported");
  return cuda_status(ssd::launch_ssu(p, (cudaStream_t)stream), "selective_state_update");
}

int ssd_causal_conv1d_fwd(const ssd_conv1d_params_t* p, ssd_stream_t stream) {
  g_err[0] = 0;
  if (!p) return fail(SSD_ERR_INVALID_ARG, "params is NULL");
  if (p->batch <= 0 || p->dim <= 0 || p->seqlen <= 0) return fail(SSD_ERR_INVALID_ARG, "dims must be positive");
  if (p->width < 1 || p->width > 8) return fail(SSD_ERR_UNSUPPORTED, "width must be 1..8");
  if (!dtype_ok(p->dtype) || !dtype_ok(p->out_dtype) || !dtype_ok(p->weight_dtype) || !dtype_ok(p->bias_dtype))
    return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (!p->x || !p->weight || !p->out) return fail(SSD_ERR_INVALID_ARG, "x, weight and out are required");
  if (p->x == p->out) return fail(SSD_ERR_INVALID_ARG, "out must not alias x");
  return cuda_status(ssd::launch_conv1d(p, (cudaStream_t)stream), "causal_conv1d");
}

int ssd_causal_conv1d_update(const ssd_conv1d_update_params_t* p, ssd_stream_t stream) {
  g_err[0] = 0;
  if (!p) return fail(SSD_ERR_INVALID_ARG, "params is NULL");
  if (p->batch <= 0 || p->dim <= 0) return fail(SSD_ERR_INVALID_ARG, "dims must be positive");
  if (p->width < 1 || p->width > 8) return fail(SSD_ERR_UNSUPPORTED, "width must be 1..8");
  if (!dtype_ok(p->x_dtype) || !dtype_ok(p->state_dtype) || !dtype_ok(p->out_dtype) ||
      !dtype_ok(p->weight_dtype) || !dtype_ok(p->bias_dtype))
    return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (!p->x_new || !p->conv_state || !p->weight || !p->out)
    return fail(SSD_ERR_INVALID_ARG, "x_new, conv_state, weight and out are required");
  return cuda_status(ssd::launch_conv1d_update(p, (cudaStream_t)stream), "causal_conv1d_update");
}

int ssd_rms_norm_gated(const ssd_rms_norm_params_t* p, ssd_stream_t stream) {
  g_err[0] = 0;
  if (!p) return fail(SSD_ERR_INVALID_ARG, "params is NULL");
  if (p->rows <= 0 || p->hidden <= 0 || p->group_size <= 0) return fail(SSD_ERR_INVALID_ARG, "dims must be positive");
  if (p->hidden % p->group_size != 0) return fail(SSD_ERR_INVALID_ARG, "hidden must be a multiple of group_size");
  if (!dtype_ok(p->x_dtype) || !dtype_ok(p->weight_dtype) || !dtype_ok(p->out_dtype) ||
      (p->z && !dtype_ok(p->z_dtype)))
    return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (!p->x || !p->weight || !p->out) return fail(SSD_ERR_INVALID_ARG, "x, weight and out are required");
  if (p->x_stride_row < p->hidden || p->out_stride_row < p->hidden || (p->z && p->z_stride_row < p->hidden))
    return fail(SSD_ERR_INVALID_ARG, "row strides must be at least hidden");
  if (!(p->eps >= 0.f)) return fail(SSD_ERR_INVALID_ARG, "eps must be non-negative");
  return cuda_status(ssd::launch_rms_norm_gated(p, (cudaStream_t)stream), "rms_norm_gated");
}

int ssd_sp_state_fixup(const ssd_sp_fixup_params_t* p, ssd_stream_t stream) {
  g_err[0] = 0;
  if (!p) return fail(SSD_ERR_INVALID_ARG, "params is NULL");
  if (p->batch <= 0 || p->seqlen <= 0 || p->nheads <= 0 || p->headdim <= 0 || p->ngroups <= 0 ||
      p->dstate <= 0 || p->chunk_size <= 0)
    return fail(SSD_ERR_INVALID_ARG, "dims must be positive");
  if (p->nheads % p->ngroups != 0) return fail(SSD_ERR_INVALID_ARG, "nheads must be a multiple of ngroups");
  if (p->headdim % 4 != 0) return fail(SSD_ERR_UNSUPPORTED, "headdim must be a multiple of 4");
  if (ssd::sp_fixup_smem_bytes(p->headdim, p->dstate) > 227 * 1024)
    return fail(SSD_ERR_UNSUPPORTED, "headdim * dstate too large for the fix-up's shared memory");
  if (!dtype_ok(p->dtype)) return fail(SSD_ERR_INVALID_ARG, "bad dtype enum");
  if (!p->C || !p->dA_cumsum || !p->state_in || !p->out)
    return fail(SSD_ERR_INVALID_ARG, "C, dA_cumsum, state_in and out are required");
  if (ssd::tc_sp_fixup_supported(p)) return ssd::tc_sp_fixup(p, (cudaStream_t)stream);
  return cuda_status(ssd::launch_sp_fixup(p, (cudaStream_t)stream), "sp_state_fixup");
}

}  // extern "C"
