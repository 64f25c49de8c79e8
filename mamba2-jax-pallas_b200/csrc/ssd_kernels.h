// Internal launcher declarations (host side).  Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ssd_b200.h"

namespace ssd {

cudaError_t launch_chunk_cumsum(const void* dt, int dt_dtype, const float* A, const float* dt_bias,
                                int softplus, float lo, float hi, int64_t b, int64_t L, int64_t H,
                                int64_t Q, float* dA_cs, float* dt_out, cudaStream_t st);
cudaError_t launch_chunk_state(const void* x, const void* B, int dtype, const float* dt,
                               const float* dA, const int32_t* seq_idx, int64_t b, int64_t L,
                               int64_t H, int64_t P, int64_t G, int64_t N, int64_t Q,
                               float* states, cudaStream_t st);
cudaError_t launch_state_passing(const float* states, const float* dA_chunk, int64_t stride_bh,
                                 int64_t stride_c, const float* init, const int32_t* seq_idx,
                                 int64_t b, int64_t nc, int64_t H, int64_t dim, int64_t L,
                                 int64_t Q, void* out, int out_dtype, float* final_states,
                                 cudaStream_t st);
cudaError_t launch_bmm_chunk(const void* a, const void* b, int dtype, const int32_t* seq_idx,
                             int causal, int64_t batch, int64_t L, int64_t G, int64_t K,
                             int64_t Q, float* out, cudaStream_t st);
cudaError_t launch_chunk_scan(const float* cb, const void* x, int dtype, const float* dt,
                              const float* dA, const void* C, const void* states, int states_dtype,
                              const float* D, int D_ndim, const void* z, const int32_t* seq_idx,
                              int64_t b, int64_t L, int64_t H, int64_t P, int64_t G, int64_t N,
                              int64_t Q, float* out, float* out_x, cudaStream_t st);
cudaError_t launch_chunk_state_varlen(const void* B, const void* x, int dtype, const float* dt,
                                      const float* dA, const int32_t* cu, int S, const void* cs,
                                      int states_dtype, int64_t T_total, int64_t H, int64_t P,
                                      int64_t G, int64_t N, int64_t Q, float* out, cudaStream_t st);
cudaError_t launch_ssu(const ssu_params_t* p, cudaStream_t st);
cudaError_t launch_conv1d(const ssd_conv1d_params_t* p, cudaStream_t st);
cudaError_t launch_conv1d_update(const ssd_conv1d_update_params_t* p, cudaStream_t st);
cudaError_t launch_rms_norm_gated(const ssd_rms_norm_params_t* p, cudaStream_t st);
cudaError_t launch_sp_fixup(const ssd_sp_fixup_params_t* p, cudaStream_t st);
size_t sp_fixup_smem_bytes(int64_t P, int64_t N);

// Set the thread-local message ssd_last_error() returns.
void set_last_error(const char* msg);

}  // namespace ssd
