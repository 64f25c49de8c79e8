// Tensor-core (tcgen05, split-bf16 "bf16x3") chunk_state, bmm_chunk and chunk_scan for
// fp32 inputs: host-side interface.  Same layouts and results (to rel-L2 ~1e-5) as the
// CUDA-core stages declared in ssd_kernels.h.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "ssd_b200.h"

namespace ssd {

bool x3_bmm_supported(const void* a, const void* b, int dtype, int64_t K, int64_t Q);
bool x3_chunk_state_supported(const void* x, const void* B, int dtype, int64_t P, int64_t N, int64_t Q);
bool x3_chunk_scan_supported(const void* x, const void* C, const void* z, const float* cb, const void* states,
                             int dtype, int states_dtype, int64_t P, int64_t N, int64_t Q, const float* out,
                             const float* out_x);

// `status` (nullable) is a device word a bounded wait that gave up writes 0x100|id to.
cudaError_t launch_x3_bmm(const float* a, const float* b, const int32_t* seq_idx, int causal, int64_t batch,
                          int64_t L, int64_t G, int64_t K, int64_t Q, float* out, unsigned* status,
                          cudaStream_t st);
cudaError_t launch_x3_chunk_state(const float* x, const float* B, const float* dt, const float* dA,
                                  const int32_t* seq_idx, int64_t b, int64_t L, int64_t H, int64_t P, int64_t G,
                                  int64_t N, int64_t Q, float* states, unsigned* status, cudaStream_t st);
cudaError_t launch_x3_chunk_scan(const float* cb, const float* x, const float* dt, const float* dA, const float* C,
                                 const float* states, const float* D, int D_ndim, const float* z,
                                 const int32_t* seq_idx, int64_t b, int64_t L, int64_t H, int64_t P, int64_t G,
                                 int64_t N, int64_t Q, float* out, float* out_x, unsigned* status,
                                 cudaStream_t st);

}  // namespace ssd
