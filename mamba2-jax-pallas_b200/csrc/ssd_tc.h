// Tensor-core (tcgen05) pipeline for bf16 inputs: host-side interface.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "ssd_b200.h"

namespace ssd {

// True when the tcgen05 pipeline covers these params (bf16 inputs, supported shape).
bool tc_supported(const ssd_fwd_params_t* p);
// Workspace bytes the tcgen05 pipeline needs besides the status word (0 when unsupported).
size_t tc_workspace_bytes(const ssd_fwd_params_t* p);
// Kernel launches one tc_combined_fwd call enqueues.
int tc_num_launches(const ssd_fwd_params_t* p);
// Enqueue the tcgen05 pipeline.  Requires tc_supported(p).  `status` is the device status
// word (cleared by the caller on the stream); a bounded wait that gives up writes there.
int tc_combined_fwd(const ssd_fwd_params_t* p, unsigned* status, void* workspace, cudaStream_t st);

// The sequence-parallel fix-up on the tensor cores (bf16 C, P = 64, N = 128 or 256).
bool tc_sp_fixup_supported(const ssd_sp_fixup_params_t* p);
int tc_sp_fixup(const ssd_sp_fixup_params_t* p, cudaStream_t st);

}  // namespace ssd
