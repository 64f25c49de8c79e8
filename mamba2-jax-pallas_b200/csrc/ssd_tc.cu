// tcgen05 pipeline (placeholder until the tensor-core kernels land).
#include "ssd_tc.h"

namespace ssd {
bool tc_supported(const ssd_fwd_params_t*) { return false; }
int tc_num_launches(const ssd_fwd_params_t*) { return 0; }
size_t tc_workspace_bytes(const ssd_fwd_params_t*) { return 0; }
int tc_combined_fwd(const ssd_fwd_params_t*, void*, cudaStream_t) { return SSD_ERR_UNSUPPORTED; }
}  // namespace ssd
