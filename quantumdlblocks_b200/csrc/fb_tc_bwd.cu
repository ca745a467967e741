// fb_tc_bwd.cu -- tcgen05 backward (placeholder until the tensor-core backward lands).
#include "fb_common.cuh"

namespace fb {
bool tc_bwd_supported(const Problem&) { return false; }
size_t tc_bwd_workspace(const Problem&) { return 0; }
int tc_bwd(const Problem&, cudaStream_t, int*) { return FB_ERR_UNSUPPORTED; }
}  // namespace fb
