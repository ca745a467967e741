// fb_tc_fwd.cu -- tcgen05 forward (placeholder until the tensor-core forward lands).
#include "fb_common.cuh"

namespace fb {
bool tc_fwd_supported(const Problem&) { return false; }
int tc_fwd(const Problem&, cudaStream_t, int*) { return FB_ERR_UNSUPPORTED; }
}  // namespace fb
