// fb_static_scratch.cu -- a backward entry point that allocates nothing.
//
// fb_born_bwd() needs device scratch (delta, 1/Z, the fp32 dQ accumulator, gradient partials)
// that the caller passes as a workspace.  Some callers cannot allocate device memory: a host
// runtime that binds only this library's C functions and has no device allocator of its own,
// or a step loop that must not call cudaMalloc (it can synchronise the device, and it fails once
// another framework's memory pool has reserved the GPU).  fb_born_bwd_static_scratch() serves
// them from a fixed array compiled into the library instead.
//
//   * The array is FB_STATIC_SCRATCH_BYTES (16 MiB) of device memory per GPU, held from the first
//     call on that device until the process exits.  Problems whose backward needs more scratch
//     than that (fb_bwd_workspace_size) are rejected with FB_ERR_SCRATCH_LIMIT.
//   * The first call on a device looks up the array's device address there (cudaGetSymbolAddress,
//     with that device current); make that first call before any stream capture begins.
//   * All calls on a device share the one array and it keeps the previous call's contents; every
//     part the kernels read is rewritten or zeroed by the call itself.  Calls whose work overlaps
//     on the GPU (different streams, or host threads without ordering) race on it.
#include <mutex>

#include "fb_common.cuh"

namespace {

constexpr size_t kScratchBytes = FB_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_bwd_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
void* g_scratch_ptr[kMaxDevices];
cudaError_t g_scratch_err[kMaxDevices];

}  // namespace

extern "C" FB_API int fb_born_bwd_static_scratch(const fb_attn_args* args, void* stream) {
  if (args == nullptr) return FB_ERR_ARG;
  fb_attn_args a = *args;
  a.tau = nullptr;  // plain Born backward only
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  if (fb_bwd_workspace_size(&a) > kScratchBytes) return FB_ERR_SCRATCH_LIMIT;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    fb::record_cuda_error(e == cudaSuccess ? cudaErrorInvalidDevice : e);
    return FB_ERR_NO_DEVICE;
  }
  // host code must not use g_bwd_scratch itself (that is a host-side stand-in): look up the
  // array's address on this device once, with this device current
  std::call_once(g_once[dev], [dev] { g_scratch_err[dev] = cudaGetSymbolAddress(&g_scratch_ptr[dev], g_bwd_scratch); });
  if (g_scratch_err[dev] != cudaSuccess) {
    fb::record_cuda_error(g_scratch_err[dev]);
    return FB_ERR_NO_DEVICE;
  }
  a.workspace = g_scratch_ptr[dev];
  a.workspace_bytes = kScratchBytes;
  return fb_born_bwd(&a, stream);
}
