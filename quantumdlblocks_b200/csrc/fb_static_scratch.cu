// fb_static_scratch.cu -- a backward entry point that allocates nothing.
//
// fb_born_bwd() needs device scratch (delta, 1/Z, the fp32 dQ accumulator, gradient partials)
// that the caller passes as a workspace.  Some callers cannot allocate device memory: a host
// runtime that binds only this library's C functions and has no device allocator of its own,
// or a step loop that must not call cudaMalloc (it can synchronise the device, and it fails once
// another framework's memory pool has reserved the GPU).  fb_born_bwd_static_scratch() serves
// them from a fixed array compiled into the library instead.
//
//   * The array is FB_STATIC_SCRATCH_BYTES (16 MiB) of device memory per GPU.  It is part of the
//     library's device module, so a GPU holds it from the time the module is loaded there until
//     the process exits: with CUDA's default lazy module loading that is the first launch of
//     any of this library's kernels on that GPU, with CUDA_MODULE_LOADING=EAGER it is context
//     creation, whether or not this entry point is ever called.  Problems whose backward needs
//     more scratch than that (fb_bwd_workspace_size) are rejected with FB_ERR_SCRATCH_LIMIT.
//   * Plain Born only: purified arguments (tau != NULL) are rejected with FB_ERR_ARG.
//   * The first successful call on a device looks up the array's device address there
//     (cudaGetSymbolAddress, with that device current); make that first call before any stream
//     capture begins.  A failed lookup is not remembered: the next call tries again.
//   * All calls on a device share the one array and it keeps the previous call's contents; every
//     part the kernels read is rewritten or zeroed by the call itself.  Calls whose work overlaps
//     on the GPU (different streams, or host threads without ordering) race on it.
#include <mutex>

#include "fb_common.cuh"

namespace {

constexpr size_t kScratchBytes = FB_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_bwd_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lookup_mutex;
void* g_scratch_ptr[kMaxDevices];  // written once per device, under g_lookup_mutex

// Device address of the array on device `dev` (current), looked up on first use; a failed
// lookup leaves the slot empty so that a later call retries it.
void* scratch_address(int dev, cudaError_t* err) {
  std::lock_guard<std::mutex> lock(g_lookup_mutex);
  *err = cudaSuccess;
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (*err == cudaSuccess) g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" FB_API int fb_born_bwd_static_scratch(const fb_attn_args* args, void* stream) {
  if (args == nullptr || args->tau != nullptr) return FB_ERR_ARG;  // plain Born backward only
  fb_attn_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  if (fb_bwd_workspace_size(&a) > kScratchBytes) return FB_ERR_SCRATCH_LIMIT;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    fb::record_cuda_error(e == cudaSuccess ? cudaErrorInvalidDevice : e);
    return FB_ERR_NO_DEVICE;
  }
  // host code must not use g_bwd_scratch itself (that is a host-side stand-in): use the array's
  // address on this device, looked up with this device current
  void* ptr = scratch_address(dev, &e);
  if (ptr == nullptr) {
    fb::record_cuda_error(e);
    return FB_ERR_NO_DEVICE;
  }
  a.workspace = ptr;
  a.workspace_bytes = kScratchBytes;
  return fb_born_bwd(&a, stream);
}
