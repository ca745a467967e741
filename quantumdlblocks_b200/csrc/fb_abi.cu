// fb_abi.cu -- the extern "C" boundary of libflashborn_b200.so.
//
// Validates the fb_attn_args of each call (host-side; no device traps), normalises them into
// fb::Problem, picks the kernel path (tcgen05 tensor-core path when applicable, else the general
// CUDA-core path) and enqueues the kernels on the caller's stream.  The library allocates no
// device memory: the backward's scratch comes from the caller's workspace.
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "fb_common.cuh"

namespace fb {

namespace {
thread_local int t_last_launches = 0;
thread_local char t_last_cuda_error[256] = "no error";

// Device status word: {code, site}.  One instance per device (the module is loaded per device);
// its device address is looked up once per device and cached.
__device__ int g_status[2];

constexpr int kMaxDevices = 64;
std::once_flag g_status_once[kMaxDevices];
int* g_status_ptr[kMaxDevices];
cudaError_t g_status_err[kMaxDevices];

int* status_ptr(int* rc) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    record_cuda_error(e == cudaSuccess ? cudaErrorInvalidDevice : e);
    *rc = FB_ERR_NO_DEVICE;
    return nullptr;
  }
  std::call_once(g_status_once[dev], [dev] {
    void* p = nullptr;
    g_status_err[dev] = cudaGetSymbolAddress(&p, g_status);
    g_status_ptr[dev] = static_cast<int*>(p);
  });
  if (g_status_err[dev] != cudaSuccess) {
    record_cuda_error(g_status_err[dev]);
    *rc = FB_ERR_NO_DEVICE;
    return nullptr;
  }
  *rc = FB_OK;
  return g_status_ptr[dev];
}

bool valid_dtype(int d) { return d == FB_F32 || d == FB_F16 || d == FB_BF16; }

int check_tensor(const void* p, const int64_t* st) {
  if (p == nullptr) return FB_ERR_ARG;
  for (int i = 0; i < 4; ++i)
    if (st[i] < 0) return FB_ERR_ALIGN;
  return FB_OK;
}

// Validates and normalises.  backward selects the extra backward checks; query_only (workspace
// and path queries) fills the backward fields without requiring their pointers.
int normalise(const fb_attn_args* a, bool purified, bool backward, Problem* p, bool query_only = false,
              bool given_norm = false) {
  if (a == nullptr) return FB_ERR_ARG;
  *p = Problem{};
  p->B = a->batch; p->H = a->heads; p->T = a->seq_len; p->D = a->head_dim;
  if (p->B < 0 || p->H < 0 || p->T < 0 || p->D < 1 || p->D > 256) return FB_ERR_SHAPE;
  if (p->B > 65535 || p->H > 65535) return FB_ERR_SHAPE;
  if (!valid_dtype(a->dtype) || !valid_dtype(a->out_dtype)) return FB_ERR_DTYPE;
  // out has the input type (plain, flash_born.py:467) or fp32 (purified, flash_born.py:1102; a
  // plain forward whose output is one partial term of a sum, combined at full precision)
  if (a->out_dtype != FB_F32 && a->out_dtype != a->dtype) return FB_ERR_DTYPE;
  if (a->window_size < 0) return FB_ERR_ARG;
  if (a->path < FB_PATH_AUTO || a->path > FB_PATH_GENERAL) return FB_ERR_ARG;
  p->dtype = a->dtype; p->out_dtype = a->out_dtype;
  p->causal = a->is_causal != 0; p->window = a->window_size;
  p->eps = a->eps; p->eps_base = a->eps_base;
  p->purified = purified;
  p->deterministic = a->deterministic != 0;
  if (a->scale == nullptr) return FB_ERR_ARG;
  if (a->scale_numel != 1 && a->scale_numel != p->H) return FB_ERR_ARG;
  p->scale = a->scale; p->scale_per_head = a->scale_numel > 1;
  if (purified) {
    if (a->tau == nullptr) return FB_ERR_ARG;
    if (a->tau_numel != 1 && a->tau_numel != p->H) return FB_ERR_ARG;
    p->tau = a->tau; p->tau_per_head = a->tau_numel > 1;
  }
  p->doc = a->doc_ids;
  p->doc_s[0] = a->doc_stride[0]; p->doc_s[1] = a->doc_stride[1];
  const bool empty = (int64_t)p->B * p->H * p->T == 0;
  auto t4 = [](const void* ptr, const int64_t* st) { Tensor4 t; t.ptr = ptr; for (int i = 0; i < 4; ++i) t.s[i] = st[i]; return t; };
  p->q = t4(a->q, a->q_stride); p->k = t4(a->k, a->k_stride); p->v = t4(a->v, a->v_stride);
  p->o = t4(a->out, a->out_stride);
  p->z = a->z;
  p->ws = a->workspace; p->ws_bytes = a->workspace_bytes;  // forward: document ranges only
  if (!empty && !query_only) {
    int rc;
    if ((rc = check_tensor(a->q, a->q_stride)) || (rc = check_tensor(a->k, a->k_stride)) ||
        (rc = check_tensor(a->v, a->v_stride)) || (rc = check_tensor(a->out, a->out_stride)))
      return rc;
    if (a->z == nullptr) return FB_ERR_ARG;
  }
  if (backward) {
    p->dout = t4(a->dout, a->dout_stride);
    p->dq = t4(a->dq, a->dq_stride); p->dk = t4(a->dk, a->dk_stride); p->dv = t4(a->dv, a->dv_stride);
    p->dscale = a->dscale; p->dtau = a->dtau;
    p->ws = a->workspace; p->ws_bytes = a->workspace_bytes;
    if (!empty && !query_only) {
      int rc;
      if ((rc = check_tensor(a->dout, a->dout_stride)) || (rc = check_tensor(a->dq, a->dq_stride)) ||
          (rc = check_tensor(a->dk, a->dk_stride)) || (rc = check_tensor(a->dv, a->dv_stride)))
        return rc;
      if (a->dscale == nullptr && !given_norm) return FB_ERR_ARG;
      if (purified && a->dtau == nullptr) return FB_ERR_ARG;
    }
  }
  return FB_OK;
}

// Tensor-core backward: the fused kernel for d = 64 (its dQ partials are added by fp32
// reduce-adds, in an order that can vary); the two-kernel backward for d = 128 and whenever the
// caller asks for deterministic gradients.
bool use_fused_bwd(const Problem& p) { return p.D == 64 && !p.deterministic && tc_bwd64_supported(p); }

int choose_path(const fb_attn_args* a, const Problem& p, bool backward) {
  const bool tc = backward ? (use_fused_bwd(p) || tc_bwd_supported(p)) : tc_fwd_supported(p);
  if (a->path == FB_PATH_GENERAL) return FB_PATH_GENERAL;
  if (a->path == FB_PATH_TCGEN05) return tc ? FB_PATH_TCGEN05 : -FB_ERR_UNSUPPORTED;
  return tc ? FB_PATH_TCGEN05 : FB_PATH_GENERAL;
}

size_t workspace_for(const Problem& p, int path, bool backward) {
  if (!backward) return path == FB_PATH_TCGEN05 ? doc_ranges_bytes(p) : 0;  // forward: document ranges
  if (path != FB_PATH_TCGEN05) return general_bwd_workspace(p);
  return use_fused_bwd(p) ? tc_bwd64_workspace(p) : tc_bwd_workspace(p);
}

// Test hook of fb_test_born_fwd_timeout: a short bound on every device-side wait and a forward
// whose CTA 0 never requests its first K tile.
struct TestHook {
  uint64_t wait_limit_ns;
};

int run(const fb_attn_args* a, void* stream, bool purified, bool backward, bool given_norm = false,
        const TestHook* hook = nullptr) {
  Problem p;
  int rc = normalise(a, purified, backward, &p, false, given_norm);
  if (rc != FB_OK) return rc;
  p.given_norm = given_norm;
  if (given_norm) p.dscale = p.dtau = nullptr;
  if ((int64_t)p.B * p.H * p.T == 0) {  // nothing to do (empty batch / heads / sequence)
    t_last_launches = 0;
    return FB_OK;
  }
  const int path = choose_path(a, p, backward);
  if (path < 0) return -path;
  if (hook != nullptr) {
    if (backward || path != FB_PATH_TCGEN05) return FB_ERR_UNSUPPORTED;
    p.wait_limit_ns = hook->wait_limit_ns;
    p.test_skip_first_k = 1;
  }
  const size_t ws_need = workspace_for(p, path, backward);
  if (p.ws_bytes < ws_need || (p.ws == nullptr && ws_need > 0)) return FB_ERR_WORKSPACE;
  p.status = status_ptr(&rc);
  if (rc != FB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int launches = 0;
  if (path == FB_PATH_TCGEN05) {
    rc = backward ? (use_fused_bwd(p) ? tc_bwd64(p, s, &launches) : tc_bwd(p, s, &launches))
                  : tc_fwd(p, s, &launches);
  } else {
    rc = backward ? general_bwd(p, s, &launches) : general_fwd(p, s, &launches);
  }
  if (rc == FB_OK) t_last_launches = launches;
  return rc;
}

}  // namespace

void set_last_launch_count(int n) { t_last_launches = n; }

cudaError_t set_smem_limit_once(const void* kernel, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const std::pair<const void*, int> key(kernel, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = done.find(key);
    if (it != done.end() && it->second >= smem) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  int& v = done[key];
  v = std::max(v, smem);
  return cudaSuccess;
}

void record_cuda_error(cudaError_t e) {
  const char* msg = cudaGetErrorString(e);
  size_t i = 0;
  for (; msg && msg[i] && i + 1 < sizeof(t_last_cuda_error); ++i) t_last_cuda_error[i] = msg[i];
  t_last_cuda_error[i] = 0;
}

}  // namespace fb

extern "C" {

int fb_born_fwd(const fb_attn_args* args, void* stream) { return fb::run(args, stream, false, false); }
int fb_born_bwd(const fb_attn_args* args, void* stream) { return fb::run(args, stream, false, true); }
int fb_purified_born_fwd(const fb_attn_args* args, void* stream) { return fb::run(args, stream, true, false); }
int fb_purified_born_bwd(const fb_attn_args* args, void* stream) { return fb::run(args, stream, true, true); }
int fb_born_bwd_term(const fb_attn_args* args, void* stream) { return fb::run(args, stream, false, true, true); }

int fb_test_born_fwd_timeout(const fb_attn_args* args, void* stream, uint32_t wait_limit_us) {
  if (wait_limit_us == 0) return FB_ERR_ARG;
  const fb::TestHook hook{static_cast<uint64_t>(wait_limit_us) * 1000ull};
  return fb::run(args, stream, false, false, false, &hook);
}

size_t fb_bwd_workspace_size(const fb_attn_args* args) {
  fb::Problem p;
  const bool purified = args != nullptr && args->tau != nullptr;
  if (fb::normalise(args, purified, true, &p, true) != FB_OK) return 0;
  const int path = fb::choose_path(args, p, true);
  if (path < 0) return 0;
  return fb::workspace_for(p, path, true);
}

size_t fb_fwd_workspace_size(const fb_attn_args* args) {
  fb::Problem p;
  const bool purified = args != nullptr && args->tau != nullptr;
  if (fb::normalise(args, purified, false, &p, true) != FB_OK) return 0;
  const int path = fb::choose_path(args, p, false);
  if (path < 0) return 0;
  return fb::workspace_for(p, path, false);
}

int fb_select_path(const fb_attn_args* args, int backward) {
  fb::Problem p;
  const bool purified = args != nullptr && args->tau != nullptr;
  int rc = fb::normalise(args, purified, backward != 0, &p, true);
  if (rc != FB_OK) return -rc;
  return fb::choose_path(args, p, backward != 0);
}

int fb_last_launch_count(void) { return fb::t_last_launches; }

int fb_device_status(void* stream, int32_t* detail) {
  int rc;
  int* st = fb::status_ptr(&rc);
  if (rc != FB_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host[2] = {0, 0};
  cudaError_t e = cudaMemcpyAsync(host, st, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(st, 0, sizeof(host), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    fb::record_cuda_error(e);
    return FB_ERR_LAUNCH;
  }
  if (detail) *detail = host[1];
  return host[0] == 0 ? FB_OK : host[0];
}

const char* fb_strerror(int status) {
  switch (status) {
    case FB_OK: return "success";
    case FB_ERR_SHAPE: return "flashborn: shape out of range (need 1 <= D <= 256, B, H <= 65535, T >= 0)";
    case FB_ERR_DTYPE: return "flashborn: unsupported dtype combination (q/k/v must share float32/float16/bfloat16; plain out = input dtype; purified out = float32 or input dtype)";
    case FB_ERR_ALIGN: return "flashborn: negative or misaligned stride";
    case FB_ERR_ARG: return "flashborn: invalid argument (null pointer, scale/tau length not 1 or H, negative window, bad path)";
    case FB_ERR_LAUNCH: return "flashborn: CUDA launch failed (see fb_last_cuda_error)";
    case FB_ERR_TIMEOUT: return "flashborn: a device-side pipeline wait exceeded its bound; the kernel stopped early and its outputs are invalid";
    case FB_ERR_WORKSPACE: return "flashborn: workspace missing or smaller than fb_bwd_workspace_size() / fb_fwd_workspace_size()";
    case FB_ERR_NO_DEVICE: return "flashborn: no usable CUDA device";
    case FB_ERR_UNSUPPORTED: return "flashborn: the forced tcgen05 path does not support this configuration";
    case FB_ERR_SCRATCH_LIMIT: return "flashborn: this backward needs more scratch than the library's static array (FB_STATIC_SCRATCH_BYTES); call fb_born_bwd with a workspace instead";
    default: return "flashborn: unknown status";
  }
}

const char* fb_last_cuda_error(void) { return fb::t_last_cuda_error; }

int fb_abi_version(void) { return FB_ABI_VERSION; }

}  // extern "C"
