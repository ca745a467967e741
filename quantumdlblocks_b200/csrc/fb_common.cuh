// fb_common.cuh -- shared definitions of the flash-Born CUDA library (sm_100a).
//
// Element conversion, the two Born pointwise maps (plain and purified), the validity mask and
// the normalised problem description that the C-ABI layer (fb_abi.cu) hands to the kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "flashborn_b200.h"  // -I include

namespace fb {

// ------------------------------------------------------------------------------------------
// Normalised problem (host side; passed by value to kernels as needed)
// ------------------------------------------------------------------------------------------
struct Tensor4 {
  const void* ptr;
  int64_t s[4];  // element strides for (B, H, T, D)
};

struct Problem {
  int B, H, T, D;
  int dtype, out_dtype;
  bool causal;
  int window;
  float eps, eps_base;
  bool purified;
  bool deterministic;  // backward without floating-point atomics
  // Backward of one term of a sum of score families that share one normaliser: o and z are the
  // whole sum's output and Z, dq/dk/dv receive this term's share, dscale/dtau are not written.
  bool given_norm;
  Tensor4 q, k, v, o, dout, dq, dk, dv;
  float* z;
  const float* scale;
  int scale_per_head;
  const float* tau;
  int tau_per_head;
  const int32_t* doc;
  int64_t doc_s[2];
  float* dscale;
  float* dtau;
  void* ws;
  size_t ws_bytes;
  int* status;  // device status word [2]: {code, site}
  // test hook (fb_test_born_fwd_timeout): bound of every device-side wait (0: the default) and
  // whether CTA 0 of the tensor-core forward skips its first K-tile copy
  uint64_t wait_limit_ns;
  int test_skip_first_k;
};

// Device status codes written into Problem::status.
enum : int { kStatusOk = 0, kStatusTimeout = FB_ERR_TIMEOUT };

// ------------------------------------------------------------------------------------------
// Element conversion
// ------------------------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// ------------------------------------------------------------------------------------------
// Validity of a (query i, key j) pair: flash_born.py:169-178 / :635-652.
//   causal: j <= i;  window > 0: i - j < window (a non-causal window leaves the future visible);
//   document ids: equal.  Keys at or beyond T are never valid.
// ------------------------------------------------------------------------------------------
//   Written with non-short-circuit & / | so that it compiles to predicate logic: the row index
//   differs between the lanes of a warp, and a short-circuit form becomes divergent branches.
__device__ __forceinline__ bool pair_valid(int i, int j, int T, bool causal, int window, int doc_i, int doc_j) {
  return (j < T) & (!causal | (j <= i)) & ((window <= 0) | (i - j < window)) & (doc_i == doc_j);
}

// ------------------------------------------------------------------------------------------
// Pointwise maps.  raw = <q_i, k_j> (unscaled).  prob() gives p_ij; grad() turns
// dP_ij = dL/dp_ij into dL/draw_ij and accumulates the parameter gradients.
// ------------------------------------------------------------------------------------------
struct PlainMap {
  float scale;
  // a = relu(scale * raw), p = a^2                                      flash_born.py:166-181
  __device__ __forceinline__ float prob(float raw, bool valid) const {
    float a = valid ? fmaxf(raw * scale, 0.f) : 0.f;
    return a * a;
  }
  // dS = 2 a dP (masked), dscale += dS * raw, dL/draw = dS * scale      flash_born.py:306-312
  __device__ __forceinline__ float grad(float raw, bool valid, float dp, float& g1, float& g2) const {
    (void)g2;
    if (!valid) return 0.f;
    float a = fmaxf(raw * scale, 0.f);
    float ds = 2.f * a * dp;
    g1 += ds * raw;
    return ds * scale;
  }
};

// Plain map without the in-loop dscale sum: the tensor-core backward takes dscale from the exact
// closed form  sum_ij dS_ij raw_ij = sum_i 2 eps delta_i / (scale Z_i)  (a raw = p / scale and
// sum_j p_ij dO_i.v_j / Z_i = delta_i), which avoids the O(N^2) cancelling sum.
struct PlainMapNoParam : PlainMap {
  __device__ __forceinline__ float grad(float raw, bool valid, float dp, float& g1, float& g2) const {
    (void)g1;
    (void)g2;
    if (!valid) return 0.f;
    float a = fmaxf(raw * scale, 0.f);
    return 2.f * a * dp * scale;
  }
};

struct PurifiedMap {
  float gamma, tau, eps_base;
  // u = relu(gamma (raw - tau)), b = relu(raw), p = u^4 + eps_base b^2  flash_born.py:782-797
  __device__ __forceinline__ float prob(float raw, bool valid) const {
    if (!valid) return 0.f;
    float u = fmaxf(gamma * (raw - tau), 0.f);
    float b = fmaxf(raw, 0.f);
    float u2 = u * u;
    return u2 * u2 + eps_base * (b * b);
  }
  // du = 4 u^3 dP; dL/draw = du gamma + 2 eps_base b dP;
  // dgamma += du (raw - tau); dtau += -du gamma                         flash_born.py:930-937
  __device__ __forceinline__ float grad(float raw, bool valid, float dp, float& g1, float& g2) const {
    if (!valid) return 0.f;
    float u = fmaxf(gamma * (raw - tau), 0.f);
    float b = fmaxf(raw, 0.f);
    float du = 4.f * (u * u * u) * dp;
    g1 += du * (raw - tau);
    g2 += -du * gamma;
    return du * gamma + 2.f * eps_base * b * dp;
  }
};

// Purified map for the tensor-core backward: d gamma via the identity
//   sum_j u^4 dP = delta eps / Z - eps_base sum_j b^2 dP      (p = u^4 + eps_base b^2)
// so  d gamma = sum du (raw - tau) = (4 / gamma) (sum_i eps delta_i / Z_i - eps_base sum b^2 dP):
// g1 accumulates eps_base b^2 dP (small terms) instead of the cancelling du (raw - tau); the
// closed-form part comes from the backward pre-pass.  d tau is accumulated as before.
struct PurifiedMapTC : PurifiedMap {
  __device__ __forceinline__ float grad(float raw, bool valid, float dp, float& g1, float& g2) const {
    if (!valid) return 0.f;
    float u = fmaxf(gamma * (raw - tau), 0.f);
    float b = fmaxf(raw, 0.f);
    float du = 4.f * (u * u * u) * dp;
    g1 += eps_base * (b * b) * dp;
    g2 += -du * gamma;
    return du * gamma + 2.f * eps_base * b * dp;
  }
};

// ------------------------------------------------------------------------------------------
// Document-mask tile ranges (fb_docs.cu): per 64-row block, the span of blocks on the other side
// that can share a document id with it (qr: key blocks of a query block; kr: query blocks of a
// key block).  Tiles outside a span hold no valid pair and are skipped.
// ------------------------------------------------------------------------------------------
constexpr int kDocBlock = 64;
__host__ __device__ inline int doc_blocks(int T) { return (T + kDocBlock - 1) / kDocBlock; }
struct DocRanges {
  const int2* qr;
  const int2* kr;
  const int2* mm;    // per 64-row block (min, max) document id
  const int2* runs;  // [B][T] positions [first, last + 1) holding each position's id (rows with mono = 1)
  const int* mono;   // [B] 1 when the row's ids never decrease along the sequence
  int nblk;
};

// True when the query rows [m0, m0 + qrows) and key rows [n0, n0 + krows) all carry one and the
// same document id (every block's min equals its max and the blocks agree): the document mask is
// then all-true on the tile and only the causal / window / length conditions remain.
__device__ __forceinline__ bool doc_single(const int2* mm, int nblk, int b, int m0, int qrows, int n0, int krows) {
  const int2* m = mm + (int64_t)b * nblk;
  const int2 a = __ldg(&m[min(m0 / kDocBlock, nblk - 1)]);
  if (a.x != a.y) return false;
  bool one = true;
  for (int x = m0 / kDocBlock; x <= min((m0 + qrows - 1) / kDocBlock, nblk - 1); ++x) {
    const int2 v = __ldg(&m[x]);
    one = one && v.x == a.x && v.y == a.x;
  }
  for (int x = n0 / kDocBlock; x <= min((n0 + krows - 1) / kDocBlock, nblk - 1); ++x) {
    const int2 v = __ldg(&m[x]);
    one = one && v.x == a.x && v.y == a.x;
  }
  return one;
}

// Narrows the other side's row range [lo, hi) of a tile whose own rows are [row0, row0 + rows) to
// the blocks that can share a document with those rows; no-op without document ids (r == null).
__device__ __forceinline__ void doc_narrow(const int2* r, int nblk, int b, int row0, int rows, int& lo, int& hi) {
  if (r == nullptr) return;
  const int x0 = row0 / kDocBlock;
  const int x1 = min((row0 + rows - 1) / kDocBlock, nblk - 1);
  int f = nblk, l = -1;
  for (int x = x0; x <= x1; ++x) {
    const int2 v = __ldg(&r[(int64_t)b * nblk + x]);
    f = min(f, v.x);
    l = max(l, v.y);
  }
  lo = max(lo, f * kDocBlock);
  hi = min(hi, (l + 1) * kDocBlock);
}

__device__ __forceinline__ void set_status(int* status, int code, int site) {
  if (status != nullptr && atomicCAS(status, 0, code) == 0) status[1] = site;
}

}  // namespace fb

// Internal host-side launchers (defined in fb_general.cu / fb_tc_*.cu).
namespace fb {
int general_fwd(const Problem& p, cudaStream_t s, int* launches);
int general_bwd(const Problem& p, cudaStream_t s, int* launches);
size_t general_bwd_workspace(const Problem& p);
bool tc_fwd_supported(const Problem& p);
int tc_fwd(const Problem& p, cudaStream_t s, int* launches);
bool tc_bwd_supported(const Problem& p);   // two-kernel backward (fb_tc_bwd.cu), d = 64 or 128
int tc_bwd(const Problem& p, cudaStream_t s, int* launches);
size_t tc_bwd_workspace(const Problem& p);
bool tc_bwd64_supported(const Problem& p);  // fused backward (fb_tc_bwd64.cu), d = 64
int tc_bwd64(const Problem& p, cudaStream_t s, int* launches);
size_t tc_bwd64_workspace(const Problem& p);
void record_cuda_error(cudaError_t e);
void set_last_launch_count(int n);  // what fb_last_launch_count reports for this host thread
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for `kernel` on the current device, made once
// per (kernel, device, size) and remembered (a failure is not), so that repeated launches spend
// no host time on it and a launch inside a stream capture makes no attribute call
cudaError_t set_smem_limit_once(const void* kernel, int smem);
// document-mask tile ranges (fb_docs.cu): bytes of workspace, and the two launches that fill it
size_t doc_ranges_bytes(const Problem& p);
int doc_ranges(const Problem& p, cudaStream_t s, void* ws, DocRanges* out);
// TMA tensor maps (fb_tmap.cu)
bool get_encoder();
bool tma_ok(const Tensor4& t);
bool bh_mergeable(const Tensor4& t, int H);
bool encode_bhtd(CUtensorMap* m, const Tensor4& t, int B, int H, int T, int D, int box_rows, bool merge_bh);
bool encode_rows_f32(CUtensorMap* m, float* base, int64_t rows);
}  // namespace fb
