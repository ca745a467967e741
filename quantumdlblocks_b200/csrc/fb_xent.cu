// fb_xent.cu -- the GPT training loss: mean cross-entropy over bf16 logits, fused.
//
// The reference's GPTs take F.cross_entropy(logits.reshape(-1, V), targets) (models/born_gpt.py:1291)
// under bf16 autocast, which upcasts the logits to an fp32 copy, runs log-softmax forward and
// backward over it and casts the gradient back: five passes over an (N, V) fp32 tensor (3.3 GB at
// the C5 shape, N = 16384, V = 50,304).  Here:
//
//   xent_fwd_kernel   one CTA per row: online max / sum of exp over the bf16 row (16-byte loads),
//                     lse_r = m + log s, loss_r = lse_r - x[r, target_r]
//   xent_bwd_kernel   one CTA per row: dx = (exp(x - lse_r) - [c == target_r]) * g / N, written
//                     bf16; g (the incoming gradient of the mean loss) is read from device memory
//
// The forward reads the logits once and the backward reads them again and writes the gradient:
// three passes over a bf16 tensor.  exp and log are CUDA's __expf / __logf; all sums are fp32.
#include <cuda_runtime.h>

#include <cmath>

#include "fb_common.cuh"

namespace fb {
namespace {

constexpr int kXentThreads = 512;

struct XentParams {
  int64_t rows;
  int V;
  int64_t ld;  // elements between rows
  const __nv_bfloat16* logits;
  const int64_t* targets;
  float* lse;
  float* loss;
  __nv_bfloat16* grad;
  const float* gscale;
  float inv_n;
};

__device__ __forceinline__ void unpack8(const uint4 w, float (&f)[8]) {
  const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(a[i] << 16);
    f[2 * i + 1] = __uint_as_float(a[i] & 0xFFFF0000u);
  }
}

// (m, s) pairs: s = sum exp(x - m).  An empty side has m = -inf, s = 0.
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;  // both empty
  s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
  m = mm;
}

__global__ void __launch_bounds__(kXentThreads) xent_fwd_kernel(const XentParams p) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = p.logits + row * p.ld;
  const int nchunk = p.V / 8;
  float m = -INFINITY, s = 0.f;
  // kUnroll chunks are requested before any is used, so each thread keeps 64 bytes in flight;
  // chunks past the row read as -inf (bf16 0xFF80), which adds nothing
  constexpr int kUnroll = 4;
  for (int c0 = threadIdx.x; c0 < nchunk; c0 += kUnroll * kXentThreads) {
    uint4 w[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * kXentThreads;
      w[u] = c < nchunk ? __ldg(reinterpret_cast<const uint4*>(x + 8 * c))
                        : make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float f[8];
      unpack8(w[u], f);
      float cm = f[0];
#pragma unroll
      for (int i = 1; i < 8; ++i) cm = fmaxf(cm, f[i]);
      if (cm == -INFINITY) continue;  // a chunk of masked columns
      if (cm > m) {
        s = s * __expf(m - cm);
        m = cm;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) s += __expf(f[i] - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) merge(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
  __shared__ float sm[kXentThreads / 32], ss[kXentThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < kXentThreads / 32 ? sm[lane] : -INFINITY;
    s = lane < kXentThreads / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      merge(m, s, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) {
      const float lse = m + __logf(s);
      const int64_t t = p.targets[row];
      const float xt = (t >= 0 && t < p.V) ? __bfloat162float(x[t]) : NAN;  // out-of-range target: NaN loss
      p.lse[row] = lse;
      p.loss[row] = lse - xt;
    }
  }
}

__global__ void __launch_bounds__(kXentThreads) xent_bwd_kernel(const XentParams p) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = p.logits + row * p.ld;
  __nv_bfloat16* dx = p.grad + row * p.ld;
  const float lse = p.lse[row];
  const float g = *p.gscale * p.inv_n;
  const int64_t t = p.targets[row];
  const int nchunk = p.V / 8;
  for (int c = threadIdx.x; c < nchunk; c += kXentThreads) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(x + 8 * c), f);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      float a = __expf(f[i] - lse) * g, b = __expf(f[i + 1] - lse) * g;
      if (8 * c + i == t) a -= g;
      if (8 * c + i + 1 == t) b -= g;
      __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
      w[i / 2] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(dx + 8 * c) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

int xent(const fb_xent_args* a, void* stream, bool backward) {
  if (a == nullptr) return FB_ERR_ARG;
  if (a->rows < 0 || a->vocab < 8 || a->vocab % 8 != 0 || a->ld < a->vocab || a->ld % 8 != 0) return FB_ERR_SHAPE;
  if (a->rows > 0x7FFFFFFF) return FB_ERR_SHAPE;
  if (a->logits == nullptr || a->targets == nullptr || a->lse == nullptr) return FB_ERR_ARG;
  if (!backward && a->loss == nullptr) return FB_ERR_ARG;
  if (backward && (a->grad == nullptr || a->gscale == nullptr)) return FB_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a->logits) & 15) != 0 || (backward && (reinterpret_cast<uintptr_t>(a->grad) & 15) != 0))
    return FB_ERR_ALIGN;
  if (a->rows == 0) {
    set_last_launch_count(0);
    return FB_OK;
  }
  XentParams p{a->rows, a->vocab, a->ld, static_cast<const __nv_bfloat16*>(a->logits), a->targets, a->lse, a->loss,
               static_cast<__nv_bfloat16*>(a->grad), a->gscale, a->rows > 0 ? 1.f / (float)a->rows : 0.f};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (backward)
    xent_bwd_kernel<<<(unsigned)a->rows, kXentThreads, 0, s>>>(p);
  else
    xent_fwd_kernel<<<(unsigned)a->rows, kXentThreads, 0, s>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return FB_ERR_LAUNCH;
  }
  set_last_launch_count(1);
  return FB_OK;
}

}  // namespace
}  // namespace fb

extern "C" {

int fb_xent_fwd(const fb_xent_args* args, void* stream) { return fb::xent(args, stream, false); }
int fb_xent_bwd(const fb_xent_args* args, void* stream) { return fb::xent(args, stream, true); }

}  // extern "C"
