// fb_prologue.cu -- the Born attention layer's Q / K prologue and row L2 normalisation, fused.
//
// The reference layer (layers/attention.py:508-589, functional.py:59-121) turns its input into
// attention operands with a chain of PyTorch ops per layer: psi = l2_normalize(x); the fused
// projection's output is reshaped, transposed and copied contiguous (:512-516); Q and K are
// rotated by the unitary RoPE (apply_unitary_rope: the two halves of each head turned by
// position-dependent angles) and normalised again (:588-589).  Each op reads and writes the whole
// activation; the backward doubles the count.  Two kernel pairs replace them:
//
//   qkv_prologue_fwd   qkv (B, T, 3 H hd) -> Q, K = l2n(rope(.)), V copied, all (B, H, T, hd)
//   qkv_prologue_bwd   dQ, dK, dV (B, H, T, hd) + qkv -> d qkv (B, T, 3 H hd)
//   l2norm_rows_fwd    y = x / sqrt(sum x^2 + eps) per row
//   l2norm_rows_bwd    dx = r (dy - y (y . dy)), r = 1 / sqrt(sum x^2 + eps)
//
// One warp per token row.  In the prologue lane l holds elements [l E, l E + E) of a head (E =
// hd / 32); the RoPE partner of element i < hd / 2 is element i + hd / 2, which sits 16 lanes away,
// so one shfl.xor 16 brings it.  Sums of squares and the backward's dot products are warp
// reductions; all arithmetic is fp32, inputs and outputs bf16 or fp32.  Memory-bound: each
// kernel reads and writes every element once (the row L2 kernels read x twice, the second time
// from L1).
#include <cuda_runtime.h>

#include "fb_common.cuh"

namespace fb {
namespace {

constexpr int kWarpsPerBlock = 8;

template <typename T, int E> struct Lane;
template <> struct Lane<__nv_bfloat16, 2> {
  __device__ static void load(const __nv_bfloat16* p, float (&f)[2]) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xFFFF0000u);
  }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[2]) {
    __nv_bfloat162 v = __floats2bfloat162_rn(f[0], f[1]);
    *reinterpret_cast<__nv_bfloat162*>(p) = v;
  }
};
template <> struct Lane<__nv_bfloat16, 4> {
  __device__ static void load(const __nv_bfloat16* p, float (&f)[4]) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    f[0] = __uint_as_float(w.x << 16);
    f[1] = __uint_as_float(w.x & 0xFFFF0000u);
    f[2] = __uint_as_float(w.y << 16);
    f[3] = __uint_as_float(w.y & 0xFFFF0000u);
  }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), b = __floats2bfloat162_rn(f[2], f[3]);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = w;
  }
};
template <> struct Lane<float, 2> {
  __device__ static void load(const float* p, float (&f)[2]) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    f[0] = v.x;
    f[1] = v.y;
  }
  __device__ static void store(float* p, const float (&f)[2]) { *reinterpret_cast<float2*>(p) = make_float2(f[0], f[1]); }
};
template <> struct Lane<float, 4> {
  __device__ static void load(const float* p, float (&f)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x;
    f[1] = v.y;
    f[2] = v.z;
    f[3] = v.w;
  }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct QkvParams {
  int B, T, H;
  float eps;
  const void* qkv;   // (B, T, 3 H hd) contiguous
  const float* cos;  // (T, hd / 2) contiguous
  const float* sin;
  void* q;           // (B, H, T, hd) contiguous: forward outputs / backward incoming gradients
  void* k;
  void* v;
  void* dqkv;        // backward output, qkv's layout
};

// Rotation of this lane's E elements: for the first half of the head (lanes 0-15)
// y = u c - u' s, for the second half y = u' s + u c, u' = the partner element 16 lanes away.
template <int E>
__device__ __forceinline__ void rope(const float (&u)[E], const float (&c)[E], const float (&s)[E], bool hi,
                                     float (&y)[E]) {
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float o = __shfl_xor_sync(0xffffffffu, u[e], 16);
    y[e] = hi ? fmaf(o, s[e], u[e] * c[e]) : fmaf(u[e], c[e], -o * s[e]);
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) qkv_prologue_fwd_kernel(const QkvParams p) {
  constexpr int E = HD / 32;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= (int64_t)p.B * p.T) return;
  const int lane = threadIdx.x & 31;
  const int b = (int)(row / p.T), t = (int)(row % p.T);
  const int D = p.H * HD;
  const T* src = static_cast<const T*>(p.qkv) + row * 3 * D + lane * E;
  float c[E], s[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int pi = (lane & 15) * E + e;  // rotation pair of this element
    c[e] = p.cos[(int64_t)t * (HD / 2) + pi];
    s[e] = p.sin[(int64_t)t * (HD / 2) + pi];
  }
  const bool hi = lane >= 16;
  for (int part = 0; part < 3; ++part) {
    T* dst = static_cast<T*>(part == 0 ? p.q : part == 1 ? p.k : p.v) + ((int64_t)b * p.H * p.T + t) * HD + lane * E;
#pragma unroll 4
    for (int h = 0; h < p.H; ++h) {
      float u[E];
      Lane<T, E>::load(src + part * D + h * HD, u);
      if (part < 2) {
        float y[E];
        rope<E>(u, c, s, hi, y);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss = fmaf(y[e], y[e], ss);
        const float r = rsqrtf(warp_sum(ss) + p.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) u[e] = y[e] * r;
      }
      Lane<T, E>::store(dst + (int64_t)h * p.T * HD, u);
    }
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) qkv_prologue_bwd_kernel(const QkvParams p) {
  constexpr int E = HD / 32;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= (int64_t)p.B * p.T) return;
  const int lane = threadIdx.x & 31;
  const int b = (int)(row / p.T), t = (int)(row % p.T);
  const int D = p.H * HD;
  const T* src = static_cast<const T*>(p.qkv) + row * 3 * D + lane * E;
  T* out = static_cast<T*>(p.dqkv) + row * 3 * D + lane * E;
  float c[E], s[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int pi = (lane & 15) * E + e;
    c[e] = p.cos[(int64_t)t * (HD / 2) + pi];
    s[e] = p.sin[(int64_t)t * (HD / 2) + pi];
  }
  const bool hi = lane >= 16;
  for (int part = 0; part < 3; ++part) {
    const T* g = static_cast<const T*>(part == 0 ? p.q : part == 1 ? p.k : p.v) + ((int64_t)b * p.H * p.T + t) * HD +
                 lane * E;
#pragma unroll 4
    for (int h = 0; h < p.H; ++h) {
      float dz[E];
      Lane<T, E>::load(g + (int64_t)h * p.T * HD, dz);
      if (part < 2) {
        float u[E], y[E];
        Lane<T, E>::load(src + part * D + h * HD, u);
        rope<E>(u, c, s, hi, y);
        float ss = 0.f, yd = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          ss = fmaf(y[e], y[e], ss);
          yd = fmaf(y[e], dz[e], yd);
        }
        const float r = rsqrtf(warp_sum(ss) + p.eps);
        const float k3 = r * r * r * warp_sum(yd);
        // d y = r dz - y r^3 (y . dz); then the transposed rotation: du = dy c + dy' s (first
        // half) and du = dy c - dy' s (second half), dy' = the partner's gradient
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float dy = fmaf(r, dz[e], -y[e] * k3);
          const float o = __shfl_xor_sync(0xffffffffu, dy, 16);
          dz[e] = hi ? fmaf(dy, c[e], -o * s[e]) : fmaf(dy, c[e], o * s[e]);
        }
      }
      Lane<T, E>::store(out + part * D + h * HD, dz);
    }
  }
}

// Row L2 normalisation: one warp per row, 16-byte chunks (8 bf16 / 4 fp32 elements).
template <typename T> struct Chunk;
template <> struct Chunk<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 w = *reinterpret_cast<const uint4*>(p);
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(a[i] << 16);
      f[2 * i + 1] = __uint_as_float(a[i] & 0xFFFF0000u);
    }
  }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[8]) {
    uint32_t a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      a[i] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(a[0], a[1], a[2], a[3]);
  }
};
template <> struct Chunk<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&f)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x;
    f[1] = v.y;
    f[2] = v.z;
    f[3] = v.w;
  }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

struct RowsParams {
  int64_t rows;
  int cols;
  float eps;
  const void* x;
  void* y;
  const void* dy;
  void* dx;
};

template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) l2norm_rows_fwd_kernel(const RowsParams p) {
  constexpr int N = Chunk<T>::N;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int lane = threadIdx.x & 31;
  const T* x = static_cast<const T*>(p.x) + row * p.cols;
  T* y = static_cast<T*>(p.y) + row * p.cols;
  float ss = 0.f;
  for (int c = lane * N; c < p.cols; c += 32 * N) {
    float f[N];
    Chunk<T>::load(x + c, f);
#pragma unroll
    for (int i = 0; i < N; ++i) ss = fmaf(f[i], f[i], ss);
  }
  const float r = rsqrtf(warp_sum(ss) + p.eps);
  for (int c = lane * N; c < p.cols; c += 32 * N) {
    float f[N];
    Chunk<T>::load(x + c, f);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] *= r;
    Chunk<T>::store(y + c, f);
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) l2norm_rows_bwd_kernel(const RowsParams p) {
  constexpr int N = Chunk<T>::N;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int lane = threadIdx.x & 31;
  const T* x = static_cast<const T*>(p.x) + row * p.cols;
  const T* dy = static_cast<const T*>(p.dy) + row * p.cols;
  T* dx = static_cast<T*>(p.dx) + row * p.cols;
  float ss = 0.f, xd = 0.f;
  for (int c = lane * N; c < p.cols; c += 32 * N) {
    float f[N], g[N];
    Chunk<T>::load(x + c, f);
    Chunk<T>::load(dy + c, g);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      ss = fmaf(f[i], f[i], ss);
      xd = fmaf(f[i], g[i], xd);
    }
  }
  const float r = rsqrtf(warp_sum(ss) + p.eps);
  const float k3 = r * r * r * warp_sum(xd);  // dx = r dy - x r^3 (x . dy)
  for (int c = lane * N; c < p.cols; c += 32 * N) {
    float f[N], g[N];
    Chunk<T>::load(x + c, f);
    Chunk<T>::load(dy + c, g);
#pragma unroll
    for (int i = 0; i < N; ++i) g[i] = fmaf(r, g[i], -f[i] * k3);
    Chunk<T>::store(dx + c, g);
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int finish_launch(int n) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return FB_ERR_LAUNCH;
  }
  set_last_launch_count(n);
  return FB_OK;
}

int qkv_prologue(const fb_qkv_args* a, void* stream, bool backward) {
  if (a == nullptr) return FB_ERR_ARG;
  if (a->batch < 1 || a->seq_len < 1 || a->heads < 1 || (a->head_dim != 64 && a->head_dim != 128))
    return FB_ERR_SHAPE;
  if (a->dtype != FB_BF16 && a->dtype != FB_F32) return FB_ERR_DTYPE;
  if (a->qkv == nullptr || a->cos == nullptr || a->sin == nullptr || a->q == nullptr || a->k == nullptr ||
      a->v == nullptr || (backward && a->dqkv == nullptr) || !(a->eps >= 0.f))
    return FB_ERR_ARG;
  if (!aligned16(a->qkv) || !aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) ||
      (backward && !aligned16(a->dqkv)))
    return FB_ERR_ALIGN;
  QkvParams p{a->batch, a->seq_len, a->heads, a->eps, a->qkv, a->cos, a->sin, a->q, a->k, a->v, a->dqkv};
  const int64_t rows = (int64_t)a->batch * a->seq_len;
  const unsigned grid = (unsigned)((rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = a->dtype == FB_BF16;
  const bool h64 = a->head_dim == 64;
  if (backward) {
    if (bf)
      h64 ? qkv_prologue_bwd_kernel<__nv_bfloat16, 64><<<grid, kWarpsPerBlock * 32, 0, s>>>(p)
          : qkv_prologue_bwd_kernel<__nv_bfloat16, 128><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
    else
      h64 ? qkv_prologue_bwd_kernel<float, 64><<<grid, kWarpsPerBlock * 32, 0, s>>>(p)
          : qkv_prologue_bwd_kernel<float, 128><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
  } else {
    if (bf)
      h64 ? qkv_prologue_fwd_kernel<__nv_bfloat16, 64><<<grid, kWarpsPerBlock * 32, 0, s>>>(p)
          : qkv_prologue_fwd_kernel<__nv_bfloat16, 128><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
    else
      h64 ? qkv_prologue_fwd_kernel<float, 64><<<grid, kWarpsPerBlock * 32, 0, s>>>(p)
          : qkv_prologue_fwd_kernel<float, 128><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
  }
  return finish_launch(1);
}

int l2norm_rows(const fb_rows_args* a, void* stream, bool backward) {
  if (a == nullptr) return FB_ERR_ARG;
  if (a->rows < 1 || a->cols < 1) return FB_ERR_SHAPE;
  if (a->dtype != FB_BF16 && a->dtype != FB_F32) return FB_ERR_DTYPE;
  const int per_chunk = a->dtype == FB_BF16 ? 8 : 4;
  if (a->cols % per_chunk != 0) return FB_ERR_ALIGN;
  if (a->x == nullptr || !(a->eps >= 0.f) || (!backward && a->y == nullptr) ||
      (backward && (a->dy == nullptr || a->dx == nullptr)))
    return FB_ERR_ARG;
  if (!aligned16(a->x) || (!backward && !aligned16(a->y)) || (backward && (!aligned16(a->dy) || !aligned16(a->dx))))
    return FB_ERR_ALIGN;
  RowsParams p{a->rows, a->cols, a->eps, a->x, a->y, a->dy, a->dx};
  const unsigned grid = (unsigned)((a->rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (backward) {
    if (a->dtype == FB_BF16)
      l2norm_rows_bwd_kernel<__nv_bfloat16><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
    else
      l2norm_rows_bwd_kernel<float><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
  } else {
    if (a->dtype == FB_BF16)
      l2norm_rows_fwd_kernel<__nv_bfloat16><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
    else
      l2norm_rows_fwd_kernel<float><<<grid, kWarpsPerBlock * 32, 0, s>>>(p);
  }
  return finish_launch(1);
}

}  // namespace
}  // namespace fb

extern "C" {

int fb_qkv_prologue_fwd(const fb_qkv_args* args, void* stream) { return fb::qkv_prologue(args, stream, false); }
int fb_qkv_prologue_bwd(const fb_qkv_args* args, void* stream) { return fb::qkv_prologue(args, stream, true); }
int fb_l2norm_rows_fwd(const fb_rows_args* args, void* stream) { return fb::l2norm_rows(args, stream, false); }
int fb_l2norm_rows_bwd(const fb_rows_args* args, void* stream) { return fb::l2norm_rows(args, stream, true); }

}  // extern "C"
