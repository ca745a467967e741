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
// One warp per token row, 16-byte accesses.  In the prologue a head spans hd / 8 (bf16) or hd / 4
// (fp32) lanes and one warp-wide access covers several heads; the RoPE partner of element
// i < hd / 2 is element i + hd / 2, half a head's lanes away, so one shfl.xor brings it.  Sums of
// squares and the backward's dot products are reductions over a head's lanes; all arithmetic is
// fp32, inputs and outputs bf16 or fp32.  Memory-bound: each
// kernel reads and writes every element once (the row L2 kernels read x twice, the second time
// from L1).
#include <cuda_runtime.h>

#include "fb_common.cuh"

namespace fb {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Row L2 normalisation: one warp per row, 16-byte chunks (8 bf16 / 4 fp32 elements).
template <typename T> struct Chunk;
template <> struct Chunk<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&f)[8]) { unpack(*reinterpret_cast<const uint4*>(p), f); }
  __device__ static void unpack(const uint4 w, float (&f)[8]) {
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
  __device__ static void load(const float* p, float (&f)[4]) { unpack(*reinterpret_cast<const uint4*>(p), f); }
  __device__ static void unpack(const uint4 w, float (&f)[4]) {
    f[0] = __uint_as_float(w.x);
    f[1] = __uint_as_float(w.y);
    f[2] = __uint_as_float(w.z);
    f[3] = __uint_as_float(w.w);
  }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

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

// The prologue works in 16-byte chunks: N elements per lane (8 bf16 or 4 fp32), LPH = hd / N
// lanes per head, 32 / LPH heads per warp-wide access.  Element i < hd / 2 of a head and its RoPE
// partner i + hd / 2 sit LPH / 2 lanes apart (one shfl.xor); a head's norm is a reduction over its
// LPH lanes.  Each lane loads G chunks before it computes, so a warp keeps G x 512 bytes of loads
// in flight.
template <typename T, int HD> struct QkvShape {
  static constexpr int N = Chunk<T>::N;
  static constexpr int LPH = HD / N;     // lanes per head
  static constexpr int HPP = 32 / LPH;   // heads per warp-wide access
  static constexpr int G = 4;            // accesses in flight per lane
  static_assert(LPH >= 2 && LPH <= 32, "head must span 2..32 lanes");
};

template <int LPH>
__device__ __forceinline__ float head_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int HD>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) qkv_prologue_fwd_kernel(const QkvParams p) {
  using S = QkvShape<T, HD>;
  constexpr int N = S::N, LPH = S::LPH, HPP = S::HPP, G = S::G;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= (int64_t)p.B * p.T) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPH, hl = lane / LPH;
  const bool hi = sub >= LPH / 2;
  const int b = (int)(row / p.T), t = (int)(row % p.T);
  const int D = p.H * HD;
  const T* __restrict__ src = static_cast<const T*>(p.qkv) + row * 3 * D + sub * N;
  float c[N], sn[N];
#pragma unroll
  for (int e = 0; e < N; ++e) {
    const int pi = (sub % (LPH / 2)) * N + e;  // rotation pair of this element
    c[e] = p.cos[(int64_t)t * (HD / 2) + pi];
    sn[e] = p.sin[(int64_t)t * (HD / 2) + pi];
  }
  for (int part = 0; part < 3; ++part) {
    T* __restrict__ dst = static_cast<T*>(part == 0 ? p.q : part == 1 ? p.k : p.v) +
                          ((int64_t)b * p.H * p.T + t) * HD + sub * N;
    for (int h0 = 0; h0 < p.H; h0 += G * HPP) {
      uint4 raw[G];  // loaded chunks stay packed until used (fewer registers, more rows in flight)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int h = h0 + g * HPP + hl;
        raw[g] = h < p.H ? *reinterpret_cast<const uint4*>(src + part * D + h * HD) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int h = h0 + g * HPP + hl;
        if (part == 2) {  // V: copied
          if (h < p.H) *reinterpret_cast<uint4*>(dst + (int64_t)h * p.T * HD) = raw[g];
          continue;
        }
        float u[N], y[N], ss = 0.f;
        Chunk<T>::unpack(raw[g], u);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float o = __shfl_xor_sync(0xffffffffu, u[e], LPH / 2);
          y[e] = hi ? fmaf(o, sn[e], u[e] * c[e]) : fmaf(u[e], c[e], -o * sn[e]);
          ss = fmaf(y[e], y[e], ss);
        }
        const float r = rsqrtf(head_sum<LPH>(ss) + p.eps);
#pragma unroll
        for (int e = 0; e < N; ++e) y[e] *= r;
        if (h < p.H) Chunk<T>::store(dst + (int64_t)h * p.T * HD, y);
      }
    }
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) qkv_prologue_bwd_kernel(const QkvParams p) {
  using S = QkvShape<T, HD>;
  constexpr int N = S::N, LPH = S::LPH, HPP = S::HPP, G = S::G;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= (int64_t)p.B * p.T) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPH, hl = lane / LPH;
  const bool hi = sub >= LPH / 2;
  const int b = (int)(row / p.T), t = (int)(row % p.T);
  const int D = p.H * HD;
  const T* __restrict__ src = static_cast<const T*>(p.qkv) + row * 3 * D + sub * N;
  T* __restrict__ out = static_cast<T*>(p.dqkv) + row * 3 * D + sub * N;
  float c[N], sn[N];
#pragma unroll
  for (int e = 0; e < N; ++e) {
    const int pi = (sub % (LPH / 2)) * N + e;
    c[e] = p.cos[(int64_t)t * (HD / 2) + pi];
    sn[e] = p.sin[(int64_t)t * (HD / 2) + pi];
  }
  for (int part = 0; part < 3; ++part) {
    const T* __restrict__ grad = static_cast<const T*>(part == 0 ? p.q : part == 1 ? p.k : p.v) +
                                 ((int64_t)b * p.H * p.T + t) * HD + sub * N;
    for (int h0 = 0; h0 < p.H; h0 += G * HPP) {
      uint4 rd[G], ru[G];  // loaded chunks stay packed until used
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int h = h0 + g * HPP + hl;
        const bool ok = h < p.H;
        rd[g] = ok ? *reinterpret_cast<const uint4*>(grad + (int64_t)h * p.T * HD) : make_uint4(0, 0, 0, 0);
        ru[g] = ok && part < 2 ? *reinterpret_cast<const uint4*>(src + part * D + h * HD) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int h = h0 + g * HPP + hl;
        if (part == 2) {  // V was copied: its gradient passes through
          if (h < p.H) *reinterpret_cast<uint4*>(out + part * D + h * HD) = rd[g];
          continue;
        }
        float dz[N], u[N], y[N], ss = 0.f, yd = 0.f;
        Chunk<T>::unpack(rd[g], dz);
        Chunk<T>::unpack(ru[g], u);
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float o = __shfl_xor_sync(0xffffffffu, u[e], LPH / 2);
          y[e] = hi ? fmaf(o, sn[e], u[e] * c[e]) : fmaf(u[e], c[e], -o * sn[e]);
          ss = fmaf(y[e], y[e], ss);
          yd = fmaf(y[e], dz[e], yd);
        }
        const float r = rsqrtf(head_sum<LPH>(ss) + p.eps);
        const float k3 = r * r * r * head_sum<LPH>(yd);
        // d y = r dz - y r^3 (y . dz); then the transposed rotation: du = dy c + dy' s (first
        // half) and du = dy c - dy' s (second half), dy' = the partner's gradient
#pragma unroll
        for (int e = 0; e < N; ++e) {
          const float dy = fmaf(r, dz[e], -y[e] * k3);
          const float o = __shfl_xor_sync(0xffffffffu, dy, LPH / 2);
          dz[e] = hi ? fmaf(dy, c[e], -o * sn[e]) : fmaf(dy, c[e], o * sn[e]);
        }
        if (h < p.H) Chunk<T>::store(out + part * D + h * HD, dz);
      }
    }
  }
}

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

// Rows of at most 32 N R elements: each lane keeps its R chunks of the row in registers (packed),
// so the row is read once and all its loads are in flight together.
template <typename T, int R>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) l2norm_rows_reg_kernel(const RowsParams p, bool bwd) {
  constexpr int N = Chunk<T>::N;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= p.rows) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const T* x = static_cast<const T*>(p.x) + row * p.cols;
  uint4 rx[R], rg[R];
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = (j * 32 + lane) * N;
    rx[j] = c < p.cols ? *reinterpret_cast<const uint4*>(x + c) : make_uint4(0u, 0u, 0u, 0u);
    if (bwd) rg[j] = c < p.cols ? *reinterpret_cast<const uint4*>(static_cast<const T*>(p.dy) + row * p.cols + c)
                                : make_uint4(0u, 0u, 0u, 0u);
  }
  float ss = 0.f, xd = 0.f;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    float f[N], g[N];
    Chunk<T>::unpack(rx[j], f);
    if (bwd) Chunk<T>::unpack(rg[j], g);
#pragma unroll
    for (int i = 0; i < N; ++i) {
      ss = fmaf(f[i], f[i], ss);
      if (bwd) xd = fmaf(f[i], g[i], xd);
    }
  }
  const float r = rsqrtf(warp_sum(ss) + p.eps);
  const float k3 = bwd ? r * r * r * warp_sum(xd) : 0.f;  // dx = r dy - x r^3 (x . dy)
  T* out = static_cast<T*>(bwd ? p.dx : p.y) + row * p.cols;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = (j * 32 + lane) * N;
    if (c >= p.cols) continue;
    float f[N], g[N];
    Chunk<T>::unpack(rx[j], f);
    if (bwd) {
      Chunk<T>::unpack(rg[j], g);
#pragma unroll
      for (int i = 0; i < N; ++i) g[i] = fmaf(r, g[i], -f[i] * k3);
    } else {
#pragma unroll
      for (int i = 0; i < N; ++i) g[i] = f[i] * r;
    }
    Chunk<T>::store(out + c, g);
  }
}

template <typename T>
bool launch_rows_reg(const RowsParams& p, bool bwd, unsigned grid, cudaStream_t s) {
  const int chunks = (p.cols + 32 * Chunk<T>::N - 1) / (32 * Chunk<T>::N);  // per lane
  if (chunks <= 2) l2norm_rows_reg_kernel<T, 2><<<grid, kWarpsPerBlock * 32, 0, s>>>(p, bwd);
  else if (chunks <= 4) l2norm_rows_reg_kernel<T, 4><<<grid, kWarpsPerBlock * 32, 0, s>>>(p, bwd);
  else if (chunks <= 8) l2norm_rows_reg_kernel<T, 8><<<grid, kWarpsPerBlock * 32, 0, s>>>(p, bwd);
  else return false;
  return true;
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
  // rows of up to 8 chunks per lane stay in registers; longer rows take the two-pass kernels
  const bool in_regs = a->dtype == FB_BF16 ? launch_rows_reg<__nv_bfloat16>(p, backward, grid, s)
                                           : launch_rows_reg<float>(p, backward, grid, s);
  if (in_regs) return finish_launch(1);
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
