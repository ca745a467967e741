// fb_families.cu -- the glue kernels of the Born attention families that run as sums of plain
// Born terms (complex phase: layers/attention.py:717-730; paired heads: :591-626).
//
//   rotate_halves_kernel  dst = a + R b per row of D = 2 h elements, R b = [-b_im | b_re] (the
//                         key rotation of the imaginary overlap) or its adjoint R^T b = [b_im | -b_re]
//                         (its gradient), a optional
//   combine_terms_kernel  O = sum_t O_t Z_t / sum_t Z_t and Z = sum_t Z_t over the terms' fp32
//                         outputs, O written in the output type through 4-D strides
//   delta_terms_kernel    per (b, h, 64-row chunk): sum_i eps (dO_i . O_i) / Z_i, the closed-form
//                         scale gradient of the family before its 2 / scale factor
//
// All three are single passes over their operands (HBM-bound), 16-byte accesses where the rows
// allow, fp32 arithmetic.
#include <cuda_runtime.h>

#include "fb_common.cuh"

namespace fb {
namespace {

template <typename T> __device__ __forceinline__ float ld_f32(const T* p);
template <> __device__ __forceinline__ float ld_f32<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <> __device__ __forceinline__ float ld_f32<__half>(const __half* p) { return __half2float(*p); }
template <typename T> __device__ __forceinline__ void st_f32(T* p, float v);
template <> __device__ __forceinline__ void st_f32<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st_f32<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ void st_f32<__half>(__half* p, float v) { *p = __float2half_rn(v); }

struct RotParams {
  int64_t rows;
  int D;
  int adjoint;
  const void* a;
  const void* b;
  void* dst;
};

// Four consecutive elements as floats: one 8-byte (bf16, fp16) or 16-byte (fp32) access when
// `vec` (16-byte aligned rows of a multiple of 4 elements), else four scalar ones.
template <typename T> __device__ __forceinline__ void ld4(const T* q, bool vec, float (&f)[4]) {
  if (vec) {
    if constexpr (sizeof(T) == 4) {
      const float4 v = *reinterpret_cast<const float4*>(q);
      f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
      return;
    } else {
      const uint2 w = *reinterpret_cast<const uint2*>(q);
      const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) f[i] = ld_f32(e + i);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) f[i] = ld_f32(q + i);
}
template <typename T> __device__ __forceinline__ void st4(T* q, bool vec, const float (&f)[4]) {
  if (vec) {
    if constexpr (sizeof(T) == 4) {
      *reinterpret_cast<float4*>(q) = make_float4(f[0], f[1], f[2], f[3]);
      return;
    } else {
      uint2 w;
      T* e = reinterpret_cast<T*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) st_f32(e + i, f[i]);
      *reinterpret_cast<uint2*>(q) = w;
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) st_f32(q + i, f[i]);
}

// One thread per (row, 4 element pairs i..i+3 < D/2) when D/2 is a multiple of 4 (else one pair
// per thread): reads b_i, b_{i+h} (and a), writes both outputs.
template <typename T, int V>
__global__ void rotate_halves_kernel(const RotParams p, bool vec) {
  const int h = p.D / 2;
  const int64_t n = p.rows * (h / V);
  const T* a = static_cast<const T*>(p.a);
  const T* b = static_cast<const T*>(p.b);
  T* d = static_cast<T*>(p.dst);
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / (h / V);
    const int i = (int)(idx % (h / V)) * V;
    const int64_t lo = row * p.D + i, hi = lo + h;
    if constexpr (V == 4) {
      float re[4], im[4], o_lo[4], o_hi[4];
      ld4(b + lo, vec, re);
      ld4(b + hi, vec, im);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o_lo[e] = p.adjoint ? im[e] : -im[e];
        o_hi[e] = p.adjoint ? -re[e] : re[e];
      }
      if (a != nullptr) {
        float al[4], ah[4];
        ld4(a + lo, vec, al);
        ld4(a + hi, vec, ah);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o_lo[e] += al[e];
          o_hi[e] += ah[e];
        }
      }
      st4(d + lo, vec, o_lo);
      st4(d + hi, vec, o_hi);
    } else {
      const float re = ld_f32(b + lo), im = ld_f32(b + hi);
      float o_lo = p.adjoint ? im : -im;
      float o_hi = p.adjoint ? -re : re;
      if (a != nullptr) {
        o_lo += ld_f32(a + lo);
        o_hi += ld_f32(a + hi);
      }
      st_f32(d + lo, o_lo);
      st_f32(d + hi, o_hi);
    }
  }
}

struct CombineParams {
  int B, H, T, D;
  int n_terms;
  const float* o[4];
  const float* z[4];
  void* out;
  int64_t os[4];
  float* z_out;
  int64_t zs[3];
};

// One thread per (row, 4 consecutive elements) (D a multiple of 4): the terms' float4s weighted
// by their Z, one output access of 4 elements when the output rows allow it.
template <typename TO>
__global__ void combine_terms_kernel(const CombineParams p, bool vec) {
  const int q4 = p.D / 4;
  const int64_t n = (int64_t)p.B * p.H * p.T * q4;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / q4;
    const int c = (int)(idx % q4) * 4;
    const int t = (int)(row % p.T);
    const int h = (int)((row / p.T) % p.H);
    const int b = (int)(row / ((int64_t)p.T * p.H));
    float zt[4], zsum = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      zt[k] = k < p.n_terms ? p.z[k][row] : 0.f;
      zsum += zt[k];
    }
    const float inv = 1.f / zsum;
    if (c == 0) p.z_out[b * p.zs[0] + h * p.zs[1] + t * p.zs[2]] = zsum;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k < p.n_terms) {
        const float4 v = *reinterpret_cast<const float4*>(p.o[k] + row * p.D + c);
        acc[0] = fmaf(v.x, zt[k], acc[0]);
        acc[1] = fmaf(v.y, zt[k], acc[1]);
        acc[2] = fmaf(v.z, zt[k], acc[2]);
        acc[3] = fmaf(v.w, zt[k], acc[3]);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] *= inv;
    TO* orow = static_cast<TO*>(p.out) + b * p.os[0] + h * p.os[1] + t * p.os[2];
    if (vec) {
      st4(orow + c, true, acc);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) st_f32(orow + (c + e) * p.os[3], acc[e]);
    }
  }
}

struct DeltaParams {
  int B, H, T, D;
  float eps;
  const void* dout;
  int64_t ds[4];
  const void* out;
  int64_t os[4];
  const float* z;  // (B, H, T) contiguous
  float* part;     // (B, H, ceil(T / kDeltaRows))
};

constexpr int kDeltaRows = 64;  // rows per block of delta_terms_kernel

// One block per (64-row chunk, h, b): each warp takes 8 rows, lanes over D; fixed-order block
// reduction into the chunk's partial.
template <typename TD, typename TO>
__global__ void __launch_bounds__(256) delta_terms_kernel(const DeltaParams p) {
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TD* dO = static_cast<const TD*>(p.dout) + b * p.ds[0] + h * p.ds[1];
  const TO* O = static_cast<const TO*>(p.out) + b * p.os[0] + h * p.os[1];
  const float* z = p.z + ((int64_t)b * p.H + h) * p.T;
  float acc = 0.f;
  const int t_end = min(p.T, (chunk + 1) * kDeltaRows);
  for (int t = chunk * kDeltaRows + warp; t < t_end; t += 8) {
    float d = 0.f;
    for (int c = lane; c < p.D; c += 32) d = fmaf(ld_f32(dO + t * p.ds[2] + c * p.ds[3]), ld_f32(O + t * p.os[2] + c * p.os[3]), d);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    acc += p.eps * d / z[t];
  }
  __shared__ float red[8];
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w];
    p.part[((int64_t)b * p.H + h) * gridDim.x + chunk] = s;
  }
}

int finish(int n) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return FB_ERR_LAUNCH;
  }
  set_last_launch_count(n);
  return FB_OK;
}

unsigned grid_for(int64_t threads) {
  const int64_t blocks = (threads + 255) / 256;
  return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

bool valid_dtype3(int d) { return d == FB_F32 || d == FB_BF16 || d == FB_F16; }

}  // namespace
}  // namespace fb

extern "C" {

int fb_rotate_halves(const fb_rot_args* a, void* stream) {
  using namespace fb;
  if (a == nullptr) return FB_ERR_ARG;
  if (a->rows < 0 || a->head_dim < 2 || a->head_dim % 2 != 0) return FB_ERR_SHAPE;
  if (!valid_dtype3(a->dtype)) return FB_ERR_DTYPE;
  if (a->b == nullptr || a->dst == nullptr) return FB_ERR_ARG;
  if (a->rows == 0) return finish(0);
  RotParams p{a->rows, a->head_dim, a->adjoint != 0, a->a, a->b, a->dst};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int h = a->head_dim / 2;
  const int elt = a->dtype == FB_F32 ? 4 : 2;
  const auto al = [&](const void* q) { return (reinterpret_cast<uintptr_t>(q) & (uintptr_t)(4 * elt - 1)) == 0; };
  const bool v4 = h % 4 == 0;
  const bool vec = v4 && al(a->b) && al(a->dst) && (a->a == nullptr || al(a->a));
  const unsigned g = grid_for(a->rows * (v4 ? h / 4 : h));
  if (a->dtype == FB_F32)
    v4 ? rotate_halves_kernel<float, 4><<<g, 256, 0, s>>>(p, vec) : rotate_halves_kernel<float, 1><<<g, 256, 0, s>>>(p, false);
  else if (a->dtype == FB_BF16)
    v4 ? rotate_halves_kernel<__nv_bfloat16, 4><<<g, 256, 0, s>>>(p, vec)
       : rotate_halves_kernel<__nv_bfloat16, 1><<<g, 256, 0, s>>>(p, false);
  else
    v4 ? rotate_halves_kernel<__half, 4><<<g, 256, 0, s>>>(p, vec) : rotate_halves_kernel<__half, 1><<<g, 256, 0, s>>>(p, false);
  return finish(1);
}

int fb_combine_terms(const fb_combine_args* a, void* stream) {
  using namespace fb;
  if (a == nullptr) return FB_ERR_ARG;
  if (a->batch < 0 || a->heads < 0 || a->seq_len < 0 || a->head_dim < 4 || a->head_dim % 4 != 0 ||
      a->n_terms < 1 || a->n_terms > 4)
    return FB_ERR_SHAPE;
  if (!valid_dtype3(a->out_dtype)) return FB_ERR_DTYPE;
  if (a->out == nullptr || a->z_out == nullptr) return FB_ERR_ARG;
  for (int k = 0; k < a->n_terms; ++k) {
    if (a->o[k] == nullptr || a->z[k] == nullptr) return FB_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(a->o[k]) & 15) != 0) return FB_ERR_ALIGN;
  }
  const int64_t rows = (int64_t)a->batch * a->heads * a->seq_len;
  if (rows == 0) return finish(0);
  CombineParams p{};
  p.B = a->batch; p.H = a->heads; p.T = a->seq_len; p.D = a->head_dim; p.n_terms = a->n_terms;
  for (int k = 0; k < 4; ++k) {
    p.o[k] = k < a->n_terms ? a->o[k] : nullptr;
    p.z[k] = k < a->n_terms ? a->z[k] : nullptr;
  }
  p.out = a->out;
  for (int i = 0; i < 4; ++i) p.os[i] = a->out_stride[i];
  p.z_out = a->z_out;
  for (int i = 0; i < 3; ++i) p.zs[i] = a->z_stride[i];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int elt = a->out_dtype == FB_F32 ? 4 : 2;
  bool vec = a->out_stride[3] == 1 && (reinterpret_cast<uintptr_t>(a->out) & (uintptr_t)(4 * elt - 1)) == 0;
  for (int i = 0; i < 3; ++i) vec = vec && a->out_stride[i] % 4 == 0;
  const unsigned g = grid_for(rows * (a->head_dim / 4));
  if (a->out_dtype == FB_F32) combine_terms_kernel<float><<<g, 256, 0, s>>>(p, vec);
  else if (a->out_dtype == FB_BF16) combine_terms_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(p, vec);
  else combine_terms_kernel<__half><<<g, 256, 0, s>>>(p, vec);
  return finish(1);
}

int fb_delta_terms(const fb_delta_args* a, void* stream) {
  using namespace fb;
  if (a == nullptr) return FB_ERR_ARG;
  if (a->batch < 0 || a->heads < 0 || a->seq_len < 0 || a->head_dim < 1 || a->batch > 65535 ||
      a->heads > 65535)
    return FB_ERR_SHAPE;
  if (!valid_dtype3(a->dout_dtype) || (a->out_dtype != FB_F32 && a->out_dtype != a->dout_dtype)) return FB_ERR_DTYPE;
  if (a->dout == nullptr || a->out == nullptr || a->z == nullptr || a->part == nullptr) return FB_ERR_ARG;
  if ((int64_t)a->batch * a->heads * a->seq_len == 0) return finish(0);
  DeltaParams p{a->batch, a->heads, a->seq_len, a->head_dim, a->eps, a->dout, {}, a->out, {}, a->z, a->part};
  for (int i = 0; i < 4; ++i) {
    p.ds[i] = a->dout_stride[i];
    p.os[i] = a->out_stride[i];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 g((a->seq_len + kDeltaRows - 1) / kDeltaRows, a->heads, a->batch);
  const bool of = a->out_dtype == FB_F32;
  if (a->dout_dtype == FB_F32) delta_terms_kernel<float, float><<<g, 256, 0, s>>>(p);
  else if (a->dout_dtype == FB_BF16)
    of ? delta_terms_kernel<__nv_bfloat16, float><<<g, 256, 0, s>>>(p)
       : delta_terms_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, s>>>(p);
  else
    of ? delta_terms_kernel<__half, float><<<g, 256, 0, s>>>(p) : delta_terms_kernel<__half, __half><<<g, 256, 0, s>>>(p);
  return finish(1);
}

}  // extern "C"
