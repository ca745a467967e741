// fb_epilogue.cu -- the Born attention layer's head epilogue (_finalize_heads), fused.
//
// After the attention call the reference layer (layers/attention.py:478-493) optionally
// subtracts a gated self-value projection from every head's output (apply_gated_xsa,
// layers/mudd_and_gates.py:45-61: r = y - tanh(alpha_h) (y . v) / (|v|^2 + eps) v), multiplies by
// an input-driven per-head gate (InputChannelGate, :17-42: g = 2 sigmoid(x[:c] . W_h + b_h) from
// the first c channels of the layer input) and merges the heads into (B, T, H hd) for out_proj.
// Each of those is a separate PyTorch pass over (B, H, T, hd) tensors; here:
//
//   heads_epilogue_fwd_kernel  Y[b, t, h hd + i] = g_bth r_bthi          (one pass: reads O, V)
//   heads_epilogue_bwd_kernel  dO, dV from dY, O, V; per (b, t, h) the scalars the parameter
//                              gradients are sums of: -(1 - tanh^2 alpha_h) s e (d alpha_h) and
//                              g (1 - g / 2) (dY . r) (d of the gate's pre-activation)
//
// One warp per token row (b, t), 16-byte accesses: a head spans hd / 8 (bf16) or hd / 4 (fp32)
// lanes, one warp-wide access covers several heads; head sums are reductions over a head's lanes.
// fp32 arithmetic; tanh, exp are CUDA's tanhf / __expf.
#include <cuda_runtime.h>

#include "fb_common.cuh"

namespace fb {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxGate = 8;  // gate channels held per lane

struct HeadsParams {
  int B, H, T, hd;
  float eps;
  const void* o;
  int64_t os[3];
  const void* v;
  int64_t vs[3];
  const float* alpha;
  const float* gx;  // (B, T, c) fp32
  int c;
  const float* gw;  // (H, c)
  const float* gb;  // (H)
  void* y;          // (B, T, H hd)
  const void* dy;   // (B, T, H hd)
  void* dO;         // (B, H, T, hd) contiguous
  void* dV;         // (B, H, T, hd) contiguous
  float* dalpha;    // (B, T, H)
  float* du;        // (B, T, H)
};

template <typename T> struct Vec;
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const void* p, float (&f)[8]) { unpack(*reinterpret_cast<const uint4*>(p), f); }
  __device__ static void unpack(const uint4 w, float (&f)[8]) {
    const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(a[i] << 16);
      f[2 * i + 1] = __uint_as_float(a[i] & 0xFFFF0000u);
    }
  }
  __device__ static void store(void* p, const float (&f)[8]) {
    uint32_t a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 v = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      a[i] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(a[0], a[1], a[2], a[3]);
  }
};
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const void* p, float (&f)[4]) { unpack(*reinterpret_cast<const uint4*>(p), f); }
  __device__ static void unpack(const uint4 w, float (&f)[4]) {
    f[0] = __uint_as_float(w.x); f[1] = __uint_as_float(w.y); f[2] = __uint_as_float(w.z); f[3] = __uint_as_float(w.w);
  }
  __device__ static void store(void* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};

template <int LPH>
__device__ __forceinline__ float head_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Gate of head h at row (b, t): 2 sigmoid(b_h + sum_c x_c W_hc); 1 without a gate.
__device__ __forceinline__ float gate_of(const HeadsParams& p, const float (&x)[kMaxGate], int h) {
  if (p.gx == nullptr) return 1.f;
  float u = p.gb[h];
#pragma unroll
  for (int k = 0; k < kMaxGate; ++k)
    if (k < p.c) u = fmaf(x[k], p.gw[(int64_t)h * p.c + k], u);
  return 2.f / (1.f + __expf(-u));
}

template <typename T, int HD, bool kBwd>
__global__ void __launch_bounds__(kWarps * 32) heads_epilogue_kernel(const HeadsParams p) {
  constexpr int N = Vec<T>::N, LPH = HD / N, HPP = 32 / LPH;
  static_assert(LPH >= 1 && LPH <= 32 && (LPH & (LPH - 1)) == 0, "head must span a power of two of lanes");
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= (int64_t)p.B * p.T) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPH, hl = lane / LPH;
  const int b = (int)(row / p.T), t = (int)(row % p.T);
  float x[kMaxGate];
#pragma unroll
  for (int k = 0; k < kMaxGate; ++k) x[k] = (p.gx != nullptr && k < p.c) ? p.gx[row * p.c + k] : 0.f;
  const int D = p.H * HD;
  // G warp-wide accesses of O, V (and dY) are requested before any is used; chunks stay packed
  constexpr int G = 4;
  const bool xsa = p.alpha != nullptr;
  const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
  for (int h00 = 0; h00 < p.H; h00 += G * HPP) {
    uint4 ro[G], rv[G], rd[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      const int h = h00 + gi * HPP + hl;
      const bool ok = h < p.H;
      const int64_t oo = (int64_t)b * p.os[0] + (int64_t)h * p.os[1] + (int64_t)t * p.os[2] + sub * N;
      const int64_t vo = (int64_t)b * p.vs[0] + (int64_t)h * p.vs[1] + (int64_t)t * p.vs[2] + sub * N;
      ro[gi] = ok ? *reinterpret_cast<const uint4*>(static_cast<const T*>(p.o) + oo) : zero4;
      rv[gi] = ok && xsa ? *reinterpret_cast<const uint4*>(static_cast<const T*>(p.v) + vo) : zero4;
      if constexpr (kBwd)
        rd[gi] = ok ? *reinterpret_cast<const uint4*>(static_cast<const T*>(p.dy) + row * D + (int64_t)h * HD + sub * N)
                    : zero4;
    }
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      const int h = h00 + gi * HPP + hl;
      const bool ok = h < p.H;
      float y[N], v[N];
      Vec<T>::unpack(ro[gi], y);
      Vec<T>::unpack(rv[gi], v);
      float nn = 0.f, dot = 0.f;
#pragma unroll
      for (int e = 0; e < N; ++e) {
        nn = fmaf(v[e], v[e], nn);
        dot = fmaf(y[e], v[e], dot);
      }
      nn = head_sum<LPH>(nn) + p.eps;
      dot = head_sum<LPH>(dot);
      const float cx = (xsa && ok) ? tanhf(p.alpha[h]) : 0.f;
      const float s = dot / nn;
      float r[N];
#pragma unroll
      for (int e = 0; e < N; ++e) r[e] = fmaf(-cx * s, v[e], y[e]);
      const float g = ok ? gate_of(p, x, h) : 1.f;
      const int64_t yo = row * D + (int64_t)(ok ? h : 0) * HD + sub * N;
      if constexpr (!kBwd) {
        float out[N];
#pragma unroll
        for (int e = 0; e < N; ++e) out[e] = g * r[e];
        if (ok) Vec<T>::store(static_cast<T*>(p.y) + yo, out);
      } else {
        float d3[N];
        Vec<T>::unpack(rd[gi], d3);
        float dg = 0.f, ee = 0.f, dr[N];
#pragma unroll
        for (int e = 0; e < N; ++e) {
          dg = fmaf(d3[e], r[e], dg);
          dr[e] = g * d3[e];
          ee = fmaf(dr[e], v[e], ee);
        }
        dg = head_sum<LPH>(dg);
        ee = head_sum<LPH>(ee);
        float dy[N], dv[N];
#pragma unroll
        for (int e = 0; e < N; ++e) {
          // r = y - c s v, s = (y . v) / n:  dy = dr - c (e / n) v,
          // dv = -c ((y - 2 s v) e / n + s dr)
          dy[e] = fmaf(-cx * ee / nn, v[e], dr[e]);
          dv[e] = -cx * fmaf((y[e] - 2.f * s * v[e]), ee / nn, s * dr[e]);
        }
        if (ok) {
          const int64_t go = (((int64_t)b * p.H + h) * p.T + t) * HD + sub * N;
          Vec<T>::store(static_cast<T*>(p.dO) + go, dy);
          if (xsa) Vec<T>::store(static_cast<T*>(p.dV) + go, dv);
          if (sub == 0) {
            const int64_t so = row * p.H + h;
            if (xsa) p.dalpha[so] = -(1.f - cx * cx) * s * ee;
            if (p.gx != nullptr) p.du[so] = dg * g * (1.f - 0.5f * g);
          }
        }
      }
    }
  }
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

template <typename T, int HD>
void launch(const HeadsParams& p, bool bwd, cudaStream_t s) {
  const unsigned grid = (unsigned)(((int64_t)p.B * p.T + kWarps - 1) / kWarps);
  if (bwd) heads_epilogue_kernel<T, HD, true><<<grid, kWarps * 32, 0, s>>>(p);
  else heads_epilogue_kernel<T, HD, false><<<grid, kWarps * 32, 0, s>>>(p);
}

int heads_epilogue(const fb_heads_args* a, void* stream, bool bwd) {
  if (a == nullptr) return FB_ERR_ARG;
  if (a->batch < 0 || a->heads < 0 || a->seq_len < 0) return FB_ERR_SHAPE;
  if (a->head_dim != 32 && a->head_dim != 64 && a->head_dim != 128) return FB_ERR_SHAPE;
  if (a->dtype != FB_BF16 && a->dtype != FB_F32) return FB_ERR_DTYPE;
  if ((int64_t)a->batch * a->seq_len * a->heads == 0) {
    set_last_launch_count(0);
    return FB_OK;
  }
  const bool gate = a->gate_x != nullptr;
  const bool xsa = a->xsa_alpha != nullptr;
  if (a->o == nullptr || (xsa && a->v == nullptr)) return FB_ERR_ARG;
  if (gate && (a->gate_channels < 1 || a->gate_channels > kMaxGate || a->gate_w == nullptr || a->gate_b == nullptr))
    return FB_ERR_ARG;
  if (!bwd && a->y == nullptr) return FB_ERR_ARG;
  if (bwd && (a->dy == nullptr || a->grad_o == nullptr || (xsa && (a->grad_v == nullptr || a->dalpha == nullptr)) ||
              (gate && a->du == nullptr)))
    return FB_ERR_ARG;
  const int n = a->dtype == FB_BF16 ? 8 : 4;
  auto strided_ok = [&](const void* ptr, const int64_t* st) {
    if (!al16(ptr) || st[3] != 1) return false;
    for (int i = 0; i < 3; ++i)
      if (st[i] % n != 0) return false;
    return true;
  };
  if (!strided_ok(a->o, a->o_stride) || (xsa && !strided_ok(a->v, a->v_stride))) return FB_ERR_ALIGN;
  if ((!bwd && !al16(a->y)) || (bwd && (!al16(a->dy) || !al16(a->grad_o) || (xsa && !al16(a->grad_v))))) return FB_ERR_ALIGN;
  HeadsParams p{};
  p.B = a->batch; p.H = a->heads; p.T = a->seq_len; p.hd = a->head_dim; p.eps = a->eps;
  p.o = a->o; p.v = a->v;
  for (int i = 0; i < 3; ++i) { p.os[i] = a->o_stride[i]; p.vs[i] = a->v_stride[i]; }
  p.alpha = a->xsa_alpha;
  p.gx = a->gate_x; p.c = a->gate_channels; p.gw = a->gate_w; p.gb = a->gate_b;
  p.y = a->y; p.dy = a->dy; p.dO = a->grad_o; p.dV = a->grad_v; p.dalpha = a->dalpha; p.du = a->du;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf = a->dtype == FB_BF16;
  switch (a->head_dim) {
    case 32: bf ? launch<__nv_bfloat16, 32>(p, bwd, s) : launch<float, 32>(p, bwd, s); break;
    case 64: bf ? launch<__nv_bfloat16, 64>(p, bwd, s) : launch<float, 64>(p, bwd, s); break;
    default: bf ? launch<__nv_bfloat16, 128>(p, bwd, s) : launch<float, 128>(p, bwd, s); break;
  }
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

int fb_heads_epilogue_fwd(const fb_heads_args* args, void* stream) { return fb::heads_epilogue(args, stream, false); }
int fb_heads_epilogue_bwd(const fb_heads_args* args, void* stream) { return fb::heads_epilogue(args, stream, true); }

}  // extern "C"
