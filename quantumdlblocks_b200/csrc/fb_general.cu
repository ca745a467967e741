// fb_general.cu -- the general flash-Born path: fp32-accumulating CUDA-core kernels.
//
// This path serves every configuration the tensor-core path does not: fp32 inputs (the
// reference's fp32 gate is max-abs 1e-4, which a single tf32 product cannot meet once p = a^2
// amplifies the error), head dims other than 64/128, and arbitrary element strides.  It keeps
// all arithmetic in fp32 (no rounding of P or dS to the input type), so it is also the most
// accurate CUDA statement of the reference math.
//
// Kernels (one (batch, head) per grid column, tiles of queries or keys per grid row):
//   general_fwd_kernel      O, Z                    flash_born.py:80-192 / :695-811
//   general_bwd_q_kernel    delta and dQ                                    :324-430 / :949-1061
//   general_bwd_kv_kernel   dK, dV, per-CTA parameter-gradient partials    :194-322 / :813-947
//
// delta.  The reference uses delta_i = sum_d dO_id O_id (:302).  Mathematically that equals
// sum_j w_ij (dO_i . v_j), and dS_ij = 2 a_ij (dO_i . v_j - delta_i) / Z_i subtracts the two.
// In a row whose weight sits on one small overlap a, any rounding difference between the two
// forms is amplified by ~2/a (Z ~ a^2); with fp32 O this alone exceeds 1e-4 in dQ at the C1
// configuration.  This path therefore computes delta_i = sum_j w_ij (dO_i . v_j) from the same
// recomputed dO.v products it later subtracts it from (a first pass of the dQ kernel), with its
// own Z'_i = sum_j p_ij + eps recomputed in the same pass (so it does not depend on how the
// forward rounded Z), and the cancellation is consistent; the dK/dV kernel reads both back.
//   general_param_reduce    fixed-order sum of the partials into dscale/dtau (deterministic;
//                           replaces the reference's atomic_add, :319-322)
#include <algorithm>

#include "fb_common.cuh"

namespace fb {
namespace {

constexpr int kThreads = 256;

struct GenArgs {
  int B, H, T, D;
  bool causal;
  int window;
  float eps, eps_base;
  Tensor4 q, k, v, o, dout, dq, dk, dv;
  float* z;
  int given_norm;  // backward: delta and Z from the given O and z (one term of a sum)
  int o_f32;       // O is fp32 (else the input type)
  const float* scale;
  int scale_per_head;
  const float* tau;
  int tau_per_head;
  const int32_t* doc;
  int64_t doc_s0, doc_s1;
  float* delta;     // B*H*T
  float* zb;        // B*H*T: Z' recomputed by the backward
  float* partials;  // [B*H*n_kv_tiles][2]
  int n_kv_tiles;
};

__device__ __forceinline__ int64_t off4(const Tensor4& t, int b, int h, int i, int d) {
  return (int64_t)b * t.s[0] + (int64_t)h * t.s[1] + (int64_t)i * t.s[2] + (int64_t)d * t.s[3];
}

template <class Map> struct MapFactory;
template <> struct MapFactory<PlainMap> {
  __device__ static PlainMap make(const GenArgs& a, int h) {
    return PlainMap{a.scale[a.scale_per_head ? h : 0]};
  }
};
template <> struct MapFactory<PurifiedMap> {
  __device__ static PurifiedMap make(const GenArgs& a, int h) {
    return PurifiedMap{a.scale[a.scale_per_head ? h : 0], a.tau[a.tau_per_head ? h : 0], a.eps_base};
  }
};

__device__ __forceinline__ int doc_at(const GenArgs& a, int b, int i) {
  if (a.doc == nullptr || i >= a.T) return 0;
  return a.doc[(int64_t)b * a.doc_s0 + (int64_t)i * a.doc_s1];
}

// Load rows [r0, r0+R) of a (b,h) slice into smem [R][KD+1] as fp32, zero-padding r >= T, d >= D.
template <typename T, int KD>
__device__ __forceinline__ void load_rows(float* dst, const Tensor4& t, int b, int h, int r0, int R, int Tn, int D) {
  const T* base = reinterpret_cast<const T*>(t.ptr);
  for (int idx = threadIdx.x; idx < R * KD; idx += kThreads) {
    int r = idx / KD, d = idx - r * KD;
    float x = 0.f;
    if (r0 + r < Tn && d < D) x = to_f32<T>(base[off4(t, b, h, r0 + r, d)]);
    dst[r * (KD + 1) + d] = x;
  }
}

// Key range [lo, hi) that can hold valid keys for queries [m0, m1).
__device__ __forceinline__ void key_range(const GenArgs& a, int m0, int m1, int& lo, int& hi) {
  lo = 0;
  hi = a.causal ? min(a.T, m1) : a.T;
  if (a.window > 0) lo = max(0, m0 - a.window + 1);
}
// Query range [lo, hi) that can hold valid queries for keys [n0, n1).
__device__ __forceinline__ void query_range(const GenArgs& a, int n0, int n1, int& lo, int& hi) {
  lo = a.causal ? n0 : 0;
  hi = a.T;
  if (a.window > 0) hi = min(a.T, n1 - 1 + a.window);
}

// ------------------------------------------------------------------------------------------
// Forward: BM=64 queries per CTA, key tiles of BN=32.
// ------------------------------------------------------------------------------------------
template <typename T, typename TO, int KD, class Map>
__global__ void __launch_bounds__(kThreads) general_fwd_kernel(GenArgs a) {
  constexpr int BM = 64, BN = 32, LD = KD + 1, LP = BN + 1;
  extern __shared__ float smem[];
  float* Qs = smem;
  float* Ks = Qs + BM * LD;
  float* Vs = Ks + BN * LD;
  float* Ps = Vs + BN * LD;
  int* docq = reinterpret_cast<int*>(Ps + BM * LP);
  int* dock = docq + BM;

  const int tile = gridDim.x - 1 - blockIdx.x;  // heaviest (latest) causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int m0 = tile * BM;
  const int tid = threadIdx.x;
  const Map map = MapFactory<Map>::make(a, h);

  load_rows<T, KD>(Qs, a.q, b, h, m0, BM, a.T, a.D);
  for (int r = tid; r < BM; r += kThreads) docq[r] = doc_at(a, b, m0 + r);

  const int orow = tid >> 2;   // 0..63
  const int ocol = tid & 3;    // owns columns ocol + 4 j
  float oacc[KD / 4];
#pragma unroll
  for (int j = 0; j < KD / 4; ++j) oacc[j] = 0.f;
  float zrow = 0.f;

  const int srow = (tid >> 4) * 4;  // 4 query rows
  const int scol = (tid & 15) * 2;  // 2 key columns

  int lo, hi;
  key_range(a, m0, min(a.T, m0 + BM), lo, hi);
  for (int n0 = lo; n0 < hi; n0 += BN) {
    __syncthreads();
    load_rows<T, KD>(Ks, a.k, b, h, n0, BN, a.T, a.D);
    load_rows<T, KD>(Vs, a.v, b, h, n0, BN, a.T, a.D);
    for (int r = tid; r < BN; r += kThreads) dock[r] = doc_at(a, b, n0 + r);
    __syncthreads();

    float acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.f;
#pragma unroll 8
    for (int d = 0; d < KD; ++d) {
      float k0 = Ks[(scol + 0) * LD + d], k1 = Ks[(scol + 1) * LD + d];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float qv = Qs[(srow + i) * LD + d];
        acc[i][0] = fmaf(qv, k0, acc[i][0]);
        acc[i][1] = fmaf(qv, k1, acc[i][1]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        int qi = m0 + srow + i, kj = n0 + scol + j;
        bool valid = pair_valid(qi, kj, a.T, a.causal, a.window, docq[srow + i], dock[scol + j]);
        Ps[(srow + i) * LP + scol + j] = map.prob(acc[i][j], valid);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int n = 0; n < BN; ++n) {
      float pv = Ps[orow * LP + n];
      zrow += pv;
#pragma unroll
      for (int j = 0; j < KD / 4; ++j) oacc[j] = fmaf(pv, Vs[n * LD + ocol + 4 * j], oacc[j]);
    }
  }

  const int qi = m0 + orow;
  if (qi < a.T) {
    const float zden = zrow + a.eps;
    TO* o = reinterpret_cast<TO*>(const_cast<void*>(a.o.ptr));
#pragma unroll
    for (int j = 0; j < KD / 4; ++j) {
      int c = ocol + 4 * j;
      if (c < a.D) o[off4(a.o, b, h, qi, c)] = from_f32<TO>(oacc[j] / zden);
    }
    if (ocol == 0) a.z[((int64_t)b * a.H + h) * a.T + qi] = zden;
  }
}

// ------------------------------------------------------------------------------------------
// Backward, key-tile parallel: dK, dV and the per-CTA parameter-gradient partials.
// BN=32 keys per CTA; query tiles of BM=32.
// ------------------------------------------------------------------------------------------
template <typename T, int KD, class Map>
__global__ void __launch_bounds__(kThreads) general_bwd_kv_kernel(GenArgs a) {
  constexpr int BN = 32, BM = 32, LD = KD + 1, LP = BM + 1;
  extern __shared__ float smem[];
  float* Ks = smem;
  float* Vs = Ks + BN * LD;
  float* Qs = Vs + BN * LD;
  float* dOs = Qs + BM * LD;
  float* Ws = dOs + BM * LD;   // [BN][BM]  w^T
  float* Gs = Ws + BN * LP;    // [BN][BM]  (dL/draw)^T
  float* zq = Gs + BN * LP;    // [BM]
  float* dq_ = zq + BM;        // [BM] delta
  int* docq = reinterpret_cast<int*>(dq_ + BM);
  int* dock = docq + BM;
  float* red = reinterpret_cast<float*>(dock + BN);  // [2][kThreads/32]

  const int tile = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int n0 = tile * BN;
  const int tid = threadIdx.x;
  const Map map = MapFactory<Map>::make(a, h);
  const int64_t bh = (int64_t)b * a.H + h;

  load_rows<T, KD>(Ks, a.k, b, h, n0, BN, a.T, a.D);
  load_rows<T, KD>(Vs, a.v, b, h, n0, BN, a.T, a.D);
  for (int r = tid; r < BN; r += kThreads) dock[r] = doc_at(a, b, n0 + r);

  const int arow = tid >> 3;  // key row 0..31
  const int acol = tid & 7;   // columns acol + 8 j
  float dk[KD / 8], dv[KD / 8];
#pragma unroll
  for (int j = 0; j < KD / 8; ++j) dk[j] = dv[j] = 0.f;
  float g1 = 0.f, g2 = 0.f;

  const int pn = (tid >> 4) * 2;  // 2 keys
  const int pm = (tid & 15) * 2;  // 2 queries

  int lo, hi;
  query_range(a, n0, min(a.T, n0 + BN), lo, hi);
  for (int m0 = lo; m0 < hi; m0 += BM) {
    __syncthreads();
    load_rows<T, KD>(Qs, a.q, b, h, m0, BM, a.T, a.D);
    load_rows<T, KD>(dOs, a.dout, b, h, m0, BM, a.T, a.D);
    for (int r = tid; r < BM; r += kThreads) {
      int qi = m0 + r;
      zq[r] = qi < a.T ? a.zb[bh * a.T + qi] : 1.f;
      dq_[r] = qi < a.T ? a.delta[bh * a.T + qi] : 0.f;
      docq[r] = doc_at(a, b, qi);
    }
    __syncthreads();

    float s[2][2], dp[2][2];
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int y = 0; y < 2; ++y) s[x][y] = dp[x][y] = 0.f;
#pragma unroll 8
    for (int d = 0; d < KD; ++d) {
      float k0 = Ks[(pn + 0) * LD + d], k1 = Ks[(pn + 1) * LD + d];
      float v0 = Vs[(pn + 0) * LD + d], v1 = Vs[(pn + 1) * LD + d];
      float q0 = Qs[(pm + 0) * LD + d], q1 = Qs[(pm + 1) * LD + d];
      float o0 = dOs[(pm + 0) * LD + d], o1 = dOs[(pm + 1) * LD + d];
      s[0][0] = fmaf(k0, q0, s[0][0]); s[0][1] = fmaf(k0, q1, s[0][1]);
      s[1][0] = fmaf(k1, q0, s[1][0]); s[1][1] = fmaf(k1, q1, s[1][1]);
      dp[0][0] = fmaf(v0, o0, dp[0][0]); dp[0][1] = fmaf(v0, o1, dp[0][1]);
      dp[1][0] = fmaf(v1, o0, dp[1][0]); dp[1][1] = fmaf(v1, o1, dp[1][1]);
    }
#pragma unroll
    for (int x = 0; x < 2; ++x) {
#pragma unroll
      for (int y = 0; y < 2; ++y) {
        int kj = n0 + pn + x, qi = m0 + pm + y;
        bool valid = qi < a.T && pair_valid(qi, kj, a.T, a.causal, a.window, docq[pm + y], dock[pn + x]);
        float zi = zq[pm + y];
        float p = map.prob(s[x][y], valid);
        float dpv = (dp[x][y] - dq_[pm + y]) / zi;
        Ws[(pn + x) * LP + pm + y] = p / zi;
        Gs[(pn + x) * LP + pm + y] = map.grad(s[x][y], valid, dpv, g1, g2);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int m = 0; m < BM; ++m) {
      float w = Ws[arow * LP + m], g = Gs[arow * LP + m];
#pragma unroll
      for (int j = 0; j < KD / 8; ++j) {
        dv[j] = fmaf(w, dOs[m * LD + acol + 8 * j], dv[j]);
        dk[j] = fmaf(g, Qs[m * LD + acol + 8 * j], dk[j]);
      }
    }
  }

  const int kj = n0 + arow;
  if (kj < a.T) {
    T* dK = reinterpret_cast<T*>(const_cast<void*>(a.dk.ptr));
    T* dV = reinterpret_cast<T*>(const_cast<void*>(a.dv.ptr));
#pragma unroll
    for (int j = 0; j < KD / 8; ++j) {
      int c = acol + 8 * j;
      if (c < a.D) {
        dK[off4(a.dk, b, h, kj, c)] = from_f32<T>(dk[j]);
        dV[off4(a.dv, b, h, kj, c)] = from_f32<T>(dv[j]);
      }
    }
  }
  // block reduction of the parameter-gradient partials (fixed order -> deterministic)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    g1 += __shfl_xor_sync(0xffffffffu, g1, o);
    g2 += __shfl_xor_sync(0xffffffffu, g2, o);
  }
  __syncthreads();
  if ((tid & 31) == 0) {
    red[tid >> 5] = g1;
    red[kThreads / 32 + (tid >> 5)] = g2;
  }
  __syncthreads();
  if (tid == 0) {
    float t1 = 0.f, t2 = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) {
      t1 += red[w];
      t2 += red[kThreads / 32 + w];
    }
    float* part = a.partials + (bh * a.n_kv_tiles + tile) * 2;
    part[0] = t1;
    part[1] = t2;
  }
}

// ------------------------------------------------------------------------------------------
// Backward, query-tile parallel: delta (pass 1) then dQ (pass 2).  BM=32 queries per CTA;
// key tiles of BN=32.  Must run before the key-tile kernel, which reads delta.
// ------------------------------------------------------------------------------------------
template <typename T, int KD, class Map>
__global__ void __launch_bounds__(kThreads) general_bwd_q_kernel(GenArgs a) {
  constexpr int BM = 32, BN = 32, LD = KD + 1, LP = BN + 1;
  extern __shared__ float smem[];
  float* Qs = smem;
  float* dOs = Qs + BM * LD;
  float* Ks = dOs + BM * LD;
  float* Vs = Ks + BN * LD;
  float* Gs = Vs + BN * LD;  // [BM][BN]
  float* zq = Gs + BM * LP;
  float* dq_ = zq + BM;
  int* docq = reinterpret_cast<int*>(dq_ + BM);
  int* dock = docq + BM;

  const int tile = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int m0 = tile * BM;
  const int tid = threadIdx.x;
  const Map map = MapFactory<Map>::make(a, h);
  const int64_t bh = (int64_t)b * a.H + h;

  load_rows<T, KD>(Qs, a.q, b, h, m0, BM, a.T, a.D);
  load_rows<T, KD>(dOs, a.dout, b, h, m0, BM, a.T, a.D);
  for (int r = tid; r < BM; r += kThreads) {
    int qi = m0 + r;
    zq[r] = 1.f;  // replaced by Z' after pass 1
    dq_[r] = 0.f;
    docq[r] = doc_at(a, b, qi);
  }

  const int arow = tid >> 3;
  const int acol = tid & 7;
  const int pm = (tid >> 4) * 2;  // 2 queries (shared by the 16 lanes of a half-warp)
  const int pn = (tid & 15) * 2;  // 2 keys

  int lo, hi;
  key_range(a, m0, min(a.T, m0 + BM), lo, hi);

  // S = Q K^T and dP = dO V^T for this thread's 2x2 pairs of the current key tile
  auto pair_products = [&](float (&s)[2][2], float (&dp)[2][2]) {
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int y = 0; y < 2; ++y) s[x][y] = dp[x][y] = 0.f;
#pragma unroll 8
    for (int d = 0; d < KD; ++d) {
      float q0 = Qs[(pm + 0) * LD + d], q1 = Qs[(pm + 1) * LD + d];
      float o0 = dOs[(pm + 0) * LD + d], o1 = dOs[(pm + 1) * LD + d];
      float k0 = Ks[(pn + 0) * LD + d], k1 = Ks[(pn + 1) * LD + d];
      float v0 = Vs[(pn + 0) * LD + d], v1 = Vs[(pn + 1) * LD + d];
      s[0][0] = fmaf(q0, k0, s[0][0]); s[0][1] = fmaf(q0, k1, s[0][1]);
      s[1][0] = fmaf(q1, k0, s[1][0]); s[1][1] = fmaf(q1, k1, s[1][1]);
      dp[0][0] = fmaf(o0, v0, dp[0][0]); dp[0][1] = fmaf(o0, v1, dp[0][1]);
      dp[1][0] = fmaf(o1, v0, dp[1][0]); dp[1][1] = fmaf(o1, v1, dp[1][1]);
    }
  };
  auto load_keys = [&](int n0) {
    __syncthreads();
    load_rows<T, KD>(Ks, a.k, b, h, n0, BN, a.T, a.D);
    load_rows<T, KD>(Vs, a.v, b, h, n0, BN, a.T, a.D);
    for (int r = tid; r < BN; r += kThreads) dock[r] = doc_at(a, b, n0 + r);
    __syncthreads();
  };

  if (a.given_norm) {
    // one term of a sum of score families: delta_i = dO_i . O_i and Z_i of the whole sum
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31;
    for (int r = warp; r < BM; r += kThreads / 32) {
      const int qi = m0 + r;
      float acc = 0.f;
      if (qi < a.T) {
        for (int c = lane; c < a.D; c += 32) {
          const int64_t off = off4(a.o, b, h, qi, c);
          const float ov = a.o_f32 ? reinterpret_cast<const float*>(a.o.ptr)[off]
                                   : to_f32<T>(reinterpret_cast<const T*>(a.o.ptr)[off]);
          acc = fmaf(dOs[r * LD + c], ov, acc);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        dq_[r] = acc;
        zq[r] = qi < a.T ? a.z[bh * a.T + qi] : 1.f;
      }
    }
    __syncthreads();
  }
  // pass 1: Z'_i = sum_j p_ij + eps and delta_i = sum_j (p_ij / Z'_i) (dO_i . v_j)
  float dsum[2] = {0.f, 0.f}, zsum[2] = {0.f, 0.f};
  for (int n0 = a.given_norm ? hi : lo; n0 < hi; n0 += BN) {
    load_keys(n0);
    float s[2][2], dp[2][2];
    pair_products(s, dp);
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int y = 0; y < 2; ++y) {
        int qi = m0 + pm + x, kj = n0 + pn + y;
        bool valid = qi < a.T && pair_valid(qi, kj, a.T, a.causal, a.window, docq[pm + x], dock[pn + y]);
        const float pv = map.prob(s[x][y], valid);
        dsum[x] += pv * dp[x][y];
        zsum[x] += pv;
      }
  }
#pragma unroll
  for (int x = 0; x < 2; ++x) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      dsum[x] += __shfl_xor_sync(0xffffffffu, dsum[x], o);
      zsum[x] += __shfl_xor_sync(0xffffffffu, zsum[x], o);
    }
  }
  __syncthreads();
  if ((tid & 15) == 0 && !a.given_norm) {
#pragma unroll
    for (int x = 0; x < 2; ++x) {
      const float zz = zsum[x] + a.eps;
      zq[pm + x] = zz;
      dq_[pm + x] = dsum[x] / zz;
    }
  }
  __syncthreads();
  for (int r = tid; r < BM; r += kThreads)
    if (m0 + r < a.T) {
      a.delta[bh * a.T + m0 + r] = dq_[r];
      a.zb[bh * a.T + m0 + r] = zq[r];
    }

  // pass 2: dQ = sum_j dL/draw_ij k_j
  float dqa[KD / 8];
#pragma unroll
  for (int j = 0; j < KD / 8; ++j) dqa[j] = 0.f;
  float g1 = 0.f, g2 = 0.f;  // parameter grads come from the key-tile kernel; discarded here
  for (int n0 = lo; n0 < hi; n0 += BN) {
    load_keys(n0);
    float s[2][2], dp[2][2];
    pair_products(s, dp);
#pragma unroll
    for (int x = 0; x < 2; ++x) {
#pragma unroll
      for (int y = 0; y < 2; ++y) {
        int qi = m0 + pm + x, kj = n0 + pn + y;
        bool valid = qi < a.T && pair_valid(qi, kj, a.T, a.causal, a.window, docq[pm + x], dock[pn + y]);
        float dpv = (dp[x][y] - dq_[pm + x]) / zq[pm + x];
        Gs[(pm + x) * LP + pn + y] = map.grad(s[x][y], valid, dpv, g1, g2);
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int n = 0; n < BN; ++n) {
      float g = Gs[arow * LP + n];
#pragma unroll
      for (int j = 0; j < KD / 8; ++j) dqa[j] = fmaf(g, Ks[n * LD + acol + 8 * j], dqa[j]);
    }
  }
  const int qi = m0 + arow;
  if (qi < a.T) {
    T* dQ = reinterpret_cast<T*>(const_cast<void*>(a.dq.ptr));
#pragma unroll
    for (int j = 0; j < KD / 8; ++j) {
      int c = acol + 8 * j;
      if (c < a.D) dQ[off4(a.dq, b, h, qi, c)] = from_f32<T>(dqa[j]);
    }
  }
}

// Sum per-(b,h,tile) partials into dscale / dtau in a fixed order (deterministic).
// Per-head parameters: one thread per head.  Shared parameters: thread 0 sums all heads.
__global__ void general_param_reduce(GenArgs a, float* dscale, float* dtau) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  auto head_sum = [&](int hh, float& t1, float& t2) {
    for (int b = 0; b < a.B; ++b) {
      const float* part = a.partials + ((int64_t)b * a.H + hh) * a.n_kv_tiles * 2;
      for (int t = 0; t < a.n_kv_tiles; ++t) {
        t1 += part[2 * t];
        t2 += part[2 * t + 1];
      }
    }
  };
  if (h < a.H) {
    float t1 = 0.f, t2 = 0.f;
    head_sum(h, t1, t2);
    if (a.scale_per_head) dscale[h] += t1;
    if (dtau != nullptr && a.tau_per_head) dtau[h] += t2;
  }
  if (h == 0 && (!a.scale_per_head || (dtau != nullptr && !a.tau_per_head))) {
    float s1 = 0.f, s2 = 0.f;
    for (int hh = 0; hh < a.H; ++hh) head_sum(hh, s1, s2);
    if (!a.scale_per_head) dscale[0] += s1;
    if (dtau != nullptr && !a.tau_per_head) dtau[0] += s2;
  }
}

GenArgs make_args(const Problem& p) {
  GenArgs a{};
  a.B = p.B; a.H = p.H; a.T = p.T; a.D = p.D;
  a.causal = p.causal; a.window = p.window; a.eps = p.eps; a.eps_base = p.eps_base;
  a.q = p.q; a.k = p.k; a.v = p.v; a.o = p.o; a.dout = p.dout; a.dq = p.dq; a.dk = p.dk; a.dv = p.dv;
  a.z = p.z;
  a.given_norm = p.given_norm ? 1 : 0;
  a.o_f32 = p.out_dtype == FB_F32 ? 1 : 0;
  a.scale = p.scale; a.scale_per_head = p.scale_per_head;
  a.tau = p.tau; a.tau_per_head = p.tau_per_head;
  a.doc = p.doc; a.doc_s0 = p.doc_s[0]; a.doc_s1 = p.doc_s[1];
  return a;
}

int kd_bucket(int D) { return D <= 32 ? 32 : D <= 64 ? 64 : D <= 128 ? 128 : 256; }

template <typename K>
int launch(K kernel, dim3 grid, size_t smem, cudaStream_t s, const GenArgs& a) {
  if (smem > 48 * 1024) {
    cudaError_t e = set_smem_limit_once(reinterpret_cast<const void*>(kernel), (int)smem);
    if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  }
  kernel<<<grid, kThreads, smem, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  return FB_OK;
}

// Dynamic shared memory of each kernel (floats + ints), matching the carve-up in the kernels.
size_t fwd_smem(int KD) { return (size_t)(128 * (KD + 1) + 64 * 33) * 4 + (64 + 32) * 4; }
size_t kv_smem(int KD) {
  return (size_t)(4 * 32 * (KD + 1) + 2 * 32 * 33 + 2 * 32) * 4 + (32 + 32) * 4 + 2 * (kThreads / 32) * 4;
}
size_t q_smem(int KD) { return (size_t)(4 * 32 * (KD + 1) + 32 * 33 + 2 * 32) * 4 + (32 + 32) * 4; }

template <typename T, typename TO, int KD, class Map>
int fwd_typed(const GenArgs& a, cudaStream_t s) {
  dim3 grid((a.T + 63) / 64, a.H, a.B);
  return launch(general_fwd_kernel<T, TO, KD, Map>, grid, fwd_smem(KD), s, a);
}

template <typename T, typename TO, class Map>
int fwd_kd(const GenArgs& a, cudaStream_t s) {
  switch (kd_bucket(a.D)) {
    case 32: return fwd_typed<T, TO, 32, Map>(a, s);
    case 64: return fwd_typed<T, TO, 64, Map>(a, s);
    case 128: return fwd_typed<T, TO, 128, Map>(a, s);
    default: return fwd_typed<T, TO, 256, Map>(a, s);
  }
}

template <typename T, typename TO, int KD, class Map>
int bwd_typed(const GenArgs& a, const Problem& p, cudaStream_t s, int* launches) {
  int rc;
  dim3 gq((a.T + 31) / 32, a.H, a.B);
  if ((rc = launch(general_bwd_q_kernel<T, KD, Map>, gq, q_smem(KD), s, a)) != FB_OK) return rc;
  dim3 gkv((a.T + 31) / 32, a.H, a.B);
  if ((rc = launch(general_bwd_kv_kernel<T, KD, Map>, gkv, kv_smem(KD), s, a)) != FB_OK) return rc;
  *launches = 2;
  if (!p.given_norm) {  // a term of a sum leaves the parameter gradients to its caller
    general_param_reduce<<<(a.H + 127) / 128, 128, 0, s>>>(a, p.dscale, p.purified ? p.dtau : nullptr);
    *launches = 3;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  return FB_OK;
}

template <typename T, typename TO, class Map>
int bwd_kd(const GenArgs& a, const Problem& p, cudaStream_t s, int* launches) {
  switch (kd_bucket(a.D)) {
    case 32: return bwd_typed<T, TO, 32, Map>(a, p, s, launches);
    case 64: return bwd_typed<T, TO, 64, Map>(a, p, s, launches);
    case 128: return bwd_typed<T, TO, 128, Map>(a, p, s, launches);
    default: return bwd_typed<T, TO, 256, Map>(a, p, s, launches);
  }
}

template <class Map>
int fwd_dispatch(const GenArgs& a, const Problem& p, cudaStream_t s) {
  if (p.dtype == FB_F32) return fwd_kd<float, float, Map>(a, s);
  if (p.dtype == FB_F16) {
    return p.out_dtype == FB_F32 ? fwd_kd<__half, float, Map>(a, s) : fwd_kd<__half, __half, Map>(a, s);
  }
  return p.out_dtype == FB_F32 ? fwd_kd<__nv_bfloat16, float, Map>(a, s)
                               : fwd_kd<__nv_bfloat16, __nv_bfloat16, Map>(a, s);
}

template <class Map>
int bwd_dispatch(const GenArgs& a, const Problem& p, cudaStream_t s, int* launches) {
  // the general backward never reads O (delta comes from its own first pass)
  if (p.dtype == FB_F32) return bwd_kd<float, float, Map>(a, p, s, launches);
  if (p.dtype == FB_F16) return bwd_kd<__half, __half, Map>(a, p, s, launches);
  return bwd_kd<__nv_bfloat16, __nv_bfloat16, Map>(a, p, s, launches);
}

}  // namespace

int general_fwd(const Problem& p, cudaStream_t s, int* launches) {
  GenArgs a = make_args(p);
  int rc = p.purified ? fwd_dispatch<PurifiedMap>(a, p, s) : fwd_dispatch<PlainMap>(a, p, s);
  if (rc == FB_OK) *launches = 1;
  return rc;
}

size_t general_bwd_workspace(const Problem& p) {
  const size_t n_kv = (size_t)((p.T + 31) / 32);
  size_t delta = (size_t)p.B * p.H * p.T * sizeof(float);
  delta = (delta + 255) & ~(size_t)255;
  return 2 * delta + (size_t)p.B * p.H * n_kv * 2 * sizeof(float);
}

int general_bwd(const Problem& p, cudaStream_t s, int* launches) {
  GenArgs a = make_args(p);
  size_t delta = (size_t)p.B * p.H * p.T * sizeof(float);
  delta = (delta + 255) & ~(size_t)255;
  a.delta = reinterpret_cast<float*>(p.ws);
  a.zb = reinterpret_cast<float*>(reinterpret_cast<char*>(p.ws) + delta);
  a.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(p.ws) + 2 * delta);
  a.n_kv_tiles = (p.T + 31) / 32;
  return p.purified ? bwd_dispatch<PurifiedMap>(a, p, s, launches) : bwd_dispatch<PlainMap>(a, p, s, launches);
}

}  // namespace fb
