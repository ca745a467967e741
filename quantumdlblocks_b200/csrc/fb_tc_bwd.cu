// fb_tc_bwd.cu -- flash-Born backward on the tcgen05 tensor cores (sm_100a), head dim 64.
//
// Three launches (all on the caller's stream):
//   1. bwd_prep_kernel   delta_i / Z_i with delta_i = sum_d dO_id O_id, 1/Z_i (per-head rows padded
//                        to a multiple of 64), and a zeroed fp32 dQ accumulator (workspace)
//   2. tc_bwd_kernel     one CTA per (batch, head, 128-key tile); walks the 64-query tiles that
//                        can hold valid pairs and accumulates dK, dV in TMEM; dQ partials are
//                        reduced into the fp32 accumulator with TMA tensor reduce-add
//   3. bwd_post_kernel   dQ = accumulator -> input dtype
//   4. bwd_param_kernel  fixed-order sums into dscale / dtau from the pre-pass's closed-form
//                        sums and the main kernel's per-CTA partials
//
// Per (key tile, query tile) the main kernel runs the five products the algorithm needs
// (the reference's two kernels run six, flash_born.py:267-312 and :398-427):
//   S^T  = K Q^T        M=128 keys, N=64 queries, K=64   A=K (smem K-major), B=Q (smem K-major)
//   dP^T = V dO^T       same shape                        A=V, B=dO
//   pointwise (thread = key row): a = relu(scale raw), p = a^2, W = p / Z_i,
//     dP = (dP^T - delta_i) / Z_i, G = dL/draw = 2 a dP scale (masked; purified: 4u^3 dP gamma +
//     2 eps_base b dP) -> W^T, G^T into TMEM (bf16, aliasing S^T / dP^T) and G into smem
//   dV  += W^T dO       M=128, N=64, K=64 queries         A=W^T (TMEM), B=dO (smem MN-major)
//   dK  += G^T Q        same                              A=G^T (TMEM), B=Q (smem MN-major)
//   dQ_t = G K          M=64 queries, N=64, K=128 keys    A=G (smem MN-major), B=K (smem MN-major)
//
// Warps (320 threads): 0 TMA producer, 1 TMEM owner + MMA issuer, 2-9 two pointwise warpgroups
// (key rows; group g takes the query tiles t with t % 2 == g, i.e. TMEM buffer g, so the two
// groups' latency chains interleave).  Before each tile a group drains the dQ partial of its
// previous tile (TMEM -> swizzled smem -> TMA tensor reduce-add into the fp32 accumulator).  S^T/dP^T/dQ are double-buffered in TMEM so
// the products of query tile t+1 overlap the pointwise work of tile t.
//
// TMEM columns: S^T[0..1] 0/64, dP^T[0..1] 128/192, dV 256, dK 320, dQ[0..1] 384/448.
#include <cuda.h>

#include "fb_common.cuh"
#include "fb_sm100.cuh"

namespace fb {
namespace {

using namespace sm100;

constexpr int kBN = 128;  // keys per CTA
constexpr int kBM = 64;   // queries per step
constexpr int kD = 64;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTS = 0, kTdP = 128, kTdV = 256, kTdK = 320, kTdQ = 384;

// shared memory carve-up (bytes from the 1024-aligned base)
constexpr uint32_t kSK = 0;                    // K tile 128 x 64 bf16     16 KB
constexpr uint32_t kSV = 16384;                // V tile                    16 KB
constexpr uint32_t kSQ = 32768;                // Q stages [2] 64 x 64       8 KB each
constexpr uint32_t kSdO = 49152;               // dO stages [2]              8 KB each
constexpr uint32_t kSG = 65536;                // G [2] 128 keys x 64 q      16 KB each
constexpr uint32_t kSStg = 98304;              // dQ staging [4 quadrants][2 groups] two 16 x 32 fp32 swizzled boxes
constexpr uint32_t kSVec = 131072;             // dlz[2][64] (delta / Z), zinv[2][64] (1 / Z) fp32
constexpr uint32_t kSDoc = kSVec + 1024;       // query doc ids [8 warps][64] int32
constexpr uint32_t kSBar = kSDoc + 2048;       // barriers + flags
constexpr uint32_t kSmemBytes = kSBar + 256;

struct BwdParams {
  int B, H, T, Tpad;
  int causal, window;
  float eps_base;
  const float* scale;
  int scale_per_head;
  const float* tau;
  int tau_per_head;
  const int32_t* doc;
  int64_t doc_s0, doc_s1;
  __nv_bfloat16* dk;
  int64_t dk_s0, dk_s1, dk_s2;
  __nv_bfloat16* dv;
  int64_t dv_s0, dv_s1, dv_s2;
  const float* dlz;    // [BH][Tpad]  delta_i / Z_i
  const float* zinv;   // [BH][Tpad]  1 / Z_i
  float* dq_acc;       // [BH][Tpad][64]
  float* partials;     // [BH][n_kv][2]
  int n_kv;
  int* status;
};

template <class Map> struct BwdMap;
template <> struct BwdMap<PlainMapNoParam> {
  __device__ static PlainMapNoParam make(const BwdParams& p, int h) {
    PlainMapNoParam m;
    m.scale = p.scale[p.scale_per_head ? h : 0];
    return m;
  }
};
template <> struct BwdMap<PurifiedMapTC> {
  __device__ static PurifiedMapTC make(const BwdParams& p, int h) {
    PurifiedMapTC m;
    m.gamma = p.scale[p.scale_per_head ? h : 0];
    m.tau = p.tau[p.tau_per_head ? h : 0];
    m.eps_base = p.eps_base;
    return m;
  }
};

// Query tiles [m_first, m_first + 64 * count) that can hold valid pairs for keys [n0, n0 + kBN).
__device__ __forceinline__ void query_tiles(const BwdParams& p, int n0, int& m_first, int& count) {
  int lo = p.causal ? n0 : 0;
  int hi = p.T;
  if (p.window > 0) hi = min(p.T, n0 + kBN - 1 + p.window);
  lo = (lo / kBM) * kBM;
  m_first = lo;
  count = hi > lo ? (hi - lo + kBM - 1) / kBM : 0;
}

template <class Map, bool kHasDoc>
__global__ void __launch_bounds__(kThreads, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
                  const __grid_constant__ CUtensorMap tmDQ, const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;     // [2]
  uint64_t* q_empty = bars + 3;    // [2]
  uint64_t* sdp_full = bars + 5;   // [2]
  uint64_t* wg_full = bars + 7;    // [2]
  uint64_t* mma_done = bars + 9;   // [2]
  uint64_t* dq_full = bars + 11;   // [2]
  uint64_t* dq_empty = bars + 13;  // [2]
  uint64_t* acc_full = bars + 15;
  uint64_t* drain = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 18);
  float* red = reinterpret_cast<float*>(bars + 19);  // [8 pointwise warps][2]
  float* vdlz = reinterpret_cast<float*>(smem + kSVec);          // [2][64]
  float* vzinv = reinterpret_cast<float*>(smem + kSVec + 512);   // [2][64]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ktile = blockIdx.x;  // early key tiles see the most queries under a causal mask
  const int h = blockIdx.y, b = blockIdx.z;
  const int n0 = ktile * kBN;
  const int64_t bh = (int64_t)b * p.H + h;
  int m_first, n_tiles;
  query_tiles(p, n0, m_first, n_tiles);
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&sdp_full[i], 1);
      mbar_init(&wg_full[i], 128);
      mbar_init(&mma_done[i], 1);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], 128);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmdO);
    prefetch_tensormap(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      bool ok = true;
      int issued = 0;
      mbar_arrive_expect_tx(kv_full, 2 * kBN * kD * 2);
      tma_load_4d(smem + kSK, &tmK, kv_full, 0, n0, h, b);
      tma_load_4d(smem + kSV, &tmV, kv_full, 0, n0, h, b);
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int st = t & 1;
        if (t >= 2) ok = mbar_wait(&q_empty[st], ((t >> 1) - 1) & 1, wc, 21);
        if (!ok) break;
        const int m0 = m_first + t * kBM;
        mbar_arrive_expect_tx(&q_full[st], 2 * kBM * kD * 2 + 2 * kBM * 4);
        tma_load_4d(smem + kSQ + st * 8192, &tmQ, &q_full[st], 0, m0, h, b);
        tma_load_4d(smem + kSdO + st * 8192, &tmdO, &q_full[st], 0, m0, h, b);
        bulk_load(vdlz + st * kBM, p.dlz + bh * p.Tpad + m0, kBM * 4, &q_full[st]);
        bulk_load(vzinv + st * kBM, p.zinv + bh * p.Tpad + m0, kBM * 4, &q_full[st]);
        issued = t + 1;
      }
      if (!ok) {
        mbar_wait_drain(kv_full, 0);
        for (int t = max(0, issued - 2); t < issued; ++t) mbar_wait_drain(&q_full[t & 1], (t >> 1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idSdP = idesc_f16(1, 0, 0, kBM, kBN);  // N = 64 queries, M = 128 keys
      constexpr uint32_t idAcc = idesc_f16(1, 0, 1, kD, kBN);   // A TMEM, B MN-major, N = 64
      constexpr uint32_t idDQ = idesc_f16(1, 1, 1, kD, kBM);    // A, B MN-major, M = 64, N = 64
      const uint32_t sK = smem_u32(smem + kSK), sV = smem_u32(smem + kSV);
      bool ok = mbar_wait(kv_full, 0, wc, 22);
      for (int t = 0; t <= n_tiles && ok; ++t) {
        if (t < n_tiles) {
          const int sb = t & 1;
          ok = mbar_wait(&q_full[sb], (t >> 1) & 1, wc, 23);
          if (ok && t >= 2) ok = mbar_wait(&mma_done[sb], ((t - 2) >> 1) & 1, wc, 24);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sQ = smem_u32(smem + kSQ + sb * 8192), sdO = smem_u32(smem + kSdO + sb * 8192);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            mma_ss(tmem + kTS + sb * kBM, sdesc_sw128(sK + kk * 32, 16, 1024), sdesc_sw128(sQ + kk * 32, 16, 1024),
                   idSdP, kk > 0);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            mma_ss(tmem + kTdP + sb * kBM, sdesc_sw128(sV + kk * 32, 16, 1024),
                   sdesc_sw128(sdO + kk * 32, 16, 1024), idSdP, kk > 0);
          mma_commit(&sdp_full[sb]);
        }
        if (t >= 1) {
          const int u = t - 1, su = u & 1;
          ok = mbar_wait(&wg_full[su], (u >> 1) & 1, wc, 25);
          if (ok && u >= 2) ok = mbar_wait(&dq_empty[su], ((u - 2) >> 1) & 1, wc, 26);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sQ = smem_u32(smem + kSQ + su * 8192), sdO = smem_u32(smem + kSdO + su * 8192);
          const uint32_t sG = smem_u32(smem + kSG + su * 16384);
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)  // 16 queries per step: 8 packed TMEM columns, 2048 B of dO
            mma_ts(tmem + kTdV, tmem + kTS + su * kBM + kk * 8, sdesc_sw128(sdO + kk * 2048, 8192, 1024), idAcc,
                   (u > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            mma_ts(tmem + kTdK, tmem + kTdP + su * kBM + kk * 8, sdesc_sw128(sQ + kk * 2048, 8192, 1024), idAcc,
                   (u > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk)  // 16 keys per step: 2048 B of G and of K
            mma_ss(tmem + kTdQ + su * kD, sdesc_sw128(sG + kk * 2048, 16384, 1024),
                   sdesc_sw128(sK + kk * 2048, 16384, 1024), idDQ, kk > 0);
          mma_commit(&q_empty[su]);
          mma_commit(&dq_full[su]);
          mma_commit(&mma_done[su]);
        }
      }
      if (ok) {
        mma_commit(acc_full);
      } else {
        mma_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
    __syncwarp();
  } else if (warp < 10) {
    // ------------------------------------------------------------------ pointwise (key rows)
    const int wg = (warp - 2) >> 2;
    const int lg = warp & 3;
    const int jr = lg * 32 + lane;  // key row within the tile == TMEM lane
    const int kj = n0 + jr;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    const Map map = BwdMap<Map>::make(p, h);
    int doc_j = 0;
    if constexpr (kHasDoc) doc_j = kj < p.T ? p.doc[(int64_t)b * p.doc_s0 + (int64_t)kj * p.doc_s1] : -2;
    int* docq = reinterpret_cast<int*>(smem + kSDoc) + (wg * 4 + lg) * kBM;
    uint8_t* g_row0 = smem + kSG + jr * 128;
    uint8_t* stg = smem + kSStg + lg * 8192 + wg * 4096;  // this warp's dQ staging (two 16 x 32 boxes)
    const bool leader = elect_one();
    float g1 = 0.f, g2 = 0.f;
    bool ok = true;
    // dQ partial of tile u (TMEM buffer wg; an M=64 accumulator keeps rows 16lg..16lg+15 in lanes
    // 0..15 of this warp's quadrant) -> swizzled staging -> TMA reduce-add into the accumulator
    auto drain_dq = [&](int u) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(&dq_full[wg], (u >> 1) & 1, wc, 29))) return false;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32(lane_addr + kTdQ + wg * kD, r0);
      tmem_ld32(lane_addr + kTdQ + wg * kD + 32, r1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&dq_empty[wg]);
      if (leader) bulk_wait_read<0>();  // the previous reduce from this staging buffer has read it
      __syncwarp();
      if (lane < 16) {
        uint8_t* row0 = stg + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(row0 + ((c ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(r0[4 * c]), __uint_as_float(r0[4 * c + 1]), __uint_as_float(r0[4 * c + 2]),
                          __uint_as_float(r0[4 * c + 3]));
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(row0 + 2048 + ((c ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(r1[4 * c]), __uint_as_float(r1[4 * c + 1]), __uint_as_float(r1[4 * c + 2]),
                          __uint_as_float(r1[4 * c + 3]));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (leader) {
        const int grow = (int)(bh * p.Tpad + m_first + u * kBM + 16 * lg);
        tma_reduce_add_2d(&tmDQ, stg, 0, grow);
        tma_reduce_add_2d(&tmDQ, stg + 2048, 32, grow);
        bulk_commit();
      }
      return true;
    };
    int t_prev = -1;
    for (int t = wg; t < n_tiles && ok; t += 2) {
      if (t_prev >= 0) {
        ok = drain_dq(t_prev);
        if (!ok) break;
      }
      t_prev = t;
      const int sb = wg;  // == t & 1
      const int m0 = m_first + t * kBM;
      if constexpr (kHasDoc) {
#pragma unroll
        for (int u = 0; u < kBM / 32; ++u) {
          const int qi = m0 + u * 32 + lane;
          docq[u * 32 + lane] = qi < p.T ? p.doc[(int64_t)b * p.doc_s0 + (int64_t)qi * p.doc_s1] : -1;
        }
        __syncwarp();
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&sdp_full[sb], (t >> 1) & 1, wc, 27));
      if (!ok) break;
      tc_fence_after();
      const bool full = !kHasDoc && (!p.causal || m0 >= n0 + kBN - 1) &&
                        (p.window <= 0 || (m0 + kBM - 1) - n0 < p.window) && (m0 + kBM <= p.T) &&
                        (n0 + kBN <= p.T);
      const float* dl = vdlz + sb * kBM;
      const float* zi = vzinv + sb * kBM;
      uint8_t* g_row = g_row0 + sb * 16384;
#pragma unroll 1
      for (int c = 0; c < kBM / 32; ++c) {
        uint32_t rs[32], rd[32];
        tmem_ld32(lane_addr + kTS + sb * kBM + c * 32, rs);
        tmem_ld32(lane_addr + kTdP + sb * kBM + c * 32, rd);
        float zc[32], dc[32];  // per-query 1/Z and delta/Z of these 32 columns (shared, broadcast)
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4) {
          const float4 z4 = reinterpret_cast<const float4*>(zi + c * 32)[v4];
          const float4 d4 = reinterpret_cast<const float4*>(dl + c * 32)[v4];
          zc[4 * v4] = z4.x; zc[4 * v4 + 1] = z4.y; zc[4 * v4 + 2] = z4.z; zc[4 * v4 + 3] = z4.w;
          dc[4 * v4] = d4.x; dc[4 * v4 + 1] = d4.y; dc[4 * v4 + 2] = d4.z; dc[4 * v4 + 3] = d4.w;
        }
        tmem_wait_ld();
        uint32_t wpk[16], gpk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float wv[2], gv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int qx = c * 32 + e + u;
            bool valid = true;
            if (!full) {
              int doc_i = 0;
              if constexpr (kHasDoc) doc_i = docq[qx];
              valid = pair_valid(m0 + qx, kj, p.T, p.causal, p.window, doc_i, doc_j);
            }
            const float raw = __uint_as_float(rs[e + u]);
            wv[u] = map.prob(raw, valid) * zc[e + u];
            gv[u] = map.grad(raw, valid, fmaf(__uint_as_float(rd[e + u]), zc[e + u], -dc[e + u]), g1, g2);
          }
          wpk[e / 2] = pack2<true>(wv[0], wv[1]);
          gpk[e / 2] = pack2<true>(gv[0], gv[1]);
        }
        tmem_st16(lane_addr + kTS + sb * kBM + c * 16, wpk);   // W^T over the consumed S^T columns
        tmem_st16(lane_addr + kTdP + sb * kBM + c * 16, gpk);  // G^T over the consumed dP^T columns
        // G (MN-major A operand of dQ): key row jr holds 64 queries = 128 B, 16-byte chunks swizzled
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int chunk = c * 4 + x;
          *reinterpret_cast<uint4*>(g_row + ((chunk ^ (jr & 7)) << 4)) =
              make_uint4(gpk[4 * x], gpk[4 * x + 1], gpk[4 * x + 2], gpk[4 * x + 3]);
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();  // G written by the generic proxy, read by the tensor core
      tc_fence_before();
      mbar_arrive(&wg_full[sb]);
    }
    if (ok && t_prev >= 0) ok = drain_dq(t_prev);
    if (leader) bulk_wait<0>();  // every reduce has finished reading shared memory
    __syncwarp();
    // dK, dV rows: group 0 stores dV, group 1 stores dK
    if (ok) ok = __all_sync(0xffffffffu, n_tiles == 0 || mbar_wait(acc_full, 0, wc, 28));
    if (ok) {
      tc_fence_after();
      {
        const int which = wg;
        __nv_bfloat16* dst = which == 0 ? p.dv + (int64_t)b * p.dv_s0 + (int64_t)h * p.dv_s1 + (int64_t)kj * p.dv_s2
                                        : p.dk + (int64_t)b * p.dk_s0 + (int64_t)h * p.dk_s1 + (int64_t)kj * p.dk_s2;
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(lane_addr + (which == 0 ? kTdV : kTdK) + c * 32, r);
          tmem_wait_ld();
          if (kj < p.T) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              w[e] = n_tiles == 0 ? 0u : pack2<true>(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
            uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) d4[v4] = make_uint4(w[4 * v4], w[4 * v4 + 1], w[4 * v4 + 2], w[4 * v4 + 3]);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      g1 += __shfl_xor_sync(0xffffffffu, g1, o);
      g2 += __shfl_xor_sync(0xffffffffu, g2, o);
    }
    if (lane == 0) {
      red[(wg * 4 + lg) * 2] = g1;
      red[(wg * 4 + lg) * 2 + 1] = g2;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    float* part = p.partials + (bh * p.n_kv + ktile) * 2;
    float t1 = 0.f, t2 = 0.f;
    for (int w = 0; w < 8; ++w) {
      t1 += red[2 * w];
      t2 += red[2 * w + 1];
    }
    part[0] = t1;
    part[1] = t2;
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Pre / post passes
// ---------------------------------------------------------------------------------------------
struct AuxParams {
  int B, H, T, Tpad, D;
  float eps;
  const float* scale;
  float* prep_part;  // [BH][Tpad / 64]: sum_i eps delta_i / Z_i over 64-row chunks
  int purified;
  const void* out;
  int64_t o_s0, o_s1, o_s2, o_s3;
  int out_f32;
  const __nv_bfloat16* dout;
  int64_t do_s0, do_s1, do_s2, do_s3;
  const float* z;
  float* dlz;
  float* zinv;
  float* dq_acc;
  __nv_bfloat16* dq;
  int64_t dq_s0, dq_s1, dq_s2;
  const float* partials;
  int n_kv;
  float* dscale;
  float* dtau;
  int scale_per_head, tau_per_head;
};

// One block per (64-row chunk, head, batch); each warp handles 8 rows: delta_i / Z_i, 1 / Z_i,
// a zeroed dQ accumulator row, and the chunk's sum_i eps delta_i / Z_i (the closed-form part of
// dscale / d gamma).
__global__ void __launch_bounds__(256) bwd_prep_kernel(const AuxParams a) {
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = (int64_t)b * a.H + h;
  __shared__ float csum_w[8];
  float csum = 0.f;
#pragma unroll 4
  for (int r = 0; r < 8; ++r) {
    const int i = chunk * 64 + warp * 8 + r;
    const int64_t row = bh * a.Tpad + i;
    float s = 0.f;
    if (i < a.T) {
      for (int d = 2 * lane; d < a.D; d += 64) {  // two adjacent elements per lane
        const int64_t oo = (int64_t)b * a.o_s0 + (int64_t)h * a.o_s1 + (int64_t)i * a.o_s2 + (int64_t)d * a.o_s3;
        const int64_t od = (int64_t)b * a.do_s0 + (int64_t)h * a.do_s1 + (int64_t)i * a.do_s2 + (int64_t)d * a.do_s3;
        float o0, o1;
        if (a.out_f32) {
          const float* op = reinterpret_cast<const float*>(a.out) + oo;
          o0 = op[0];
          o1 = op[a.o_s3];
        } else {
          const __nv_bfloat16* op = reinterpret_cast<const __nv_bfloat16*>(a.out) + oo;
          o0 = __bfloat162float(op[0]);
          o1 = __bfloat162float(op[a.o_s3]);
        }
        s += o0 * __bfloat162float(a.dout[od]) + o1 * __bfloat162float(a.dout[od + a.do_s3]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      const float zi = i < a.T ? 1.f / a.z[bh * a.T + i] : 0.f;
      a.dlz[row] = s * zi;
      a.zinv[row] = zi;
      csum += a.eps * s * zi;
    }
    float2* acc = reinterpret_cast<float2*>(a.dq_acc + row * a.D);
    for (int d = lane; d < a.D / 2; d += 32) acc[d] = make_float2(0.f, 0.f);
  }
  if (lane == 0) csum_w[warp] = csum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += csum_w[w];
    a.prep_part[bh * (a.Tpad / 64) + chunk] = t;
  }
}

// dQ accumulator -> bf16 (one thread per 8 elements)
__global__ void __launch_bounds__(256) bwd_post_kernel(const AuxParams a) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = a.D / 8;
  const int64_t rows = (int64_t)a.B * a.H * a.T;
  if (idx >= rows * per_row) return;
  const int c8 = (int)(idx % per_row);
  const int64_t r = idx / per_row;
  const int i = (int)(r % a.T);
  const int64_t bh = r / a.T;
  const int h = (int)(bh % a.H), b = (int)(bh / a.H);
  const float4* src = reinterpret_cast<const float4*>(a.dq_acc + ((bh * a.Tpad + i) * a.D + c8 * 8));
  const float4 x = src[0], y = src[1];
  uint4 o;
  o.x = sm100::pack2<true>(x.x, x.y);
  o.y = sm100::pack2<true>(x.z, x.w);
  o.z = sm100::pack2<true>(y.x, y.y);
  o.w = sm100::pack2<true>(y.z, y.w);
  *reinterpret_cast<uint4*>(a.dq + (int64_t)b * a.dq_s0 + (int64_t)h * a.dq_s1 + (int64_t)i * a.dq_s2 + c8 * 8) = o;
}

// Fixed-order sums into dscale / dtau (deterministic; replaces atomics, flash_born.py:319-322):
//   plain     dscale_h = (2 / scale_h) sum_{b,i} eps delta_i / Z_i
//   purified  dgamma_h = (4 / gamma_h) (sum_{b,i} eps delta_i / Z_i - sum eps_base b^2 dP),
//             dtau_h   = sum -4 u^3 dP gamma        (the last two from the main kernel's partials)
__global__ void bwd_param_kernel(const AuxParams a) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  auto head_terms = [&](int hh, float& d1, float& d2) {
    float tp = 0.f, t1 = 0.f, t2 = 0.f;
    const int nc = a.Tpad / 64;
    for (int b = 0; b < a.B; ++b) {
      const int64_t bhh = (int64_t)b * a.H + hh;
      for (int t = 0; t < nc; ++t) tp += a.prep_part[bhh * nc + t];
      if (a.purified) {
        const float* part = a.partials + bhh * a.n_kv * 2;
        for (int t = 0; t < a.n_kv; ++t) {
          t1 += part[2 * t];
          t2 += part[2 * t + 1];
        }
      }
    }
    const float sc = a.scale[a.scale_per_head ? hh : 0];
    d1 = a.purified ? (4.f / sc) * (tp - t1) : (2.f / sc) * tp;
    d2 = t2;
  };
  if (h < a.H) {
    float d1, d2;
    head_terms(h, d1, d2);
    if (a.scale_per_head) a.dscale[h] += d1;
    if (a.dtau != nullptr && a.tau_per_head) a.dtau[h] += d2;
  }
  if (h == 0 && (!a.scale_per_head || (a.dtau != nullptr && !a.tau_per_head))) {
    float s1 = 0.f, s2 = 0.f;
    for (int hh = 0; hh < a.H; ++hh) {
      float d1, d2;
      head_terms(hh, d1, d2);
      s1 += d1;
      s2 += d2;
    }
    if (!a.scale_per_head) a.dscale[0] += s1;
    if (a.dtau != nullptr && !a.tau_per_head) a.dtau[0] += s2;
  }
}

struct WsLayout {
  size_t dlz, zinv, dq_acc, partials, prep_part, total;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

WsLayout ws_layout(const Problem& p) {
  const int Tpad = (p.T + kBM - 1) / kBM * kBM;
  const size_t BH = (size_t)p.B * p.H;
  const int n_kv = (p.T + kBN - 1) / kBN;
  WsLayout w;
  w.dlz = 0;
  w.zinv = align256(w.dlz + BH * Tpad * 4);
  w.dq_acc = align256(w.zinv + BH * Tpad * 4);
  w.partials = align256(w.dq_acc + BH * Tpad * kD * 4);
  w.prep_part = align256(w.partials + BH * n_kv * 2 * 4);
  w.total = align256(w.prep_part + BH * (Tpad / 64) * 4);
  return w;
}

bool rows16(const Tensor4& t) {  // 16-byte vector row stores of bf16 rows
  if ((reinterpret_cast<uintptr_t>(t.ptr) & 15) != 0 || t.s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t.s[i] % 8 != 0) return false;
  return true;
}

template <class Map, bool kHasDoc>
int launch_main(const Problem& pr, cudaStream_t s, const BwdParams& bp, const CUtensorMap& mk, const CUtensorMap& mv,
                const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mdq) {
  auto kernel = tc_bwd_kernel<Map, kHasDoc>;
  const uint32_t smem = kSmemBytes + 1024;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  dim3 grid(bp.n_kv, pr.H, pr.B);
  kernel<<<grid, kThreads, smem, s>>>(mk, mv, mq, mdo, mdq, bp);
  e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  return FB_OK;
}

}  // namespace

bool tc_bwd_supported(const Problem& p) {
  if (p.dtype != FB_BF16 || p.D != kD) return false;
  if (p.out_dtype != FB_BF16 && p.out_dtype != FB_F32) return false;
  if (!tma_ok(p.q) || !tma_ok(p.k) || !tma_ok(p.v) || !tma_ok(p.dout)) return false;
  if (!rows16(p.dq) || !rows16(p.dk) || !rows16(p.dv)) return false;
  return true;
}

size_t tc_bwd_workspace(const Problem& p) { return ws_layout(p).total; }

int tc_bwd(const Problem& pr, cudaStream_t s, int* launches) {
  if (!get_encoder()) return FB_ERR_NO_DEVICE;
  CUtensorMap mk, mv, mq, mdo;
  if (!encode_bhtd(&mk, pr.k, pr.B, pr.H, pr.T, pr.D, kBN) || !encode_bhtd(&mv, pr.v, pr.B, pr.H, pr.T, pr.D, kBN) ||
      !encode_bhtd(&mq, pr.q, pr.B, pr.H, pr.T, pr.D, kBM) || !encode_bhtd(&mdo, pr.dout, pr.B, pr.H, pr.T, pr.D, kBM))
    return FB_ERR_ALIGN;
  const WsLayout w = ws_layout(pr);
  char* ws = static_cast<char*>(pr.ws);
  const int Tpad = (pr.T + kBM - 1) / kBM * kBM;
  const int n_kv = (pr.T + kBN - 1) / kBN;

  AuxParams a{};
  a.B = pr.B; a.H = pr.H; a.T = pr.T; a.Tpad = Tpad; a.D = pr.D;
  a.eps = pr.eps;
  a.scale = pr.scale;
  a.prep_part = reinterpret_cast<float*>(ws + w.prep_part);
  a.purified = pr.purified;
  a.out = pr.o.ptr;
  a.o_s0 = pr.o.s[0]; a.o_s1 = pr.o.s[1]; a.o_s2 = pr.o.s[2]; a.o_s3 = pr.o.s[3];
  a.out_f32 = pr.out_dtype == FB_F32;
  a.dout = static_cast<const __nv_bfloat16*>(pr.dout.ptr);
  a.do_s0 = pr.dout.s[0]; a.do_s1 = pr.dout.s[1]; a.do_s2 = pr.dout.s[2]; a.do_s3 = pr.dout.s[3];
  a.z = pr.z;
  a.dlz = reinterpret_cast<float*>(ws + w.dlz);
  a.zinv = reinterpret_cast<float*>(ws + w.zinv);
  a.dq_acc = reinterpret_cast<float*>(ws + w.dq_acc);
  a.dq = static_cast<__nv_bfloat16*>(const_cast<void*>(pr.dq.ptr));
  a.dq_s0 = pr.dq.s[0]; a.dq_s1 = pr.dq.s[1]; a.dq_s2 = pr.dq.s[2];
  a.partials = reinterpret_cast<float*>(ws + w.partials);
  a.n_kv = n_kv;
  a.dscale = pr.dscale;
  a.dtau = pr.purified ? pr.dtau : nullptr;
  a.scale_per_head = pr.scale_per_head;
  a.tau_per_head = pr.tau_per_head;

  BwdParams bp{};
  bp.B = pr.B; bp.H = pr.H; bp.T = pr.T; bp.Tpad = Tpad;
  bp.causal = pr.causal; bp.window = pr.window; bp.eps_base = pr.eps_base;
  bp.scale = pr.scale; bp.scale_per_head = pr.scale_per_head;
  bp.tau = pr.tau; bp.tau_per_head = pr.tau_per_head;
  bp.doc = pr.doc; bp.doc_s0 = pr.doc_s[0]; bp.doc_s1 = pr.doc_s[1];
  bp.dk = static_cast<__nv_bfloat16*>(const_cast<void*>(pr.dk.ptr));
  bp.dk_s0 = pr.dk.s[0]; bp.dk_s1 = pr.dk.s[1]; bp.dk_s2 = pr.dk.s[2];
  bp.dv = static_cast<__nv_bfloat16*>(const_cast<void*>(pr.dv.ptr));
  bp.dv_s0 = pr.dv.s[0]; bp.dv_s1 = pr.dv.s[1]; bp.dv_s2 = pr.dv.s[2];
  bp.dlz = a.dlz; bp.zinv = a.zinv; bp.dq_acc = a.dq_acc;
  bp.partials = reinterpret_cast<float*>(ws + w.partials);
  bp.n_kv = n_kv;
  bp.status = pr.status;

  CUtensorMap mdq;
  if (!encode_rows_f32(&mdq, a.dq_acc, (int64_t)pr.B * pr.H * Tpad)) return FB_ERR_ALIGN;
  bwd_prep_kernel<<<dim3(Tpad / 64, pr.H, pr.B), 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  int rc;
  if (pr.purified)
    rc = pr.doc ? launch_main<PurifiedMapTC, true>(pr, s, bp, mk, mv, mq, mdo, mdq)
                : launch_main<PurifiedMapTC, false>(pr, s, bp, mk, mv, mq, mdo, mdq);
  else
    rc = pr.doc ? launch_main<PlainMapNoParam, true>(pr, s, bp, mk, mv, mq, mdo, mdq)
                : launch_main<PlainMapNoParam, false>(pr, s, bp, mk, mv, mq, mdo, mdq);
  if (rc != FB_OK) return rc;
  const int64_t post_threads = (int64_t)pr.B * pr.H * pr.T * (pr.D / 8);
  bwd_post_kernel<<<(unsigned)((post_threads + 255) / 256), 256, 0, s>>>(a);
  bwd_param_kernel<<<(pr.H + 127) / 128, 128, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  *launches = 4;
  return FB_OK;
}

}  // namespace fb
