// fb_tc_bwd.cu -- flash-Born backward on the tcgen05 tensor cores (sm_100a), head dim 64 or 128.
//
// Four launches (all on the caller's stream):
//   1. bwd_prep_kernel   (1 / Z_i, delta_i / Z_i) pairs with delta_i = sum_d dO_id O_id (per-head
//                        rows padded to a multiple of 128), plus the closed-form sums of dscale /
//                        dgamma
//   2. tc_dkdv_kernel    persistent, key-major: one CTA per SM walks work items (batch, head,
//                        128-key tile) in L2-resident windows of heads (bwd_next); each item walks
//                        the 64-query tiles that can hold valid pairs and accumulates dK and dV in
//                        TMEM (four products per tile)
//   3. tc_dq_kernel      persistent, query-major: work items (batch, head, 128-query tile), heaviest
//                        first; each item walks 64-key tiles, recomputes S and dP and accumulates
//                        dQ = G K in TMEM (three products per tile), then stores dQ once
//   4. bwd_param_kernel  fixed-order sums into dscale / dtau from the pre-pass's closed-form sums
//                        and the dK/dV kernel's per-warp partials
// dQ is accumulated in TMEM by the CTA that owns its rows and written once: no fp32 atomics, so
// every gradient is deterministic.  Splitting dQ off the key-major kernel frees the TMEM columns
// its accumulators would take; the key-major kernel spends them on a third S^T/dP^T buffer (d=64)
// or on the wider dK/dV accumulators (d=128).
//
// Per (key tile, query tile) the algorithm needs (flash_born.py:267-312 and :398-427):
//   S^T  = K Q^T, dP^T = V dO^T                         (raw scores and dO.v, transposed)
//   pointwise: a = relu(scale raw), p = a^2, W = p / Z_i, dP = (dP^T - delta_i) / Z_i,
//              G = dL/draw = 2 a dP scale (masked; purified: 4u^3 dP gamma + 2 eps_base b dP)
//   dV += W^T dO, dK += G^T Q                            (key-major kernel)
//   S = Q K^T, dP = dO V^T, pointwise G, dQ += G K       (query-major kernel)
//
// Warps (384 threads, both main kernels): 0 TMA producers (copies issued by one thread complete
// one after another, about 0.3 us each, so each operand stream has its own lane), 1 TMEM owner +
// issuer of the raw-score product (S^T / S), 2-9 two pointwise warpgroups (group g takes the
// tiles t with t % 2 == g), 10 issuer of the dO.v product (dP^T / dP), 11 issuer of the gradient
// products.  One thread issues a tcgen05.mma at most every ~50 cycles (a commit costs about as
// much), about the execution time of an N = 64 product, so each product has its own issuing
// warp; barriers that both score products feed count two arrivals.  The score issuers run up to
// kNB - 1 tiles ahead of the gradient issuer (kNB TMEM buffers), so a group finds its next
// tile's scores ready when it finishes the current one.
//
// TMEM columns, key-major kernel:   d=64  S^T[3] 0/64/128, dP^T[3] 192/256/320, dV 384, dK 448
//                                   d=128 S^T[2] 0/64, dP^T[2] 128/192, dV 256, dK 384
//                 query-major kernel: S[3] 0/64/128, dP[3] 192/256/320, dQ 384 (d columns)
// W^T / G^T (bf16) are written over the consumed S^T / dP^T columns, G over the consumed S columns.
#include <cuda.h>

#include <algorithm>

#include "fb_common.cuh"
#include "fb_sm100.cuh"

namespace fb {
namespace {

using namespace sm100;

constexpr int kThreads = 384;  // 12 warps
constexpr uint32_t kTmemCols = 512;
constexpr int kRowPad = 128;  // per-head rows of the prep vectors are padded to this

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
  __nv_bfloat16* dq;
  int64_t dq_s0, dq_s1, dq_s2;
  const float* zd;     // [BH][Tpad][2]  (1 / Z_i, delta_i / Z_i)
  int map3;            // tensor maps address (b, h) as one merged dimension
  float* partials;     // [BH][n_kv][8 warps][2]
  int n_kv, n_items;   // key-major kernel: 128-key tiles per head, work items
  int n_mt, n_qitems;  // query-major kernel: 128-query tiles per head, work items
  const int2* doc_qr;  // document spans of the query / key blocks (null without document ids)
  const int2* doc_kr;
  int nblk;
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

// =============================================================================================
// Key-major kernel: dK, dV
// =============================================================================================
template <int D>
struct KvCfg {
  static constexpr int kBN = 128;  // keys per item (M of every product)
  static constexpr int kBM = 64;   // queries per tile
  static constexpr int kNB = D == 64 ? 3 : 2;    // S^T / dP^T TMEM buffers
  static constexpr int kKVB = D == 64 ? 2 : 1;   // K / V item buffers (d=64: the next item's are prefetched)
  static constexpr int kQS = D == 64 ? 8 : 4;    // Q / dO / vector stages
  static constexpr uint32_t kKTile = kBN * D * 2;
  static constexpr uint32_t kKHalf = kBN * 128;  // one 64-column half of a K or V tile
  static constexpr uint32_t kQTile = kBM * D * 2;
  static constexpr uint32_t kQHalf = kBM * 128;
  static constexpr uint32_t kSK = 0;
  static constexpr uint32_t kSV = kKVB * kKTile;
  static constexpr uint32_t kSQ = 2 * kKVB * kKTile;
  static constexpr uint32_t kSdO = kSQ + kQS * kQTile;
  static constexpr uint32_t kSVec = kSdO + kQS * kQTile;  // [kQS][64 queries] (1/Z, delta/Z) fp32 pairs
  static constexpr uint32_t kSDoc = kSVec + kQS * 512;     // query doc ids [8 warps][64] int32
  static constexpr uint32_t kSBar = kSDoc + 8 * kBM * 4;
  static constexpr uint32_t kSmem = kSBar + 512;
  static constexpr uint32_t kTS = 0, kTdP = kNB * 64, kTdV = 2 * kNB * 64, kTdK = kTdV + D;
  static_assert(kTdK + D <= kTmemCols, "TMEM columns");
  static_assert(kSmem + 1024 <= 227 * 1024, "shared memory per CTA");
  static_assert(4 + 4 * kQS + 3 * kNB + 5 <= 60, "barrier area");
};

struct BwdItem {
  int b, h, kt, n0, m_first, n_tiles;
};

// Work item (bh, kt): keys [n0, n0 + 128) of head bh; query tiles [m_first, m_first + 64 n_tiles)
// can hold valid pairs for them (at least one: the key tile starts below T).
__device__ __forceinline__ BwdItem bwd_item(const BwdParams& p, int bh, int kt) {
  BwdItem it;
  it.kt = kt;
  it.b = bh / p.H;
  it.h = bh % p.H;
  it.n0 = it.kt * 128;
  int lo = p.causal ? it.n0 : 0;
  int hi = p.T;
  if (p.window > 0) hi = min(p.T, it.n0 + 128 - 1 + p.window);
  doc_narrow(p.doc_kr, p.nblk, it.b, it.n0, 128, lo, hi);  // queries that can share a document
  lo = (lo / 64) * 64;
  it.m_first = lo;
  it.n_tiles = hi > lo ? (hi - lo + 63) / 64 : 0;
  return it;
}

// Schedule.  Items are numbered head-major, u = bh n_kv + kt, and the numbering is cut into
// windows of 2 gridDim.x consecutive items (about 2 gridDim.x / n_kv heads).  Every item of a
// head reads all of that head's Q, dO and 1/Z rows, so while the CTAs work through one window
// only a few heads' rows are live and they stay in L2.  Inside a window the items are sorted by
// key tile (under a causal mask the early key tiles have the most query tiles) and dealt out as
// a snake: CTA c takes window positions c and 2 gridDim.x - 1 - c, one long and one short item.
// bwd_next: the item of this CTA's slot k, moving k past empty slots (the last window can be
// short); false once the CTA has no items left.  Every role walks the same sequence.
__device__ __forceinline__ bool bwd_next(const BwdParams& p, int& k, BwdItem& it) {
  const int W = 2 * (int)gridDim.x;
  for (;; ++k) {
    const int a = (k >> 1) * W;  // first item of the window (n_items < 2^31)
    if (a >= p.n_items) return false;
    const int e = min(a + W, p.n_items);
    int rem = (k & 1) ? W - 1 - (int)blockIdx.x : (int)blockIdx.x;
    if (rem >= e - a) continue;
    // a = A n_kv + ra, e = E n_kv + re: the window holds key tile kt of heads
    // A + [kt < ra] ..., (E - A) - [kt < ra] + [kt < re] of them
    const int A = a / p.n_kv, ra = a - A * p.n_kv;
    const int E = e / p.n_kv, re = e - E * p.n_kv;
    for (int kt = 0; kt < p.n_kv; ++kt) {
      const int c = (E - A) - (kt < ra ? 1 : 0) + (kt < re ? 1 : 0);
      if (rem < c) {
        it = bwd_item(p, A + (kt < ra ? 1 : 0) + rem, kt);
        return true;
      }
      rem -= c;
    }
    return false;  // not reached: the per-key-tile counts add up to e - a
  }
}

template <int D, class Map, bool kHasDoc>
__global__ void __launch_bounds__(kThreads, 1)
    tc_dkdv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
                   const BwdParams p) {
  using C = KvCfg<D>;
  constexpr int NB = C::kNB, KVB = C::kKVB, QS = C::kQS, BM = C::kBM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kSBar);
  uint64_t* kv_full = bars + 0;                // [2] per item
  uint64_t* kv_empty = bars + 2;               // [2]
  uint64_t* q_full = bars + 4;                 // [QS] per query-tile stage: Q
  uint64_t* o_full = bars + 4 + QS;            // [QS] dO
  uint64_t* vec_full = bars + 4 + 2 * QS;      // [QS] (1/Z, delta/Z) of the tile's queries
  uint64_t* q_empty = bars + 4 + 3 * QS;       // [QS] the whole stage
  uint64_t* sdp_full = bars + 4 + 4 * QS;      // [NB] per score buffer
  uint64_t* wg_full = sdp_full + NB;           // [NB]
  uint64_t* mma_done = wg_full + NB;           // [NB]
  uint64_t* acc_full = mma_done + NB;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 60);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 61);
  float* vzd = reinterpret_cast<float*>(smem + C::kSVec);  // [QS][64][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int i = 0; i < QS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&vec_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);  // both score products
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&sdp_full[i], 2);  // S^T and dP^T
      mbar_init(&wg_full[i], 128);
      mbar_init(&mma_done[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    for (int r = 0; r < 3; ++r) mbar_init(drain + r, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmdO);
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
    // ------------------------------------------------------------------ TMA producers
    // Copies issued by one thread complete one after another, so the streams are split over
    // lanes: lane 0 requests K / V of the items and Q of the query tiles, lane 1 dO, lane 2 the
    // (1/Z, delta/Z) pairs; each walks the same tile sequence.
    if (lane < 3) {
      bool ok = true;
      int g = 0, i = 0, kv_issued = 0, issued = 0;  // issued: this lane's query-tile copies requested
      uint64_t* full = lane == 0 ? q_full : (lane == 1 ? o_full : vec_full);
      auto load_kv = [&](int item_seq, const BwdItem& it) -> bool {
        const int kb = item_seq % KVB;
        if (item_seq >= KVB && !mbar_wait(&kv_empty[kb], ((item_seq / KVB) - 1) & 1, wc, 20)) return false;
        mbar_arrive_expect_tx(&kv_full[kb], 2 * C::kKTile);
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf) {
          tma_load_bhtd(smem + C::kSK + kb * C::kKTile + hf * C::kKHalf, &tmK, &kv_full[kb], p.map3, hf * 64, it.n0, it.h,
                        it.b, p.H);
          tma_load_bhtd(smem + C::kSV + kb * C::kKTile + hf * C::kKHalf, &tmV, &kv_full[kb], p.map3, hf * 64, it.n0, it.h,
                        it.b, p.H);
        }
        kv_issued = item_seq + 1;
        return true;
      };
      int k = 0;
      BwdItem it;
      for (; ok && bwd_next(p, k, it); ++k, ++i) {
        const int64_t bh = (int64_t)it.b * p.H + it.h;
        if (lane == 0 && kv_issued <= i) ok = load_kv(i, it);
        for (int t = 0; t < it.n_tiles && ok; ++t, ++g) {
          const int st = g % QS;
          if (g >= QS) ok = mbar_wait(&q_empty[st], ((g / QS) - 1) & 1, wc, 21);
          if (!ok) break;
          const int m0 = it.m_first + t * BM;
          if (lane < 2) {
            mbar_arrive_expect_tx(&full[st], C::kQTile);
            const CUtensorMap* map = lane == 0 ? &tmQ : &tmdO;
            uint8_t* dst = smem + (lane == 0 ? C::kSQ : C::kSdO) + st * C::kQTile;
#pragma unroll
            for (int hf = 0; hf < D / 64; ++hf)
              tma_load_bhtd(dst + hf * C::kQHalf, map, &full[st], p.map3, hf * 64, m0, it.h, it.b, p.H);
          } else {
            mbar_arrive_expect_tx(&full[st], 2 * BM * 4);
            bulk_load(vzd + st * 2 * BM, p.zd + (bh * p.Tpad + m0) * 2, 2 * BM * 4, &full[st]);
          }
          issued = g + 1;
          // with two K/V buffers, the next item's K and V are requested once this item's first
          // query tile is on its way
          if (KVB == 2 && lane == 0 && t == 0) {
            int kn = k + 1;
            BwdItem nit;
            if (bwd_next(p, kn, nit)) ok = load_kv(i + 1, nit);
          }
        }
      }
      if (!ok) {
        // abandoned: let this lane's copies already in flight land before the CTA exits
        for (int gg = max(0, issued - QS); gg < issued; ++gg) mbar_wait_drain(&full[gg % QS], (gg / QS) & 1);
        for (int ii = max(0, kv_issued - KVB); ii < kv_issued; ++ii)
          mbar_wait_drain(&kv_full[ii % KVB], (ii / KVB) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp >= 10) {
    // ------------------------------------------------------------------ MMA issuers
    // warp 1: S^T, warp 10: dP^T (score cursor); warp 11: dV, dK (gradient cursor)
    if (elect_one()) {
      constexpr uint32_t idSdP = idesc_f16(1, 0, 0, BM, C::kBN);  // M = 128 keys, N = 64 queries
      constexpr uint32_t idAcc = idesc_f16(1, 0, 1, D, C::kBN);   // A TMEM, B MN-major, N = D
      bool ok = true;
      // score cursor (S^T, dP^T) and gradient cursor (dV, dK) walk the same tile sequence; the
      // score cursor runs up to NB - 1 tiles ahead
      int s_k = 0, s_i = 0, s_t = 0, s_g = 0;
      int u_k = 0, u_i = 0, u_t = 0, u_g = 0;
      BwdItem s_it, u_it;
      bool s_have = bwd_next(p, s_k, s_it);
      bool u_have = bwd_next(p, u_k, u_it);
      // which = 0: S^T = K Q^T into S^T[b]; which = 1: dP^T = V dO^T into dP^T[b]
      auto issue_sdp = [&](int which) -> bool {
        const int b = s_g % NB;
        const int qs = s_g % QS;
        const int kb = s_i % KVB;
        if (s_t == 0 && !mbar_wait(&kv_full[kb], (s_i / KVB) & 1, wc, 22)) return false;
        if (!mbar_wait(which == 0 ? &q_full[qs] : &o_full[qs], (s_g / QS) & 1, wc, 23 + 5 * which)) return false;
        // buffer b is free once the gradient products of tile s_g - NB have read W^T / G^T
        if (s_g >= NB && !mbar_wait(&mma_done[b], ((s_g / NB) - 1) & 1, wc, 24)) return false;
        tc_fence_after();
        const uint64_t dA = sdesc_sw128(smem_u32(smem + (which ? C::kSV : C::kSK) + kb * C::kKTile), 16, 1024);
        const uint64_t dB = sdesc_sw128(smem_u32(smem + (which ? C::kSdO : C::kSQ) + qs * C::kQTile), 16, 1024);
        const uint32_t dst = tmem + (which ? C::kTdP : C::kTS) + b * 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // 16 head-dim elements per step (32 B along a row)
          const uint32_t ok_ = ((kk >> 2) * C::kKHalf + (kk & 3) * 32) >> 4;
          const uint32_t oq_ = ((kk >> 2) * C::kQHalf + (kk & 3) * 32) >> 4;
          mma_ss(dst, dA + ok_, dB + oq_, idSdP, kk > 0);
        }
        mma_commit(&sdp_full[b]);
        // K and V feed only the score products: the item's buffer is free after its last one
        if (s_t == s_it.n_tiles - 1) mma_commit(&kv_empty[kb]);
        ++s_g;
        if (++s_t == s_it.n_tiles) {
          s_t = 0;
          ++s_i;
          ++s_k;
          s_have = bwd_next(p, s_k, s_it);
        }
        return true;
      };
      auto issue_grads = [&]() -> bool {
        const int b = u_g % NB;
        const int qs = u_g % QS;
        if (!mbar_wait(&wg_full[b], (u_g / NB) & 1, wc, 25)) return false;
        if (u_t == 0 && u_i >= 1 && !mbar_wait(acc_empty, (u_i - 1) & 1, wc, 27)) return false;
        tc_fence_after();
        // MN-major Q / dO (N = head dim): 64-column blocks kQHalf apart, a K step of 16 queries
        // is 16 rows = 2048 B
        const uint64_t dQmn = sdesc_sw128(smem_u32(smem + C::kSQ + qs * C::kQTile), C::kQHalf, 1024);
        const uint64_t ddOmn = sdesc_sw128(smem_u32(smem + C::kSdO + qs * C::kQTile), C::kQHalf, 1024);
        const uint32_t acc = (u_t == 0) ? 0u : 1u;
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)  // 16 queries per step: 8 packed TMEM columns
          mma_ts(tmem + C::kTdV, tmem + C::kTS + b * 64 + kk * 8, ddOmn + kk * 128, idAcc, (kk == 0) ? acc : 1u);
#pragma unroll
        for (int kk = 0; kk < BM / 16; ++kk)
          mma_ts(tmem + C::kTdK, tmem + C::kTdP + b * 64 + kk * 8, dQmn + kk * 128, idAcc, (kk == 0) ? acc : 1u);
        mma_commit(&q_empty[qs]);
        mma_commit(&mma_done[b]);
        if (u_t == u_it.n_tiles - 1) mma_commit(acc_full);
        ++u_g;
        if (++u_t == u_it.n_tiles) {
          u_t = 0;
          ++u_i;
          ++u_k;
          u_have = bwd_next(p, u_k, u_it);
        }
        return true;
      };
      const int role = warp == 1 ? 0 : warp - 9;  // 0: S^T, 1: dP^T, 2: dV / dK
      if (role < 2) {
        while (ok && s_have) ok = issue_sdp(role);
      } else {
        while (ok && u_have) ok = issue_grads();
      }
      if (!ok) {  // wait for this thread's products in flight before TMEM is released
        mma_commit(drain + role);
        mbar_wait_drain(drain + role, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ pointwise (key rows), warps 2-9
    const int wg = (warp - 2) >> 2;
    const int lg = warp & 3;
    const int jr = lg * 32 + lane;  // key row within the tile == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    int* docq = reinterpret_cast<int*>(smem + C::kSDoc) + (wg * 4 + lg) * BM;
    bool ok = true;
    int g = 0, i = 0;
    // per-item parameters (map, this key row's document id) come from global memory; those of
    // the next item are requested before the current item's end-of-item work hides their latency
    int k = 0;
    BwdItem it_n;
    bool have_n = bwd_next(p, k, it_n);
    Map map_n{};
    int doc_n = 0;
    auto fetch = [&]() {
      map_n = BwdMap<Map>::make(p, it_n.h);
      if constexpr (kHasDoc) {
        const int kr = it_n.n0 + jr;
        doc_n = kr < p.T ? p.doc[(int64_t)it_n.b * p.doc_s0 + (int64_t)kr * p.doc_s1] : -2;
      }
    };
    if (have_n) fetch();
    for (; ok && have_n; ++i) {
      const BwdItem it = it_n;
      const Map map = map_n;
      const int doc_j = doc_n;
      (void)doc_j;
      const int64_t bh = (int64_t)it.b * p.H + it.h;
      const int n0 = it.n0;
      const int kj = n0 + jr;
      float g1 = 0.f, g2 = 0.f;
      for (int t = (wg - g) & 1; t < it.n_tiles && ok; t += 2) {
        const int gg = g + t;  // gg % 2 == wg
        const int b = gg % NB;
        const int qs = gg % QS;
        const int m0 = it.m_first + t * BM;
        if constexpr (kHasDoc) {
#pragma unroll
          for (int u = 0; u < BM / 32; ++u) {
            const int qi = m0 + u * 32 + lane;
            docq[u * 32 + lane] = qi < p.T ? p.doc[(int64_t)it.b * p.doc_s0 + (int64_t)qi * p.doc_s1] : -1;
          }
          __syncwarp();
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&vec_full[qs], (gg / QS) & 1, wc, 32));
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sdp_full[b], (gg / NB) & 1, wc, 30));
        if (!ok) break;
        tc_fence_after();
        const bool full = !kHasDoc && (!p.causal || m0 >= n0 + C::kBN - 1) &&
                          (p.window <= 0 || (m0 + BM - 1) - n0 < p.window) && (m0 + BM <= p.T) &&
                          (n0 + C::kBN <= p.T);
        const float4* zd4 = reinterpret_cast<const float4*>(vzd + qs * 2 * BM);  // (z, d) of two queries each
        const uint32_t s_col = lane_addr + C::kTS + b * 64, p_col = lane_addr + C::kTdP + b * 64;
        // Partial tiles: the raw score of every invalid pair is replaced by NaN before the map,
        // which turns it into p = 0 and dL/draw = 0 (fmaxf returns its non-NaN operand and no
        // other term of these maps touches raw), so one branch-free body serves every tile.
        const int lo_q = p.causal ? kj - m0 : -BM;  // causal: query column qx is valid iff qx >= kj - m0
        const int hi_q = kj < p.T ? p.T - m0 : 0;   // queries below T; a padded key row has none
        auto mask16 = [&](int sc, uint32_t (&rs)[16]) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int qx = sc * 16 + e;
            bool v = (qx >= lo_q) & (qx < hi_q) & ((p.window <= 0) | ((m0 + qx) - kj < p.window));
            if constexpr (kHasDoc) v = v & (docq[qx] == doc_j);
            rs[e] = v ? rs[e] : 0x7FC00000u;
          }
        };
        // one 16-query sub-chunk: W^T, G^T -> TMEM over the consumed S^T / dP^T columns
        auto sub16 = [&](int sc, const uint32_t (&rs)[16], const uint32_t (&rd)[16]) {
          float zc[16], dc[16];
#pragma unroll
          for (int v2 = 0; v2 < 8; ++v2) {
            const float4 f = zd4[sc * 8 + v2];
            zc[2 * v2] = f.x; dc[2 * v2] = f.y; zc[2 * v2 + 1] = f.z; dc[2 * v2 + 1] = f.w;
          }
          uint32_t wpk[8], gpk[8];
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            float wv[2], gv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float raw = __uint_as_float(rs[e + u]);
              wv[u] = map.prob(raw, true) * zc[e + u];
              gv[u] = map.grad(raw, true, fmaf(__uint_as_float(rd[e + u]), zc[e + u], -dc[e + u]), g1, g2);
            }
            wpk[e / 2] = pack2<true>(wv[0], wv[1]);
            gpk[e / 2] = pack2<true>(gv[0], gv[1]);
          }
          tmem_st8(s_col + sc * 8, wpk);
          tmem_st8(p_col + sc * 8, gpk);
        };
        {
          // software pipeline: the TMEM loads of sub-chunk s+1 are in flight while s is computed
          uint32_t sA[16], dA[16], sB[16], dB[16];
          tmem_ld16(s_col, sA);
          tmem_ld16(p_col, dA);
          tmem_wait_ld();
#pragma unroll
          for (int sc = 0; sc < BM / 16; sc += 2) {
            tmem_ld16(s_col + (sc + 1) * 16, sB);
            tmem_ld16(p_col + (sc + 1) * 16, dB);
            if (!full) mask16(sc, sA);
            sub16(sc, sA, dA);
            tmem_wait_ld();
            if (sc + 2 < BM / 16) {
              tmem_ld16(s_col + (sc + 2) * 16, sA);
              tmem_ld16(p_col + (sc + 2) * 16, dA);
            }
            if (!full) mask16(sc + 1, sB);
            sub16(sc + 1, sB, dB);
            tmem_wait_ld();
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&wg_full[b]);
      }
      if (!ok) break;
      ++k;
      have_n = bwd_next(p, k, it_n);
      if (have_n) fetch();
      // ---- end of the item: dK / dV rows (group 0 stores dV, group 1 stores dK), partials
      ok = __all_sync(0xffffffffu, mbar_wait(acc_full, i & 1, wc, 31));
      if (!ok) break;
      tc_fence_after();
      {
        const uint32_t acc_col = lane_addr + (wg == 0 ? C::kTdV : C::kTdK);
        __nv_bfloat16* dst = wg == 0 ? p.dv + (int64_t)it.b * p.dv_s0 + (int64_t)it.h * p.dv_s1 + (int64_t)kj * p.dv_s2
                                     : p.dk + (int64_t)it.b * p.dk_s0 + (int64_t)it.h * p.dk_s1 + (int64_t)kj * p.dk_s2;
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf) {
          uint32_t r0[32], r1[32];
          tmem_ld32(acc_col + hf * 64, r0);
          tmem_ld32(acc_col + hf * 64 + 32, r1);
          tmem_wait_ld();
          if (hf == D / 64 - 1) {
            tc_fence_before();
            mbar_arrive(acc_empty);
          }
          if (kj < p.T) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + hf * 64);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              d4[v4] = make_uint4(pack2<true>(__uint_as_float(r0[8 * v4]), __uint_as_float(r0[8 * v4 + 1])),
                                  pack2<true>(__uint_as_float(r0[8 * v4 + 2]), __uint_as_float(r0[8 * v4 + 3])),
                                  pack2<true>(__uint_as_float(r0[8 * v4 + 4]), __uint_as_float(r0[8 * v4 + 5])),
                                  pack2<true>(__uint_as_float(r0[8 * v4 + 6]), __uint_as_float(r0[8 * v4 + 7])));
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              d4[4 + v4] = make_uint4(pack2<true>(__uint_as_float(r1[8 * v4]), __uint_as_float(r1[8 * v4 + 1])),
                                      pack2<true>(__uint_as_float(r1[8 * v4 + 2]), __uint_as_float(r1[8 * v4 + 3])),
                                      pack2<true>(__uint_as_float(r1[8 * v4 + 4]), __uint_as_float(r1[8 * v4 + 5])),
                                      pack2<true>(__uint_as_float(r1[8 * v4 + 6]), __uint_as_float(r1[8 * v4 + 7])));
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        g1 += __shfl_xor_sync(0xffffffffu, g1, o);
        g2 += __shfl_xor_sync(0xffffffffu, g2, o);
      }
      if (lane == 0) {
        float* part = p.partials + ((bh * p.n_kv + it.kt) * 8 + (wg * 4 + lg)) * 2;
        part[0] = g1;
        part[1] = g2;
      }
      g += it.n_tiles;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// =============================================================================================
// Query-major kernel: dQ
// =============================================================================================
template <int D>
struct DqCfg {
  static constexpr int kBM = 128;  // queries per item (M of every product)
  static constexpr int kBN = 64;   // keys per tile
  static constexpr int kNB = 3;    // S / dP TMEM buffers
  static constexpr int kQB = D == 64 ? 2 : 1;   // Q / dO item buffers (d=64: the next item's are prefetched)
  static constexpr int kKS = D == 64 ? 8 : 5;   // K stages (held until dQ += G K of the tile)
  static constexpr int kVS = D == 64 ? 6 : 4;   // V stages (held until dP of the tile)
  static constexpr uint32_t kQTile = kBM * D * 2;
  static constexpr uint32_t kQHalf = kBM * 128;
  static constexpr uint32_t kKTile = kBN * D * 2;
  static constexpr uint32_t kKHalf = kBN * 128;
  static constexpr uint32_t kSQ = 0;
  static constexpr uint32_t kSdO = kQB * kQTile;
  static constexpr uint32_t kSK = 2 * kQB * kQTile;
  static constexpr uint32_t kSV = kSK + kKS * kKTile;
  static constexpr uint32_t kSDoc = kSV + kVS * kKTile;  // key doc ids [8 warps][64] int32
  static constexpr uint32_t kSBar = kSDoc + 8 * kBN * 4;
  static constexpr uint32_t kSmem = kSBar + 512;
  static constexpr uint32_t kTS = 0, kTdP = kNB * 64, kTdQ = 2 * kNB * 64;
  static_assert(kTdQ + D <= kTmemCols, "TMEM columns");
  static_assert(kSmem + 1024 <= 227 * 1024, "shared memory per CTA");
  static_assert(4 + 2 * kKS + 2 * kVS + 3 * kNB + 5 <= 60, "barrier area");
};

struct QItem {
  int b, h, m0, n_first, n_count;
};

// Work item idx of the query-major kernel: latest query tiles (the most keys under a causal
// mask) first, then (b, h).  Keys [n_first, n_first + 64 n_count) can be valid for its rows.
__device__ __forceinline__ QItem q_item(const BwdParams& p, int idx) {
  const int bh_total = p.B * p.H;
  const int mt = p.n_mt - 1 - idx / bh_total;
  const int bh = idx % bh_total;
  QItem it;
  it.b = bh / p.H;
  it.h = bh % p.H;
  it.m0 = mt * 128;
  int lo = 0, hi = p.T;
  if (p.causal) hi = min(p.T, it.m0 + 128);
  if (p.window > 0) lo = max(0, it.m0 - p.window + 1);
  doc_narrow(p.doc_qr, p.nblk, it.b, it.m0, 128, lo, hi);  // keys that can share a document
  lo = (lo / 64) * 64;
  it.n_first = lo;
  it.n_count = hi > lo ? (hi - lo + 63) / 64 : 0;
  return it;
}

// Global index of this CTA's j-th query-major item, or -1 when it has no more: rows of gridDim.x
// items dealt left to right on even rows and right to left on odd ones (snake order), which keeps
// every CTA's total within about one item of the others for items sorted heaviest first; with
// document ids (sizes that follow the documents) every row is dealt left to right.
__device__ __forceinline__ int q_slot(const BwdParams& p, int j) {
  const int G = (int)gridDim.x;
  const bool back = (j & 1) && p.doc_qr == nullptr;
  const int idx = j * G + (back ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
  return idx < p.n_qitems ? idx : -1;
}


template <int D, class Map, bool kHasDoc>
__global__ void __launch_bounds__(kThreads, 1)
    tc_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmdO,
                 const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const BwdParams p) {
  using C = DqCfg<D>;
  constexpr int NB = C::kNB, QB = C::kQB, KS = C::kKS, VS = C::kVS, BN = C::kBN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kSBar);
  uint64_t* q_full = bars + 0;           // [2] per item
  uint64_t* q_empty = bars + 2;          // [2]
  uint64_t* k_full = bars + 4;           // [KS]
  uint64_t* k_empty = k_full + KS;       // [KS]
  uint64_t* v_full = k_empty + KS;       // [VS]
  uint64_t* v_empty = v_full + VS;       // [VS]
  uint64_t* s_full = v_empty + VS;       // [NB] per score buffer
  uint64_t* g_full = s_full + NB;        // [NB]
  uint64_t* mma_done = g_full + NB;      // [NB]
  uint64_t* dq_full = mma_done + NB;
  uint64_t* dq_empty = dq_full + 1;
  uint64_t* drain = dq_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 60);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 61);
  int* docs_all = reinterpret_cast<int*>(smem + C::kSDoc);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);  // Q by the S product, dO by the dP product
    }
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&s_full[i], 2);  // S and dP
      mbar_init(&g_full[i], 128);
      mbar_init(&mma_done[i], 1);
    }
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 256);
    for (int r = 0; r < 3; ++r) mbar_init(drain + r, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmdO);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
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
    // ------------------------------------------------------------------ TMA producers
    // lane 0 requests Q / dO of the items and K of the key tiles, lane 1 V (copies issued by one
    // thread complete one after another)
    if (lane < 2) {
      bool ok = true;
      int g = 0, i = 0, q_issued = 0, issued = 0;  // issued: K (lane 0) or V (lane 1) tiles requested
      const int NS = lane == 0 ? KS : VS;
      uint64_t* full = lane == 0 ? k_full : v_full;
      uint64_t* empty = lane == 0 ? k_empty : v_empty;
      const CUtensorMap* map = lane == 0 ? &tmK : &tmV;
      uint8_t* ring = smem + (lane == 0 ? C::kSK : C::kSV);
      auto load_q = [&](int item_seq, const QItem& it) -> bool {
        const int qb = item_seq % QB;
        if (item_seq >= QB && !mbar_wait(&q_empty[qb], ((item_seq / QB) - 1) & 1, wc, 40)) return false;
        mbar_arrive_expect_tx(&q_full[qb], 2 * C::kQTile);
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf) {
          tma_load_bhtd(smem + C::kSQ + qb * C::kQTile + hf * C::kQHalf, &tmQ, &q_full[qb], p.map3, hf * 64, it.m0, it.h,
                        it.b, p.H);
          tma_load_bhtd(smem + C::kSdO + qb * C::kQTile + hf * C::kQHalf, &tmdO, &q_full[qb], p.map3, hf * 64, it.m0,
                        it.h, it.b, p.H);
        }
        q_issued = item_seq + 1;
        return true;
      };
      for (int idx = q_slot(p, 0); idx >= 0 && ok; idx = q_slot(p, i + 1), ++i) {
        const QItem it = q_item(p, idx);
        if (lane == 0 && q_issued <= i) ok = load_q(i, it);
        for (int t = 0; t < it.n_count && ok; ++t, ++g) {
          const int st = g % NS;
          const int n0 = it.n_first + t * BN;
          // a K stage is free once dQ += G K of its tile has completed, a V stage once dP has
          if (g >= NS) ok = mbar_wait(&empty[st], ((g / NS) - 1) & 1, wc, 41 + lane);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[st], C::kKTile);
#pragma unroll
          for (int hf = 0; hf < D / 64; ++hf)
            tma_load_bhtd(ring + st * C::kKTile + hf * C::kKHalf, map, &full[st], p.map3, hf * 64, n0, it.h, it.b, p.H);
          issued = g + 1;
          // with two Q / dO buffers, the next item's are requested once this item's first key
          // tile is on its way
          if (QB == 2 && lane == 0 && t == 0 && q_slot(p, i + 1) >= 0)
            ok = load_q(i + 1, q_item(p, q_slot(p, i + 1)));
        }
      }
      if (!ok) {
        // abandoned: let this lane's copies already in flight land before the CTA exits
        for (int gg = max(0, issued - NS); gg < issued; ++gg) mbar_wait_drain(&full[gg % NS], (gg / NS) & 1);
        for (int qq = max(0, q_issued - QB); qq < q_issued; ++qq) mbar_wait_drain(&q_full[qq % QB], (qq / QB) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp >= 10) {
    // ------------------------------------------------------------------ MMA issuers
    // warp 1: S, warp 10: dP (score cursor); warp 11: dQ += G K (gradient cursor)
    if (elect_one()) {
      constexpr uint32_t idS = idesc_f16(1, 0, 0, BN, C::kBM);  // M = 128 queries, N = 64 keys
      constexpr uint32_t idQ = idesc_f16(1, 0, 1, D, C::kBM);   // A TMEM (G), B MN-major (K), N = D
      bool ok = true;
      int s_idx = q_slot(p, 0), s_i = 0, s_t = 0, s_g = 0;
      int u_idx = q_slot(p, 0), u_i = 0, u_t = 0, u_g = 0;
      QItem s_it{}, u_it{};
      bool s_have = s_idx >= 0, u_have = u_idx >= 0;
      if (s_have) s_it = q_item(p, s_idx);
      if (u_have) u_it = q_item(p, u_idx);
      // which = 0: S = Q K^T into S[b]; which = 1: dP = dO V^T into dP[b]
      auto issue_sdp = [&](int which) -> bool {
        const int b = s_g % NB;
        const int qb = s_i % QB;
        if (s_t == 0 && !mbar_wait(&q_full[qb], (s_i / QB) & 1, wc, 43)) return false;
        if (which == 0 && !mbar_wait(&k_full[s_g % KS], (s_g / KS) & 1, wc, 44)) return false;
        if (which == 1 && !mbar_wait(&v_full[s_g % VS], (s_g / VS) & 1, wc, 45)) return false;
        // buffer b is free once dQ += G K of tile s_g - NB has read G
        if (s_g >= NB && !mbar_wait(&mma_done[b], ((s_g / NB) - 1) & 1, wc, 46)) return false;
        tc_fence_after();
        const uint64_t dA = sdesc_sw128(smem_u32(smem + (which ? C::kSdO : C::kSQ) + qb * C::kQTile), 16, 1024);
        const uint64_t dB = sdesc_sw128(
            smem_u32(smem + (which ? C::kSV + (s_g % VS) * C::kKTile : C::kSK + (s_g % KS) * C::kKTile)), 16, 1024);
        const uint32_t dst = tmem + (which ? C::kTdP : C::kTS) + b * 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t oq_ = ((kk >> 2) * C::kQHalf + (kk & 3) * 32) >> 4;
          const uint32_t ok_ = ((kk >> 2) * C::kKHalf + (kk & 3) * 32) >> 4;
          mma_ss(dst, dA + oq_, dB + ok_, idS, kk > 0);
        }
        mma_commit(&s_full[b]);
        if (which == 1) mma_commit(&v_empty[s_g % VS]);  // V feeds only dP
        if (s_t == s_it.n_count - 1) mma_commit(&q_empty[qb]);  // Q and dO feed only the score products
        ++s_g;
        if (++s_t == s_it.n_count) {
          s_t = 0;
          ++s_i;
          s_idx = q_slot(p, s_i);
          s_have = s_idx >= 0;
          if (s_have) s_it = q_item(p, s_idx);
        }
        return true;
      };
      auto issue_dq = [&]() -> bool {
        const int b = u_g % NB;
        if (!mbar_wait(&g_full[b], (u_g / NB) & 1, wc, 47)) return false;
        if (u_t == 0 && u_i >= 1 && !mbar_wait(dq_empty, (u_i - 1) & 1, wc, 48)) return false;
        tc_fence_after();
        // K as the MN-major B operand (N = head dim): 64-column blocks kKHalf apart, a K step of
        // 16 keys is 16 rows = 2048 B
        const uint64_t dKmn = sdesc_sw128(smem_u32(smem + C::kSK + (u_g % KS) * C::kKTile), C::kKHalf, 1024);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)  // 16 keys per step: 8 packed TMEM columns of G
          mma_ts(tmem + C::kTdQ, tmem + C::kTS + b * 64 + kk * 8, dKmn + kk * 128, idQ, (u_t == 0 && kk == 0) ? 0u : 1u);
        mma_commit(&k_empty[u_g % KS]);
        mma_commit(&mma_done[b]);
        if (u_t == u_it.n_count - 1) mma_commit(dq_full);
        ++u_g;
        if (++u_t == u_it.n_count) {
          u_t = 0;
          ++u_i;
          u_idx = q_slot(p, u_i);
          u_have = u_idx >= 0;
          if (u_have) u_it = q_item(p, u_idx);
        }
        return true;
      };
      const int role = warp == 1 ? 0 : warp - 9;  // 0: S, 1: dP, 2: dQ
      if (role < 2) {
        while (ok && s_have) ok = issue_sdp(role);
      } else {
        while (ok && u_have) ok = issue_dq();
      }
      if (!ok) {  // wait for this thread's products in flight before TMEM is released
        mma_commit(drain + role);
        mbar_wait_drain(drain + role, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ pointwise (query rows), warps 2-9
    const int wg = (warp - 2) >> 2;
    const int lg = warp & 3;
    const int row = lg * 32 + lane;  // query row within the item == TMEM lane
    int* docs_k = docs_all + (wg * 4 + lg) * BN;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    bool ok = true;
    int g = 0, i = 0;
    // per-item, per-row parameters from global memory; the next item's are requested before the
    // current item's epilogue
    QItem it_n{};
    Map map_n{};
    int doc_n = 0;
    float zinv_n = 0.f, dlz_n = 0.f;
    auto fetch = [&](int idx) {
      it_n = q_item(p, idx);
      map_n = BwdMap<Map>::make(p, it_n.h);
      const int q = it_n.m0 + row;
      const int64_t vrow = ((int64_t)it_n.b * p.H + it_n.h) * p.Tpad + q;  // q < Tpad (a multiple of 128)
      const float2 zd = reinterpret_cast<const float2*>(p.zd)[vrow];
      zinv_n = zd.x;
      dlz_n = zd.y;
      if constexpr (kHasDoc) doc_n = q < p.T ? p.doc[(int64_t)it_n.b * p.doc_s0 + (int64_t)q * p.doc_s1] : -1;
    };
    if (q_slot(p, 0) >= 0) fetch(q_slot(p, 0));
    for (int idx = q_slot(p, 0); idx >= 0 && ok; idx = q_slot(p, i + 1), ++i) {
      const QItem it = it_n;
      const Map map = map_n;
      const int doc_i = doc_n;
      const float zinv = zinv_n, dlz = dlz_n;
      (void)doc_i;
      const int qi = it.m0 + row;
      float unused1 = 0.f, unused2 = 0.f;
      for (int t = (wg - g) & 1; t < it.n_count && ok; t += 2) {
        const int gg = g + t;  // gg % 2 == wg
        const int b = gg % NB;
        const int n0 = it.n_first + t * BN;
        if constexpr (kHasDoc) {
#pragma unroll
          for (int u = 0; u < BN / 32; ++u) {
            const int kj = n0 + u * 32 + lane;
            docs_k[u * 32 + lane] = kj < p.T ? p.doc[(int64_t)it.b * p.doc_s0 + (int64_t)kj * p.doc_s1] : -2;
          }
          __syncwarp();
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (gg / NB) & 1, wc, 50));
        if (!ok) break;
        tc_fence_after();
        const bool full = !kHasDoc && (!p.causal || n0 + BN - 1 <= it.m0) &&
                          (p.window <= 0 || (it.m0 + C::kBM - 1) - n0 < p.window) && (n0 + BN <= p.T);
        const uint32_t s_col = lane_addr + C::kTS + b * 64, p_col = lane_addr + C::kTdP + b * 64;
        // Partial tiles: invalid pairs get raw = NaN before the map, which yields dL/draw = 0
        // (fmaxf returns its non-NaN operand), so one branch-free body serves every tile.
        // Two 32-key chunks; chunk c writes G (16 packed columns) over S columns [16c, 16c + 16),
        // which chunk 0 has already read.
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t rs[32], rd[32];
          tmem_ld32(s_col + c * 32, rs);
          tmem_ld32(p_col + c * 32, rd);
          tmem_wait_ld();
          if (!full) {
            const int kbase = n0 + c * 32;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              int doc_j = 0;
              if constexpr (kHasDoc) doc_j = docs_k[c * 32 + e];
              const bool v = pair_valid(qi, kbase + e, p.T, p.causal, p.window, doc_i, doc_j);
              rs[e] = v ? rs[e] : 0x7FC00000u;
            }
          }
          uint32_t gpk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float gv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u)
              gv[u] = map.grad(__uint_as_float(rs[e + u]), true, fmaf(__uint_as_float(rd[e + u]), zinv, -dlz), unused1,
                               unused2);
            gpk[e / 2] = pack2<true>(gv[0], gv[1]);
          }
          tmem_st16(s_col + c * 16, gpk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&g_full[b]);
      }
      if (!ok) break;
      if (q_slot(p, i + 1) >= 0) fetch(q_slot(p, i + 1));
      // ---- epilogue of the item: dQ rows (group wg stores head-dim columns [wg D/2, (wg+1) D/2))
      ok = __all_sync(0xffffffffu, mbar_wait(dq_full, i & 1, wc, 51));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[D / 2];
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc)
        tmem_ld32(lane_addr + C::kTdQ + wg * (D / 2) + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(r + cc * 32));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dq_empty);
      if (qi < p.T) {
        uint4* dst = reinterpret_cast<uint4*>(p.dq + (int64_t)it.b * p.dq_s0 + (int64_t)it.h * p.dq_s1 +
                                              (int64_t)qi * p.dq_s2 + wg * (D / 2));
#pragma unroll
        for (int v4 = 0; v4 < D / 16; ++v4)
          dst[v4] = make_uint4(pack2<true>(__uint_as_float(r[8 * v4]), __uint_as_float(r[8 * v4 + 1])),
                               pack2<true>(__uint_as_float(r[8 * v4 + 2]), __uint_as_float(r[8 * v4 + 3])),
                               pack2<true>(__uint_as_float(r[8 * v4 + 4]), __uint_as_float(r[8 * v4 + 5])),
                               pack2<true>(__uint_as_float(r[8 * v4 + 6]), __uint_as_float(r[8 * v4 + 7])));
      }
      g += it.n_count;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Pre pass and parameter sums
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
  float* zd;  // [BH][Tpad][2]  (1 / Z_i, delta_i / Z_i)
  const float* partials;
  int n_kv;
  float* dscale;
  float* dtau;
  int scale_per_head, tau_per_head;
};

// One block per (64-row chunk, head, batch): delta_i / Z_i, 1 / Z_i (delta_i = sum_d dO_id O_id;
// rows at or beyond T get zeros), and the chunk's sum_i eps delta_i / Z_i (the closed-form part of
// dscale / d gamma).  Eight lanes share a row (D / 8 elements each, 16-byte loads), so a warp
// reads four rows per step.
template <int D>
__global__ void __launch_bounds__(256) bwd_prep_kernel(const AuxParams a) {
  constexpr int kPer = D / 8;  // elements per lane
  const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane >> 3, part = lane & 7;  // row within the group of 4, slice of the row
  const int64_t bh = (int64_t)b * a.H + h;
  __shared__ float csum_w[8];
  float csum = 0.f;
#pragma unroll
  for (int r4 = 0; r4 < 2; ++r4) {
    const int i = chunk * 64 + warp * 8 + r4 * 4 + sub;
    const int64_t row = bh * a.Tpad + i;
    float s = 0.f;
    if (i < a.T) {
      const int d0 = part * kPer;
      const __nv_bfloat16* dop = a.dout + (int64_t)b * a.do_s0 + (int64_t)h * a.do_s1 + (int64_t)i * a.do_s2 + d0;
      const int64_t oo = (int64_t)b * a.o_s0 + (int64_t)h * a.o_s1 + (int64_t)i * a.o_s2 + d0;
#pragma unroll
      for (int v = 0; v < kPer / 8; ++v) {
        const uint4 dv = reinterpret_cast<const uint4*>(dop)[v];
        float o[8];
        if (a.out_f32) {
          const float4 x = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.out) + oo)[2 * v];
          const float4 y = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.out) + oo)[2 * v + 1];
          o[0] = x.x; o[1] = x.y; o[2] = x.z; o[3] = x.w; o[4] = y.x; o[5] = y.y; o[6] = y.z; o[7] = y.w;
        } else {
          const uint4 ov = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.out) + oo)[v];
          const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            o[2 * x] = sm100::bf16_lo(ow[x]);
            o[2 * x + 1] = sm100::bf16_hi(ow[x]);
          }
        }
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int x = 0; x < 4; ++x) s += o[2 * x] * sm100::bf16_lo(dw[x]) + o[2 * x + 1] * sm100::bf16_hi(dw[x]);
      }
    }
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (part == 0) {
      const float zi = i < a.T ? 1.f / a.z[bh * a.T + i] : 0.f;
      reinterpret_cast<float2*>(a.zd)[row] = make_float2(zi, s * zi);
      csum += a.eps * s * zi;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, off);
  if (lane == 0) csum_w[warp] = csum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += csum_w[w];
    a.prep_part[bh * (a.Tpad / 64) + chunk] = t;
  }
}

// Fixed-order sums into dscale / dtau (deterministic; replaces atomics, flash_born.py:319-322):
//   plain     dscale_h = (2 / scale_h) sum_{b,i} eps delta_i / Z_i
//   purified  dgamma_h = (4 / gamma_h) (sum_{b,i} eps delta_i / Z_i - sum eps_base b^2 dP),
//             dtau_h   = sum -4 u^3 dP gamma        (the last two from the dK/dV kernel's partials)
// One block per head: each thread sums a fixed strided subset, then a fixed-shape tree; the
// per-head terms are folded together for shared (scalar) parameters by a second kernel.
__global__ void __launch_bounds__(256) bwd_param_kernel(const AuxParams a, float* head_terms) {
  const int h = blockIdx.x;
  const int nc = a.Tpad / 64;
  __shared__ float r1[256], r2[256], rp[256];
  float tp = 0.f, t1 = 0.f, t2 = 0.f;
  for (int b = 0; b < a.B; ++b) {
    const int64_t bhh = (int64_t)b * a.H + h;
    for (int t = threadIdx.x; t < nc; t += 256) tp += a.prep_part[bhh * nc + t];
    if (a.purified) {
      const float* part = a.partials + bhh * a.n_kv * 16;
      for (int t = threadIdx.x; t < a.n_kv * 8; t += 256) {
        t1 += part[2 * t];
        t2 += part[2 * t + 1];
      }
    }
  }
  rp[threadIdx.x] = tp;
  r1[threadIdx.x] = t1;
  r2[threadIdx.x] = t2;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      rp[threadIdx.x] += rp[threadIdx.x + w];
      r1[threadIdx.x] += r1[threadIdx.x + w];
      r2[threadIdx.x] += r2[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float sc = a.scale[a.scale_per_head ? h : 0];
    const float d1 = a.purified ? (4.f / sc) * (rp[0] - r1[0]) : (2.f / sc) * rp[0];
    const float d2 = r2[0];
    if (a.scale_per_head) a.dscale[h] += d1;
    if (a.dtau != nullptr && a.tau_per_head) a.dtau[h] += d2;
    head_terms[2 * h] = d1;
    head_terms[2 * h + 1] = d2;
  }
}

// shared (scalar) scale / tau: the per-head terms added in head order
__global__ void bwd_param_shared_kernel(const AuxParams a, const float* head_terms) {
  float s1 = 0.f, s2 = 0.f;
  for (int hh = 0; hh < a.H; ++hh) {
    s1 += head_terms[2 * hh];
    s2 += head_terms[2 * hh + 1];
  }
  if (!a.scale_per_head) a.dscale[0] += s1;
  if (a.dtau != nullptr && !a.tau_per_head) a.dtau[0] += s2;
}

struct WsLayout {
  size_t zd, partials, prep_part, head_terms, docs, total;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int row_pad(int T) { return (T + kRowPad - 1) / kRowPad * kRowPad; }

WsLayout ws_layout(const Problem& p) {
  const int Tpad = row_pad(p.T);
  const size_t BH = (size_t)p.B * p.H;
  const int n_kv = (p.T + 127) / 128;
  WsLayout w;
  w.zd = 0;
  w.partials = align256(w.zd + BH * Tpad * 8);
  w.prep_part = align256(w.partials + BH * n_kv * 8 * 2 * 4);
  w.head_terms = align256(w.prep_part + BH * (Tpad / 64) * 4);
  w.docs = align256(w.head_terms + (size_t)p.H * 2 * 4);
  w.total = align256(w.docs + doc_ranges_bytes(p));
  return w;
}

int bwd_num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      n = v;
    else
      n = 148;
  }
  return n;
}

bool rows16(const Tensor4& t) {  // 16-byte vector row stores of bf16 rows
  if ((reinterpret_cast<uintptr_t>(t.ptr) & 15) != 0 || t.s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t.s[i] % 8 != 0) return false;
  return true;
}

template <int D, class Map, bool kHasDoc>
int launch_kv(cudaStream_t s, const BwdParams& bp, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq,
              const CUtensorMap& mdo) {
  auto kernel = tc_dkdv_kernel<D, Map, kHasDoc>;
  const uint32_t smem = KvCfg<D>::kSmem + 1024;  // + alignment slack
  cudaError_t e = set_smem_limit_once(reinterpret_cast<const void*>(kernel), (int)smem);
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  kernel<<<std::min(bp.n_items, bwd_num_sms()), kThreads, smem, s>>>(mk, mv, mq, mdo, bp);
  e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  return FB_OK;
}

template <int D, class Map, bool kHasDoc>
int launch_dq(cudaStream_t s, const BwdParams& bp, const CUtensorMap& mq, const CUtensorMap& mdo, const CUtensorMap& mk,
              const CUtensorMap& mv) {
  auto kernel = tc_dq_kernel<D, Map, kHasDoc>;
  const uint32_t smem = DqCfg<D>::kSmem + 1024;
  cudaError_t e = set_smem_limit_once(reinterpret_cast<const void*>(kernel), (int)smem);
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  kernel<<<std::min(bp.n_qitems, bwd_num_sms()), kThreads, smem, s>>>(mq, mdo, mk, mv, bp);
  e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  return FB_OK;
}

template <int D, class Map>
int launch_main(const Problem& pr, cudaStream_t s, const BwdParams& bp) {
  CUtensorMap kk, kv, kq, kdo, qq, qdo, qk, qv;
  const bool m3 = bp.map3 != 0;
  // key-major kernel: K / V boxes of 128 rows, Q / dO of 64; query-major: the other way round
  if (!encode_bhtd(&kk, pr.k, pr.B, pr.H, pr.T, D, 128, m3) || !encode_bhtd(&kv, pr.v, pr.B, pr.H, pr.T, D, 128, m3) ||
      !encode_bhtd(&kq, pr.q, pr.B, pr.H, pr.T, D, 64, m3) || !encode_bhtd(&kdo, pr.dout, pr.B, pr.H, pr.T, D, 64, m3) ||
      !encode_bhtd(&qq, pr.q, pr.B, pr.H, pr.T, D, 128, m3) || !encode_bhtd(&qdo, pr.dout, pr.B, pr.H, pr.T, D, 128, m3) ||
      !encode_bhtd(&qk, pr.k, pr.B, pr.H, pr.T, D, 64, m3) || !encode_bhtd(&qv, pr.v, pr.B, pr.H, pr.T, D, 64, m3))
    return FB_ERR_ALIGN;
  int rc = pr.doc ? launch_kv<D, Map, true>(s, bp, kk, kv, kq, kdo) : launch_kv<D, Map, false>(s, bp, kk, kv, kq, kdo);
  if (rc != FB_OK) return rc;
  return pr.doc ? launch_dq<D, Map, true>(s, bp, qq, qdo, qk, qv) : launch_dq<D, Map, false>(s, bp, qq, qdo, qk, qv);
}

}  // namespace

bool tc_bwd_supported(const Problem& p) {
  if (p.dtype != FB_BF16 || (p.D != 64 && p.D != 128)) return false;
  if (p.out_dtype != FB_BF16 && p.out_dtype != FB_F32) return false;
  if (!tma_ok(p.q) || !tma_ok(p.k) || !tma_ok(p.v) || !tma_ok(p.dout)) return false;
  if (!rows16(p.dq) || !rows16(p.dk) || !rows16(p.dv)) return false;
  // the pre-pass reads O rows as 16-byte vectors
  const int oelt = p.out_dtype == FB_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(p.o.ptr) & 15) != 0 || p.o.s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if ((p.o.s[i] * oelt) % 16 != 0) return false;
  return true;
}

size_t tc_bwd_workspace(const Problem& p) { return ws_layout(p).total; }

int tc_bwd(const Problem& pr, cudaStream_t s, int* launches) {
  if (!get_encoder()) return FB_ERR_NO_DEVICE;
  const WsLayout w = ws_layout(pr);
  char* ws = static_cast<char*>(pr.ws);
  const int Tpad = row_pad(pr.T);
  const int n_kv = (pr.T + 127) / 128;
  const int n_mt = (pr.T + 127) / 128;

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
  a.zd = reinterpret_cast<float*>(ws + w.zd);
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
  bp.dq = static_cast<__nv_bfloat16*>(const_cast<void*>(pr.dq.ptr));
  bp.dq_s0 = pr.dq.s[0]; bp.dq_s1 = pr.dq.s[1]; bp.dq_s2 = pr.dq.s[2];
  bp.zd = a.zd;
  bp.partials = reinterpret_cast<float*>(ws + w.partials);
  bp.n_kv = n_kv;
  bp.n_items = n_kv * pr.B * pr.H;
  bp.n_mt = n_mt;
  bp.n_qitems = n_mt * pr.B * pr.H;
  bp.status = pr.status;
  bp.map3 = bh_mergeable(pr.q, pr.H) && bh_mergeable(pr.k, pr.H) && bh_mergeable(pr.v, pr.H) &&
            bh_mergeable(pr.dout, pr.H);
  DocRanges dr;
  const int drc = doc_ranges(pr, s, ws + w.docs, &dr);
  if (drc != FB_OK) return drc;
  bp.doc_qr = dr.qr;
  bp.doc_kr = dr.kr;
  bp.nblk = dr.nblk;

  if (pr.D == 64)
    bwd_prep_kernel<64><<<dim3(Tpad / 64, pr.H, pr.B), 256, 0, s>>>(a);
  else
    bwd_prep_kernel<128><<<dim3(Tpad / 64, pr.H, pr.B), 256, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  int rc;
  if (pr.D == 64)
    rc = pr.purified ? launch_main<64, PurifiedMapTC>(pr, s, bp) : launch_main<64, PlainMapNoParam>(pr, s, bp);
  else
    rc = pr.purified ? launch_main<128, PurifiedMapTC>(pr, s, bp) : launch_main<128, PlainMapNoParam>(pr, s, bp);
  if (rc != FB_OK) return rc;
  float* head_terms = reinterpret_cast<float*>(ws + w.head_terms);
  int n = 3 + (pr.doc != nullptr ? 2 : 0);
  if (!pr.given_norm) {  // a term of a sum leaves the parameter gradients to its caller
    bwd_param_kernel<<<pr.H, 256, 0, s>>>(a, head_terms);
    ++n;
  }
  if (!pr.given_norm && (!pr.scale_per_head || (pr.purified && !pr.tau_per_head))) {
    bwd_param_shared_kernel<<<1, 1, 0, s>>>(a, head_terms);
    ++n;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  *launches = n;
  return FB_OK;
}

}  // namespace fb
