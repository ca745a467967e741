// fb_tc_fwd.cu -- flash-Born forward on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Persistent kernel: one CTA per SM walks work items (batch, head, 128-query tile), heaviest
// first (longest-processing-time order for the causal mask), dealt out in snake order.  Each item
// walks the key tiles (128 keys) that can hold valid pairs (causal / window tile skipping, as
// flash_born.py:152-156).  The tile sequence is flattened across items, so the TMA ring, the
// TMEM double buffers and the mbarrier phases run on from one item into the next and the
// per-item set-up latency is hidden.  Warp-specialised pipeline (480 threads for d=64, 352 for
// d=128, which has no epilogue warpgroup):
//
//   warp 0      TMA producers: copies issued by one thread complete one after another (about
//               0.3 us each, whatever their size), so lane 0 requests Q of an item (double-
//               buffered, the next item's Q is fetched while the current one runs) and K_j, and
//               lane 1 requests V_j, through rings of kStages stages with separate full and empty
//               barriers: a K stage is released when S_j completes, a V stage when O += P_j V_j does
//   warp 1      TMEM owner + S issuer (one elected lane):
//                 S_g = Q K_g^T      tcgen05.mma kind::f16, A = Q (smem, K-major),
//                                    B = K_g (smem, K-major), D = S[g%2] in TMEM (fp32)
//   warp 10     O += P V issuer (one elected lane; one thread issues a tcgen05.mma at most every
//               ~50 cycles, longer than an N = 80 product takes, so the two products get a warp each):
//                 O  += P_g V_g      A = P[g%2] (TMEM, bf16 packed), B = V_g (smem, MN-major),
//                                    D = O in TMEM (fp32); the first tile of an item overwrites O.
//                                    For d=64 the same MMA also produces the row sums: N = 80,
//                                    and the B columns 64..79 are a ones tile in shared memory
//                                    (reached through the descriptor's leading-byte offset), so
//                                    TMEM columns O[64..80) accumulate Z = P 1.
//               S_{g+2} waits until the pointwise group has read S_g (p_full), so S runs up to
//               two tiles ahead of O += P V and the tensor core works while the pointwise warps
//               turn S_g into P_g.
//   warps 2-9   two pointwise ("Born") warpgroups; group w handles the tiles with g % 2 == w
//               (TMEM buffers S[w], P[w]); thread r of a group owns TMEM lane r = query row r.
//               tcgen05.ld S row -> a = relu(scale s) (masked), p = a^2, P = bf16(p) ->
//               tcgen05.st into P[w], Z += the bf16-rounded p.  No exp, no running max, no
//               rescale of O.  d=64: at an item's end the groups go straight on to the next
//               item.  d=128: the groups add their row sums, read O once, multiply by 1 / Z and
//               store O (each group half the columns) and Z.
//   warps 11-14 (d=64) epilogue warpgroup: per item, once the last O += P V has landed, read O (and Z)
//               from TMEM, release O to the next item's first product, store O * (1 / Z) and Z
//               (Z = sum p + eps).  The pointwise groups never wait at item boundaries: in
//               traces of the earlier layout, where they ran the epilogue themselves, about a
//               third of a CTA's time went to waiting for the item's last product and the store.
//
// Numerics: S and O accumulate in fp32 and PV consumes p rounded to bf16, as in the reference
// kernel (flash_born.py:156-191).  Z sums the same bf16-rounded p that PV consumes (the reference
// sums the unrounded p), so O is an exact convex combination of the v rows: a row with a single
// valid key returns that key's v exactly, and the backward's delta = dO.O cancels against dO.v
// without the bf16 rounding of p (which the 2/a factor of dS would otherwise amplify).
//
// TMEM columns (512): S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384) O [384,384+D);
// for d=64 also Z [448,464) right after O: the row sums, produced by the PV product itself.
#include <cuda.h>

#include <algorithm>
#include <type_traits>

#include "fb_common.cuh"
#include "fb_sm100.cuh"

namespace fb {
namespace {

using namespace sm100;

constexpr int kBM = 128;       // queries per item (one M=128 MMA)
constexpr int kBN = 128;       // keys per tile
constexpr int kMaxThreads = 480;  // 15 warps (d = 64), 11 warps (d = 128)
constexpr uint32_t kTmemCols = 512;

template <int D>
struct FwdCfg {
  // d=64 runs the item epilogue in a warpgroup of its own (warps 11-14); d=128 keeps it in the
  // pointwise groups: its pointwise body wants ~170 registers, more than 480 threads can have
  static constexpr bool kEpiWarps = D == 64;
  static constexpr int kThreads = kEpiWarps ? 480 : 352;
  static constexpr int kStages = D == 64 ? 5 : 2;
  // d=64: Z comes from the tensor core (the PV product is widened to N = 80 with a ones block
  // as the extra B columns, into the 16 TMEM columns after O); d=128 has no spare columns and
  // sums Z in the pointwise warps
  static constexpr bool kTcZ = D == 64;
  static constexpr int kHalves = D / 64;                // 64-column halves of a head
  static constexpr uint32_t kTileBytes = kBN * D * 2;   // one K or V tile (== one Q tile)
  static constexpr uint32_t kHalfBytes = kBN * 64 * 2;  // 16 KB
  static constexpr uint32_t kQOff = 0;                  // Q[2]
  static constexpr uint32_t kKOff = 2 * kTileBytes;
  static constexpr uint32_t kVOff = kKOff + kStages * kTileBytes;
  // 16 rows x 128 B of bf16 ones; above every V stage, so the leading-byte offset from a V
  // sub-tile to it is positive
  static constexpr uint32_t kOnesOff = kVOff + kStages * kTileBytes;
  static constexpr uint32_t kBarOff = kOnesOff + 2048;
  static constexpr uint32_t kDocOff = kBarOff + 512;             // [8 warps][kBN] int32
  static constexpr uint32_t kZOff = kDocOff + 8 * kBN * 4;         // [2 items][2 groups][kBM] fp32
  static constexpr uint32_t kSmemBytes = kZOff + 4 * kBM * 4;
  static constexpr uint32_t kTmemS = 0, kTmemP = 256, kTmemO = 384, kTmemZ = 448;
  static_assert(!kTcZ || kTmemZ == kTmemO + D, "Z columns follow O: one N = D + 16 product writes both");
};

struct FwdParams {
  int B, H, T;
  int map3;           // tensor maps address (b, h) as one merged dimension
  int n_mt, n_items;  // query tiles per head, work items
  int causal, window;
  float eps, eps_base;
  const float* scale;
  int scale_per_head;
  const float* tau;
  int tau_per_head;
  const int32_t* doc;
  int64_t doc_s0, doc_s1;
  const int2* doc_qr;  // document spans of the query blocks (null without document ids)
  const int2* doc_mm;  // per-block (min, max) document ids
  const int2* doc_runs;  // [B][T] run of equal ids around each position (rows with doc_mono = 1)
  const int* doc_mono;   // [B] the row's ids never decrease
  int nblk;
  void* out;
  int64_t o_s0, o_s1, o_s2;
  float* z;
  int* status;
  uint64_t wait_limit_ns;  // bound of every wait
  int skip_first_k;        // test hook: CTA 0 never issues its first K-tile copy
};

template <class Map> struct TcMap;
template <> struct TcMap<PlainMap> {
  __device__ static PlainMap make(const FwdParams& p, int h) { return PlainMap{p.scale[p.scale_per_head ? h : 0]}; }
};
template <> struct TcMap<PurifiedMap> {
  __device__ static PurifiedMap make(const FwdParams& p, int h) {
    return PurifiedMap{p.scale[p.scale_per_head ? h : 0], p.tau[p.tau_per_head ? h : 0], p.eps_base};
  }
};

struct Item {
  int b, h, m0, n_first, n_count;
};

// Work item idx: latest query tiles (the most keys under a causal mask) first, then (b, h).  Its
// key tiles span the causal / window range, narrowed to the documents of its rows.
__device__ __forceinline__ Item item_at(const FwdParams& p, int idx) {
  const int bh_total = p.B * p.H;
  const int mt = p.n_mt - 1 - idx / bh_total;
  const int bh = idx % bh_total;
  Item it;
  it.b = bh / p.H;
  it.h = bh % p.H;
  it.m0 = mt * kBM;
  int lo = 0, hi = p.T;
  if (p.causal) hi = min(p.T, it.m0 + kBM);
  if (p.window > 0) lo = max(0, it.m0 - p.window + 1);
  doc_narrow(p.doc_qr, p.nblk, it.b, it.m0, kBM, lo, hi);  // keys that can share a document
  lo = (lo / kBN) * kBN;
  it.n_first = lo;
  it.n_count = hi > lo ? (hi - lo + kBN - 1) / kBN : 0;
  return it;
}

// Global index of this CTA's j-th work item, or -1 when it has no more.  The items (sorted
// heaviest first by item_at) are dealt out in rows of gridDim.x, left to right on even rows and
// right to left on odd ones (snake order): every CTA's total stays within about one item of the
// others, where dealing every row left to right hands the first CTAs the heaviest item of each
// row (C2: the busiest CTA 119 key tiles against 125, the mean being 117.6; a quarter of C2's
// heads: 31 against 38).  With document ids the item sizes follow the documents, not the order,
// and every row is dealt left to right (measured faster at C4).
__device__ __forceinline__ int fwd_slot(const FwdParams& p, int j) {
  const int G = (int)gridDim.x;
  const bool back = (j & 1) && p.doc_qr == nullptr;
  const int idx = j * G + (back ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
  return idx < p.n_items ? idx : -1;
}

template <int D, class Map, bool kHasDoc, typename TO>
__global__ void __launch_bounds__(FwdCfg<D>::kThreads, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using Cfg = FwdCfg<D>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* q_full = bars + 0;           // [2]
  uint64_t* q_empty = bars + 2;          // [2]
  uint64_t* k_full = bars + 4;           // [S]
  uint64_t* v_full = bars + 4 + S;       // [S]
  uint64_t* k_empty = bars + 4 + 2 * S;  // [S]
  uint64_t* v_empty = bars + 4 + 3 * S;  // [S]
  uint64_t* s_full = bars + 4 + 4 * S;   // [2]
  uint64_t* p_full = bars + 6 + 4 * S;   // [2]
  uint64_t* pv_done = bars + 8 + 4 * S;  // [2]
  uint64_t* o_full = bars + 10 + 4 * S;
  uint64_t* o_empty = bars + 11 + 4 * S;
  uint64_t* z_bar = bars + 12 + 4 * S;   // the groups' row sums (d = 128)
  uint64_t* drain = bars + 13 + 4 * S;   // [2]
  static_assert(15 + 4 * S <= 48, "barrier area");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 48);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 49);
  int* docs_all = reinterpret_cast<int*>(smem + Cfg::kDocOff);
  float* zpart = reinterpret_cast<float*>(smem + Cfg::kZOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtx wc{abort_flag, p.status, p.wait_limit_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    for (int st = 0; st < S; ++st) {
      mbar_init(&k_full[st], 1);
      mbar_init(&v_full[st], 1);
      mbar_init(&k_empty[st], 1);
      mbar_init(&v_empty[st], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, Cfg::kEpiWarps ? 128 : 256);  // the epilogue warpgroup, or both pointwise groups
    mbar_init(z_bar, 256);
    mbar_init(drain, 1);
    mbar_init(drain + 1, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if constexpr (Cfg::kTcZ) {  // the ones tile read by the Z product (B operand)
    uint32_t* ones = reinterpret_cast<uint32_t*>(smem + Cfg::kOnesOff);
    for (int x = threadIdx.x; x < 2048 / 4; x += Cfg::kThreads) ones[x] = 0x3F803F80u;  // bf16 1.0 pairs
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmQ);
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
    // Copies issued by one thread complete one after another, so the streams are split over
    // lanes: lane 0 requests Q and K, lane 1 requests V; each walks the same tile sequence.
    if (lane < 2) {
      bool ok = true;
      int g = 0, i = 0, q_issued = 0, issued = 0;  // issued: K (lane 0) or V (lane 1) tiles requested
      uint64_t* full = lane == 0 ? k_full : v_full;
      uint64_t* empty = lane == 0 ? k_empty : v_empty;
      const CUtensorMap* map = lane == 0 ? &tmK : &tmV;
      uint8_t* ring = smem + (lane == 0 ? Cfg::kKOff : Cfg::kVOff);
      auto load_q = [&](int item_seq, const Item& it) -> bool {
        const int qb = item_seq & 1;
        if (item_seq >= 2 && !mbar_wait(&q_empty[qb], ((item_seq >> 1) - 1) & 1, wc, 1)) return false;
        mbar_arrive_expect_tx(&q_full[qb], Cfg::kTileBytes);
#pragma unroll
        for (int hf = 0; hf < Cfg::kHalves; ++hf)
          tma_load_bhtd(smem + Cfg::kQOff + qb * Cfg::kTileBytes + hf * Cfg::kHalfBytes, &tmQ, &q_full[qb], p.map3,
                        hf * 64, it.m0, it.h, it.b, p.H);
        q_issued = item_seq + 1;
        return true;
      };
      for (int idx = fwd_slot(p, 0); idx >= 0 && ok; idx = fwd_slot(p, i + 1), ++i) {
        const Item it = item_at(p, idx);
        if (lane == 0 && q_issued <= i) ok = load_q(i, it);
        for (int t = 0; t < it.n_count && ok; ++t, ++g) {
          const int st = g % S;
          // stage st is free once S_{g-S} (K) or O += P_{g-S} V_{g-S} (V) has completed
          if (g >= S) ok = mbar_wait(&empty[st], ((g / S) - 1) & 1, wc, 2 + 10 * lane);
          if (!ok) break;
          const int n0 = it.n_first + t * kBN;
          if (lane == 0 && p.skip_first_k && blockIdx.x == 0 && g == 0) {
            // test hook: this copy is never requested, so every wait on it runs into its bound
            // and the CTA takes the abort path (fb_test_born_fwd_timeout)
            issued = g + 1;
            continue;
          }
          mbar_arrive_expect_tx(&full[st], Cfg::kTileBytes);
#pragma unroll
          for (int hf = 0; hf < Cfg::kHalves; ++hf)
            tma_load_bhtd(ring + st * Cfg::kTileBytes + hf * Cfg::kHalfBytes, map, &full[st], p.map3, hf * 64, n0, it.h,
                          it.b, p.H);
          issued = g + 1;
          // once the first K of this item is on its way, fetch the next item's Q
          if (lane == 0 && t == 0 && fwd_slot(p, i + 1) >= 0) ok = load_q(i + 1, item_at(p, fwd_slot(p, i + 1)));
        }
      }
      if (!ok) {
        // abandoned: let this lane's copies already in flight land before the CTA exits
        for (int gg = max(0, issued - S); gg < issued; ++gg) mbar_wait_drain(&full[gg % S], (gg / S) & 1, wc.limit_ns);
        for (int qq = max(0, q_issued - 2); qq < q_issued; ++qq)
          mbar_wait_drain(&q_full[qq & 1], (qq >> 1) & 1, wc.limit_ns);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ S issuer
    if (elect_one()) {
      constexpr uint32_t idS = idesc_f16(1, 0, 0, kBN, kBM);  // S: A K-major, B K-major, N = 128
      bool ok = true;
      int g = 0, i = 0;
      for (int idx = fwd_slot(p, 0); idx >= 0 && ok; idx = fwd_slot(p, i + 1), ++i) {
        const Item it = item_at(p, idx);
        ok = mbar_wait(&q_full[i & 1], (i >> 1) & 1, wc, 3);
        const uint32_t q_base = smem_u32(smem + Cfg::kQOff + (i & 1) * Cfg::kTileBytes);
        for (int t = 0; t < it.n_count && ok; ++t, ++g) {
          const int st = g % S;
          ok = mbar_wait(&k_full[st], (g / S) & 1, wc, 4);
          // S[g % 2] still holds S_{g-2} until the pointwise group has read it (p_full)
          if (ok && g >= 2) ok = mbar_wait(&p_full[g & 1], ((g - 2) >> 1) & 1, wc, 13);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + Cfg::kKOff + st * Cfg::kTileBytes);
          const uint32_t d_s = tmem + Cfg::kTmemS + (g & 1) * kBN;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * Cfg::kHalfBytes + (kk & 3) * 32;
            mma_ss(d_s, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024), idS, kk > 0);
          }
          mma_commit(&s_full[g & 1]);
          mma_commit(&k_empty[st]);
          if (t == it.n_count - 1) mma_commit(&q_empty[i & 1]);
        }
      }
      if (!ok) {  // wait for this thread's products in flight before TMEM is released
        mma_commit(drain);
        mbar_wait_drain(drain, 0, wc.limit_ns);
      }
    }
    __syncwarp();
  } else if (warp == 10) {
    // ------------------------------------------------------------------ O += P V issuer
    if (elect_one()) {
      // O (and for d=64 Z): A TMEM, B MN-major, N = D (+16 ones columns)
      constexpr uint32_t idO = idesc_f16(1, 0, 1, Cfg::kTcZ ? D + 16 : D, kBM);
      const uint32_t ones_base = smem_u32(smem + Cfg::kOnesOff);
      bool ok = true;
      int g = 0, i = 0;
      for (int idx = fwd_slot(p, 0); idx >= 0 && ok; idx = fwd_slot(p, i + 1), ++i) {
        const Item it = item_at(p, idx);
        for (int t = 0; t < it.n_count && ok; ++t, ++g) {
          const int st = g % S;
          ok = mbar_wait(&p_full[g & 1], (g >> 1) & 1, wc, 5);
          if (ok) ok = mbar_wait(&v_full[st], (g / S) & 1, wc, 6);
          // the first product of an item overwrites O: the previous item's epilogue must have read it
          if (ok && t == 0 && i >= 1) ok = mbar_wait(o_empty, (i - 1) & 1, wc, 7);
          if (!ok) break;
          tc_fence_after();
          const uint32_t v_base = smem_u32(smem + Cfg::kVOff + st * Cfg::kTileBytes);
          const uint32_t a_p = tmem + Cfg::kTmemP + (g & 1) * (kBN / 2);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            // 16 keys per step: 8 packed TMEM columns of P; 16 V rows = 2048 B of the MN-major tile.
            // The leading-byte offset is the distance to the next 64-column block of B: the second
            // half of V for d=128; for d=64 the ones tile (every B row of it is ones, whatever the
            // swizzle, so each K step may read the same 2 KB)
            const uint32_t sub = v_base + kk * 2048;
            const uint32_t lbo = Cfg::kTcZ ? ones_base - sub : Cfg::kHalfBytes;
            mma_ts(tmem + Cfg::kTmemO, a_p + kk * 8, sdesc_sw128(sub, lbo, 1024), idO, (t == 0 && kk == 0) ? 0u : 1u);
          }
          mma_commit(&v_empty[st]);
          mma_commit(&pv_done[g & 1]);
          if (t == it.n_count - 1) mma_commit(o_full);
        }
      }
      if (!ok) {
        mma_commit(drain + 1);
        mbar_wait_drain(drain + 1, 0, wc.limit_ns);
      }
    }
    __syncwarp();
  } else if (Cfg::kEpiWarps && warp >= 11) {
    // ------------------------------------------------------------------ epilogue warpgroup (warps 11-14)
    // Per item: wait until the last O += P V has landed, read O and Z from TMEM, release O to the next item's first product, and store
    // O * (1 / Z) and Z.  Thread r of the group owns TMEM lane r = query row r (warp 11 + x
    // reads lane quadrant (11 + x) % 4).
    const int lg = warp & 3;
    const int row = lg * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    bool ok = true;
    int i = 0;
    for (int idx = fwd_slot(p, 0); idx >= 0 && ok; idx = fwd_slot(p, i + 1), ++i) {
      const Item it = item_at(p, idx);
      const int qi = it.m0 + row;
      static_assert(!Cfg::kEpiWarps || Cfg::kTcZ, "the epilogue warpgroup reads Z from TMEM");
      ok = __all_sync(0xffffffffu, mbar_wait(o_full, i & 1, wc, 11));
      if (!ok) break;
      tc_fence_after();
      const float zden = __uint_as_float(tmem_ld1(lane_addr + Cfg::kTmemZ)) + p.eps;
      const float inv = 1.f / zden;
      TO* orow = reinterpret_cast<TO*>(p.out) + (int64_t)it.b * p.o_s0 + (int64_t)it.h * p.o_s1 + (int64_t)qi * p.o_s2;
      // 64 columns per round (d = 128: two rounds), O released after the last round's loads
#pragma unroll
      for (int hf = 0; hf < D / 64; ++hf) {
        uint32_t r[64];
        tmem_ld32(lane_addr + Cfg::kTmemO + hf * 64, *reinterpret_cast<uint32_t(*)[32]>(r));
        tmem_ld32(lane_addr + Cfg::kTmemO + hf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
        tmem_wait_ld();
        if (hf == D / 64 - 1) {
          tc_fence_before();
          mbar_arrive(o_empty);
        }
        if (qi < p.T) {
          if constexpr (sizeof(TO) == 2) {
            uint4* dst = reinterpret_cast<uint4*>(orow + hf * 64);
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4)
              dst[v4] = make_uint4(pack2<true>(__uint_as_float(r[8 * v4]) * inv, __uint_as_float(r[8 * v4 + 1]) * inv),
                                   pack2<true>(__uint_as_float(r[8 * v4 + 2]) * inv, __uint_as_float(r[8 * v4 + 3]) * inv),
                                   pack2<true>(__uint_as_float(r[8 * v4 + 4]) * inv, __uint_as_float(r[8 * v4 + 5]) * inv),
                                   pack2<true>(__uint_as_float(r[8 * v4 + 6]) * inv, __uint_as_float(r[8 * v4 + 7]) * inv));
          } else {
            float4* dst = reinterpret_cast<float4*>(orow + hf * 64);
#pragma unroll
            for (int v4 = 0; v4 < 16; ++v4)
              dst[v4] = make_float4(__uint_as_float(r[4 * v4]) * inv, __uint_as_float(r[4 * v4 + 1]) * inv,
                                    __uint_as_float(r[4 * v4 + 2]) * inv, __uint_as_float(r[4 * v4 + 3]) * inv);
          }
        }
      }
      if (qi < p.T) p.z[((int64_t)it.b * p.H + it.h) * p.T + qi] = zden;
    }
  } else {
    // ------------------------------------------------------------------ pointwise warpgroups (warps 2-9)
    const int wg = (warp - 2) >> 2;
    const int lg = warp & 3;              // TMEM lane group of this warp
    const int row = lg * 32 + lane;       // query row within the tile == TMEM lane
    int* docs_k = docs_all + (wg * 4 + lg) * kBN;  // this warp's copy of the key tile's doc ids
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    const uint32_t s_addr = lane_addr + Cfg::kTmemS + wg * kBN;
    const uint32_t p_addr = lane_addr + Cfg::kTmemP + wg * (kBN / 2);
    bool ok = true;
    int g = 0, i = 0;
    // Per-item parameters (score map, this row's document id) come from global memory; those of
    // the next item are requested before the current item's epilogue, which hides their latency.
    Item it_n{};
    Map map_n{};
    int doc_n = 0, mono_n = 0;
    int2 run_n = make_int2(0, 0);
    auto fetch = [&](int idx) {
      it_n = item_at(p, idx);
      map_n = TcMap<Map>::make(p, it_n.h);
      if constexpr (kHasDoc) {
        const int q = it_n.m0 + row;
        doc_n = q < p.T ? p.doc[(int64_t)it_n.b * p.doc_s0 + (int64_t)q * p.doc_s1] : -1;
        mono_n = p.doc_mono[it_n.b];
        run_n = q < p.T ? p.doc_runs[(int64_t)it_n.b * p.T + q] : make_int2(0, 0);
      }
    };
    if (fwd_slot(p, 0) >= 0) fetch(fwd_slot(p, 0));
    for (int idx = fwd_slot(p, 0); idx >= 0 && ok; idx = fwd_slot(p, i + 1), ++i) {
      const Item it = it_n;
      const Map map = map_n;
      const int doc_i = doc_n;
      const int qi = it.m0 + row;
      (void)doc_i;
      // This row's valid keys as one range [klo, khi): causal, window and T always; with document
      // ids whose row never decreases (packed documents), the row's run of equal ids too.  Other
      // rows with document ids compare ids pair by pair (cmp).
      const bool cmp = kHasDoc && mono_n == 0;
      int klo = p.window > 0 ? qi - p.window + 1 : 0;
      int khi = p.causal ? min(p.T, qi + 1) : p.T;
      if constexpr (kHasDoc) {
        if (!cmp) {
          klo = max(klo, run_n.x);
          khi = min(khi, run_n.y);
        }
      }
      // d=128: row sum of the bf16-rounded p, in two independent packed-pair chains (a single
      // running sum would serialise 128 dependent adds per tile)
      f32x2 zacc[2] = {f2_make(0.f, 0.f), f2_make(0.f, 0.f)};
      auto zadd = [&](int e2, uint32_t wv) { zacc[e2 & 1] = f2_add(zacc[e2 & 1], f2_make(bf16_lo(wv), bf16_hi(wv))); };
      for (int t = (wg - g) & 1; t < it.n_count && ok; t += 2) {
        const int gg = g + t;  // gg % 2 == wg
        const int n0 = it.n_first + t * kBN;
        if (cmp) {
#pragma unroll
          for (int u = 0; u < kBN / 32; ++u) {
            const int kj = n0 + u * 32 + lane;
            docs_k[u * 32 + lane] = kj < p.T ? p.doc[(int64_t)it.b * p.doc_s0 + (int64_t)kj * p.doc_s1] : -2;
          }
          __syncwarp();
        }
        // with document ids: every row of the tile in one document?  (read before the wait, so the
        // loads' latency hides behind it)
        bool one_doc = !kHasDoc;
        if constexpr (kHasDoc) one_doc = doc_single(p.doc_mm, p.nblk, it.b, it.m0, kBM, n0, kBN);
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[wg], (gg >> 1) & 1, wc, 8));  // warp-uniform
        if (!ok) break;
        tc_fence_after();
        // whole tile valid?  (below the causal diagonal, inside the window, inside T, and with
        // document ids every row of the tile in one document)
        const bool full = one_doc && (!p.causal || n0 + kBN - 1 <= it.m0) &&
                          (p.window <= 0 || (it.m0 + kBM - 1) - n0 < p.window) && (n0 + kBN <= p.T);
        if (gg >= 2) {  // P[wg] is free once O += P_{gg-2} V_{gg-2} has completed
          ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[wg], ((gg - 2) >> 1) & 1, wc, 9));
          if (!ok) break;
        }
        // causal diagonal tile (the item's own 128 keys): chunk c of warp lg is entirely valid for
        // c < lg, entirely masked for c > lg, and valid for column e <= lane when c == lg
        const bool diag = !full && one_doc && p.causal && p.window <= 0 && n0 == it.m0;
        if (full) {
          // four 32-column chunks, software pipelined: the TMEM load of chunk c+1 is in flight
          // while chunk c is turned into P (the loads would otherwise expose their latency)
          uint32_t ra[32], rb[32];
          f32x2 sc2{};
          if constexpr (std::is_same<Map, PlainMap>::value) sc2 = f2_make(map.scale, map.scale);
          auto chunk = [&](int c, const uint32_t (&r)[32]) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              if constexpr (std::is_same<Map, PlainMap>::value) {
                // p = relu(x)^2 = relu(x |x|) with x = scale raw: one packed multiply for the
                // pair, one multiply each (|x| is an operand modifier) and the ReLU in the cvt
                const f32x2 x = f2_mul(f2_make(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), sc2);
                const float x0 = f2_lo(x), x1 = f2_hi(x);
                w[e / 2] = relu_bf16x2(x0 * fabsf(x0), x1 * fabsf(x1));
              } else {
                w[e / 2] = pack2<true>(map.prob(__uint_as_float(r[e]), true), map.prob(__uint_as_float(r[e + 1]), true));
              }
              if constexpr (!Cfg::kTcZ) zadd(e / 2, w[e / 2]);
            }
            tmem_st16(p_addr + c * 16, w);
          };
          tmem_ld32(s_addr, ra);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < kBN / 32; c += 2) {
            tmem_ld32(s_addr + (c + 1) * 32, rb);
            chunk(c, ra);
            tmem_wait_ld();
            if (c + 2 < kBN / 32) tmem_ld32(s_addr + (c + 2) * 32, ra);
            chunk(c + 1, rb);
            tmem_wait_ld();
          }
        } else if (diag) {
#pragma unroll 1
          for (int c = 0; c < kBN / 32; ++c) {
            uint32_t w[16];
            if (c > lg) {  // keys above the diagonal for every row of this warp
#pragma unroll
              for (int e = 0; e < 16; ++e) w[e] = 0u;
            } else {
              uint32_t r[32];
              tmem_ld32(s_addr + c * 32, r);
              tmem_wait_ld();
              const int lim = c < lg ? 31 : lane;
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                w[e / 2] = pack2<true>(map.prob(__uint_as_float(r[e]), e <= lim),
                                       map.prob(__uint_as_float(r[e + 1]), e + 1 <= lim));
                if constexpr (!Cfg::kTcZ) zadd(e / 2, w[e / 2]);
              }
            }
            tmem_st16(p_addr + c * 16, w);
          }
        } else if (!cmp) {
          // Compact loops (not unrolled over chunks) keep the masked variants small in the
          // instruction cache (a fully unrolled 128-column body with both variants does not fit).
          // Key column e of chunk c is valid iff klo <= n0 + 32 c + e < khi.
#pragma unroll 1
          for (int c = 0; c < kBN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(s_addr + c * 32, r);
            tmem_wait_ld();
            uint32_t w[16];
            const int lo = klo - (n0 + c * 32), hi = khi - (n0 + c * 32);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              w[e / 2] = pack2<true>(map.prob(__uint_as_float(r[e]), (e >= lo) & (e < hi)),
                                     map.prob(__uint_as_float(r[e + 1]), (e + 1 >= lo) & (e + 1 < hi)));
              if constexpr (!Cfg::kTcZ) zadd(e / 2, w[e / 2]);
            }
            tmem_st16(p_addr + c * 16, w);
          }
        } else {
          if constexpr (kHasDoc) {
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
              uint32_t r[32];
              tmem_ld32(s_addr + c * 32, r);
              tmem_wait_ld();
              uint32_t w[16];
              const int kbase = n0 + c * 32;
              const int* dk = docs_k + c * 32;
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                float pr[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  const bool valid = pair_valid(qi, kbase + e + u, p.T, p.causal, p.window, doc_i, dk[e + u]);
                  pr[u] = map.prob(__uint_as_float(r[e + u]), valid);
                }
                w[e / 2] = pack2<true>(pr[0], pr[1]);
                if constexpr (!Cfg::kTcZ) zadd(e / 2, w[e / 2]);
              }
              tmem_st16(p_addr + c * 16, w);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[wg]);
      }
      if (fwd_slot(p, i + 1) >= 0) fetch(fwd_slot(p, i + 1));
      if constexpr (Cfg::kEpiWarps) {  // the epilogue warpgroup takes the item's O; go straight on
        g += it.n_count;
        continue;
      }
      // ---- epilogue of the item (d = 128): Z (the two groups' row sums), O * (1 / Z)
      float* zp = zpart + (i & 1) * 2 * kBM;
      if constexpr (!Cfg::kTcZ) {
        zp[wg * kBM + row] = (f2_lo(zacc[0]) + f2_hi(zacc[0])) + (f2_lo(zacc[1]) + f2_hi(zacc[1]));
        mbar_arrive(z_bar);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(z_bar, i & 1, wc, 10));
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_full, i & 1, wc, 11));
      if (!ok) break;
      tc_fence_after();
      float zden;
      if constexpr (Cfg::kTcZ) {
        zden = __uint_as_float(tmem_ld1(lane_addr + Cfg::kTmemZ)) + p.eps;
      } else {
        zden = zp[row] + zp[kBM + row] + p.eps;
      }
      const float inv = 1.f / zden;
      uint32_t r[D / 2];
      // group wg handles output columns [wg D/2, (wg+1) D/2)
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) tmem_ld32(lane_addr + Cfg::kTmemO + wg * (D / 2) + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(r + cc * 32));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(o_empty);
      if (qi < p.T) {
        TO* orow = reinterpret_cast<TO*>(p.out) + (int64_t)it.b * p.o_s0 + (int64_t)it.h * p.o_s1 +
                   (int64_t)qi * p.o_s2 + wg * (D / 2);
        if constexpr (sizeof(TO) == 2) {
          uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
          for (int v4 = 0; v4 < D / 16; ++v4)
            dst[v4] = make_uint4(pack2<true>(__uint_as_float(r[8 * v4]) * inv, __uint_as_float(r[8 * v4 + 1]) * inv),
                                 pack2<true>(__uint_as_float(r[8 * v4 + 2]) * inv, __uint_as_float(r[8 * v4 + 3]) * inv),
                                 pack2<true>(__uint_as_float(r[8 * v4 + 4]) * inv, __uint_as_float(r[8 * v4 + 5]) * inv),
                                 pack2<true>(__uint_as_float(r[8 * v4 + 6]) * inv, __uint_as_float(r[8 * v4 + 7]) * inv));
        } else {
          float4* dst = reinterpret_cast<float4*>(orow);
#pragma unroll
          for (int v4 = 0; v4 < D / 8; ++v4)
            dst[v4] = make_float4(__uint_as_float(r[4 * v4]) * inv, __uint_as_float(r[4 * v4 + 1]) * inv,
                                  __uint_as_float(r[4 * v4 + 2]) * inv, __uint_as_float(r[4 * v4 + 3]) * inv);
        }
        if (wg == 0) p.z[((int64_t)it.b * p.H + it.h) * p.T + qi] = zden;
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
// Host side
// ---------------------------------------------------------------------------------------------
int num_sms() {
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

template <int D, class Map, bool kHasDoc, typename TO>
int launch_fwd(const Problem& pr, cudaStream_t s, const FwdParams& fp, const CUtensorMap& mq, const CUtensorMap& mk,
               const CUtensorMap& mv) {
  auto kernel = tc_fwd_kernel<D, Map, kHasDoc, TO>;
  const uint32_t smem = FwdCfg<D>::kSmemBytes + 1024;  // + alignment slack
  cudaError_t e = set_smem_limit_once(reinterpret_cast<const void*>(kernel), (int)smem);
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  dim3 grid(std::min(fp.n_items, num_sms()));
  kernel<<<grid, FwdCfg<D>::kThreads, smem, s>>>(mq, mk, mv, fp);
  e = cudaGetLastError();
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  return FB_OK;
}

template <int D, class Map>
int fwd_doc(const Problem& pr, cudaStream_t s, const FwdParams& fp, const CUtensorMap& mq, const CUtensorMap& mk,
            const CUtensorMap& mv) {
  const bool f32out = pr.out_dtype == FB_F32;
  if (pr.doc != nullptr)
    return f32out ? launch_fwd<D, Map, true, float>(pr, s, fp, mq, mk, mv)
                  : launch_fwd<D, Map, true, __nv_bfloat16>(pr, s, fp, mq, mk, mv);
  return f32out ? launch_fwd<D, Map, false, float>(pr, s, fp, mq, mk, mv)
                : launch_fwd<D, Map, false, __nv_bfloat16>(pr, s, fp, mq, mk, mv);
}

}  // namespace

bool tc_fwd_supported(const Problem& p) {
  if (p.dtype != FB_BF16) return false;  // f16 P could overflow (p = a^2 > 65504); fp32 needs the exact path
  if (p.D != 64 && p.D != 128) return false;
  if (!tma_ok(p.q) || !tma_ok(p.k) || !tma_ok(p.v)) return false;
  if ((reinterpret_cast<uintptr_t>(p.o.ptr) & 15) != 0 || p.o.s[3] != 1) return false;
  const int oelt = p.out_dtype == FB_F32 ? 4 : 2;
  for (int i = 0; i < 3; ++i)
    if ((p.o.s[i] * oelt) % 16 != 0) return false;
  if (p.out_dtype != FB_F32 && p.out_dtype != FB_BF16) return false;
  return true;
}

int tc_fwd(const Problem& pr, cudaStream_t s, int* launches) {
  if (!get_encoder()) return FB_ERR_NO_DEVICE;
  CUtensorMap mq, mk, mv;
  const bool map3 = bh_mergeable(pr.q, pr.H) && bh_mergeable(pr.k, pr.H) && bh_mergeable(pr.v, pr.H);
  if (!encode_bhtd(&mq, pr.q, pr.B, pr.H, pr.T, pr.D, kBM, map3) ||
      !encode_bhtd(&mk, pr.k, pr.B, pr.H, pr.T, pr.D, kBN, map3) ||
      !encode_bhtd(&mv, pr.v, pr.B, pr.H, pr.T, pr.D, kBN, map3))
    return FB_ERR_ALIGN;
  FwdParams fp{};
  fp.map3 = map3;
  fp.B = pr.B; fp.H = pr.H; fp.T = pr.T;
  fp.n_mt = (pr.T + kBM - 1) / kBM;
  fp.n_items = fp.n_mt * pr.B * pr.H;
  fp.causal = pr.causal; fp.window = pr.window;
  fp.eps = pr.eps; fp.eps_base = pr.eps_base;
  fp.scale = pr.scale; fp.scale_per_head = pr.scale_per_head;
  fp.tau = pr.tau; fp.tau_per_head = pr.tau_per_head;
  fp.doc = pr.doc; fp.doc_s0 = pr.doc_s[0]; fp.doc_s1 = pr.doc_s[1];
  DocRanges dr;
  const int drc = doc_ranges(pr, s, pr.ws, &dr);  // workspace of doc_ranges_bytes(pr) bytes
  if (drc != FB_OK) return drc;
  fp.doc_qr = dr.qr;
  fp.doc_mm = dr.mm;
  fp.doc_runs = dr.runs;
  fp.doc_mono = dr.mono;
  fp.nblk = dr.nblk;
  fp.out = const_cast<void*>(pr.o.ptr);
  fp.o_s0 = pr.o.s[0]; fp.o_s1 = pr.o.s[1]; fp.o_s2 = pr.o.s[2];
  fp.z = pr.z;
  fp.status = pr.status;
  fp.wait_limit_ns = pr.wait_limit_ns ? pr.wait_limit_ns : sm100::kWaitLimitNs;
  fp.skip_first_k = pr.test_skip_first_k;
  int rc;
  if (pr.D == 64)
    rc = pr.purified ? fwd_doc<64, PurifiedMap>(pr, s, fp, mq, mk, mv) : fwd_doc<64, PlainMap>(pr, s, fp, mq, mk, mv);
  else
    rc = pr.purified ? fwd_doc<128, PurifiedMap>(pr, s, fp, mq, mk, mv) : fwd_doc<128, PlainMap>(pr, s, fp, mq, mk, mv);
  if (rc == FB_OK) *launches = 1 + (pr.doc != nullptr ? 2 : 0);
  return rc;
}

}  // namespace fb
