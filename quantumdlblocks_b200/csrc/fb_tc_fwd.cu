// fb_tc_fwd.cu -- flash-Born forward on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// One CTA owns a tile of 128 queries of one (batch, head) and walks the key tiles (128 keys)
// that can hold valid pairs (causal / window tile skipping, as flash_born.py:152-156).
// Warp-specialised pipeline (320 threads):
//
//   warp 0      TMA producer: Q tile once, then K_j / V_j through an smem ring of kStages stages
//   warp 1      TMEM owner + MMA issuer (one elected lane):
//                 S_j = Q K_j^T      tcgen05.mma kind::f16, A = Q (smem, K-major),
//                                    B = K_j (smem, K-major), D = S[j%2] in TMEM (fp32)
//                 O  += P_j V_j      A = P[j%2] (TMEM, bf16 packed), B = V_j (smem, MN-major),
//                                    D = O in TMEM (fp32)
//               S_{j+1} is issued before O += P_j V_j so the tensor core works while the
//               pointwise warps turn S_j into P_j.
//   warps 2-9   two pointwise ("Born") warpgroups; group g handles key tiles j with j % 2 == g
//               (TMEM buffers S[g], P[g]); thread r of a group owns TMEM lane r = query row r.
//               tcgen05.ld S row -> a = relu(scale s) (masked), p = a^2, Z += p (fp32),
//               P = bf16(p) -> tcgen05.st into P[g].  No exp, no running max, no rescale of O:
//               the epilogue adds the two groups' row sums, reads O once, divides by
//               Z = sum p + eps and stores O (each group half the columns) and Z.
//
// Numerics: S and O accumulate in fp32 and PV consumes p rounded to bf16, as in the reference
// kernel (flash_born.py:156-191).  Z sums the same bf16-rounded p that PV consumes (the reference
// sums the unrounded p), so O is an exact convex combination of the v rows: a row with a single
// valid key returns that key's v exactly, and the backward's delta = dO.O cancels against dO.v
// without the bf16 rounding of p (which the 2/a factor of dS would otherwise amplify).
//
// TMEM columns (512 allocated): S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384) O [384,384+D).
#include <cuda.h>

#include "fb_common.cuh"
#include "fb_sm100.cuh"

namespace fb {
namespace {

using namespace sm100;

constexpr int kBM = 128;      // queries per CTA (one M=128 MMA)
constexpr int kBN = 128;      // keys per tile
constexpr int kThreads = 320; // 10 warps
constexpr uint32_t kTmemCols = 512;

template <int D>
struct FwdCfg {
  static constexpr int kStages = D == 64 ? 3 : 2;
  static constexpr int kHalves = D / 64;                // 64-column halves of a head
  static constexpr uint32_t kTileBytes = kBN * D * 2;   // one K or V tile (== one Q tile)
  static constexpr uint32_t kHalfBytes = kBN * 64 * 2;  // 16 KB
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKOff = kTileBytes;
  static constexpr uint32_t kVOff = kKOff + kStages * kTileBytes;
  static constexpr uint32_t kBarOff = kVOff + kStages * kTileBytes;
  static constexpr uint32_t kDocOff = kBarOff + 256;             // [8 warps][kBN] int32
  static constexpr uint32_t kZOff = kDocOff + 8 * kBN * 4;         // [2 groups][kBM] fp32 row sums
  static constexpr uint32_t kSmemBytes = kZOff + 2 * kBM * 4;
  static constexpr uint32_t kTmemS = 0, kTmemP = 256, kTmemO = 384;
};

struct FwdParams {
  int B, H, T;
  int causal, window;
  float eps, eps_base;
  const float* scale;
  int scale_per_head;
  const float* tau;
  int tau_per_head;
  const int32_t* doc;
  int64_t doc_s0, doc_s1;
  void* out;
  int64_t o_s0, o_s1, o_s2;
  float* z;
  int* status;
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

// Key-tile range [first, first + count) of query tile m0 (tiles of kBN keys, aligned to kBN).
__device__ __forceinline__ void key_tiles(const FwdParams& p, int m0, int& n_first, int& n_count) {
  int lo = 0, hi = p.T;
  if (p.causal) hi = min(p.T, m0 + kBM);
  if (p.window > 0) lo = max(0, m0 - p.window + 1);
  lo = (lo / kBN) * kBN;
  n_first = lo;
  n_count = hi > lo ? (hi - lo + kBN - 1) / kBN : 0;
}

template <int D, class Map, bool kHasDoc, typename TO>
__global__ void __launch_bounds__(kThreads, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FwdParams p) {
  using Cfg = FwdCfg<D>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;             // [S]
  uint64_t* kv_empty = bars + 1 + S;        // [S]
  uint64_t* s_full = bars + 1 + 2 * S;      // [2]
  uint64_t* p_full = bars + 3 + 2 * S;      // [2]
  uint64_t* pv_done = bars + 5 + 2 * S;     // [2]
  uint64_t* o_full = bars + 7 + 2 * S;
  uint64_t* drain = bars + 8 + 2 * S;
  uint64_t* z_bar = bars + 9 + 2 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 17);
  int* docs_all = reinterpret_cast<int*>(smem + Cfg::kDocOff);  // per pointwise warp: [kBN]
  float* zpart = reinterpret_cast<float*>(smem + Cfg::kZOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = gridDim.x - 1 - blockIdx.x;  // latest (heaviest causal) query tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int m0 = tile * kBM;
  int n_first, n_count;
  key_tiles(p, m0, n_first, n_count);
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    mbar_init(z_bar, 256);
    *abort_flag = 0;
    fence_mbar_init();
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
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int issued = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, Cfg::kTileBytes);
#pragma unroll
      for (int hf = 0; hf < Cfg::kHalves; ++hf)
        tma_load_4d(smem + Cfg::kQOff + hf * Cfg::kHalfBytes, &tmQ, q_full, hf * 64, m0, h, b);
      for (int j = 0; j < n_count && ok; ++j) {
        const int st = j % S;
        if (j >= S) ok = mbar_wait(&kv_empty[st], ((j / S) - 1) & 1, wc, 1);
        if (!ok) break;
        const int n0 = n_first + j * kBN;
        mbar_arrive_expect_tx(&kv_full[st], 2 * Cfg::kTileBytes);
#pragma unroll
        for (int hf = 0; hf < Cfg::kHalves; ++hf) {
          tma_load_4d(smem + Cfg::kKOff + st * Cfg::kTileBytes + hf * Cfg::kHalfBytes, &tmK, &kv_full[st], hf * 64,
                      n0, h, b);
          tma_load_4d(smem + Cfg::kVOff + st * Cfg::kTileBytes + hf * Cfg::kHalfBytes, &tmV, &kv_full[st], hf * 64,
                      n0, h, b);
        }
        issued = j + 1;
      }
      if (!ok) {
        // abandoned: let the copies already in flight land before the CTA exits
        for (int j = max(0, issued - S); j < issued; ++j) mbar_wait_drain(&kv_full[j % S], (j / S) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = idesc_f16(1, 0, 0, kBN, kBM);  // S: A K-major, B K-major, N = 128
      constexpr uint32_t idO = idesc_f16(1, 0, 1, D, kBM);    // O: A TMEM, B MN-major, N = D
      const uint32_t q_base = smem_u32(smem + Cfg::kQOff);
      bool ok = mbar_wait(q_full, 0, wc, 3);
      for (int j = 0; j <= n_count && ok; ++j) {
        if (j < n_count) {
          const int st = j % S;
          ok = mbar_wait(&kv_full[st], (j / S) & 1, wc, 4);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + Cfg::kKOff + st * Cfg::kTileBytes);
          const uint32_t d_s = tmem + Cfg::kTmemS + (j & 1) * kBN;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * Cfg::kHalfBytes + (kk & 3) * 32;
            mma_ss(d_s, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024), idS, kk > 0);
          }
          mma_commit(&s_full[j & 1]);
        }
        if (j >= 1) {
          const int jj = j - 1;
          const int st = jj % S;
          ok = mbar_wait(&p_full[jj & 1], (jj >> 1) & 1, wc, 5);
          if (!ok) break;
          tc_fence_after();
          const uint32_t v_base = smem_u32(smem + Cfg::kVOff + st * Cfg::kTileBytes);
          const uint32_t a_p = tmem + Cfg::kTmemP + (jj & 1) * (kBN / 2);
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            // 16 keys per step: 8 packed TMEM columns of P; 16 V rows = 2048 B of the MN-major tile
            mma_ts(tmem + Cfg::kTmemO, a_p + kk * 8, sdesc_sw128(v_base + kk * 2048, Cfg::kHalfBytes, 1024), idO,
                   (jj > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&kv_empty[st]);
          mma_commit(&pv_done[jj & 1]);
        }
      }
      if (ok) {
        mma_commit(o_full);
      } else {
        mma_commit(drain);  // wait for every MMA in flight before TMEM is released
        mbar_wait_drain(drain, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ pointwise warpgroups
    // Warpgroup g (warps 2+4g .. 5+4g) turns the S tiles j with j % 2 == g into P, so it always
    // uses TMEM buffer S[g]/P[g]; the two groups' TMEM latency chains interleave on the SM.
    const int wg = (warp - 2) >> 2;
    const int lg = warp & 3;              // TMEM lane group of this warp
    const int row = lg * 32 + lane;       // query row within the tile == TMEM lane
    const int qi = m0 + row;
    int* docs_k = docs_all + (wg * 4 + lg) * kBN;  // this warp's copy of the key tile's doc ids
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    const uint32_t s_addr = lane_addr + Cfg::kTmemS + wg * kBN;
    const uint32_t p_addr = lane_addr + Cfg::kTmemP + wg * (kBN / 2);
    const Map map = TcMap<Map>::make(p, h);
    int doc_i = 0;
    if constexpr (kHasDoc) doc_i = qi < p.T ? p.doc[(int64_t)b * p.doc_s0 + (int64_t)qi * p.doc_s1] : -1;
    float zsum = 0.f;
    bool ok = true;
    for (int j = wg; j < n_count && ok; j += 2) {
      const int n0 = n_first + j * kBN;
      if constexpr (kHasDoc) {
#pragma unroll
        for (int u = 0; u < kBN / 32; ++u) {
          const int kj = n0 + u * 32 + lane;
          docs_k[u * 32 + lane] = kj < p.T ? p.doc[(int64_t)b * p.doc_s0 + (int64_t)kj * p.doc_s1] : -2;
        }
        __syncwarp();
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[wg], (j >> 1) & 1, wc, 7));  // warp-uniform
      if (!ok) break;
      tc_fence_after();
      // whole tile valid?  (below the causal diagonal, inside the window, inside T, no doc ids)
      const bool full = !kHasDoc && (!p.causal || n0 + kBN - 1 <= m0) &&
                        (p.window <= 0 || (m0 + kBM - 1) - n0 < p.window) && (n0 + kBN <= p.T);
      if (j >= 2) {  // P[wg] is free once O += P_{j-2} V_{j-2} has completed
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[wg], ((j - 2) >> 1) & 1, wc, 8));
        if (!ok) break;
      }
      if (full) {
        // 64 columns per round, both loads in flight before one wait
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t r0[32], r1[32];
          tmem_ld32(s_addr + hh * 64, r0);
          tmem_ld32(s_addr + hh * 64 + 32, r1);
          tmem_wait_ld();
          uint32_t w0[16], w1[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            w0[e / 2] = pack2<true>(map.prob(__uint_as_float(r0[e]), true), map.prob(__uint_as_float(r0[e + 1]), true));
            w1[e / 2] = pack2<true>(map.prob(__uint_as_float(r1[e]), true), map.prob(__uint_as_float(r1[e + 1]), true));
            zsum += (bf16_lo(w0[e / 2]) + bf16_hi(w0[e / 2])) + (bf16_lo(w1[e / 2]) + bf16_hi(w1[e / 2]));
          }
          tmem_st16(p_addr + hh * 32, w0);
          tmem_st16(p_addr + hh * 32 + 16, w1);
        }
      } else {
        // Compact loop (not unrolled over chunks): keeps the masked variant small in the
        // instruction cache (a fully unrolled 128-column body with both variants does not fit).
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
              int doc_j = 0;
              if constexpr (kHasDoc) doc_j = dk[e + u];
              const bool valid = pair_valid(qi, kbase + e + u, p.T, p.causal, p.window, doc_i, doc_j);
              pr[u] = map.prob(__uint_as_float(r[e + u]), valid);
            }
            w[e / 2] = pack2<true>(pr[0], pr[1]);
            zsum += bf16_lo(w[e / 2]) + bf16_hi(w[e / 2]);
          }
          tmem_st16(p_addr + c * 16, w);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[wg]);
    }
    // combine the two groups' partial row sums
    zpart[wg * kBM + row] = zsum;
    mbar_arrive(z_bar);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(z_bar, 0, wc, 10));
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_full, 0, wc, 9));
    if (ok) {
      tc_fence_after();
      const float zden = zpart[row] + zpart[kBM + row] + p.eps;
      TO* orow = reinterpret_cast<TO*>(p.out) + (int64_t)b * p.o_s0 + (int64_t)h * p.o_s1 + (int64_t)qi * p.o_s2;
      // group g stores output columns [g D/2, (g+1) D/2)
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int c = wg * (D / 64) + cc;
        uint32_t r[32];
        tmem_ld32(lane_addr + Cfg::kTmemO + c * 32, r);
        tmem_wait_ld();
        if (qi < p.T) {
          if constexpr (sizeof(TO) == 2) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
              w[e] = pack2<true>(__uint_as_float(r[2 * e]) / zden, __uint_as_float(r[2 * e + 1]) / zden);
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) dst[v4] = make_uint4(w[4 * v4], w[4 * v4 + 1], w[4 * v4 + 2], w[4 * v4 + 3]);
          } else {
            float4* dst = reinterpret_cast<float4*>(orow + c * 32);
#pragma unroll
            for (int v4 = 0; v4 < 8; ++v4)
              dst[v4] = make_float4(__uint_as_float(r[4 * v4]) / zden, __uint_as_float(r[4 * v4 + 1]) / zden,
                                    __uint_as_float(r[4 * v4 + 2]) / zden, __uint_as_float(r[4 * v4 + 3]) / zden);
          }
        }
      }
      if (qi < p.T && wg == 0) p.z[((int64_t)b * p.H + h) * p.T + qi] = zden;
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
template <int D, class Map, bool kHasDoc, typename TO>
int launch_fwd(const Problem& pr, cudaStream_t s, const FwdParams& fp, const CUtensorMap& mq, const CUtensorMap& mk,
               const CUtensorMap& mv) {
  auto kernel = tc_fwd_kernel<D, Map, kHasDoc, TO>;
  const uint32_t smem = FwdCfg<D>::kSmemBytes + 1024;  // + alignment slack
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) { record_cuda_error(e); return FB_ERR_LAUNCH; }
  dim3 grid((pr.T + kBM - 1) / kBM, pr.H, pr.B);
  kernel<<<grid, kThreads, smem, s>>>(mq, mk, mv, fp);
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
  if (!encode_bhtd(&mq, pr.q, pr.B, pr.H, pr.T, pr.D, kBM) || !encode_bhtd(&mk, pr.k, pr.B, pr.H, pr.T, pr.D, kBN) ||
      !encode_bhtd(&mv, pr.v, pr.B, pr.H, pr.T, pr.D, kBN))
    return FB_ERR_ALIGN;
  FwdParams fp{};
  fp.B = pr.B; fp.H = pr.H; fp.T = pr.T;
  fp.causal = pr.causal; fp.window = pr.window;
  fp.eps = pr.eps; fp.eps_base = pr.eps_base;
  fp.scale = pr.scale; fp.scale_per_head = pr.scale_per_head;
  fp.tau = pr.tau; fp.tau_per_head = pr.tau_per_head;
  fp.doc = pr.doc; fp.doc_s0 = pr.doc_s[0]; fp.doc_s1 = pr.doc_s[1];
  fp.out = const_cast<void*>(pr.o.ptr);
  fp.o_s0 = pr.o.s[0]; fp.o_s1 = pr.o.s[1]; fp.o_s2 = pr.o.s[2];
  fp.z = pr.z;
  fp.status = pr.status;
  int rc;
  if (pr.D == 64)
    rc = pr.purified ? fwd_doc<64, PurifiedMap>(pr, s, fp, mq, mk, mv) : fwd_doc<64, PlainMap>(pr, s, fp, mq, mk, mv);
  else
    rc = pr.purified ? fwd_doc<128, PurifiedMap>(pr, s, fp, mq, mk, mv) : fwd_doc<128, PlainMap>(pr, s, fp, mq, mk, mv);
  if (rc == FB_OK) *launches = 1;
  return rc;
}

}  // namespace fb
