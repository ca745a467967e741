// fb_docs.cu -- document-mask tile ranges for the tensor-core kernels.
//
// With document ids (flash_born.py:169-178: pairs are valid only within one document) most of a
// causal tile grid holds no valid pair: packed sequences of short documents leave only blocks
// near the diagonal.  Two small launches describe, for every 64-row block, which blocks of the
// other side can share a document:
//   doc_block_minmax_kernel   [B][nblk] (min, max) document id over the block's rows below T
//   doc_block_ranges_kernel   qr[b][x] = first / last key block y (y <= x when causal) whose id
//                             range meets query block x's; kr[b][x] = first / last query block
//                             (y >= x when causal) whose range meets key block x's
// Blocks whose id ranges are disjoint cannot hold a pair with equal ids, so a kernel may skip
// every tile outside [first, last]: exact for ids that increase along the sequence (packed
// documents), conservative for arbitrary ids (tiles inside the span are still processed and
// masked pair by pair).  A block always meets itself, so every span is non-empty.
//
// The same two launches also describe the runs: runs[b][t] = [first, last + 1) of the positions
// holding position t's id, and mono[b] = 1 when row b's ids never decrease along the sequence
// (the reference's document ids, a running count of end-of-text tokens, layers/attention.py:308-315,
// always do).  In such a row two positions hold the same id exactly when they lie in the same
// run, so a kernel can fold the document mask of its row into the row's valid-column range
// (two compares per pair instead of an id load and compare); rows with mono[b] = 0 keep the
// pair-by-pair compare and never read runs.
#include <climits>

#include "fb_common.cuh"

namespace fb {
namespace {

// First position in [lo, hi) whose id is above `id` (upper) or not below it (lower), for a row
// whose ids never decrease.
__device__ __forceinline__ int doc_bound(const int32_t* row, int64_t s1, int lo, int hi, int id, bool upper) {
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    const int v = row[(int64_t)mid * s1];
    if (upper ? v <= id : v < id)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(64) doc_block_minmax_kernel(const int32_t* doc, int64_t s0, int64_t s1, int T,
                                                              int nblk, int2* mm, int* srt, int2* runs) {
  const int b = blockIdx.y, blk = blockIdx.x;
  const int r = blk * kDocBlock + threadIdx.x;
  const int32_t* row = doc + (int64_t)b * s0;
  int lo = INT_MAX, hi = INT_MIN;
  bool down = false;  // the id falls from position r - 1 to r
  if (r < T) {
    const int id = row[(int64_t)r * s1];
    lo = hi = id;
    down = r > 0 && row[(int64_t)(r - 1) * s1] > id;
    // the run of id around r, valid when the whole row is non-decreasing (mono[b] = 1)
    runs[(int64_t)b * T + r] = make_int2(doc_bound(row, s1, 0, r, id, false), doc_bound(row, s1, r + 1, T, id, true));
  }
  down = __syncthreads_or(down);
  if (threadIdx.x == 0) srt[(int64_t)b * nblk + blk] = down ? 0 : 1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  __shared__ int2 w[2];
  if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = make_int2(lo, hi);
  __syncthreads();
  if (threadIdx.x == 0) mm[(int64_t)b * nblk + blk] = make_int2(min(w[0].x, w[1].x), max(w[0].y, w[1].y));
}

__global__ void __launch_bounds__(128) doc_block_ranges_kernel(const int2* mm, const int* srt, int nblk, int causal,
                                                               int2* qr, int2* kr, int* mono) {
  const int b = blockIdx.y;
  const int x = blockIdx.x * blockDim.x + threadIdx.x;
  if (x == 0) {  // the row's ids never decrease: every block sorted, its first id not below the previous block's last
    int all = 1;
    for (int y = 0; y < nblk; ++y) all &= srt[(int64_t)b * nblk + y];
    mono[b] = all;
  }
  if (x >= nblk) return;
  const int2* m = mm + (int64_t)b * nblk;
  const int2 a = m[x];
  int f = -1, l = -1;
  for (int y = 0; y < (causal ? x + 1 : nblk); ++y) {  // key blocks of query block x
    const int2 c = m[y];
    if (c.x <= a.y && a.x <= c.y) {
      if (f < 0) f = y;
      l = y;
    }
  }
  qr[(int64_t)b * nblk + x] = make_int2(f, l);
  f = l = -1;
  for (int y = causal ? x : 0; y < nblk; ++y) {  // query blocks of key block x
    const int2 c = m[y];
    if (c.x <= a.y && a.x <= c.y) {
      if (f < 0) f = y;
      l = y;
    }
  }
  kr[(int64_t)b * nblk + x] = make_int2(f, l);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

// workspace: mm, qr, kr [B][nblk] int2; srt [B][nblk] int; mono [B] int; runs [B][T] int2
size_t doc_ranges_bytes(const Problem& p) {
  if (p.doc == nullptr) return 0;
  const size_t n = (size_t)p.B * doc_blocks(p.T);
  return 3 * align256(n * sizeof(int2)) + align256(n * sizeof(int)) + align256((size_t)p.B * sizeof(int)) +
         align256((size_t)p.B * p.T * sizeof(int2));
}

int doc_ranges(const Problem& p, cudaStream_t s, void* ws, DocRanges* out) {
  out->qr = out->kr = out->mm = out->runs = nullptr;
  out->mono = nullptr;
  out->nblk = doc_blocks(p.T);
  if (p.doc == nullptr) return FB_OK;
  const size_t n = (size_t)p.B * out->nblk;
  const size_t n2 = align256(n * sizeof(int2));
  char* base = static_cast<char*>(ws);
  int2* mm = reinterpret_cast<int2*>(base);
  int2* qr = reinterpret_cast<int2*>(base + n2);
  int2* kr = reinterpret_cast<int2*>(base + 2 * n2);
  int* srt = reinterpret_cast<int*>(base + 3 * n2);
  int* mono = reinterpret_cast<int*>(base + 3 * n2 + align256(n * sizeof(int)));
  int2* runs = reinterpret_cast<int2*>(base + 3 * n2 + align256(n * sizeof(int)) + align256((size_t)p.B * sizeof(int)));
  doc_block_minmax_kernel<<<dim3(out->nblk, p.B), kDocBlock, 0, s>>>(p.doc, p.doc_s[0], p.doc_s[1], p.T, out->nblk, mm,
                                                                     srt, runs);
  doc_block_ranges_kernel<<<dim3((out->nblk + 127) / 128, p.B), 128, 0, s>>>(mm, srt, out->nblk, p.causal ? 1 : 0, qr,
                                                                           kr, mono);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return FB_ERR_LAUNCH;
  }
  out->qr = qr;
  out->kr = kr;
  out->mm = mm;
  out->runs = runs;
  out->mono = mono;
  return FB_OK;
}

}  // namespace fb
