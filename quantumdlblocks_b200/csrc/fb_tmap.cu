// fb_tmap.cu -- host-side TMA tensor maps over (B, H, T, D) bf16 tensors.
#include <cudaTypedefs.h>

#include <mutex>

#include "fb_common.cuh"

namespace fb {
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
bool get_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// TMA needs a 16-byte aligned base, unit inner stride and 16-byte multiples for the others.
bool tma_ok(const Tensor4& t) {
  if ((reinterpret_cast<uintptr_t>(t.ptr) & 15) != 0) return false;
  if (t.s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (t.s[i] % 8 != 0 || t.s[i] <= 0) return false;
  return true;
}

// (B, H) can be addressed as one dimension of B*H when the batch stride is H head strides.
bool bh_mergeable(const Tensor4& t, int H) { return t.s[0] == (int64_t)H * t.s[1]; }

// Map over a (B, H, T, D) bf16 tensor with box (64, box_rows) of 128-byte-swizzled rows.  With
// merge_bh the map is 3-D, dims (D, T, B*H), coordinates (x, row, b*H + h); otherwise 4-D, dims
// (D, T, H, B).  A TMA copy through a 3-D map takes less time than through a 4-D one.  Rows at or
// beyond T read as zeros (per head, since T is its own dimension).
bool encode_bhtd(CUtensorMap* m, const Tensor4& t, int B, int H, int T, int D, int box_rows, bool merge_bh) {
  if (!get_encoder()) return false;
  if (merge_bh && !bh_mergeable(t, H)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)t.s[2] * 2, (cuuint64_t)t.s[1] * 2, (cuuint64_t)t.s[0] * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  cuuint32_t rank = 4;
  if (merge_bh) {
    dims[2] = (cuuint64_t)B * H;
    rank = 3;
  }
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(t.ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D map over a row-major fp32 matrix [rows][64] (the dQ accumulator): box (32 floats, 16 rows),
// 128-byte swizzle.
bool encode_rows_f32(CUtensorMap* m, float* base, int64_t rows) {
  if (!get_encoder()) return false;
  cuuint64_t dims[2] = {64, (cuuint64_t)rows};
  cuuint64_t strides[1] = {64 * 4};
  cuuint32_t box[2] = {32, 16};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace fb
