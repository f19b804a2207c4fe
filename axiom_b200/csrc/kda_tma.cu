// Host side of the TMA tile maps (see kda_tma.cuh for the map's geometry).
#include <mutex>

#include "kda_tma.cuh"

namespace kda {
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's encoder, looked up once through the runtime (no -lcuda link).
EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

}  // namespace

bool make_tile_map(CUtensorMap* map, const void* base, int B, int T, int H) {
  if (T <= 0 || T % 8 != 0 || B <= 0 || H <= 0 || (reinterpret_cast<uintptr_t>(base) & 15u)) return false;
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t row = static_cast<cuuint64_t>(H) * 128 * 2;  // bytes between tokens
  const cuuint64_t dims[5] = {8, 8, static_cast<cuuint64_t>(H) * 16, static_cast<cuuint64_t>(T) / 8,
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[4] = {row, 16, 8 * row, static_cast<cuuint64_t>(T) * row};
  const cuuint32_t box[5] = {8, 8, 16, 8, 1};
  const cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box,
             elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_out_map(CUtensorMap* map, const void* base, int B, int T, int H) {
  if (T <= 0 || B <= 0 || H <= 0 || (reinterpret_cast<uintptr_t>(base) & 15u)) return false;
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t row = static_cast<cuuint64_t>(H) * 128 * 2;  // bytes between tokens
  const cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {256, row, static_cast<cuuint64_t>(T) * row};
  const cuuint32_t box[4] = {64, 1, 64, 1};
  const cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
             elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace kda
