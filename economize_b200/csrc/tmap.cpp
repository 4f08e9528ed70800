// Tensor-map (TMA descriptor) creation. cuTensorMapEncodeTiled is a driver API call; it is resolved once through
// cudaGetDriverEntryPoint so the extension needs no link against libcuda.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "launchers.h"

namespace ecz {

// Programmatic dependent launch is on unless ECZ_PDL=0.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ECZ_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeFn>(p);
    }
  });
  return fn;
}
}  // namespace

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                      uint32_t box_rows) {
  EncodeFn fn = encode_fn();
  if (fn == nullptr) return -2;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_elems * 2) % 16 != 0) return -3;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

int make_tmap_2d(CUtensorMap* map, int elem_bytes, const void* base, uint64_t rows, uint64_t cols,
                 uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, int swizzle_bytes) {
  EncodeFn fn = encode_fn();
  if (fn == nullptr) return -2;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || row_stride_bytes % 16 != 0) return -3;
  if ((box_cols * elem_bytes) % 16 != 0) return -3;
  CUtensorMapDataType dt;
  switch (elem_bytes) {
    case 1: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case 2: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case 4: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: return -3;
  }
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return -3;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

}  // namespace ecz
