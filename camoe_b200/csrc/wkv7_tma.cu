// Host-side tensor-map encoding for the TMA tile loads (see wkv7_tma.cuh).
// cuTensorMapEncodeTiled is a driver API function; it is resolved once
// through the runtime's driver entry-point query, so the library needs no
// link-time dependency on libcuda.
#include <mutex>

#include "wkv7_tma.cuh"

namespace camoe {
namespace tma {
namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

}  // namespace

bool bind_context() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess;
}

bool encode_bhtn(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H) {
  const EncodeFn fn = encode_fn();
  if (fn == nullptr || B <= 0 || T <= 0 || H <= 0) return false;
  const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kRowBytes),
                                 static_cast<cuuint64_t>(H) * kRowBytes,
                                 static_cast<cuuint64_t>(T) * H * kRowBytes};
  const cuuint32_t box[4] = {64, 1, 16, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
            box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_2d_sw128(CUtensorMap* map, const void* base, int64_t inner, int64_t rows,
                     int box_rows) {
  const EncodeFn fn = encode_fn();
  if (fn == nullptr || inner < 64 || rows <= 0 || (inner * 2) % 16 != 0 || box_rows <= 0 ||
      box_rows > 256)
    return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estride[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_bhtn_f32(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H) {
  const EncodeFn fn = encode_fn();
  if (fn == nullptr || B <= 0 || T <= 0 || H <= 0) return false;
  const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {256, static_cast<cuuint64_t>(H) * 256,
                                 static_cast<cuuint64_t>(T) * H * 256};
  const cuuint32_t box[4] = {64, 1, 16, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box,
            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_bhtn_cols(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t H,
                      int n_box, bool f32) {
  const EncodeFn fn = encode_fn();
  if (fn == nullptr || B <= 0 || T <= 0 || H <= 0 || n_box <= 0 || n_box > 64 || n_box % 8 != 0)
    return false;
  const cuuint64_t row = f32 ? 256 : kRowBytes;
  const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {row, static_cast<cuuint64_t>(H) * row,
                                 static_cast<cuuint64_t>(T) * H * row};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(n_box), 1, 16, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  return fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
            const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tma
}  // namespace camoe
