// Host half of tma.cuh: tensor-map encoding through the driver entry point
// (the runtime hands out cuTensorMapEncodeTiled, so the library needs no
// link against libcuda).
#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace wkvm {
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
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(f);
  });
  return fn;
}

}  // namespace

int encode_rows(CUtensorMap* map, const void* base, int64_t tokens, int heads, int D, int rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return WKVM_ERR_CUDA;
  if (D <= 0 || D % 64 || rows <= 0 || rows > 256 || tokens <= 0 || heads <= 0)
    return WKVM_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(base) & 15u) return WKVM_ERR_ALIGN;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)tokens};
  // byte strides of dims 1 and 2 (multiples of 16)
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2};
  const cuuint32_t box[3] = {64u, 1u, (cuuint32_t)rows};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? WKVM_OK : WKVM_ERR_INVALID_ARG;
}

}  // namespace tma
}  // namespace wkvm
