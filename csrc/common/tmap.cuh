// Host-side TMA tensor-map construction for the tcgen05 kernels that load their
// operands with cp.async.bulk.tensor (no multicast anywhere). The driver's
// encoder is resolved through the runtime, so the extension does not link
// libcuda and imports on machines without a driver.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tmap {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// Rank-`rank` tiled map with 128-byte swizzle. dims/box are innermost first; strides (bytes) are given for
// dims 1..rank-1. The innermost box extent times the element size must be 128 bytes (one swizzle row).
inline bool encode(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box) {
  EncodeTiledFn fn = encoder();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) {
      if (strides[i - 1] % 16) return false;
      s[i - 1] = strides[i - 1];
    }
  }
  return fn(map, type, rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tmap
