// tma_host.h — host-side TMA tensor-map creation (driver entry point, no -lcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "capi_internal.h"

namespace hxm {

// 4-D bf16 tensor map with a {64, box_rows, 1, 1} box (box_rows <= 256; 128 unless given) and
// 128-byte swizzle.  dims / strides are innermost-first; strides in bytes for dims 1..3.
inline hxm_status make_map_bf16_4d(CUtensorMap* map, const void* base, const uint64_t dims[4],
                                   const uint64_t stride_bytes[3], const char* who, uint32_t box_rows = 128) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error("%s: cuTensorMapEncodeTiled unavailable", who);
      return HXM_ECUDA;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) {
    set_error("%s: tensor base %p not 16-byte aligned", who, base);
    return HXM_EBADARG;
  }
  for (int i = 0; i < 3; ++i)
    if (stride_bytes[i] % 16 != 0) {
      set_error("%s: stride %llu bytes not a multiple of 16", who, (unsigned long long)stride_bytes[i]);
      return HXM_EBADARG;
    }
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t st[3] = {stride_bytes[0], stride_bytes[1], stride_bytes[2]};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), d, st, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (%d)", who, (int)r);
    return HXM_ECUDA;
  }
  return HXM_OK;
}

}  // namespace hxm
