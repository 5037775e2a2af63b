// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace ipuc {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D tile map over a [d2][d1][d0] tensor (d0 innermost, element strides s1, s2),
// box {b0, b1, 1}, 128-byte swizzle, zero fill out of bounds.
inline ipuc_status make_map_3d(CUtensorMap *map, CUtensorMapDataType dtype, size_t elem_bytes, const void *base,
                               uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0,
                               uint32_t b1, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return fail(IPUC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {d0, d1, d2 ? d2 : 1};
  cuuint64_t strides[2] = {s1 * elem_bytes, (s2 ? s2 : s1 * d1) * elem_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu box %u x %u", (int)r,
             (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, b0, b1);
    return fail(IPUC_ERR_CUDA, buf);
  }
  return IPUC_OK;
}

// 4-D tile map over a [d3][d2][d1][d0] tensor (d0 innermost, element strides
// s1, s2, s3 of dims 1-3), box {b0, 1, b2, 1}, 128-byte swizzle, zero fill.
// Used to read one head's rows out of a [batch][rows][heads * head_dim]
// activation: d0 = head_dim, d1 = heads, d2 = rows, d3 = batch.
inline ipuc_status make_map_4d_rows(CUtensorMap *map, CUtensorMapDataType dtype, size_t elem_bytes, const void *base,
                                    uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1, uint64_t s2,
                                    uint64_t s3, uint32_t b0, uint32_t b2) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return fail(IPUC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1 * elem_bytes, s2 * elem_bytes, s3 * elem_bytes};
  cuuint32_t box[4] = {b0, 1, b2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dtype, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[192];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu x %llu box %u x %u", (int)r,
             (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, (unsigned long long)d3, b0, b2);
    return fail(IPUC_ERR_CUDA, buf);
  }
  return IPUC_OK;
}

}  // namespace ipuc
