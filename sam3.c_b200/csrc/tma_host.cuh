// tma_host.cuh - host-side creation of TMA tensor maps (cuTensorMapEncodeTiled
// reached through the runtime's driver entry point, so the library needs no
// link-time dependency on libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

namespace s3 {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor [rows, cols] of `elem` bytes per element, row pitch
// `ld` elements; box = [box_rows, box_cols].  Returns false on failure
// (misaligned base/pitch, bad box, missing driver entry point).
inline bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem,
                         uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                         uint32_t box_cols, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = get_encode_tiled();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if ((ld * elem) % 16 != 0) return false;
  if ((box_cols * elem) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// NHWC tensor [n, h, w, c] (dense), boxes of (box_c, box_w, box_h, 1).
inline bool make_tmap_nhwc(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem, uint64_t n,
                           uint64_t h, uint64_t w, uint64_t c, uint32_t box_c, uint32_t box_w, uint32_t box_h,
                           CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = get_encode_tiled();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if ((c * elem) % 16 != 0 || (box_c * elem) % 16 != 0) return false;
  cuuint64_t dims[4] = {c, w, h, n};
  cuuint64_t strides[3] = {c * elem, w * c * elem, h * w * c * elem};
  cuuint32_t box[4] = {box_c, box_w, box_h, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace s3
