// TMA tensor maps for the tcgen05 kernels: the driver's cuTensorMapEncodeTiled
// (looked up once through the runtime), 128-byte swizzle, zero fill for
// out-of-range coordinates.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "rbln_attn.h"

namespace rbln {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// rank-N tiled map, innermost dim first; strides in bytes for dims 1..N-1.
inline bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, void* base, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = strides_bytes[i];
  return fn(m, dt, rank, base, d, s, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline CUtensorMapDataType tmap_dtype(int dt) {
  return dt == RBLN_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// cache [NB, Hkv, rows, D] (element strides block, head, row) -> 4-D map, box {64, rpb, 1, 1}
inline bool map_kv(CUtensorMap* m, const void* c, int dt, int NB, int Hkv, int rows, int D, int64_t s_blk,
                   int64_t s_head, int64_t s_row, int rpb) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)rows, (uint64_t)Hkv, (uint64_t)NB};
  uint64_t str[3] = {(uint64_t)s_row * 2, (uint64_t)s_head * 2, (uint64_t)s_blk * 2};
  uint32_t box[4] = {64, (uint32_t)rpb, 1, 1};
  return make_map(m, tmap_dtype(dt), 4, const_cast<void*>(c), dims, str, box);
}

}  // namespace rbln
