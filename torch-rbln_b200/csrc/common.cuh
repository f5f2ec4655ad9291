// Device helpers shared by the sm_100a attention kernels: warp-level MMA
// wrappers, fragment transposes, fp8 conversion, streaming loads and the
// dtype-generic scalar loads used for masks and block tables.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "rbln_attn.h"

namespace rbln {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
__device__ __forceinline__ float pos_nan() { return __int_as_float(0x7fc00000); }

// ---------------------------------------------------------------------------
// Loads. KV tiles are streamed once, so they bypass L1 allocation. They use
// the coherent path (not .nc) because a decode/prefill launch may write the
// appended rows before reading them.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// 32-bit shared-state-space address of a shared-memory pointer.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Scalar loads of a runtime-typed element, used for block tables and masks.
__device__ __forceinline__ int64_t load_index(const void* base, int dtype, int64_t i) {
  switch (dtype) {
    case RBLN_DT_I16: return static_cast<const int16_t*>(base)[i];
    case RBLN_DT_I64: return static_cast<const int64_t*>(base)[i];
    default: return static_cast<const int32_t*>(base)[i];
  }
}
__device__ __forceinline__ bool load_keep(const void* base, int dtype, int64_t i) {
  switch (dtype) {
    case RBLN_DT_F32: return static_cast<const float*>(base)[i] > 0.f;
    case RBLN_DT_F16: return __half2float(static_cast<const __half*>(base)[i]) > 0.f;
    case RBLN_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]) > 0.f;
    default: return static_cast<const uint8_t*>(base)[i] != 0;
  }
}

// ---------------------------------------------------------------------------
// Warp MMA m16n8k16, fp32 accumulate. A row-major 16x16, B col-major 16x8.
// Fragment ownership (gid = lane/4, tig = lane%4):
//   A: a0 (gid, 2tig..+1) a1 (gid+8, 2tig..) a2 (gid, 2tig+8..) a3 (gid+8, 2tig+8..)
//   B: b0 (k 2tig..+1, n gid) b1 (k 2tig+8.., n gid)
//   C: c0,c1 (gid, 2tig..+1)  c2,c3 (gid+8, 2tig..+1)
// ---------------------------------------------------------------------------
template <bool kBF16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (kBF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Transpose of an 8x8 b16 matrix held one 32-bit pair per lane
// (row gid, cols 2tig..2tig+1) -> same layout of the transpose.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <bool kBF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if constexpr (kBF16) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
}

// Four e4m3 values (bytes 0..3 of w) to two f16 pairs: lo = (b0, b1),
// hi = (b2, b3); exact, every e4m3 value is representable in f16. The
// 16-bit halves are taken as register halves, with no mask or shift.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

// 2^x on the SFU.
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max_xor_rows(float v) {
  // reduce over lanes that share tig (lane%4): xor 4, 8, 16
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}
__device__ __forceinline__ float warp_sum_xor_rows(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

}  // namespace rbln
