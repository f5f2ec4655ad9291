// Thin wrappers over the sm_100a primitives used by the tensor-core kernels:
// mbarriers (with bounded waits), TMA tensor loads, tcgen05 MMA / TMEM
// alloc / load / store, and the UMMA shared-memory and instruction
// descriptors. Descriptor bit layouts follow the PTX ISA (tcgen05 "matrix
// descriptor" and "instruction descriptor" for kind::f16).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace rbln {
namespace sm100 {

// A wait that has not completed after this many SM clock cycles (~1-2 s)
// gives up: the kernel raises an error flag and returns instead of hanging.
constexpr long long kWaitLimitCycles = 4000000000LL;

using rbln::smem_u32;

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase with `parity` completed; false after the
// wait limit or when *abort is set by another role of the CTA.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort = 1;
      return false;
    }
  }
}

// --------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
// Untiled bulk copy global -> shared (no multicast); both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z,
                                            int w, int v) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
      "%7}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// Generic-proxy shared-memory writes -> visible to the async proxy (MMA/TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Per-warpgroup register reallocation (all 4 warps of the warpgroup execute
// it). The counts of all warpgroups must add up to no more than the
// registers the CTA was launched with.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/f16 in, f32 acc)
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16: A (M=128 rows on the 128
// TMEM lanes, K along the columns, two 16-bit elements per 32-bit column,
// lower k in the low half) is read from tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive on `bar` when all tcgen05.mma issued so far by this thread complete.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns per warp: thread t gets lane
// (quadrant*32 + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100
// version bits = 1. `addr` is the shared-state-space byte address of the
// (1024-byte aligned) swizzle atom's first row plus the in-row k offset.
//   K-major operand : lbo unused (16 B), sbo = 1024 B (8 rows x 128 B)
//   MN-major operand: lbo = distance between 64-element MN panels,
//                     sbo = 1024 B (8 k-rows x 128 B)
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for tcgen05.mma kind::f16 with f32 accumulation.
//   bits [4,6) D format (1 = f32); [7,10) A format, [10,13) B format
//   (0 = f16, 1 = bf16); bit 15 A major, bit 16 B major (0 = K, 1 = MN);
//   [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Packed fp32 pairs (sm_100a f32x2 instructions): one issue slot for two
// values.
__device__ __forceinline__ void fma2(float& a, float& b, float m0, float m1, float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rm, rc;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rm, {%2, %3};\n\t"
      "mov.b64 rc, {%4, %5};\n\tfma.rn.f32x2 ra, ra, rm, rc;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a), "+f"(b)
      : "f"(m0), "f"(m1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& a, float& b, float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rc;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rc, {%2, %3};\n\t"
      "add.rn.f32x2 ra, ra, rc;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a), "+f"(b)
      : "f"(c0), "f"(c1));
}
__device__ __forceinline__ void mul2(float& a, float& b, float m0, float m1) {
  asm("{\n\t.reg .b64 ra, rm;\n\tmov.b64 ra, {%0, %1};\n\tmov.b64 rm, {%2, %3};\n\t"
      "mul.rn.f32x2 ra, ra, rm;\n\tmov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a), "+f"(b)
      : "f"(m0), "f"(m1));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of x <= 8 on the FMA pipe (no SFU or conversion-unit
// instruction): x = n + f with n = round(x) taken by adding 1.5 * 2^23 (the
// rounding happens in the add), f in [-0.5, 0.5]; 2^f by a cubic with
// minimax relative error 7.5e-5 (2^-13.7) on that interval; 2^n built as the
// float with exponent field n + 127 by an integer multiply-add on the bits of
// the shifted value. x is clamped to -127 first, where the scale is exactly
// 0, so masked scores (-inf) give exactly 0.
__device__ __forceinline__ void exp2_poly2(float& x0, float& x1) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  x0 = fmaxf(x0, -127.f);
  x1 = fmaxf(x1, -127.f);
  float t0 = x0, t1 = x1;
  add2(t0, t1, kRound, kRound);
  float f0 = t0, f1 = t1;
  add2(f0, f1, -kRound, -kRound);        // round(x)
  fma2(f0, f1, -1.f, -1.f, x0, x1);      // f = x - round(x)
  float p0 = 0.05517132207751274f, p1 = 0.05517132207751274f;
  fma2(p0, p1, f0, f1, 0.24261054396629333f, 0.24261054396629333f);
  fma2(p0, p1, f0, f1, 0.6932609677314758f, 0.6932609677314758f);
  fma2(p0, p1, f0, f1, 0.9999281167984009f, 0.9999281167984009f);
  // bits(t) = 0x4B400000 + n, and 0x4B400000 * 2^23 = 0 (mod 2^32)
  const float s0 = __uint_as_float(__float_as_uint(t0) * 0x800000u + 0x3F800000u);
  const float s1 = __uint_as_float(__float_as_uint(t1) * 0x800000u + 0x3F800000u);
  mul2(p0, p1, s0, s1);
  x0 = p0;
  x1 = p1;
}

}  // namespace sm100
}  // namespace rbln
