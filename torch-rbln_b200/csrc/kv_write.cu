// Paged KV-cache write as a standalone kernel: new k/v rows [B, Hkv, S, D]
// written at logical positions [seq[b], seq[b] + S) of each sequence through
// the block table. This is the append step the decode and prefill kernels
// perform in-line (paged_decode.cu append_token, attn_prefill.cu
// paged_append_kernel; the reference's ops do it inside their compiled
// graphs, test/rbln/test_custom_kernel.py:63-79, 182-186), for callers that
// fill a cache without attending in the same call.
//
// bf16 / f16 caches: a copy. fp8-e4m3 caches with one fp32 scale per
// (block, KV head): the scale of every block the write touches is recomputed
// from the block's valid rows -- the rows the sequence already holds in that
// block (positions before seq[b]) and the new ones -- as
// scale = max(amax, 1e-6) / 448; the held rows are re-quantized from the old
// scale to the new one and the new rows quantized with it (x * (1 / scale)
// in float32, round to nearest even, saturated to +-448). Rows of the block
// past the write are left untouched.
//
// One warp per (touched block slot, KV head, K or V, sequence), HBM-bound:
// 16-byte loads of the new rows, an amax by warp shuffles, then one
// correctly rounded reciprocal of the scale per block and one multiply per
// element (q = e4m3(x * (1 / scale))). For fp8 caches whose blocks hold at
// most 256 16-byte chunks of new rows (bs x D / 8; bs <= 16 at D = 128,
// bs <= 32 at D = 64) the warp bulk-copies the block's new rows into shared
// memory as soon as the sequence start is known -- their addresses need
// nothing else -- and reads the block-table entry while they land. Larger
// blocks stream the new rows twice (amax, then quantization; the second
// read mostly hits L2).

#include "common.cuh"
#include "sm100.cuh"

namespace rbln {
namespace {

constexpr int kWriteThreads = 256;
constexpr float kFp8Max = 448.f;
constexpr int kStageChunks = 256;  // 16-byte chunks of new rows one warp stages (4 KB)

struct WriteArgs {
  const char* k_new;
  const char* v_new;
  int64_t kn_b, kn_h, kn_s, vn_b, vn_h, vn_s;  // bytes
  char* kcache;
  char* vcache;
  int64_t cs_block, cs_head, cs_tok;  // elements
  float* k_scale;
  float* v_scale;
  int64_t ss_block, ss_head;
  const int32_t* seq;
  int64_t seq_stride;
  const void* bt;
  int bt_dtype;
  int64_t bt_stride;
  int B, Hkv, S, D, bs, max_blocks, num_blocks;
  uint32_t* err;
};

__device__ __forceinline__ float from_e4m3(uint8_t q) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)q, __NV_E4M3);
  return __half2float(__half(h));
}

// 8 new values (16 bytes of bf16 / f16) as floats
template <bool IN_BF16>
__device__ __forceinline__ void unpack8(uint4 w, float (&x)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2<IN_BF16>(u[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
// 8 e4m3 values (8 bytes) as floats, times `s`
__device__ __forceinline__ void unpack8_e4m3(uint2 w, float s, float (&x)[8]) {
  const uint32_t u[2] = {w.x, w.y};
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) x[4 * i + k] = from_e4m3((uint8_t)(u[i] >> (8 * k))) * s;
}
// round to nearest even after saturating to +-448, 8 values -> 8 bytes
__device__ __forceinline__ uint2 pack8_e4m3(const float (&x)[8], float inv) {
  uint32_t u[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(x[4 * i] * inv, x[4 * i + 1] * inv), __NV_SATFINITE,
                                                 __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(x[4 * i + 2] * inv, x[4 * i + 3] * inv),
                                                 __NV_SATFINITE, __NV_E4M3);
    u[i] = (lo & 0xffffu) | (hi << 16);
  }
  return make_uint2(u[0], u[1]);
}
// pack8_e4m3 with the products x * inv taken in pairs (mul.rn.f32x2, the
// same rounding as one multiply each)
__device__ __forceinline__ uint2 pack8_e4m3x2(const float (&x)[8], float inv) {
  uint32_t u[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float a0 = x[4 * i], a1 = x[4 * i + 1], a2 = x[4 * i + 2], a3 = x[4 * i + 3];
    sm100::mul2(a0, a1, inv, inv);
    sm100::mul2(a2, a3, inv, inv);
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a0, a1), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(a2, a3), __NV_SATFINITE, __NV_E4M3);
    u[i] = (lo & 0xffffu) | (hi << 16);
  }
  return make_uint2(u[0], u[1]);
}

// Running max of |x| over 8 new values (16 bytes of bf16 / f16) kept as a
// packed pair of 16-bit values: sign bits cleared, then max.{bf16,f16}x2,
// which, like fmaxf, returns the other operand when one is NaN. Exact: the
// pair converts to floats without rounding.
template <bool IN_BF16>
__device__ __forceinline__ uint32_t amax8_packed(uint4 w, uint32_t acc) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a = u[i] & 0x7fff7fffu;
    if constexpr (IN_BF16) asm("max.bf16x2 %0, %0, %1;" : "+r"(acc) : "r"(a));
    else asm("max.f16x2 %0, %0, %1;" : "+r"(acc) : "r"(a));
  }
  return acc;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per (touched block slot j, KV head h, K or V, sequence b); the
// block's rows are walked in 8-element chunks, lane-strided, so a warp moves
// 512 contiguous source bytes per step.
template <bool IN_BF16, bool FP8>
__global__ void __launch_bounds__(kWriteThreads) paged_kv_write_kernel(const WriteArgs a, int slots) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * (kWriteThreads / 32) + warp;
  const int64_t units = (int64_t)slots * a.Hkv * 2 * a.B;
  if (unit >= units) return;
  const int j = (int)(unit % slots);
  const int64_t rest = unit / slots;
  const int part = (int)(rest & 1), h = (int)((rest >> 1) % a.Hkv), b = (int)(rest / (2 * a.Hkv));
  const int s0 = a.seq[b * a.seq_stride];
  if (s0 < 0 || (int64_t)s0 + a.S > (int64_t)a.max_blocks * a.bs) {
    if (lane == 0 && j == 0 && h == 0 && part == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_SEQ_RANGE);
    return;
  }
  const int bi = s0 / a.bs + j;
  if (bi > (s0 + a.S - 1) / a.bs) return;
  const int64_t phys = load_index(a.bt, a.bt_dtype, b * a.bt_stride + bi);
  if (phys < 0 || phys >= a.num_blocks) {
    if (lane == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
    return;
  }
  const int base = bi * a.bs;
  const int lo = max(s0, base) - base;               // first new row in the block
  const int hi = min(s0 + a.S, base + a.bs) - base;  // one past the last
  const int held = s0 > base ? lo : 0;               // rows [0, held) hold the sequence's context
  const char* src = part == 0 ? a.k_new + b * a.kn_b + h * a.kn_h : a.v_new + b * a.vn_b + h * a.vn_h;
  const int64_t src_s = part == 0 ? a.kn_s : a.vn_s;
  char* cache = part == 0 ? a.kcache : a.vcache;
  const int64_t cbase = phys * a.cs_block + (int64_t)h * a.cs_head;  // elements
  const int cpr = a.D / 8;                                           // 8-element chunks per row
  auto new_row = [&](int r) { return src + (int64_t)(base + r - s0) * src_s; };

  if constexpr (!FP8) {
    for (int i = lane; i < (hi - lo) * cpr; i += 32) {
      const int r = lo + i / cpr, c = i - (i / cpr) * cpr;
      const uint4 v = *reinterpret_cast<const uint4*>(new_row(r) + c * 16);
      *reinterpret_cast<uint4*>(cache + (cbase + (int64_t)r * a.cs_tok) * 2 + c * 16) = v;
    }
  } else {
    float* sp = (part == 0 ? a.k_scale : a.v_scale) + phys * a.ss_block + (int64_t)h * a.ss_head;
    const float old = *sp;
    uint8_t* c8 = reinterpret_cast<uint8_t*>(cache) + cbase;
    float m = 0.f;
    for (int i = lane; i < held * cpr; i += 32) {
      const int r = i / cpr, c = i - r * cpr;
      float x[8];
      unpack8_e4m3(*reinterpret_cast<const uint2*>(c8 + (int64_t)r * a.cs_tok + c * 8), old, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(x[e]));
    }
    for (int i = lane; i < (hi - lo) * cpr; i += 32) {
      const int r = lo + i / cpr, c = i - (i / cpr) * cpr;
      float x[8];
      unpack8<IN_BF16>(*reinterpret_cast<const uint4*>(new_row(r) + c * 16), x);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(x[e]));
    }
    const float scale = __fdiv_rn(fmaxf(warp_max(m), 1e-6f), kFp8Max);
    const float inv = __frcp_rn(scale);
    if (held > 0 && scale != old) {
      for (int i = lane; i < held * cpr; i += 32) {
        const int r = i / cpr, c = i - r * cpr;
        uint2* q = reinterpret_cast<uint2*>(c8 + (int64_t)r * a.cs_tok + c * 8);
        float x[8];
        unpack8_e4m3(*q, old, x);
        *q = pack8_e4m3(x, inv);
      }
    }
    for (int i = lane; i < (hi - lo) * cpr; i += 32) {
      const int r = lo + i / cpr, c = i - (i / cpr) * cpr;
      float x[8];
      unpack8<IN_BF16>(*reinterpret_cast<const uint4*>(new_row(r) + c * 16), x);
      *reinterpret_cast<uint2*>(c8 + (int64_t)r * a.cs_tok + c * 8) = pack8_e4m3(x, inv);
    }
    __syncwarp();  // every lane has read `old` before it is replaced
    if (lane == 0) *sp = scale;
  }
}

// fp8 caches, blocks of at most kStageChunks chunks: one warp per (touched
// block slot j, KV head h, K or V, sequence b), as above. Lane t copies new
// row t of the block into the warp's 4 KB stage with one bulk copy; the
// bytes in flight cost no registers, so an SM keeps 6 CTAs (48 warps, the
// limit of both the registers and the shared memory) with up to 32 KB of
// rows each in flight. The warp does not leave before its copies
// have landed (a bounded wait; on expiry it raises RBLN_DEVERR_TIMEOUT).
template <bool IN_BF16>
__global__ void __launch_bounds__(kWriteThreads) paged_kv_write_staged_kernel(const WriteArgs a, int slots) {
  constexpr int kWarps = kWriteThreads / 32;
  __shared__ __align__(128) uint4 stage[kWarps][kStageChunks];
  __shared__ __align__(8) uint64_t bars[kWarps];
  __shared__ int aborts[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t units = (int64_t)slots * a.Hkv * 2 * a.B;
  if (unit >= units) return;
  const int j = (int)(unit % slots);
  const int64_t rest = unit / slots;
  const int part = (int)(rest & 1), h = (int)((rest >> 1) % a.Hkv), b = (int)(rest / (2 * a.Hkv));
  const int s0 = a.seq[b * a.seq_stride];
  if (s0 < 0 || (int64_t)s0 + a.S > (int64_t)a.max_blocks * a.bs) {
    if (lane == 0 && j == 0 && h == 0 && part == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_SEQ_RANGE);
    return;
  }
  const int bi = s0 / a.bs + j;
  if (bi > (s0 + a.S - 1) / a.bs) return;
  const int base = bi * a.bs;
  const int lo = max(s0, base) - base;               // first new row in the block
  const int hi = min(s0 + a.S, base + a.bs) - base;  // one past the last
  const int held = s0 > base ? lo : 0;               // rows [0, held) hold the sequence's context
  const char* src = part == 0 ? a.k_new + b * a.kn_b + h * a.kn_h : a.v_new + b * a.vn_b + h * a.vn_h;
  const int64_t src_s = part == 0 ? a.kn_s : a.vn_s;
  const int cpr = a.D / 8;  // 8-element chunks per row (8 or 16)
  const int cshift = a.D == 128 ? 4 : 3;
  const int rows = hi - lo;  // at most bs <= 32: one lane per row
  const uint32_t rbytes = (uint32_t)a.D * 2;

  // stage the new rows: 16-byte aligned rows (the host checks the base and
  // the strides), rbytes a multiple of 16
  const uint32_t bar = smem_u32(&bars[warp]);
  volatile int* abort = &aborts[warp];
  if (lane == 0) {
    *abort = 0;
    sm100::mbar_init(bar, 1);
    sm100::fence_mbar_init();
    sm100::mbar_arrive_expect_tx(bar, (uint32_t)rows * rbytes);
  }
  __syncwarp();
  if (lane < rows)
    sm100::bulk_load(smem_u32(&stage[warp][lane * cpr]), src + (int64_t)(base + lo + lane - s0) * src_s, rbytes, bar);

  // while the rows land: block-table entry, old scale, held rows' amax
  const int64_t phys = load_index(a.bt, a.bt_dtype, b * a.bt_stride + bi);
  const bool bad = phys < 0 || phys >= a.num_blocks;
  if (bad && lane == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
  float* sp = nullptr;
  uint8_t* c8 = nullptr;
  float old = 0.f, m = 0.f;
  if (!bad) {
    sp = (part == 0 ? a.k_scale : a.v_scale) + phys * a.ss_block + (int64_t)h * a.ss_head;
    old = *sp;
    c8 = reinterpret_cast<uint8_t*>(part == 0 ? a.kcache : a.vcache) + phys * a.cs_block + (int64_t)h * a.cs_head;
    for (int i = lane; i < held * cpr; i += 32) {
      const int r = i >> cshift, c = i & (cpr - 1);
      float x[8];
      unpack8_e4m3(*reinterpret_cast<const uint2*>(c8 + (int64_t)r * a.cs_tok + c * 8), old, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(x[e]));
    }
  }
  if (!__all_sync(0xffffffffu, sm100::mbar_wait(bar, 0, abort))) {
    if (lane == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_TIMEOUT);
    return;
  }
  if (bad) return;

  const int n_new = rows << cshift;  // staged chunks; chunk i is row lo + (i >> cshift)
  const uint4* st = stage[warp];
  uint32_t am = 0;  // packed +0, +0
#pragma unroll
  for (int k = 0; k < kStageChunks / 32; ++k) {
    const int i = lane + 32 * k;
    if (i < n_new) am = amax8_packed<IN_BF16>(st[i], am);
  }
  {
    const float2 f = unpack2<IN_BF16>(am);
    m = fmaxf(m, fmaxf(f.x, f.y));
  }
  const float scale = __fdiv_rn(fmaxf(warp_max(m), 1e-6f), kFp8Max);
  const float inv = __frcp_rn(scale);
  if (held > 0 && scale != old) {
    for (int i = lane; i < held * cpr; i += 32) {
      const int r = i >> cshift, c = i & (cpr - 1);
      uint2* q = reinterpret_cast<uint2*>(c8 + (int64_t)r * a.cs_tok + c * 8);
      float x[8];
      unpack8_e4m3(*q, old, x);
      *q = pack8_e4m3(x, inv);
    }
  }
#pragma unroll
  for (int k = 0; k < kStageChunks / 32; ++k) {
    const int i = lane + 32 * k;
    if (i < n_new) {
      float x[8];
      unpack8<IN_BF16>(st[i], x);
      const int r = lo + (i >> cshift), c = i & (cpr - 1);
      *reinterpret_cast<uint2*>(c8 + (int64_t)r * a.cs_tok + c * 8) = pack8_e4m3x2(x, inv);
    }
  }
  __syncwarp();  // every lane has read `old` before it is replaced
  if (lane == 0) *sp = scale;
}

}  // namespace
}  // namespace rbln

extern "C" int rbln_paged_kv_write(const rbln_paged_attn_params_t* p, cudaStream_t stream) {
  using namespace rbln;
  if (!p || p->batch < 0 || p->num_kv_heads <= 0 || p->q_len < 0 || p->block_size <= 0 || p->max_blocks <= 0 ||
      p->num_blocks <= 0)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->batch == 0 || p->q_len == 0) return RBLN_OK;
  if (p->head_dim != 64 && p->head_dim != 128) return RBLN_ERR_UNSUPPORTED;
  if (p->q_dtype != RBLN_DT_BF16 && p->q_dtype != RBLN_DT_F16) return RBLN_ERR_UNSUPPORTED;
  const bool fp8 = p->kv_dtype == RBLN_DT_FP8_E4M3;
  if (!fp8 && p->kv_dtype != p->q_dtype) return RBLN_ERR_UNSUPPORTED;
  if (!p->k_new || !p->v_new || !p->kcache || !p->vcache || !p->seq || !p->block_table)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (fp8 && (!p->k_scale || !p->v_scale)) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->block_table_dtype != RBLN_DT_I16 && p->block_table_dtype != RBLN_DT_I32 &&
      p->block_table_dtype != RBLN_DT_I64)
    return RBLN_ERR_UNSUPPORTED;
  {  // 16-byte vector loads of the new rows; 16-byte (copy) or 8-byte (fp8) stores
    auto al = [](const void* q, unsigned m) { return (reinterpret_cast<uintptr_t>(q) & m) == 0; };
    const unsigned cm = fp8 ? 7u : 15u;
    const int csz = fp8 ? 1 : 2;
    if (!al(p->k_new, 15u) || !al(p->v_new, 15u) || !al(p->kcache, cm) || !al(p->vcache, cm))
      return RBLN_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 3; ++i)
      if ((p->k_new_stride[i] * 2) % 16 || (p->v_new_stride[i] * 2) % 16 || (p->cache_stride[i] * csz) % (cm + 1))
        return RBLN_ERR_INVALID_ARGUMENT;
  }
  WriteArgs a{};
  a.k_new = static_cast<const char*>(p->k_new);
  a.v_new = static_cast<const char*>(p->v_new);
  a.kn_b = p->k_new_stride[0] * 2; a.kn_h = p->k_new_stride[1] * 2; a.kn_s = p->k_new_stride[2] * 2;
  a.vn_b = p->v_new_stride[0] * 2; a.vn_h = p->v_new_stride[1] * 2; a.vn_s = p->v_new_stride[2] * 2;
  a.kcache = static_cast<char*>(p->kcache);
  a.vcache = static_cast<char*>(p->vcache);
  a.cs_block = p->cache_stride[0]; a.cs_head = p->cache_stride[1]; a.cs_tok = p->cache_stride[2];
  a.k_scale = const_cast<float*>(p->k_scale);
  a.v_scale = const_cast<float*>(p->v_scale);
  a.ss_block = p->scale_stride[0]; a.ss_head = p->scale_stride[1];
  a.seq = p->seq; a.seq_stride = p->seq_stride;
  a.bt = p->block_table; a.bt_dtype = p->block_table_dtype; a.bt_stride = p->block_table_stride;
  a.B = p->batch; a.Hkv = p->num_kv_heads; a.S = p->q_len; a.D = p->head_dim; a.bs = p->block_size;
  a.max_blocks = p->max_blocks; a.num_blocks = p->num_blocks;
  a.err = p->error_flags;
  // blocks one sequence's write can touch: S rows starting anywhere in a block
  const int slots = (p->q_len + p->block_size - 1) / p->block_size + 1;
  const int64_t units = (int64_t)slots * p->num_kv_heads * 2 * p->batch;
  const int64_t ctas = (units + kWriteThreads / 32 - 1) / (kWriteThreads / 32);
  if (ctas > INT32_MAX) return RBLN_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)ctas);
  const bool bf = p->q_dtype == RBLN_DT_BF16;
  if (fp8 && p->block_size * (p->head_dim / 8) <= kStageChunks) {
    if (bf) paged_kv_write_staged_kernel<true><<<grid, kWriteThreads, 0, stream>>>(a, slots);
    else paged_kv_write_staged_kernel<false><<<grid, kWriteThreads, 0, stream>>>(a, slots);
  } else if (fp8) {
    if (bf) paged_kv_write_kernel<true, true><<<grid, kWriteThreads, 0, stream>>>(a, slots);
    else paged_kv_write_kernel<false, true><<<grid, kWriteThreads, 0, stream>>>(a, slots);
  } else {
    if (bf) paged_kv_write_kernel<true, false><<<grid, kWriteThreads, 0, stream>>>(a, slots);
    else paged_kv_write_kernel<false, false><<<grid, kWriteThreads, 0, stream>>>(a, slots);
  }
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}
