// Flash-attention forward on the sm_100a tensor cores (tcgen05 + TMEM + TMA),
// shared by the paged chunked-prefill ops and dense SDPA.
//
// Reference semantics:
//   rbln_custom_ops::paged_causal_attn_prefill / paged_attn_prefill
//     (test/rbln/test_custom_kernel.py:31-92, 262-343): write the chunk's new
//     k/v rows at positions [seq[b], seq[b] + S_q), then attend; generalised
//     to a real block table and to a causal mask offset by seq[b];
//   aten::_scaled_dot_product_fused_attention_overrideable
//     (torch_rbln/_internal/kernels/sdpa.py:670-751 with the math of
//     _sdpa_cpu_fallback, sdpa.py:244-289): softmax(Q K^T * scale + mask) V,
//     GQA by head ratio, top-left causal.
//
// One CTA computes a 128-row query tile: the G query heads that share a KV
// head are stacked into the M dimension (rows = G heads x 128/G tokens), so
// each K/V tile fetched from HBM feeds all G heads. Warp roles:
//   warp 0     TMA producer: Q once; K and V tiles of 128 keys into a
//              2-stage ring of 128B-swizzled shared-memory panels. Paged K/V
//              are fetched block by block through the block table (4-D tensor
//              map over [num_blocks, Hkv, block_size, D]); a block outside the
//              table or the pool is fetched at an out-of-range coordinate,
//              which the TMA unit fills with zeros.
//   warp 1     TMEM owner and MMA issuer (one thread): S = Q K^T into one of
//              two TMEM buffers (128 fp32 columns each), O += P V into a third.
//   warps 2-5  softmax: thread = query row (TMEM lane), fp32 online softmax
//              in the log2 domain with lazy rescaling of O (only when the
//              running max grows by more than 8), P written to shared memory
//              as bf16/f16 in the operand layout of the PV MMA; epilogue.
// The QK MMA of tile j+1 is issued before the PV MMA of tile j, so the tensor
// cores work while the softmax warps process the previous tile.
// Every mbarrier wait is bounded (sm100.cuh); on timeout the CTA raises
// RBLN_DEVERR_TIMEOUT, drains its copies and MMAs, frees TMEM and returns.

#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_map.cuh"

namespace rbln {
namespace {

using namespace sm100;

constexpr int BM = 128;                 // query rows per CTA
constexpr int BN = 128;                 // keys per KV tile
constexpr int kThreads = 192;           // 6 warps
constexpr int kPanelBytes = 128 * 128;  // 128 rows x 128 bytes

enum MaskMode : int {
  MM_CAUSAL = 0,  // key <= seq_off + s
  MM_NONE = 1,    // every written key (paged: < seq_off + S_q; dense: < S)
  MM_KEEP = 2,    // keep-mask value > 0 (paged_attn_prefill)
};

struct AttnArgs {
  // output rows [B, Hkv, G, S_q, D]; strides in bytes
  char* out;
  int64_t os_b, os_h, os_g, os_s;
  float* lse;  // optional [B, Hkv, G, S_q] (natural-log logsumexp), element strides
  int64_t ls_b, ls_h, ls_g, ls_s;
  const int32_t* seq;  // per-sequence start offset (nullptr = 0)
  int64_t seq_stride;
  const void* bt;  // block table (nullptr = dense: block id = b)
  int bt_dtype;
  int64_t bt_stride;
  int max_blocks;
  int num_blocks;  // pool size (dense: B)
  int bs;          // tokens per block (dense: S rounded up to 128)
  int span;        // addressable keys per sequence
  int kv_extra;    // dense: number of keys S
  int B, Hkv, G, S_q, QT, q_tiles;
  int mask_mode;
  const void* mask;  // keep-mask (paged) or SDPA mask
  int mask_dtype;
  int mask_additive;  // 1: add mask * log2e to scores (SDPA float mask)
  int mask_len;
  int64_t m_b, m_h, m_s;  // element strides (h indexes query heads h*G+g); key stride 1
  const void* pmask;      // optional position keep-mask [B, L]
  int pmask_dtype;
  int pmask_len;
  int64_t pm_b;
  float scale;
  const float* scale_dev;
  uint32_t* err;
  const int* work;  // optional: items (b * q_tiles + tile) in launch order, longest first
  int* counter;     // optional: next unit of a persistent launch (zeroed by the schedule pre-pass)
  const float* sinks;  // optional [Hkv * G] sink logits (natural-log units), index h * G + g
  // 128-key kernel with a keep rule other than plain causal / bidirectional
  // (a keep-mask, or a position mask): written by the mask pre-pass
  const uint4* kbits;  // [B][S_q][nkt]: bit e of word w keeps key 128 * kt + 32 * w + e for that query row
  const int* tlist;    // [items][nkt]: each item's key tiles with a kept key, bit 31 set when not all kept
  const int* tcount;   // [items]: entries of each item's list
  int nkt;             // key tiles per row, ceil(span / 128)
};

__device__ __forceinline__ float mask_value(const void* base, int dt, int64_t i) {
  switch (dt) {
    case RBLN_DT_F32: return static_cast<const float*>(base)[i];
    case RBLN_DT_F16: return __half2float(static_cast<const __half*>(base)[i]);
    case RBLN_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
    default: return static_cast<const uint8_t*>(base)[i] ? 1.f : 0.f;
  }
}

// Keys this CTA must visit, [0, kv_end).
__device__ __forceinline__ int cta_kv_end(const AttnArgs& a, int s0, int seq_off) {
  const int s_hi = min(s0 + a.QT, a.S_q);  // exclusive
  int end;
  if (a.mask_mode == MM_KEEP) {
    end = min(a.span, a.mask_len);
  } else if (a.mask_mode == MM_CAUSAL) {
    end = seq_off + s_hi;
  } else {
    end = (a.bt == nullptr) ? a.kv_extra : seq_off + a.S_q;
  }
  if (a.bt == nullptr) end = min(end, a.kv_extra);
  return max(0, min(end, a.span));
}

template <int D>
struct SmemLayout {
  static constexpr int NP = D / 64;                    // 64-element panels along D
  static constexpr int Q = 0;                          // NP panels
  static constexpr int K0 = Q + NP * kPanelBytes;      // stage s: K0 + s*NP*panel
  static constexpr int V0 = K0 + 2 * NP * kPanelBytes;
  static constexpr int P = V0 + 2 * NP * kPanelBytes;  // 2 panels (128 keys)
  static constexpr int BAR = P + 2 * kPanelBytes;      // mbarriers
  static constexpr int TMEM_SLOT = BAR + 16 * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int TOTAL = ABORT + 8;
  // + alignment slack; at least 120 KB so that only one CTA (which holds all
  // 512 TMEM columns) is resident per SM
  static constexpr int ALLOC = (TOTAL + 1024 > 120 * 1024) ? TOTAL + 1024 : 120 * 1024;
};

enum Bar { B_Q = 0, B_KF0, B_KF1, B_VF0, B_VF1, B_KE0, B_KE1, B_SF0, B_SF1, B_SR0, B_SR1, B_PF, B_PV, B_DONE, B_COUNT };

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  using L = SmemLayout<D>;
  constexpr int NP = L::NP;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  volatile int* abort = reinterpret_cast<volatile int*>(sgen + L::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + L::TMEM_SLOT);
  auto bar = [&](int i) { return sbase + L::BAR + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = qtile * a.QT;
  const int seq_off = a.seq ? a.seq[b * a.seq_stride] : 0;
  const int kv_end = (seq_off < 0) ? 0 : cta_kv_end(a, s0, seq_off);
  const int ntiles = (kv_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    *abort = 0;
    for (int i = 0; i < B_COUNT; ++i) {
      const uint32_t cnt = (i == B_SR0 || i == B_SR1 || i == B_PF) ? 4u : 1u;
      mbar_init(bar(i), cnt);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (ntiles > 0) {
      if (lane == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        // the Q box holds QT x G rows (fewer than 128 when G does not divide 128)
        mbar_arrive_expect_tx(bar(B_Q), NP * a.QT * a.G * 128);
        for (int p = 0; p < NP; ++p)
          tma_load_5d(sbase + L::Q + p * kPanelBytes, &tm_q, bar(B_Q), p * 64, s0, 0, h, b);
      }
      const int rpb = min(a.bs, BN);
      const int nbox = BN / rpb;
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        // warp-uniform decision: every lane of the producer warp waits, all break together
        if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(bar(B_KE0 + st), ((j >> 1) - 1) & 1, abort))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(bar(B_KF0 + st), NP * kPanelBytes);
          mbar_arrive_expect_tx(bar(B_VF0 + st), NP * kPanelBytes);
        }
        __syncwarp();
        const int t0 = j * BN;
        for (int i = lane; i < nbox; i += 32) {
          const int key = t0 + i * rpb;
          int blk = a.num_blocks;  // out of range -> zero fill
          int row = 0;
          if (key < kv_end) {
            if (a.bt == nullptr) {
              blk = b;
              row = key;
            } else {
              const int bi = key / a.bs;
              row = key - bi * a.bs;
              if (bi < a.max_blocks) {
                const int64_t v = load_index(a.bt, a.bt_dtype, b * a.bt_stride + bi);
                if (v >= 0 && v < a.num_blocks) {
                  blk = (int)v;
                } else if (a.err) {
                  atomicOr(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
                }
              }
            }
          }
          const uint32_t koff = sbase + L::K0 + st * NP * kPanelBytes + i * rpb * 128;
          const uint32_t voff = sbase + L::V0 + st * NP * kPanelBytes + i * rpb * 128;
          for (int p = 0; p < NP; ++p) {
            tma_load_4d(koff + p * kPanelBytes, &tm_k, bar(B_KF0 + st), p * 64, row, h, blk);
            tma_load_4d(voff + p * kPanelBytes, &tm_v, bar(B_VF0 + st), p * 64, row, h, blk);
          }
        }
        issued = j + 1;
      }
      if (*abort) {
        // let the copies already issued land before the CTA's memory goes away
        for (int j = max(0, issued - 2); j < issued; ++j) {
          const int st = j & 1;
          const long long t0c = clock64();
          while (!mbar_try_wait(bar(B_KF0 + st), (j >> 1) & 1) && clock64() - t0c < 2000000) {
          }
          while (!mbar_try_wait(bar(B_VF0 + st), (j >> 1) & 1) && clock64() - t0c < 4000000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (lane == 0 && ntiles > 0) {
      const uint32_t id_qk = idesc_f16(BF16, BM, BN, false);
      const uint32_t id_pv = idesc_f16(BF16, BM, D, true);
      auto issue_pv = [&](int jj) -> bool {
        const int sp = jj & 1;
        if (!mbar_wait(bar(B_PF), jj & 1, abort)) return false;
        if (!mbar_wait(bar(B_VF0 + sp), (jj >> 1) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t vb = sbase + L::V0 + sp * NP * kPanelBytes;
        const uint32_t pb = sbase + L::P;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sw128_desc(pb + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(vb + kk * 16 * 128, kPanelBytes, 1024);
          umma_f16_ss(t_o, ad, bd, id_pv, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar(B_PV));
        umma_commit(bar(B_KE0 + sp));
        return true;
      };
      bool ok = mbar_wait(bar(B_Q), 0, abort);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j & 1;
        if (!mbar_wait(bar(B_KF0 + st), (j >> 1) & 1, abort)) {
          ok = false;
          break;
        }
        if (j >= 2 && !mbar_wait(bar(B_SR0 + st), ((j >> 1) - 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = sbase + L::K0 + st * NP * kPanelBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = sw128_desc(sbase + L::Q + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(kb + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
          umma_f16_ss(t_s[st], ad, bd, id_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(B_SF0 + st));
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = issue_pv(ntiles - 1);
      if (!ok) {
        // abort: let the MMAs already issued finish before TMEM is freed
        umma_commit(bar(B_DONE));
        const long long t0c = clock64();
        while (!mbar_try_wait(bar(B_DONE), 0) && clock64() - t0c < 4000000) {
        }
      }
    }
  } else {
    // --------------------------------------------------------- softmax
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row == TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int g = r / a.QT, i = r - g * a.QT;
    const int s = s0 + i;
    const bool row_ok = (g < a.G) && (s < a.S_q);
    const int qpos = seq_off + s;  // absolute position of this query
    const int none_limit = (a.bt == nullptr) ? a.kv_extra : seq_off + a.S_q;
    const float scale = a.scale_dev ? *a.scale_dev : a.scale;
    const float qk_mult = scale * kLog2e;
    float m_run = neg_inf(), l_run = 0.f;
    const int64_t mrow = a.mask ? (b * a.m_b + (int64_t)(h * a.G + g) * a.m_h + (int64_t)s * a.m_s) : 0;
    bool ok = true;

    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      // tcgen05.ld below is .sync.aligned: the whole warp must take the same path
      if (!__all_sync(0xffffffffu, mbar_wait(bar(B_SF0 + st), (j >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[BN];
      __syncwarp();
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t tmp[32];
        tmem_ld32(t_s[st] + lane_off + c * 32, tmp);
#pragma unroll
        for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(tmp[e]);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_SR0 + st));

      const int t0 = j * BN;
      const bool interior = (a.mask_mode == MM_CAUSAL) ? (t0 + BN - 1 <= seq_off + s0) && (t0 + BN <= kv_end)
                                                       : (a.mask_mode == MM_NONE && t0 + BN <= kv_end);
      float mt = neg_inf();
      if (interior && row_ok && a.mask == nullptr && a.pmask == nullptr) {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          x[c] *= qk_mult;
          mt = fmaxf(mt, x[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const int key = t0 + c;
          bool keep = row_ok && key < kv_end;
          if (a.mask_mode == MM_CAUSAL) keep = keep && key <= qpos;
          if (a.mask_mode == MM_NONE) keep = keep && key < none_limit;
          float add = 0.f;
          if (keep && a.mask) {
            const float mv = mask_value(a.mask, a.mask_dtype, mrow + key);
            if (a.mask_additive) add = mv * kLog2e;
            else keep = mv > 0.f;
          }
          if (keep && a.pmask)
            keep = key < a.pmask_len && mask_value(a.pmask, a.pmask_dtype, b * a.pm_b + key) > 0.f;
          x[c] = keep ? fmaf(x[c], qk_mult, add) : neg_inf();
          mt = fmaxf(mt, x[c]);
        }
      }
      const float m_new = fmaxf(m_run, mt);
      const bool grow = m_new > m_run + 8.f;
      float factor = 1.f;
      if (grow) {
        factor = exp2_approx(m_run - m_new);  // 0 when m_run = -inf
        l_run *= factor;
        m_run = m_new;
      }
      const float mu = (m_run == neg_inf()) ? 0.f : m_run;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        x[c] = exp2_approx(x[c] - mu);
        lsum += x[c];
      }
      l_run += lsum;

      // O and the P buffer are free once the PV MMA of tile j-1 completed
      if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(bar(B_PV), (j - 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j >= 1 && __any_sync(0xffffffffu, grow && factor != 1.f)) {
        __syncwarp();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(t_o + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          tmem_st32(t_o + lane_off + c * 32, o);
        }
        tmem_wait_st();
      }
      // P row -> shared memory, K-major 128B-swizzled (two 64-key panels)
      uint8_t* prow = sgen + L::P + r * 128;
#pragma unroll
      for (int ch = 0; ch < BN / 8; ++ch) {
        uint4 v;
        v.x = pack2<BF16>(x[ch * 8 + 0], x[ch * 8 + 1]);
        v.y = pack2<BF16>(x[ch * 8 + 2], x[ch * 8 + 3]);
        v.z = pack2<BF16>(x[ch * 8 + 4], x[ch * 8 + 5]);
        v.w = pack2<BF16>(x[ch * 8 + 6], x[ch * 8 + 7]);
        const int pan = ch >> 3, c16 = (ch & 7) ^ (r & 7);
        *reinterpret_cast<uint4*>(prow + pan * kPanelBytes + c16 * 16) = v;
      }
      // keys past kv_end in the last tile may hold unwritten memory: zero their V rows
      if (j == ntiles - 1 && t0 + BN > kv_end) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar(B_VF0 + st), (j >> 1) & 1, abort))) {
          ok = false;
          break;
        }
        if (t0 + r >= kv_end) {
          uint8_t* vrow = sgen + L::V0 + st * NP * kPanelBytes + r * 128;
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int c16 = 0; c16 < 8; ++c16)
              *reinterpret_cast<uint4*>(vrow + p * kPanelBytes + c16 * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PF));
    }

    // ------------------------------------------------------------ epilogue
    // warp-uniform from here: the TMEM loads are .sync.aligned; only the
    // global stores depend on the lane's row
    ok = __all_sync(0xffffffffu, ok);
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PV), (ntiles - 1) & 1, abort));
    tc_fence_after();
    if (ok) {
      // l_run == 0 -> inf -> NaN (all keys masked). A sink adds e^{sink - m}
      // to the denominator only (all keys masked then gives 0).
      const float inv =
          1.f / (a.sinks && g < a.G ? l_run + exp2f(a.sinks[h * a.G + g] * kLog2e - m_run) : l_run);
      char* orow = a.out + b * a.os_b + h * a.os_h + g * a.os_g + (int64_t)s * a.os_s;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (ntiles > 0) {
          __syncwarp();
          tmem_ld32(t_o + lane_off + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 v;
            v.x = pack2<BF16>(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
            v.y = pack2<BF16>(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
            v.z = pack2<BF16>(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
            v.w = pack2<BF16>(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + (c * 32 + q4 * 8) * 2) = v;
          }
        }
      }
      if (row_ok && a.lse) {
        const float v =
            (m_run == neg_inf() || l_run == 0.f) ? neg_inf() : (m_run + __log2f(l_run)) * 0.6931471805599453f;
        a.lse[b * a.ls_b + h * a.ls_h + g * a.ls_g + (int64_t)s * a.ls_s] = v;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Two-tile variant for the mask-free paths (causal / bidirectional), the hot
// path of chunked prefill and SDPA.
//
// A CTA owns two 128-row query tiles (A: tokens [s0, s0+QT), B: the next QT
// tokens) and streams 64-key K/V tiles through a 3-stage ring. Each query
// tile has its own softmax warpgroup and its own TMEM buffers (S double
// buffered, 64 columns each; O up to 128 columns), so while one warpgroup
// turns S into P the tensor core runs the other tile's MMAs:
//   warp 0       TMA producer          warp 1   MMA issuer / TMEM owner
//   warps 2-5    softmax, tile A       warps 6-9 softmax, tile B
// Per KV tile j the MMA thread issues QK_A(j), QK_B(j), then PV_A(j-1),
// PV_B(j-1). Shared memory: Q 2x32 KB, K/V 3x32 KB, P 2x16 KB (D = 128).
// Half of the softmax exponentials are evaluated on the FMA pipe with a
// polynomial (exp2_fma) so the SFU is not the bottleneck. CTAs take their
// (sequence, query-tile) items longest-first from a list that
// prefill_schedule_kernel sorts on the device by key count.
// ---------------------------------------------------------------------------
constexpr int BN2 = 64;          // keys per KV tile
constexpr int kStages2 = 3;
constexpr int kThreads2 = 320;   // 10 warps
constexpr int kPanel64 = 64 * 128;  // 64 rows x 128 bytes

// 2^x for x <= 8 on the FMA pipe: x = n + f, f in [0,1); 2^f by a cubic
// least-squares fit at Chebyshev nodes (max relative error 7.7e-5, 2^-13.7),
// 2^n by adding n to the exponent field. Inputs below -126 (masked scores
// are -inf) give exactly 0.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -126.f);
  const float n = floorf(xc);
  const float f = xc - n;
  float p = fmaf(0.07790716737508774f, f, 0.22623319923877716f);
  p = fmaf(p, f, 0.6957771182060242f);
  p = fmaf(p, f, 0.999927818775177f);
  const float r = __int_as_float(__float_as_int(p) + (static_cast<int>(n) << 23));
  return x < -126.f ? 0.f : r;
}

template <int D>
struct SmemLayout2 {
  static constexpr int NP = D / 64;
  static constexpr int QA = 0;                                  // NP panels of 128 rows
  static constexpr int QB = QA + NP * kPanelBytes;
  static constexpr int K0 = QB + NP * kPanelBytes;              // stage s: K0 + s*NP*kPanel64
  static constexpr int V0 = K0 + kStages2 * NP * kPanel64;
  static constexpr int PA = V0 + kStages2 * NP * kPanel64;      // one 128-row panel (64 keys)
  static constexpr int PB = PA + kPanelBytes;
  static constexpr int BAR = PB + kPanelBytes;
  static constexpr int TMEM_SLOT = BAR + 32 * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int TOTAL = ABORT + 8;
  static constexpr int ALLOC = (TOTAL + 1024 > 120 * 1024) ? TOTAL + 1024 : 120 * 1024;
};

enum Bar2 {
  C_Q = 0,
  C_KF0, C_KF1, C_KF2,
  C_VF0, C_VF1, C_VF2,
  C_KE0, C_KE1, C_KE2,
  C_SFA0, C_SFA1, C_SFB0, C_SFB1,
  C_SRA0, C_SRA1, C_SRB0, C_SRB1,
  C_PFA, C_PFB, C_PVA, C_PVB, C_DONE, C_COUNT
};

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads2, 1)
    attn_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  using L = SmemLayout2<D>;
  constexpr int NP = L::NP;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  volatile int* abort = reinterpret_cast<volatile int*>(sgen + L::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + L::TMEM_SLOT);
  auto bar = [&](int i) { return sbase + L::BAR + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid over (item, KV head), items longest first: from the sorted list
  // when there is one, else latest query tiles (most keys) first
  const int item = (int)(blockIdx.x / a.Hkv), h = (int)(blockIdx.x % a.Hkv);
  int b, qtile;
  if (a.work) {
    const int w = a.work[item];
    b = w / a.q_tiles;
    qtile = w - b * a.q_tiles;
  } else {
    b = item / a.q_tiles;
    qtile = a.q_tiles - 1 - (item - b * a.q_tiles);
  }
  const int s0 = qtile * 2 * a.QT;
  const int seq_off = a.seq ? a.seq[b * a.seq_stride] : 0;
  // keys for both tiles: the CTA spans 2*QT query tokens
  int kv_end = 0;
  if (seq_off >= 0) {
    const int s_hi = min(s0 + 2 * a.QT, a.S_q);
    int end = (a.mask_mode == MM_CAUSAL) ? seq_off + s_hi : ((a.bt == nullptr) ? a.kv_extra : seq_off + a.S_q);
    if (a.bt == nullptr) end = min(end, a.kv_extra);
    kv_end = max(0, min(end, a.span));
  }
  const int ntiles = (kv_end + BN2 - 1) / BN2;

  if (threadIdx.x == 0) {
    *abort = 0;
    for (int i = 0; i < C_COUNT; ++i) {
      const bool four = (i >= C_SRA0 && i <= C_SRB1) || i == C_PFA || i == C_PFB;
      mbar_init(bar(i), four ? 4u : 1u);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S_A[2] 0/64, S_B[2] 128/192, O_A 256, O_B 384
  auto t_s = [&](int x, int sb) { return tmem + x * 128 + sb * 64; };
  auto t_o = [&](int x) { return tmem + 256 + x * 128; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (ntiles > 0) {
      if (lane == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        mbar_arrive_expect_tx(bar(C_Q), 2 * NP * a.QT * a.G * 128);
        for (int p = 0; p < NP; ++p) {
          tma_load_5d(sbase + L::QA + p * kPanelBytes, &tm_q, bar(C_Q), p * 64, s0, 0, h, b);
          tma_load_5d(sbase + L::QB + p * kPanelBytes, &tm_q, bar(C_Q), p * 64, s0 + a.QT, 0, h, b);
        }
      }
      const int rpb = min(a.bs, BN2);
      const int nbox = BN2 / rpb;
      int issued = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % kStages2;
        if (j >= kStages2 &&
            !__all_sync(0xffffffffu, mbar_wait(bar(C_KE0 + st), ((j / kStages2) - 1) & 1, abort)))
          break;
        if (lane == 0) {
          mbar_arrive_expect_tx(bar(C_KF0 + st), NP * kPanel64);
          mbar_arrive_expect_tx(bar(C_VF0 + st), NP * kPanel64);
        }
        __syncwarp();
        const int t0 = j * BN2;
        for (int i = lane; i < nbox; i += 32) {
          const int key = t0 + i * rpb;
          int blk = a.num_blocks;  // out of range -> zero fill
          int row = 0;
          if (key < kv_end) {
            if (a.bt == nullptr) {
              blk = b;
              row = key;
            } else {
              const int bi = key / a.bs;
              row = key - bi * a.bs;
              if (bi < a.max_blocks) {
                const int64_t v = load_index(a.bt, a.bt_dtype, b * a.bt_stride + bi);
                if (v >= 0 && v < a.num_blocks) {
                  blk = (int)v;
                } else if (a.err) {
                  atomicOr(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
                }
              }
            }
          }
          const uint32_t koff = sbase + L::K0 + st * NP * kPanel64 + i * rpb * 128;
          const uint32_t voff = sbase + L::V0 + st * NP * kPanel64 + i * rpb * 128;
          for (int p = 0; p < NP; ++p) {
            tma_load_4d(koff + p * kPanel64, &tm_k, bar(C_KF0 + st), p * 64, row, h, blk);
            tma_load_4d(voff + p * kPanel64, &tm_v, bar(C_VF0 + st), p * 64, row, h, blk);
          }
        }
        issued = j + 1;
      }
      if (*abort) {
        for (int j = max(0, issued - kStages2); j < issued; ++j) {
          const int st = j % kStages2;
          const long long t0c = clock64();
          while (!mbar_try_wait(bar(C_KF0 + st), (j / kStages2) & 1) && clock64() - t0c < 2000000) {
          }
          while (!mbar_try_wait(bar(C_VF0 + st), (j / kStages2) & 1) && clock64() - t0c < 4000000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (lane == 0 && ntiles > 0) {
      const uint32_t id_qk = idesc_f16(BF16, 128, BN2, false);
      const uint32_t id_pv = idesc_f16(BF16, 128, D, true);
      auto issue_pv = [&](int jj) -> bool {
        const int stp = jj % kStages2;
        const uint32_t vb = sbase + L::V0 + stp * NP * kPanel64;
        if (!mbar_wait(bar(C_VF0 + stp), (jj / kStages2) & 1, abort)) return false;
        for (int x = 0; x < 2; ++x) {
          if (!mbar_wait(bar(x == 0 ? C_PFA : C_PFB), jj & 1, abort)) return false;
          tc_fence_after();
          const uint32_t pb = sbase + (x == 0 ? L::PA : L::PB);
#pragma unroll
          for (int kk = 0; kk < BN2 / 16; ++kk) {
            const uint64_t ad = sw128_desc(pb + kk * 32, 16, 1024);
            const uint64_t bd = sw128_desc(vb + kk * 16 * 128, kPanel64, 1024);
            umma_f16_ss(t_o(x), ad, bd, id_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar(x == 0 ? C_PVA : C_PVB));
        }
        umma_commit(bar(C_KE0 + stp));
        return true;
      };
      bool ok = mbar_wait(bar(C_Q), 0, abort);
      for (int j = 0; ok && j < ntiles; ++j) {
        const int st = j % kStages2, sb = j & 1;
        if (!mbar_wait(bar(C_KF0 + st), (j / kStages2) & 1, abort)) {
          ok = false;
          break;
        }
        const uint32_t kb = sbase + L::K0 + st * NP * kPanel64;
        for (int x = 0; x < 2 && ok; ++x) {
          if (j >= 2 && !mbar_wait(bar((x == 0 ? C_SRA0 : C_SRB0) + sb), ((j >> 1) - 1) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qb = sbase + (x == 0 ? L::QA : L::QB);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = sw128_desc(qb + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sw128_desc(kb + (kk >> 2) * kPanel64 + (kk & 3) * 32, 16, 1024);
            umma_f16_ss(t_s(x, sb), ad, bd, id_qk, kk > 0 ? 1u : 0u);
          }
          umma_commit(bar((x == 0 ? C_SFA0 : C_SFB0) + sb));
        }
        if (ok && j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok) ok = issue_pv(ntiles - 1);
      if (!ok) {
        umma_commit(bar(C_DONE));
        const long long t0c = clock64();
        while (!mbar_try_wait(bar(C_DONE), 0) && clock64() - t0c < 4000000) {
        }
      }
    }
  } else {
    // --------------------------------------------------------- softmax
    const int x = (warp >= 6) ? 1 : 0;  // query tile
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int g = r / a.QT, i = r - g * a.QT;
    const int s = s0 + x * a.QT + i;
    const bool row_ok = (g < a.G) && (s < a.S_q);
    const int qpos = seq_off + s;
    const int none_limit = (a.bt == nullptr) ? a.kv_extra : seq_off + a.S_q;
    // first key any row of this tile may not see (tile-uniform bound for the fast path)
    const int tile_first_q = seq_off + s0 + x * a.QT;
    const float scale = a.scale_dev ? *a.scale_dev : a.scale;
    const float qk_mult = scale * kLog2e;
    const int bar_sf = x == 0 ? C_SFA0 : C_SFB0, bar_sr = x == 0 ? C_SRA0 : C_SRB0;
    const int bar_pf = x == 0 ? C_PFA : C_PFB, bar_pv = x == 0 ? C_PVA : C_PVB;
    uint8_t* pbuf = sgen + (x == 0 ? L::PA : L::PB);
    float m_run = neg_inf(), l_run = 0.f;
    bool ok = true;

    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(bar_sf + sb), (j >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float xv[BN2];
      __syncwarp();
#pragma unroll
      for (int c = 0; c < BN2 / 32; ++c) {
        uint32_t tmp[32];
        tmem_ld32(t_s(x, sb) + lane_off + c * 32, tmp);
#pragma unroll
        for (int e = 0; e < 32; ++e) xv[c * 32 + e] = __uint_as_float(tmp[e]);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(bar_sr + sb));

      const int t0 = j * BN2;
      const bool interior = (a.mask_mode == MM_CAUSAL) ? (t0 + BN2 - 1 <= tile_first_q) && (t0 + BN2 <= kv_end)
                                                       : (t0 + BN2 <= kv_end);
      float mt = neg_inf();
      if (interior && row_ok) {
#pragma unroll
        for (int c = 0; c < BN2; ++c) {
          xv[c] *= qk_mult;
          mt = fmaxf(mt, xv[c]);
        }
      } else {
        const int lim = (a.mask_mode == MM_CAUSAL) ? min(qpos + 1, kv_end) : min(none_limit, kv_end);
#pragma unroll
        for (int c = 0; c < BN2; ++c) {
          const bool keep = row_ok && (t0 + c < lim);
          xv[c] = keep ? xv[c] * qk_mult : neg_inf();
          mt = fmaxf(mt, xv[c]);
        }
      }
      const float m_new = fmaxf(m_run, mt);
      const bool grow = m_new > m_run + 8.f;
      float factor = 1.f;
      if (grow) {
        factor = exp2_approx(m_run - m_new);
        l_run *= factor;
        m_run = m_new;
      }
      const float mu = (m_run == neg_inf()) ? 0.f : m_run;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < BN2; ++c) {
        const float e = (c & 1) ? exp2_fma(xv[c] - mu) : exp2_approx(xv[c] - mu);
        xv[c] = e;
        lsum += e;
      }
      l_run += lsum;

      if (j >= 1 && !__all_sync(0xffffffffu, mbar_wait(bar(bar_pv), (j - 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j >= 1 && __any_sync(0xffffffffu, grow && factor != 1.f)) {
        __syncwarp();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(t_o(x) + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          tmem_st32(t_o(x) + lane_off + c * 32, o);
        }
        tmem_wait_st();
      }
      uint8_t* prow = pbuf + r * 128;
#pragma unroll
      for (int ch = 0; ch < BN2 / 8; ++ch) {
        uint4 v;
        v.x = pack2<BF16>(xv[ch * 8 + 0], xv[ch * 8 + 1]);
        v.y = pack2<BF16>(xv[ch * 8 + 2], xv[ch * 8 + 3]);
        v.z = pack2<BF16>(xv[ch * 8 + 4], xv[ch * 8 + 5]);
        v.w = pack2<BF16>(xv[ch * 8 + 6], xv[ch * 8 + 7]);
        *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) * 16)) = v;
      }
      // keys past kv_end in the last tile may hold unwritten memory: tile A's
      // warpgroup zeroes their V rows before its P is released (both PV MMAs
      // of this tile come after that release)
      if (x == 0 && j == ntiles - 1 && t0 + BN2 > kv_end) {
        const int st = j % kStages2;
        if (!__all_sync(0xffffffffu, mbar_wait(bar(C_VF0 + st), (j / kStages2) & 1, abort))) {
          ok = false;
          break;
        }
        if (r < BN2 && t0 + r >= kv_end) {
          uint8_t* vrow = sgen + L::V0 + st * NP * kPanel64 + r * 128;
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int c16 = 0; c16 < 8; ++c16)
              *reinterpret_cast<uint4*>(vrow + p * kPanel64 + c16 * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(bar_pf));
    }

    ok = __all_sync(0xffffffffu, ok);
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(bar_pv), (ntiles - 1) & 1, abort));
    tc_fence_after();
    if (ok) {
      const float inv = 1.f / l_run;
      char* orow = a.out + b * a.os_b + h * a.os_h + g * a.os_g + (int64_t)s * a.os_s;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (ntiles > 0) {
          __syncwarp();
          tmem_ld32(t_o(x) + lane_off + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 v;
            v.x = pack2<BF16>(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
            v.y = pack2<BF16>(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
            v.z = pack2<BF16>(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
            v.w = pack2<BF16>(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + (c * 32 + q4 * 8) * 2) = v;
          }
        }
      }
      if (row_ok && a.lse) {
        const float v =
            (m_run == neg_inf() || l_run == 0.f) ? neg_inf() : (m_run + __log2f(l_run)) * 0.6931471805599453f;
        a.lse[b * a.ls_b + h * a.ls_h + g * a.ls_g + (int64_t)s * a.ls_s] = v;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// 128-key kernel for the mask-free paths (causal / bidirectional), the hot
// path of chunked prefill and SDPA.
//
// Same roles and two query tiles per CTA as the two-tile kernel above, with
// KV tiles of 128 keys so that every QK MMA is 128 x 128 x 16 (an N = 64 MMA
// occupies the tensor pipe about as long as an N = 128 one on B200). TMEM
// holds one S buffer per query tile (128 columns) and one O (D columns):
//   S_A 0..127, S_B 128..255, O_A 256.., O_B 384..
// The softmax warpgroup of a tile reads S, writes P as bf16/f16 pairs over
// the first 64 columns of the same buffer, and the PV MMA takes its A operand
// from there, so P never goes through shared memory. The MMA thread issues,
// per KV tile j,
//   PV_A(j-1), QK_A(j), PV_B(j-1), QK_B(j)
// so a query tile's S buffer is overwritten only after the PV that read its
// P (tcgen05.mma executes in issue order), and while one warpgroup works on
// its S the tensor core runs the other tile's PV and QK. The commit after
// QK_x(j) tracks every earlier MMA too, so when S_x(j) is ready PV_x(j-1) has
// completed and O_x may be rescaled. K and V have their own TMA rings, since
// a K tile is released after the QKs and a V tile after the PVs one step
// later. The CTA has 12 warps; the producer/MMA warpgroup hands registers to
// the two softmax warpgroups (setmaxnreg), so a softmax thread holds its
// whole row of 128 scores (one TMEM round trip per tile); the softmax
// arithmetic uses packed f32x2 instructions, and every POLY-th pair
// of exponentials runs on the FMA pipe (exp2_poly2) instead of the SFU.
// Shared memory (D = 128): Q 2x32 KB, K 2x32 KB, V 2x32 KB.
// ---------------------------------------------------------------------------
constexpr int BN3 = 128;
constexpr int kThreads3 = 384;  // 12 warps: softmax A 0-3, softmax B 4-7, producer 8, MMA 9, 10-11 idle
// Registers per thread after the split (launch: 168 each, 12 warps): the
// softmax warpgroups hold a whole 128-score row, the third warpgroup little.
constexpr uint32_t kRegsSoftmax3 = 216, kRegsOther3 = 64;
static_assert(2 * 128 * kRegsSoftmax3 + 128 * kRegsOther3 <= 12 * 32 * 168, "register split exceeds the launch");

template <int D>
struct SmemLayout3 {
  static constexpr int NP = D / 64;
  static constexpr int KS = D == 128 ? 2 : 3;  // K ring stages
  static constexpr int VS = D == 128 ? 2 : 3;  // V ring stages
  static constexpr int TILE = NP * kPanelBytes;  // 128 rows x D
  static constexpr int QA = 0;
  static constexpr int QB = QA + TILE;
  static constexpr int K0 = QB + TILE;
  static constexpr int V0 = K0 + KS * TILE;
  static constexpr int BAR = V0 + VS * TILE;
  static constexpr int TMEM_SLOT = BAR + 32 * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int UNITS = ABORT + 8;  // ring of kUnitRing unit ids
  static constexpr int TOTAL = UNITS + 4 * 4;
  static constexpr int ALLOC = (TOTAL + 1024 > 120 * 1024) ? TOTAL + 1024 : 120 * 1024;
};

constexpr int kUnitRing = 4;

enum Bar3 {
  E_Q = 0,
  E_KF0, E_KF1, E_KF2, E_KE0, E_KE1, E_KE2,
  E_VF0, E_VF1, E_VF2, E_VE0, E_VE1, E_VE2,
  E_SFA, E_SFB,  // S of query tile A / B computed (and every earlier MMA done)
  E_PFA, E_PFB,  // P of A / B written to TMEM (4 softmax warps each)
  E_OA, E_OB,    // last PV of A / B of a unit complete
  E_QE,          // every QK of a unit complete: Q may be reloaded
  E_OEA, E_OEB,  // O of A / B read by the softmax (4 warps each)
  E_UF0,         // kUnitRing barriers: unit id of a ring slot written (producer)
  E_UE0 = E_UF0 + kUnitRing,  // kUnitRing barriers: slot read (MMA thread + 8 softmax warps)
  E_DONE = E_UE0 + kUnitRing, E_COUNT
};

// Unit u of a launch of the 128-key kernel: (item, KV head), the item taken
// from the longest-first list when there is one, else in reverse query-tile
// order. Every role of a CTA derives the same units, in the same order.
struct Unit3 {
  int b, h, s0, seq_off, kv_end, ntiles;
  const int* list;  // masked launch: the item's key tiles (entry j: tile, bit 31 = not all kept); else null
};
__device__ __forceinline__ Unit3 unit3(const AttnArgs& a, int u) {
  Unit3 t;
  const int item = u / a.Hkv;
  t.h = u - item * a.Hkv;
  int qtile;
  if (a.work) {
    const int w = a.work[item];
    t.b = w / a.q_tiles;
    qtile = w - t.b * a.q_tiles;
  } else {
    t.b = item / a.q_tiles;
    qtile = a.q_tiles - 1 - (item - t.b * a.q_tiles);
  }
  t.s0 = qtile * 2 * a.QT;
  t.seq_off = a.seq ? a.seq[t.b * a.seq_stride] : 0;
  t.kv_end = 0;
  t.list = nullptr;
  if (t.seq_off >= 0) {
    const int s_hi = min(t.s0 + 2 * a.QT, a.S_q);
    int end = (a.mask_mode == MM_CAUSAL) ? t.seq_off + s_hi
              : (a.mask_mode == MM_KEEP) ? a.mask_len
              : ((a.bt == nullptr) ? a.kv_extra : t.seq_off + a.S_q);
    if (a.bt == nullptr) end = min(end, a.kv_extra);
    t.kv_end = max(0, min(end, a.span));
  }
  if (a.tcount) {
    // the mask pre-pass listed the tiles with a kept key (none for seq < 0)
    const int it = t.b * a.q_tiles + qtile;
    t.ntiles = a.tcount[it];
    t.list = a.tlist + (int64_t)it * a.nkt;
  } else {
    t.ntiles = (t.kv_end + BN3 - 1) / BN3;
  }
  return t;
}

// Key tile (index) and "not every key kept" flag of entry j of a unit.
__device__ __forceinline__ int unit3_tile(const Unit3& t, int j, bool& mixed) {
  if (t.list == nullptr) {
    mixed = false;
    return j;
  }
  const int e = t.list[j];
  mixed = e < 0;
  return e & 0x7fffffff;
}

// Persistent: one CTA per SM. The producer takes the next unit from the
// launch's counter (the units are in longest-first order, so a free CTA
// takes the longest unit left) or, without one, every gridDim.x-th unit, and
// passes its id to the MMA thread and the softmax warps through a small ring
// in shared memory. Ring stages and barrier parities follow a running count
// T of the CTA's KV tiles and `act` of its units with work, so the producer
// loads the next unit's Q and K/V while the softmax finishes the previous
// one. Q is reloaded after the previous unit's last QK (E_QE); a unit's
// first PV overwrites O only after the softmax has read the previous O
// (E_OEA/B).
template <int D, bool BF16, int POLY, bool MASKED>
__global__ void __launch_bounds__(kThreads3, 1)
    attn_fwd_tc3_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const AttnArgs a, const int n_units) {
  using L = SmemLayout3<D>;
  constexpr int NP = L::NP, KS = L::KS, VS = L::VS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  volatile int* abort = reinterpret_cast<volatile int*>(sgen + L::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + L::TMEM_SLOT);
  auto bar = [&](int i) { return sbase + L::BAR + 8u * i; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0;
    for (int i = 0; i < E_COUNT; ++i)
      mbar_init(bar(i), (i == E_PFA || i == E_PFB || i == E_OEA || i == E_OEB) ? 4u
                        : (i >= E_UE0 && i < E_UE0 + kUnitRing)          ? 9u
                                                                         : 1u);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched as a programmatic dependent of the append kernel on the paged
  // path: the set-up above (barriers, TMEM) reads no global memory and
  // overlaps the previous grid; everything below reads its results (the
  // appended rows, the schedule), so it waits for that grid here. Without a
  // programmatic launch this returns at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  auto t_s = [&](int x) { return tmem + x * 128; };
  auto t_o = [&](int x) { return tmem + 256 + x * 128; };
  volatile int* units = reinterpret_cast<volatile int*>(sgen + L::UNITS);

  // Each warpgroup changes its register count at the top of its own branch,
  // so the code of the branch is compiled for that count.
  if (warp >= 8) {
   setmaxnreg_dec<kRegsOther3>();
   if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
    }
    const int rpb = min(a.bs, BN3);
    const int nbox = BN3 / rpb;  // <= 16 (block size >= 8)
    int T = 0, act = 0, k_issued = 0, v_issued = 0;
    bool ok = true;
    for (int kq = 0; ok; ++kq) {
      // next unit: from the launch's counter (longest first, taken by
      // whichever CTA is free), else every gridDim.x-th; -1 ends the loop
      const int slot = kq % kUnitRing;
      if (kq >= kUnitRing &&
          !__all_sync(0xffffffffu, mbar_wait(bar(E_UE0 + slot), ((kq / kUnitRing) - 1) & 1, abort))) {
        ok = false;
        break;
      }
      int u = 0;
      if (lane == 0) {
        u = a.counter ? atomicAdd(a.counter, 1) : (int)blockIdx.x + kq * (int)gridDim.x;
        if (u >= n_units) u = -1;
        units[slot] = u;
        mbar_arrive(bar(E_UF0 + slot));
      }
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u < 0) break;
      const Unit3 t = unit3(a, u);
      if (t.ntiles == 0) continue;
      // Q of this unit once every QK of the previous one has completed
      if (act >= 1 && !__all_sync(0xffffffffu, mbar_wait(bar(E_QE), (act - 1) & 1, abort))) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(bar(E_Q), 2 * NP * a.QT * a.G * 128);
        for (int p = 0; p < NP; ++p) {
          tma_load_5d(sbase + L::QA + p * kPanelBytes, &tm_q, bar(E_Q), p * 64, t.s0, 0, t.h, t.b);
          tma_load_5d(sbase + L::QB + p * kPanelBytes, &tm_q, bar(E_Q), p * 64, t.s0 + a.QT, 0, t.h, t.b);
        }
      }
      for (int j = 0; j < t.ntiles; ++j) {
        const int Tj = T + j;
        // lane i < nbox fetches rows [i*rpb, (i+1)*rpb) of the tile
        int blk = a.num_blocks;  // out of range -> zero fill
        int row = 0;
        bool mixed;
        const int key = (MASKED ? unit3_tile(t, j, mixed) : j) * BN3 + lane * rpb;
        if (lane < nbox && key < t.kv_end) {
          if (a.bt == nullptr) {
            blk = t.b;
            row = key;
          } else {
            const int bi = key / a.bs;
            row = key - bi * a.bs;
            if (bi < a.max_blocks) {
              const int64_t v = load_index(a.bt, a.bt_dtype, t.b * a.bt_stride + bi);
              if (v >= 0 && v < a.num_blocks) {
                blk = (int)v;
              } else if (a.err) {
                atomicOr(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
              }
            }
          }
        }
        const int sk = Tj % KS;
        if (Tj >= KS && !__all_sync(0xffffffffu, mbar_wait(bar(E_KE0 + sk), ((Tj / KS) - 1) & 1, abort))) {
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive_expect_tx(bar(E_KF0 + sk), NP * kPanelBytes);
        __syncwarp();
        if (lane < nbox)
          for (int p = 0; p < NP; ++p)
            tma_load_4d(sbase + L::K0 + sk * L::TILE + p * kPanelBytes + lane * rpb * 128, &tm_k, bar(E_KF0 + sk),
                        p * 64, row, t.h, blk);
        k_issued = Tj + 1;
        const int sv = Tj % VS;
        if (Tj >= VS && !__all_sync(0xffffffffu, mbar_wait(bar(E_VE0 + sv), ((Tj / VS) - 1) & 1, abort))) {
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive_expect_tx(bar(E_VF0 + sv), NP * kPanelBytes);
        __syncwarp();
        if (lane < nbox)
          for (int p = 0; p < NP; ++p)
            tma_load_4d(sbase + L::V0 + sv * L::TILE + p * kPanelBytes + lane * rpb * 128, &tm_v, bar(E_VF0 + sv),
                        p * 64, row, t.h, blk);
        v_issued = Tj + 1;
      }
      T += t.ntiles;
      ++act;
    }
    if (*abort) {
      // let the copies in flight land before the CTA exits
      const long long t0c = clock64();
      for (int j = max(0, k_issued - KS); j < k_issued; ++j)
        while (!mbar_try_wait(bar(E_KF0 + j % KS), (j / KS) & 1) && clock64() - t0c < 4000000) {
        }
      for (int j = max(0, v_issued - VS); j < v_issued; ++j)
        while (!mbar_try_wait(bar(E_VF0 + j % VS), (j / VS) & 1) && clock64() - t0c < 8000000) {
        }
    }
   } else if (warp == 9) {
    // ------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(BF16, 128, BN3, false);
      const uint32_t id_pv = idesc_f16(BF16, 128, D, true);
      int T = 0, act = 0;
      bool ok = true;
      for (int kq = 0; ok; ++kq) {
        const int slot = kq % kUnitRing;
        if (!mbar_wait(bar(E_UF0 + slot), (kq / kUnitRing) & 1, abort)) {
          ok = false;
          break;
        }
        const int u = units[slot];
        mbar_arrive(bar(E_UE0 + slot));
        if (u < 0) break;
        const int nt = unit3(a, u).ntiles;
        if (nt == 0) continue;
        if (!mbar_wait(bar(E_Q), act & 1, abort)) {
          ok = false;
          break;
        }
        for (int j = 0; ok && j <= nt; ++j) {
          const int Tj = T + j;
          if (j < nt && !mbar_wait(bar(E_KF0 + Tj % KS), (Tj / KS) & 1, abort)) {
            ok = false;
            break;
          }
          if (j >= 1 && !mbar_wait(bar(E_VF0 + (Tj - 1) % VS), ((Tj - 1) / VS) & 1, abort)) {
            ok = false;
            break;
          }
          for (int x = 0; x < 2; ++x) {
            if (j >= 1) {
              // PV_x(j-1): A = P in S_x (TMEM), B = V tile j-1; the unit's
              // first PV overwrites O_x once the previous unit's O is read
              if (!mbar_wait(bar(x == 0 ? E_PFA : E_PFB), (Tj - 1) & 1, abort) ||
                  (j == 1 && act >= 1 && !mbar_wait(bar(x == 0 ? E_OEA : E_OEB), (act - 1) & 1, abort))) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t vb = sbase + L::V0 + ((Tj - 1) % VS) * L::TILE;
#pragma unroll
              for (int kk = 0; kk < BN3 / 16; ++kk) {
                const uint64_t bd = sw128_desc(vb + kk * 16 * 128, kPanelBytes, 1024);
                umma_f16_ts(t_o(x), t_s(x) + kk * 8, bd, id_pv, (j > 1 || kk > 0) ? 1u : 0u);
              }
              if (j == nt) umma_commit(bar(x == 0 ? E_OA : E_OB));
            } else {
              tc_fence_after();
            }
            if (j < nt) {
              // QK_x(j) into S_x
              const uint32_t qb = sbase + (x == 0 ? L::QA : L::QB);
              const uint32_t kb = sbase + L::K0 + (Tj % KS) * L::TILE;
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint64_t ad = sw128_desc(qb + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
                const uint64_t bd = sw128_desc(kb + (kk >> 2) * kPanelBytes + (kk & 3) * 32, 16, 1024);
                umma_f16_ss(t_s(x), ad, bd, id_qk, kk > 0 ? 1u : 0u);
              }
              umma_commit(bar(x == 0 ? E_SFA : E_SFB));
            }
          }
          if (!ok) break;
          if (j < nt) {
            umma_commit(bar(E_KE0 + Tj % KS));
            if (j == nt - 1) umma_commit(bar(E_QE));
          }
          if (j >= 1) umma_commit(bar(E_VE0 + (Tj - 1) % VS));
        }
        T += nt;
        ++act;
      }
      if (!ok) {
        umma_commit(bar(E_DONE));
        const long long t0c = clock64();
        while (!mbar_try_wait(bar(E_DONE), 0) && clock64() - t0c < 4000000) {
        }
      }
    }
   }
  } else {
    setmaxnreg_inc<kRegsSoftmax3>();
    // --------------------------------------------------------- softmax
    const int x = warp >> 2;  // query tile
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int g = r / a.QT, i = r - g * a.QT;
    const float scale = a.scale_dev ? *a.scale_dev : a.scale;
    const float qk_mult = scale * kLog2e;
    const float mult = qk_mult > 0.f ? qk_mult : 1.f;
    const int bar_sf = x == 0 ? E_SFA : E_SFB, bar_pf = x == 0 ? E_PFA : E_PFB, bar_o = x == 0 ? E_OA : E_OB;
    const int bar_oe = x == 0 ? E_OEA : E_OEB;
    int T = 0, act = 0;
    bool ok = true;
    for (int kq = 0; ok; ++kq) {
      const int slot = kq % kUnitRing;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(E_UF0 + slot), (kq / kUnitRing) & 1, abort))) {
        ok = false;
        break;
      }
      const int u = units[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(E_UE0 + slot));
      if (u < 0) break;
      const Unit3 t = unit3(a, u);
      const int s = t.s0 + x * a.QT + i;
      const bool row_ok = (g < a.G) && (s < a.S_q);
      const int qpos = t.seq_off + s;
      const int none_limit = (a.bt == nullptr) ? a.kv_extra : t.seq_off + a.S_q;
      // first key any row of this tile may not see (tile-uniform bound for the fast path)
      const int tile_first_q = t.seq_off + t.s0 + x * a.QT;
      const int kv_end = t.kv_end, ntiles = t.ntiles;
      float m_run = neg_inf(), l_run = 0.f;

      for (int j = 0; j < ntiles; ++j) {
        const int Tj = T + j;
        bool mixed = false;
        const int t0 = (MASKED ? unit3_tile(t, j, mixed) : j) * BN3;
        // a partly kept tile: the row's keep bits, loaded before the wait for S
        uint4 kb = make_uint4(0u, 0u, 0u, 0u);
        if (MASKED && mixed && row_ok) kb = a.kbits[((int64_t)t.b * a.S_q + s) * a.nkt + t0 / BN3];
        if (!__all_sync(0xffffffffu, mbar_wait(bar(bar_sf), Tj & 1, abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
        __syncwarp();
        const bool interior = MASKED ? !mixed
                              : (a.mask_mode == MM_CAUSAL) ? (t0 + BN3 - 1 <= tile_first_q) && (t0 + BN3 <= kv_end)
                                                           : (t0 + BN3 <= kv_end);
        const int lim = (a.mask_mode == MM_CAUSAL) ? min(qpos + 1, kv_end) : min(none_limit, kv_end);
        // the row's 128 scores: four loads, one wait
        float xv[BN3];
        {
          uint32_t r0[32], r1[32], r2[32], r3[32];
          tmem_ld32(t_s(x) + lane_off + 0, r0);
          tmem_ld32(t_s(x) + lane_off + 32, r1);
          tmem_ld32(t_s(x) + lane_off + 64, r2);
          tmem_ld32(t_s(x) + lane_off + 96, r3);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            xv[e] = __uint_as_float(r0[e]);
            xv[32 + e] = __uint_as_float(r1[e]);
            xv[64 + e] = __uint_as_float(r2[e]);
            xv[96 + e] = __uint_as_float(r3[e]);
          }
        }
        // Scores stay unscaled until the exponent: the max is taken on raw
        // scores (a positive multiplier keeps the order) and the scale is
        // folded into the packed x*mult - m step.
        if (!(qk_mult > 0.f)) {
#pragma unroll
          for (int e = 0; e < BN3; e += 2) mul2(xv[e], xv[e + 1], qk_mult, qk_mult);
        }
        if (!(interior && row_ok)) {
          if constexpr (MASKED) {  // keep bits of the row (all zero for a row outside the chunk)
            const uint32_t kw[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int e = 0; e < BN3; ++e)
              if (!((kw[e >> 5] >> (e & 31)) & 1u)) xv[e] = neg_inf();
          } else {
#pragma unroll
            for (int e = 0; e < BN3; ++e)
              if (!(row_ok && t0 + e < lim)) xv[e] = neg_inf();
          }
        }
        float mx0 = neg_inf(), mx1 = neg_inf(), mx2 = neg_inf(), mx3 = neg_inf();
#pragma unroll
        for (int e = 0; e < BN3; e += 8) {
          mx0 = max3(mx0, xv[e], xv[e + 1]);
          mx1 = max3(mx1, xv[e + 2], xv[e + 3]);
          mx2 = max3(mx2, xv[e + 4], xv[e + 5]);
          mx3 = max3(mx3, xv[e + 6], xv[e + 7]);
        }
        const float mt = max3(mx0, mx1, fmaxf(mx2, mx3)) * mult;
        const float m_new = fmaxf(m_run, mt);
        const bool grow = m_new > m_run + 8.f;
        float factor = 1.f;
        if (grow) {
          factor = exp2_approx(m_run - m_new);
          l_run *= factor;
          m_run = m_new;
        }
        // S_x(j) ready means PV_x(j-1) has completed: O may be rescaled now,
        // before this tile's PV (which waits for this tile's P)
        if (j >= 1 && __any_sync(0xffffffffu, grow && factor != 1.f)) {
          __syncwarp();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o(x) + lane_off + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
            tmem_st32(t_o(x) + lane_off + c * 32, o);
          }
          tmem_wait_st();
        }
        const float nmu = (m_run == neg_inf()) ? 0.f : -m_run;
#pragma unroll
        for (int e = 0; e < BN3; e += 2) fma2(xv[e], xv[e + 1], mult, mult, nmu, nmu);
#pragma unroll
        for (int e = 0; e < BN3; e += 2) {
          if (POLY > 0 && (e / 2) % (POLY > 0 ? POLY : 1) == POLY - 1) {
            exp2_poly2(xv[e], xv[e + 1]);
          } else {
            xv[e] = exp2_approx(xv[e]);
            xv[e + 1] = exp2_approx(xv[e + 1]);
          }
        }
        float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
#pragma unroll
        for (int e = 0; e < BN3; e += 4) {
          add2(sa0, sa1, xv[e], xv[e + 1]);
          add2(sb0, sb1, xv[e + 2], xv[e + 3]);
        }
        l_run += (sa0 + sa1) + (sb0 + sb1);
        // P of the row over the first 64 columns of S_x (all of S is in registers)
        __syncwarp();
#pragma unroll
        for (int c4 = 0; c4 < BN3 / 32; ++c4) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = pack2<BF16>(xv[32 * c4 + 2 * e], xv[32 * c4 + 2 * e + 1]);
          tmem_st16(t_s(x) + lane_off + c4 * 16, pk);
        }
        tmem_wait_st();
        // keys past kv_end in the tile that holds kv_end may be unwritten
        // memory: tile A's warpgroup zeroes their V rows before its P is
        // released (both PV MMAs of this tile come after that release)
        if (x == 0 && t0 < kv_end && t0 + BN3 > kv_end) {
          const int sv = Tj % VS;
          if (!__all_sync(0xffffffffu, mbar_wait(bar(E_VF0 + sv), (Tj / VS) & 1, abort))) {
            ok = false;
            break;
          }
          if (t0 + r >= kv_end) {
            uint8_t* vrow = sgen + L::V0 + sv * L::TILE + r * 128;
#pragma unroll
            for (int p = 0; p < NP; ++p)
#pragma unroll
              for (int c16 = 0; c16 < 8; ++c16)
                *reinterpret_cast<uint4*>(vrow + p * kPanelBytes + c16 * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();  // the zeroed rows are read by the PV MMA (async proxy)
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(bar_pf));
      }

      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (ntiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(bar_o), act & 1, abort));
      if (!ok) break;
      tc_fence_after();
      // an attention sink adds e^{sink} (relative to the running max) to the
      // denominator only; a row with no visible key then gives 0, not NaN
      float lsum = l_run;
      if (a.sinks && row_ok) lsum += exp2f(a.sinks[t.h * a.G + g] * kLog2e - m_run);
      const float inv = 1.f / lsum;
      char* orow = a.out + t.b * a.os_b + t.h * a.os_h + g * a.os_g + (int64_t)s * a.os_s;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (ntiles > 0) {
          __syncwarp();
          tmem_ld32(t_o(x) + lane_off + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (row_ok) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 v;
            v.x = pack2<BF16>(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
            v.y = pack2<BF16>(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
            v.z = pack2<BF16>(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
            v.w = pack2<BF16>(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + (c * 32 + q4 * 8) * 2) = v;
          }
        }
      }
      if (row_ok && a.lse) {
        const float v =
            (m_run == neg_inf() || l_run == 0.f) ? neg_inf() : (m_run + __log2f(l_run)) * 0.6931471805599453f;
        a.lse[t.b * a.ls_b + t.h * a.ls_h + g * a.ls_g + (int64_t)s * a.ls_s] = v;
      }
      if (ntiles > 0) {
        // O_x has been read: the next unit's first PV may overwrite it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(bar_oe));
        ++act;
      }
      T += ntiles;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0 && a.err) atomicOr(a.err, RBLN_DEVERR_TIMEOUT);
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Orders the (sequence, query-tile) items of a two-tile prefill launch by
// the number of keys they attend, longest first (ties: lower index first),
// so that the longest CTAs start in the first wave. One CTA; each thread
// ranks items by counting the items that go before them.
__global__ void __launch_bounds__(256) prefill_schedule_kernel(const int32_t* seq, int64_t seq_stride, int B,
                                                               int q_tiles, int S_q, int tile_tokens, int span,
                                                               int causal, const int* tcount, int* work) {
  extern __shared__ int cost[];
  const int n = B * q_tiles;
  if (threadIdx.x == 0) work[n] = 0;  // unit counter of a persistent launch
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (tcount) {  // masked launch: the key tiles the mask pre-pass listed
      cost[i] = tcount[i];
      continue;
    }
    const int b = i / q_tiles, t = i - b * q_tiles;
    const int off = max(0, seq[b * seq_stride]);
    const int hi = min((t + 1) * tile_tokens, S_q);
    cost[i] = min(span, causal ? off + hi : off + S_q);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int ci = cost[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const int cj = cost[j];
      rank += (cj > ci) || (cj == ci && j < i);
    }
    work[rank] = i;
  }
}

// ---------------------------------------------------------------------------
// Mask pre-pass of the 128-key kernel. For a keep rule other than plain
// causal / bidirectional (a keep-mask with value > 0 keeping a key, or a
// position mask on top of causal / bidirectional), every query row of the
// chunk gets 128 keep bits per 128-key tile, and every (item, key tile) a
// class: no key kept (the tile is skipped), every key of every row kept
// (no masking), or mixed (the softmax applies the row's bits). Each mask
// element is read once; a key at or past the span is never kept, nor is any
// key of a sequence whose start offset is negative.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool keep_key(const AttnArgs& a, int b, int s, int t, int seq_off) {
  if (seq_off < 0 || t >= a.span) return false;
  bool keep;
  if (a.mask_mode == MM_KEEP) {
    keep = t < a.mask_len && mask_value(a.mask, a.mask_dtype, b * a.m_b + (int64_t)s * a.m_s + t) > 0.f;
  } else if (a.mask_mode == MM_CAUSAL) {
    keep = t <= seq_off + s;
  } else {
    keep = t < seq_off + a.S_q;
  }
  if (keep && a.pmask) keep = t < a.pmask_len && mask_value(a.pmask, a.pmask_dtype, b * a.pm_b + t) > 0.f;
  return keep;
}

// 32 keep bits from 32 16-bit mask values (bf16 or f16 bit patterns, 4
// x 16-byte words): value > 0 <=> sign clear, not zero, not NaN, i.e. the
// pattern lies in [1, +inf].
__device__ __forceinline__ uint32_t keep_bits16(const uint4* src, uint32_t inf_bits) {
  uint32_t bits = 0;
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint4 x = src[v];
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t h = (w[k >> 1] >> (16 * (k & 1))) & 0xffffu;
      bits |= (uint32_t)(h - 1u < inf_bits) << (v * 8 + k);
    }
  }
  return bits;
}

// grid (nkt, items), 256 threads: rows [s0, s0 + 2 QT) of item (b,
// query-tile pair) x keys [128 kt, 128 kt + 128). A thread makes one
// (row, 32-key word) at a time with all 32 tests independent, so its loads
// are in flight together; a bf16 / f16 keep-mask whose row segment is
// 16-byte aligned and inside the mask is read as four 16-byte words.
// Class: 0 no key kept, 1 all kept, 2 mixed (over the chunk's rows).
__global__ void __launch_bounds__(256) prefill_mask_bits_kernel(const AttnArgs a, uint4* kbits, uint8_t* cls) {
  const int kt = blockIdx.x, item = blockIdx.y;
  const int b = item / a.q_tiles, qp = item - b * a.q_tiles;
  const int s0 = qp * 2 * a.QT;
  const int rows = min(2 * a.QT, a.S_q - s0);
  const int seq_off = a.seq ? a.seq[b * a.seq_stride] : 0;
  const bool half_mask = a.mask_mode == MM_KEEP && !a.pmask && seq_off >= 0 &&
                         (a.mask_dtype == RBLN_DT_BF16 || a.mask_dtype == RBLN_DT_F16);
  const uint32_t inf_bits = a.mask_dtype == RBLN_DT_BF16 ? 0x7f80u : 0x7c00u;
  bool any_keep = false, any_drop = false;
  for (int task = threadIdx.x; task < rows * 4; task += blockDim.x) {
    const int i = task >> 2, w = task & 3;
    const int s = s0 + i;
    const int t0 = kt * 128 + w * 32;
    uint32_t bits = 0;
    const int64_t e0 = b * a.m_b + (int64_t)s * a.m_s + t0;
    const uint16_t* hp = static_cast<const uint16_t*>(a.mask) + e0;
    if (half_mask && t0 + 32 <= min(a.mask_len, a.span) && (reinterpret_cast<uintptr_t>(hp) & 15u) == 0) {
      bits = keep_bits16(reinterpret_cast<const uint4*>(hp), inf_bits);
    } else {
#pragma unroll 8
      for (int e = 0; e < 32; ++e) bits |= (uint32_t)keep_key(a, b, s, t0 + e, seq_off) << e;
    }
    reinterpret_cast<uint32_t*>(kbits + ((int64_t)b * a.S_q + s) * a.nkt + kt)[w] = bits;
    any_keep |= bits != 0u;
    any_drop |= bits != 0xffffffffu;
  }
  any_keep = __syncthreads_or(any_keep);
  any_drop = __syncthreads_or(any_drop);
  if (threadIdx.x == 0) cls[(int64_t)item * a.nkt + kt] = any_keep ? (any_drop ? 2 : 1) : 0;
}

// One warp per item: the key tiles with a kept key, in order, as
// tile | (mixed << 31), and their number.
__global__ void __launch_bounds__(256) prefill_mask_list_kernel(const uint8_t* cls, int nkt, int items, int* tlist,
                                                                int* tcount) {
  const int item = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (item >= items) return;
  int n = 0;
  for (int k0 = 0; k0 < nkt; k0 += 32) {
    const int kt = k0 + lane;
    const int c = kt < nkt ? cls[(int64_t)item * nkt + kt] : 0;
    const uint32_t m = __ballot_sync(0xffffffffu, c != 0);
    if (c) tlist[(int64_t)item * nkt + n + __popc(m & ((1u << lane) - 1u))] = kt | (c == 2 ? (int)0x80000000 : 0);
    n += __popc(m);
  }
  if (lane == 0) tcount[item] = n;
}

// Writes the chunk's new k/v rows into the paged cache at [seq[b], seq[b]+S_q).
// One warp per 16 consecutive tokens of one (sequence, KV head): lanes 0-15
// look up the 16 tokens' blocks at once, then every lane copies 16-byte
// pieces of the 32 rows (16 K, 16 V), 8 loads issued before their stores, so
// a warp moves 8 KB (D = 128) behind a few round trips. One warp per token
// moved 512 bytes behind three and ran at 1.7 TB/s.
constexpr int kAppendTok = 16;  // tokens per warp
template <int D>
__global__ void __launch_bounds__(256)
    paged_append_kernel(const char* k_new, const char* v_new, int64_t kn_b, int64_t kn_h, int64_t kn_s, int64_t vn_b,
                        int64_t vn_h, int64_t vn_s, char* kcache, char* vcache, int64_t cs_block, int64_t cs_head,
                        int64_t cs_tok, const int32_t* seq, int64_t seq_stride, const void* bt, int bt_dtype,
                        int64_t bt_stride, int bs, int span, int num_blocks, int S_q, uint32_t* err) {
  constexpr int CPR = D / 8;                             // 16-byte pieces per row
  constexpr int PER_LANE = 2 * kAppendTok * CPR / 32;    // pieces per lane: 16 (D = 128) or 8 (D = 64)
  constexpr int BATCH = 8;
  static_assert(PER_LANE % BATCH == 0, "pieces per lane");
  // the attention kernel after this one may be scheduled now: it waits in
  // its own code for this grid to complete before reading the cache
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = (blockIdx.x * 8 + warp) * kAppendTok;
  const int h = blockIdx.y, b = blockIdx.z;
  if (tok0 >= S_q) return;
  const int s0 = seq[b * seq_stride];
  // lane t < 16: the block of token tok0 + t (-1: no row to write)
  int64_t my_row = -1;
  if (lane < kAppendTok) {
    const int tok = tok0 + lane, pos = s0 + tok;
    if (tok < S_q) {
      if (s0 < 0 || pos >= span) {
        if (err) atomicOr(err, RBLN_DEVERR_SEQ_RANGE);
      } else {
        const int64_t blk = load_index(bt, bt_dtype, b * bt_stride + pos / bs);
        if (blk < 0 || blk >= num_blocks) {
          if (err) atomicOr(err, RBLN_DEVERR_BLOCK_ID_RANGE);
        } else {
          my_row = (blk * cs_block + h * cs_head + (int64_t)(pos % bs) * cs_tok) * 2;
        }
      }
    }
  }
  const char* ksrc = k_new + b * kn_b + h * kn_h;
  const char* vsrc = v_new + b * vn_b + h * vn_h;
#pragma unroll
  for (int i0 = 0; i0 < PER_LANE; i0 += BATCH) {
    uint4 val[BATCH];
    int64_t dst[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = (i0 + u) * 32 + lane;  // piece c: row c / CPR (K rows 0-15, V rows 16-31), part c % CPR
      const int r = c / CPR, j = c - r * CPR;
      const int t = r & (kAppendTok - 1);
      const int64_t row = __shfl_sync(0xffffffffu, my_row, t);
      dst[u] = row < 0 ? -1 : row + j * 16;
      const char* src = (r < kAppendTok ? ksrc + (int64_t)(tok0 + t) * kn_s : vsrc + (int64_t)(tok0 + t) * vn_s) + j * 16;
      val[u] = row < 0 ? make_uint4(0, 0, 0, 0) : *reinterpret_cast<const uint4*>(src);
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = (i0 + u) * 32 + lane;
      if (dst[u] >= 0) *reinterpret_cast<uint4*>(((c / CPR) < kAppendTok ? kcache : vcache) + dst[u]) = val[u];
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct TcLaunch {
  CUtensorMap tq, tk, tv;
  AttnArgs a;
  int D;
  bool bf16;
  bool dependent = false;  // 128-key kernel: programmatic dependent of the previous launch
};

template <int D, bool BF16>
int launch_tc(const TcLaunch& Lc, cudaStream_t st) {
  using SL = SmemLayout<D>;
  // per-device attribute: set on every launch (cheap, host-side only)
  if (cudaFuncSetAttribute(attn_fwd_tc_kernel<D, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::ALLOC) !=
      cudaSuccess)
    return RBLN_ERR_LAUNCH;
  dim3 grid(Lc.a.q_tiles, Lc.a.Hkv, Lc.a.B);
  attn_fwd_tc_kernel<D, BF16><<<grid, kThreads, SL::ALLOC, st>>>(Lc.tq, Lc.tk, Lc.tv, Lc.a);
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

template <int D, bool BF16>
int launch_tc2(const TcLaunch& Lc, cudaStream_t st) {
  using SL = SmemLayout2<D>;
  if (cudaFuncSetAttribute(attn_fwd_tc2_kernel<D, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::ALLOC) !=
      cudaSuccess)
    return RBLN_ERR_LAUNCH;
  const long long n = (long long)Lc.a.q_tiles * Lc.a.B * Lc.a.Hkv;
  if (n > 2147483647LL) return RBLN_ERR_UNSUPPORTED;
  attn_fwd_tc2_kernel<D, BF16><<<(unsigned)n, kThreads2, SL::ALLOC, st>>>(Lc.tq, Lc.tk, Lc.tv, Lc.a);
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

int launch_tc2_any(const TcLaunch& Lc, cudaStream_t st) {
  if (Lc.D == 128) return Lc.bf16 ? launch_tc2<128, true>(Lc, st) : launch_tc2<128, false>(Lc, st);
  return Lc.bf16 ? launch_tc2<64, true>(Lc, st) : launch_tc2<64, false>(Lc, st);
}

// Streaming multiprocessors of the current device (looked up once per device).
int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

template <int D, bool BF16, int POLY, bool MASKED>
int launch_tc3(const TcLaunch& Lc, cudaStream_t st) {
  using SL = SmemLayout3<D>;
  // The warpgroups' setmaxnreg split assumes 168 registers per thread at
  // launch; with fewer, a warpgroup raising its count would never be served.
  static const bool regs_ok = [] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, attn_fwd_tc3_kernel<D, BF16, POLY, MASKED>) == cudaSuccess &&
           2 * 128 * kRegsSoftmax3 + 128 * kRegsOther3 <= (uint32_t)fa.numRegs * kThreads3;
  }();
  if (!regs_ok) return RBLN_ERR_LAUNCH;
  if (cudaFuncSetAttribute(attn_fwd_tc3_kernel<D, BF16, POLY, MASKED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SL::ALLOC) != cudaSuccess)
    return RBLN_ERR_LAUNCH;
  const long long n = (long long)Lc.a.q_tiles * Lc.a.B * Lc.a.Hkv;
  if (n > 2147483647LL) return RBLN_ERR_UNSUPPORTED;
  // persistent: one CTA per SM, each striding through the units
  const int grid = (int)std::min<long long>(n, sm_count());
  if (grid == 0) return RBLN_OK;
  if (!Lc.dependent) {
    attn_fwd_tc3_kernel<D, BF16, POLY, MASKED><<<grid, kThreads3, SL::ALLOC, st>>>(Lc.tq, Lc.tk, Lc.tv, Lc.a, (int)n);
    return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads3);
  cfg.dynamicSmemBytes = SL::ALLOC;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attn_fwd_tc3_kernel<D, BF16, POLY, MASKED>, Lc.tq, Lc.tk, Lc.tv, Lc.a, (int)n) ==
                 cudaSuccess
             ? RBLN_OK
             : RBLN_ERR_LAUNCH;
}

// Share of the 128-key kernel's exponentials evaluated on the FMA pipe:
// every POLY-th pair (0: none). Default 8 (one in eight), best of 0/4/8 on
// B200; RBLN_ATTN_PREFILL_POLY in {0, 2, 4, 8} overrides it.
int prefill_poly() {
  static const int v = [] {
    const char* e = std::getenv("RBLN_ATTN_PREFILL_POLY");
    const int x = e ? std::atoi(e) : -1;
    return (x == 0 || x == 2 || x == 4 || x == 8) ? x : 8;
  }();
  return v;
}

template <int D, bool BF16>
int launch_tc3_poly(const TcLaunch& Lc, cudaStream_t st) {
  switch (prefill_poly()) {
    case 2: return launch_tc3<D, BF16, 2, false>(Lc, st);
    case 4: return launch_tc3<D, BF16, 4, false>(Lc, st);
    case 8: return launch_tc3<D, BF16, 8, false>(Lc, st);
    default: return launch_tc3<D, BF16, 0, false>(Lc, st);
  }
}

int launch_tc3_any(const TcLaunch& Lc, cudaStream_t st) {
  if (Lc.a.tcount) {  // masked launch (mask pre-pass lists): the default exponential split only
    if (Lc.D == 128) return Lc.bf16 ? launch_tc3<128, true, 8, true>(Lc, st) : launch_tc3<128, false, 8, true>(Lc, st);
    return Lc.bf16 ? launch_tc3<64, true, 8, true>(Lc, st) : launch_tc3<64, false, 8, true>(Lc, st);
  }
  if (Lc.D == 128) return Lc.bf16 ? launch_tc3_poly<128, true>(Lc, st) : launch_tc3_poly<128, false>(Lc, st);
  return Lc.bf16 ? launch_tc3_poly<64, true>(Lc, st) : launch_tc3_poly<64, false>(Lc, st);
}

// Kernel for the mask-free paths: 3 = 128-key tiles (default), 2 = 64-key
// tiles (RBLN_ATTN_PREFILL_KERNEL=2).
int mask_free_kernel() {
  static const int v = [] {
    const char* e = std::getenv("RBLN_ATTN_PREFILL_KERNEL");
    return (e && std::atoi(e) == 2) ? 2 : 3;
  }();
  return v;
}

// The two-tile kernel serves mask-free causal/bidirectional attention whose
// block size gives 1 KB-aligned 64-row boxes.
bool use_tc2(const AttnArgs& a) {
  if (a.mask || a.pmask || a.mask_mode == MM_KEEP) return false;
  if (a.bt == nullptr) return true;
  return (a.bs >= 8 && a.bs <= BN2 && BN2 % a.bs == 0) || (a.bs >= BN2 && a.bs % BN2 == 0);
}

int launch_tc_any(const TcLaunch& Lc, cudaStream_t st) {
  if (Lc.D == 128) return Lc.bf16 ? launch_tc<128, true>(Lc, st) : launch_tc<128, false>(Lc, st);
  return Lc.bf16 ? launch_tc<64, true>(Lc, st) : launch_tc<64, false>(Lc, st);
}

// q [B, Hkv, G, S, D] (element strides b, hkv, g, s) -> 5-D map, box {64, QT, G, 1, 1}
bool map_q(CUtensorMap* m, const void* q, int dt, int B, int Hkv, int G, int S, int D, const int64_t* qs, int QT) {
  uint64_t dims[5] = {(uint64_t)D, (uint64_t)S, (uint64_t)G, (uint64_t)Hkv, (uint64_t)B};
  uint64_t str[4] = {(uint64_t)qs[3] * 2, (uint64_t)qs[2] * 2, (uint64_t)qs[1] * 2, (uint64_t)qs[0] * 2};
  uint32_t box[5] = {64, (uint32_t)QT, (uint32_t)G, 1, 1};
  return make_map(m, tmap_dtype(dt), 5, const_cast<void*>(q), dims, str, box);
}


bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Items ranked by prefill_schedule_kernel (its shared memory holds one int each).
constexpr int kMaxScheduledItems = 8192;

constexpr size_t round256(size_t x) { return (x + 255) / 256 * 256; }

// Workspace of a two-tile (128-key kernel) prefill launch, 256-byte regions:
//   work     items + 1 ints (longest-first order, then the unit counter),
//            when items <= kMaxScheduledItems
//   masked launches (p->mask set) also:
//   tcount   items ints; tlist items x nkt ints; cls items x nkt bytes;
//   kbits    B x S_q x nkt x 16 bytes
struct PrefillWs {
  size_t work = 0, tcount = 0, tlist = 0, cls = 0, kbits = 0, total = 0;
  long long items = 0;
  int nkt = 0;
};

PrefillWs prefill_ws_layout(const rbln_paged_attn_params_t* p) {
  PrefillWs w;
  if (!p || p->group <= 0 || p->group > BM || p->batch <= 0 || p->q_len <= 0 || p->max_blocks <= 0 ||
      p->block_size <= 0)
    return w;
  const int QT = BM / p->group;
  w.items = (long long)p->batch * ((p->q_len + 2 * QT - 1) / (2 * QT));
  size_t off = 0;
  if (w.items <= kMaxScheduledItems) {
    w.work = off;
    off += round256((size_t)(w.items + 1) * sizeof(int));
  }
  if (p->mask) {
    const long long span = (long long)p->max_blocks * p->block_size;
    w.nkt = (int)((span + BN3 - 1) / BN3);
    w.tcount = off;
    off += round256((size_t)w.items * sizeof(int));
    w.tlist = off;
    off += round256((size_t)w.items * w.nkt * sizeof(int));
    w.cls = off;
    off += round256((size_t)w.items * w.nkt);
    w.kbits = off;
    off += round256((size_t)p->batch * p->q_len * w.nkt * 16);
  }
  w.total = off ? off + 256 : 0;  // + slack to align the base to 256 bytes
  return w;
}

size_t prefill_ws_bytes(const rbln_paged_attn_params_t* p) { return prefill_ws_layout(p).total; }

int run_prefill(const rbln_paged_attn_params_t* p, cudaStream_t st, bool keep_mask_op) {
  if (!p || p->batch < 0 || p->num_kv_heads <= 0 || p->group <= 0 || p->block_size <= 0 || p->max_blocks <= 0 ||
      p->num_blocks <= 0 || p->q_len < 0)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->head_dim != 64 && p->head_dim != 128) return RBLN_ERR_UNSUPPORTED;
  if (p->q_dtype != RBLN_DT_BF16 && p->q_dtype != RBLN_DT_F16) return RBLN_ERR_UNSUPPORTED;
  if (p->kv_dtype != p->q_dtype) return RBLN_ERR_UNSUPPORTED;
  if (p->group > BM) return RBLN_ERR_UNSUPPORTED;
  const int bs = p->block_size;
  // TMA boxes of min(bs, 128) rows must start on 1 KB (8-row) swizzle atoms
  if (!((bs >= 8 && bs <= BN && BN % bs == 0) || (bs >= BN && bs % BN == 0))) return RBLN_ERR_UNSUPPORTED;
  if (keep_mask_op && !p->mask) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->batch == 0 || p->q_len == 0) return RBLN_OK;
  if (!p->q || !p->out || !p->kcache || !p->vcache || !p->seq || !p->block_table) return RBLN_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->q) || !aligned16(p->out) || !aligned16(p->kcache) || !aligned16(p->vcache))
    return RBLN_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < 4; ++i)
    if ((p->q_stride[i] * 2) % 16 || (p->out_stride[i] * 2) % 16) return RBLN_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < 3; ++i)
    if ((p->cache_stride[i] * 2) % 16) return RBLN_ERR_INVALID_ARGUMENT;
  const int64_t span64 = (int64_t)p->max_blocks * bs;
  if (span64 > (1 << 30)) return RBLN_ERR_UNSUPPORTED;
  const int D = p->head_dim, G = p->group;
  const int QT = BM / G;
  const int q_tiles = (p->q_len + QT - 1) / QT;
  if (q_tiles > 65535 || p->num_kv_heads > 65535 || p->batch > 65535) return RBLN_ERR_UNSUPPORTED;

  // 1) write the chunk's k/v rows into the cache
  if (p->k_new) {
    if (!p->v_new || !aligned16(p->k_new) || !aligned16(p->v_new)) return RBLN_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 3; ++i)
      if ((p->k_new_stride[i] * 2) % 16 || (p->v_new_stride[i] * 2) % 16) return RBLN_ERR_INVALID_ARGUMENT;
    dim3 grid((p->q_len + 8 * kAppendTok - 1) / (8 * kAppendTok), p->num_kv_heads, p->batch);
    auto* kn = static_cast<const char*>(p->k_new);
    auto* vn = static_cast<const char*>(p->v_new);
    if (D == 128)
      paged_append_kernel<128><<<grid, 256, 0, st>>>(
          kn, vn, p->k_new_stride[0] * 2, p->k_new_stride[1] * 2, p->k_new_stride[2] * 2, p->v_new_stride[0] * 2,
          p->v_new_stride[1] * 2, p->v_new_stride[2] * 2, (char*)p->kcache, (char*)p->vcache, p->cache_stride[0],
          p->cache_stride[1], p->cache_stride[2], p->seq, p->seq_stride, p->block_table, p->block_table_dtype,
          p->block_table_stride, bs, (int)span64, p->num_blocks, p->q_len, p->error_flags);
    else
      paged_append_kernel<64><<<grid, 256, 0, st>>>(
          kn, vn, p->k_new_stride[0] * 2, p->k_new_stride[1] * 2, p->k_new_stride[2] * 2, p->v_new_stride[0] * 2,
          p->v_new_stride[1] * 2, p->v_new_stride[2] * 2, (char*)p->kcache, (char*)p->vcache, p->cache_stride[0],
          p->cache_stride[1], p->cache_stride[2], p->seq, p->seq_stride, p->block_table, p->block_table_dtype,
          p->block_table_stride, bs, (int)span64, p->num_blocks, p->q_len, p->error_flags);
    if (cudaGetLastError() != cudaSuccess) return RBLN_ERR_LAUNCH;
  }

  // 2) attention: the 128-key kernel (3) unless RBLN_ATTN_PREFILL_KERNEL=2
  // picks the 64-key one; a keep-mask or position mask needs the mask
  // pre-pass and its workspace, and falls back to the one-tile kernel (1)
  // without it (as do sinks on the 64-key kernel)
  TcLaunch Lc{};
  Lc.D = D;
  Lc.bf16 = p->q_dtype == RBLN_DT_BF16;
  const int mfk = mask_free_kernel();
  const bool masked = keep_mask_op || p->mask != nullptr;
  const PrefillWs wl = prefill_ws_layout(p);
  const bool ws_ok = p->workspace != nullptr && wl.total > 0 && p->workspace_bytes >= wl.total;
  int kern;
  if (masked)
    kern = (mfk == 3 && ws_ok && wl.nkt > 0 && wl.items <= 65535) ? 3 : 1;
  else if (mfk == 3)
    kern = 3;
  else
    kern = (!p->sinks && ((bs >= 8 && bs <= BN2 && BN2 % bs == 0) || (bs >= BN2 && bs % BN2 == 0))) ? 2 : 1;
  const bool two_tile = kern != 1;
  const int rpb = std::min(bs, kern == 2 ? BN2 : BN);
  if (!map_q(&Lc.tq, p->q, p->q_dtype, p->batch, p->num_kv_heads, G, p->q_len, D, p->q_stride, QT))
    return RBLN_ERR_LAUNCH;
  if (!map_kv(&Lc.tk, p->kcache, p->kv_dtype, p->num_blocks, p->num_kv_heads, bs, D, p->cache_stride[0],
              p->cache_stride[1], p->cache_stride[2], rpb))
    return RBLN_ERR_LAUNCH;
  if (!map_kv(&Lc.tv, p->vcache, p->kv_dtype, p->num_blocks, p->num_kv_heads, bs, D, p->cache_stride[0],
              p->cache_stride[1], p->cache_stride[2], rpb))
    return RBLN_ERR_LAUNCH;
  AttnArgs& a = Lc.a;
  a.out = (char*)p->out;
  a.os_b = p->out_stride[0] * 2;
  a.os_h = p->out_stride[1] * 2;
  a.os_g = p->out_stride[2] * 2;
  a.os_s = p->out_stride[3] * 2;
  a.seq = p->seq;
  a.seq_stride = p->seq_stride;
  a.bt = p->block_table;
  a.bt_dtype = p->block_table_dtype;
  a.bt_stride = p->block_table_stride;
  a.max_blocks = p->max_blocks;
  a.num_blocks = p->num_blocks;
  a.bs = bs;
  a.span = (int)span64;
  a.kv_extra = 0;
  a.B = p->batch;
  a.Hkv = p->num_kv_heads;
  a.G = G;
  a.S_q = p->q_len;
  a.QT = QT;
  a.q_tiles = two_tile ? (p->q_len + 2 * QT - 1) / (2 * QT) : q_tiles;
  if (keep_mask_op) {
    a.mask_mode = MM_KEEP;
    a.mask = p->mask;
    a.mask_dtype = p->mask_dtype;
    a.mask_len = p->mask_len;
    a.m_b = p->mask_stride[0];
    a.m_h = 0;
    a.m_s = p->mask_stride[1];
  } else {
    a.mask_mode = p->causal ? MM_CAUSAL : MM_NONE;
    if (p->mask) {  // optional position mask [B, L]
      a.pmask = p->mask;
      a.pmask_dtype = p->mask_dtype;
      a.pmask_len = p->mask_len;
      a.pm_b = p->mask_stride[0];
    }
  }
  a.scale = p->scale;
  a.scale_dev = p->scale_dev;
  a.err = p->error_flags;
  a.sinks = p->sinks;
  if (two_tile && ws_ok) {
    char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(p->workspace) + 255) & ~uintptr_t(255));
    const int n = p->batch * a.q_tiles;  // == wl.items
    if (kern == 3 && masked) {
      // keep bits and tile classes, then each item's list of key tiles
      a.nkt = wl.nkt;
      a.kbits = reinterpret_cast<const uint4*>(base + wl.kbits);
      a.tlist = reinterpret_cast<const int*>(base + wl.tlist);
      a.tcount = reinterpret_cast<const int*>(base + wl.tcount);
      prefill_mask_bits_kernel<<<dim3(wl.nkt, n), 256, 0, st>>>(a, reinterpret_cast<uint4*>(base + wl.kbits),
                                                                 reinterpret_cast<uint8_t*>(base + wl.cls));
      prefill_mask_list_kernel<<<(n + 7) / 8, 256, 0, st>>>(reinterpret_cast<const uint8_t*>(base + wl.cls), wl.nkt,
                                                            n, reinterpret_cast<int*>(base + wl.tlist),
                                                            reinterpret_cast<int*>(base + wl.tcount));
      if (cudaGetLastError() != cudaSuccess) return RBLN_ERR_LAUNCH;
    }
    if (n <= kMaxScheduledItems) {
      int* work = reinterpret_cast<int*>(base + wl.work);
      prefill_schedule_kernel<<<1, 256, n * sizeof(int), st>>>(p->seq, p->seq_stride, p->batch, a.q_tiles, p->q_len,
                                                               2 * QT, (int)span64, p->causal, a.tcount, work);
      if (cudaGetLastError() != cudaSuccess) return RBLN_ERR_LAUNCH;
      a.work = work;
      a.counter = work + n;
    }
  }
  if (p->prof_events[0]) cudaEventRecord(static_cast<cudaEvent_t>(p->prof_events[0]), st);
  // the 128-key kernel's set-up overlaps the append (or schedule) kernel before it
  Lc.dependent = kern == 3;
  const int rc = kern == 3 ? launch_tc3_any(Lc, st) : kern == 2 ? launch_tc2_any(Lc, st) : launch_tc_any(Lc, st);
  if (p->prof_events[1]) cudaEventRecord(static_cast<cudaEvent_t>(p->prof_events[1]), st);
  return rc;
}

}  // namespace

// Dense attention on the same kernel (used by rbln_sdpa_fwd, sdpa.cu).
// q [B, Hkv, G, L, D] by element strides qs = {b, hkv, g, l}; k/v [B, Hkv, S, D]
// by strides {b, h, s}; mask [B|1, Hq|1, L, S] by strides {b, hq, l} (key stride 1).
int attn_tc_dense(const void* q, const int64_t* qs, void* out, const int64_t* os, float* lse, const int64_t* ls,
                  const void* k, const void* v, const int64_t* ks, const int64_t* vs, int dtype, int B, int Hkv,
                  int G, int L, int S, int D, int causal, const void* mask, int mask_dtype, int mask_additive,
                  const int64_t* ms, float scale, uint32_t* err, cudaStream_t st) {
  if (D != 64 && D != 128) return RBLN_ERR_UNSUPPORTED;
  if (G > BM || S <= 0) return RBLN_ERR_UNSUPPORTED;
  TcLaunch Lc{};
  Lc.D = D;
  Lc.bf16 = dtype == RBLN_DT_BF16;
  const int QT = BM / G;
  const int q_tiles = (L + QT - 1) / QT;
  if (q_tiles > 65535 || Hkv > 65535 || B > 65535) return RBLN_ERR_UNSUPPORTED;
  if (!map_q(&Lc.tq, q, dtype, B, Hkv, G, L, D, qs, QT)) return RBLN_ERR_LAUNCH;
  const bool two_tile = (mask == nullptr);
  const int mfk = mask_free_kernel();
  const int rows_per_box = (two_tile && mfk == 2) ? BN2 : BN;
  // k [B, Hkv, S, D] seen as a pool of B blocks of S rows
  if (!map_kv(&Lc.tk, k, dtype, B, Hkv, S, D, ks[0], ks[1], ks[2], rows_per_box)) return RBLN_ERR_LAUNCH;
  if (!map_kv(&Lc.tv, v, dtype, B, Hkv, S, D, vs[0], vs[1], vs[2], rows_per_box)) return RBLN_ERR_LAUNCH;
  AttnArgs& a = Lc.a;
  a.out = (char*)out;
  a.os_b = os[0] * 2;
  a.os_h = os[1] * 2;
  a.os_g = os[2] * 2;
  a.os_s = os[3] * 2;
  a.lse = lse;
  if (lse) {
    a.ls_b = ls[0];
    a.ls_h = ls[1];
    a.ls_g = ls[2];
    a.ls_s = ls[3];
  }
  a.seq = nullptr;
  a.bt = nullptr;
  a.max_blocks = 1;
  a.num_blocks = B;
  a.bs = ((S + BN - 1) / BN) * BN;
  a.span = a.bs;
  a.kv_extra = S;
  a.B = B;
  a.Hkv = Hkv;
  a.G = G;
  a.S_q = L;
  a.QT = QT;
  a.q_tiles = q_tiles;
  a.mask_mode = causal ? MM_CAUSAL : MM_NONE;
  if (mask) {
    a.mask = mask;
    a.mask_dtype = mask_dtype;
    a.mask_additive = mask_additive;
    a.mask_len = S;
    a.m_b = ms[0];
    a.m_h = ms[1];
    a.m_s = ms[2];
  }
  a.scale = scale;
  a.err = err;
  if (two_tile) {
    a.q_tiles = (L + 2 * QT - 1) / (2 * QT);
    return mfk == 3 ? launch_tc3_any(Lc, st) : launch_tc2_any(Lc, st);
  }
  return launch_tc_any(Lc, st);
}

}  // namespace rbln

extern "C" {

int rbln_paged_prefill_workspace_size(const rbln_paged_attn_params_t* p, size_t* bytes) {
  if (!p || !bytes) return RBLN_ERR_INVALID_ARGUMENT;
  *bytes = (size_t)rbln::prefill_ws_bytes(p);
  return RBLN_OK;
}

int rbln_paged_causal_attn_prefill(const rbln_paged_attn_params_t* p, cudaStream_t stream) {
  return rbln::run_prefill(p, stream, /*keep_mask_op=*/false);
}

int rbln_paged_attn_prefill(const rbln_paged_attn_params_t* p, cudaStream_t stream) {
  return rbln::run_prefill(p, stream, /*keep_mask_op=*/true);
}

}  // extern "C"
