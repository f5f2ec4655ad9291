// Scaled dot-product attention backward on the sm_100a tensor cores
// (aten::_scaled_dot_product_fused_attention_overrideable_backward on CUDA).
//
// Reference semantics: torch_rbln/_internal/kernels/sdpa.py:754-821 with the
// math of _sdpa_backward_fallback (sdpa.py:614-667) and grad_attn_bias
// (sdpa.py:800-818). With P = softmax(scale * Q K^T + mask) the forward's
// attention weights:
//   dV = P^T dO,  dP = dO V^T,  dS = P * (dP - rowsum(dP * P)),
//   dQ = scale * dS K,  dK = scale * dS^T Q,  dbias = dS,
// with GQA gradients of K and V summed over the query heads of each KV head.
// rowsum(dP * P) equals rowsum(dO * O), which is what is computed here.
//
// The reference keeps the forward's P in a cache keyed by the output
// tensor. Here P is recomputed tile by tile from Q, K and the forward's
// logsumexp, as flash-attention backward passes do: nothing of size L x S
// is stored unless dbias is asked for.
//
// Three launches:
//   sdpa_bwd_rows_kernel  one pass over O and dO: per query row
//                         {lse * log2(e), rowsum(dO * O)}, padded per head to
//                         a multiple of 128 rows (padding rows: {+inf, 0}, so
//                         their P and dS are 0).
//   sdpa_bwd_kv_kernel    one CTA per (128-key tile, KV head, batch): K and V
//                         tiles stay in shared memory while Q and dO tiles of
//                         every query head of the group stream through a
//                         2-stage TMA ring. Per tile, in TMEM:
//                           S^T = K Q^T and dP^T = V dO^T (128 x 128 each),
//                         the compute warps (thread = key row = TMEM lane)
//                         turn them into P^T and dS^T as bf16/f16 pairs
//                         written back over columns 32-95 of their own
//                         buffers (see kPackOff), and
//                           dV += P^T dO, dK += dS^T Q
//                         read those as the A operand straight from TMEM.
//                         Each tile is handled in two halves of 64 query rows
//                         with their own barriers, pipelined across tiles.
//                         The grid is 1-D, key tile major: under a causal
//                         mask the first key tiles see the most query tiles,
//                         so the longest CTAs launch first.
//   sdpa_bwd_q_kernel     persistent, one CTA per SM walking the units (128-query
//                         tile, query head, batch): per unit Q and dO stay, K
//                         and V tiles stream; S = Q K^T, dP = dO V^T, dS over
//                         S's buffer, dQ += dS K (two halves of 64 keys,
//                         pipelined the same way, and on across units).
// No atomics: every output element has one writer.
//
// Warp roles in both tile kernels (384 threads): warp 0 issues the TMA copies
// (one thread; in the dK/dV kernel also a bulk copy of the tile's 128 row
// pairs into shared memory), warp 1 owns TMEM and issues the MMAs (one
// thread), warps 2-3 idle, warps 4-11 compute: thread = TMEM lane, the two
// warps of a lane quadrant each take 64 of the tile's 128 columns. The
// compute warpgroups take 192 registers per thread, the first one 112 (the
// largest compute share with no spills in either). The mask, the dbias store
// and the causal test are compile-time or per-32-column-chunk decisions, so
// an unmasked chunk costs one FMA, one exp2, two FP ops and a pack per
// element. Every mbarrier wait is bounded (sm100.cuh);
// on timeout the CTA raises RBLN_DEVERR_TIMEOUT, drains its copies and MMAs,
// frees TMEM and returns.

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_map.cuh"

namespace rbln {
namespace {

using namespace sm100;

constexpr int BT = 128;                 // rows per tile: keys (kv kernel) or queries (q kernel)
constexpr int kPanel = 128 * 128;       // 128 rows x 64 16-bit elements, 128B-swizzled

struct BwdArgs {
  int B, H, Hkv, G, L, S, Lp;  // Lp: rows per head in `rows`, L rounded up to 128
  int causal;
  float qk_mult;  // scale * log2(e)
  float scale;
  const float2* rows;  // [B * H][Lp] {lse * log2(e) (+inf: no key), rowsum(dO * O)}
  const void* mask;
  int mask_dtype, mask_additive;
  int64_t m_b, m_h, m_l;  // element strides (query-head index), key stride 1
  float* dbias;           // optional [B, H, L, S]
  char* dq;
  int64_t dq_b, dq_h, dq_l;  // bytes
  char* dk;
  int64_t dk_b, dk_h, dk_l;
  char* dv;
  int64_t dv_b, dv_h, dv_l;
  uint32_t* err;
};

__device__ __forceinline__ float bias_value(const void* base, int dt, int64_t i) {
  switch (dt) {
    case RBLN_DT_F32: return static_cast<const float*>(base)[i];
    case RBLN_DT_F16: return __half2float(static_cast<const __half*>(base)[i]);
    case RBLN_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
    default: return static_cast<const uint8_t*>(base)[i] ? 1.f : 0.f;
  }
}

// ---------------------------------------------------------------------------
// per-row pre-pass
// ---------------------------------------------------------------------------
template <int D, bool BF16>
__global__ void __launch_bounds__(256) sdpa_bwd_rows_kernel(const char* out, int64_t os_b, int64_t os_h,
                                                            int64_t os_l, const char* dout, int64_t ds_b,
                                                            int64_t ds_h, int64_t ds_l, const float* lse,
                                                            int64_t ls_b, int64_t ls_h, int64_t ls_l,
                                                            float2* rows, int H, int L, int Lp, int64_t nrows) {
  constexpr int TPR = D / 8;  // threads per row, 8 elements (16 bytes) each
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int64_t row = gid / TPR;  // in [0, B * H * Lp)
  const int part = (int)(gid % TPR);
  float acc = 0.f;
  int b = 0, h = 0, l = 0;
  const bool in_range = row < nrows;
  if (in_range) {
    l = (int)(row % Lp);
    const int64_t bh = row / Lp;
    h = (int)(bh % H);
    b = (int)(bh / H);
    if (l < L) {
      const uint4 o = *reinterpret_cast<const uint4*>(out + b * os_b + h * os_h + l * os_l + part * 16);
      const uint4 d = *reinterpret_cast<const uint4*>(dout + b * ds_b + h * ds_h + l * ds_l + part * 16);
      const uint32_t ow[4] = {o.x, o.y, o.z, o.w}, dw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 of = unpack2<BF16>(ow[i]), df = unpack2<BF16>(dw[i]);
        acc = fmaf(of.x, df.x, acc);
        acc = fmaf(of.y, df.y, acc);
      }
    }
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (in_range && part == 0) {
    float2 r = make_float2(__int_as_float(0x7f800000), 0.f);  // +inf: P = 0
    if (l < L) {
      const float v = lse[b * ls_b + h * ls_h + (int64_t)l * ls_l];
      if (v != neg_inf()) r.x = v * kLog2e;
      r.y = acc;
    }
    rows[row] = r;
  }
}

// ---------------------------------------------------------------------------
// dK / dV
// ---------------------------------------------------------------------------
template <int D>
struct KvLayout {
  static constexpr int NP = D / 64;
  static constexpr int K = 0;
  static constexpr int V = K + NP * kPanel;
  static constexpr int Q0 = V + NP * kPanel;     // stage s at Q0 + s * NP * kPanel
  static constexpr int DO0 = Q0 + 2 * NP * kPanel;
  static constexpr int RI0 = DO0 + 2 * NP * kPanel;  // stage s: the tile's 128 row pairs (1 KB)
  static constexpr int BAR = RI0 + 2 * BT * 8;
  static constexpr int TMEM_SLOT = BAR + 16 * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int TOTAL = ABORT + 8;
  // + alignment slack; at least 120 KB so that one CTA (which holds all 512
  // TMEM columns) is resident per SM
  static constexpr int ALLOC = (TOTAL + 1024 > 120 * 1024) ? TOTAL + 1024 : 120 * 1024;
};

// SF/PF come in two halves (A: the tile's columns 0-63, B: 64-127): the
// compute warps of half A start while the tensor cores compute half B, and
// dV / dK of half A run while the compute warps of half B work.
enum KvBar { KB_KV = 0, KB_QF0, KB_QF1, KB_QE0, KB_QE1, KB_SFA, KB_SFB, KB_PFA, KB_PFB, KB_DONE, KB_COUNT };

// Tile i of a kv CTA: query head g of the group, query tile qt.
__device__ __forceinline__ void kv_tile(int i, int per_g, int qt0, int& g, int& qt) {
  g = i / per_g;
  qt = qt0 + (i - g * per_g);
}

// Packed (16-bit pairs) outputs of the compute warps sit at column offset
// kPackOff of the S / dP buffers: chunk c (32 fp32 columns) packs into
// columns [kPackOff + 16c, kPackOff + 16c + 16). The warp of half 0 reads
// chunks 0-1 (columns [0, 64)) and processes chunk 1 first; the warp of
// half 1 reads chunks 2-3 ([64, 128)) and processes chunk 2 first. So every
// packed store lands on columns its own warp has already read, and the two
// warps of a lane quadrant never touch each other's columns.
constexpr int kPackOff = 32;

// 12 warps: producer 0, MMA 1, 2-3 idle, and 8 compute warps (4..11) with
// lane quadrant warp % 4 and column half (warp - 4) / 4. The first warpgroup
// gives registers up (setmaxnreg) so that a compute thread holds both of its
// chunks of S and dP without spilling (168 per thread at launch).
constexpr int kBwdThreads = 384;
constexpr int kComputeWarps = 8;
constexpr uint32_t kRegsCompute = 192, kRegsCtl = 112;
static_assert(2 * 128 * kRegsCompute + 128 * kRegsCtl <= kBwdThreads * 168, "register split exceeds the launch");

// The split needs the 168 registers per thread at launch: with fewer, a
// warpgroup raising its count would never be served.
template <typename K>
bool bwd_regs_ok(K* kernel) {
  cudaFuncAttributes fa{};
  return cudaFuncGetAttributes(&fa, kernel) == cudaSuccess &&
         2 * 128 * kRegsCompute + 128 * kRegsCtl <= (uint32_t)fa.numRegs * kBwdThreads;
}

template <int D, bool BF16, bool MASK, bool DBIAS>
__global__ void __launch_bounds__(kBwdThreads, 1)
    sdpa_bwd_kv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                       const BwdArgs a) {
  using Lay = KvLayout<D>;
  constexpr int NP = Lay::NP;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  volatile int* abort = reinterpret_cast<volatile int*>(sgen + Lay::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + Lay::TMEM_SLOT);
  auto bar = [&](int i) { return sbase + Lay::BAR + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // one-dimensional grid, key tile major: under a causal mask the first key
  // tiles see the most query tiles, so the longest CTAs launch first
  const int hb = (int)(blockIdx.x % (unsigned)(a.Hkv * a.B));
  const int kt = (int)(blockIdx.x / (unsigned)(a.Hkv * a.B)), h = hb % a.Hkv, b = hb / a.Hkv;
  const int t0 = kt * BT;
  const int nq = (a.L + BT - 1) / BT;
  // top-left causal: query l sees key t only when t <= l, so tiles before
  // the one holding query t0 contribute nothing
  const int qt0 = a.causal ? min(t0 / BT, nq) : 0;
  const int per_g = nq - qt0;
  const int ntiles = a.G * per_g;

  if (threadIdx.x == 0) {
    *abort = 0;
    for (int i = 0; i < KB_COUNT; ++i)
      mbar_init(bar(i), (i == KB_PFA || i == KB_PFB) ? (uint32_t)(kComputeWarps / 2) : 1u);
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
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 384;

  // Each warpgroup changes its register count at the top of its own branch,
  // so the code of the branch is compiled for that count.
  if (warp < 4) {
   setmaxnreg_dec<kRegsCtl>();
   if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntiles > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      prefetch_tmap(&tm_do);
      mbar_arrive_expect_tx(bar(KB_KV), 2 * NP * kPanel);
      for (int p = 0; p < NP; ++p) {
        tma_load_4d(sbase + Lay::K + p * kPanel, &tm_k, bar(KB_KV), p * 64, t0, h, b);
        tma_load_4d(sbase + Lay::V + p * kPanel, &tm_v, bar(KB_KV), p * 64, t0, h, b);
      }
      int issued = 0;
      for (int i = 0; i < ntiles; ++i) {
        const int st = i & 1;
        if (i >= 2 && !mbar_wait(bar(KB_QE0 + st), ((i >> 1) - 1) & 1, abort)) break;
        int g, qt;
        kv_tile(i, per_g, qt0, g, qt);
        const int hq = h * a.G + g;
        mbar_arrive_expect_tx(bar(KB_QF0 + st), 2 * NP * kPanel + BT * 8);
        for (int p = 0; p < NP; ++p) {
          tma_load_4d(sbase + Lay::Q0 + (st * NP + p) * kPanel, &tm_q, bar(KB_QF0 + st), p * 64, qt * BT, hq, b);
          tma_load_4d(sbase + Lay::DO0 + (st * NP + p) * kPanel, &tm_do, bar(KB_QF0 + st), p * 64, qt * BT, hq,
                      b);
        }
        // {lse, delta} of the tile's 128 query rows: 1 KB at a 1 KB-aligned offset
        bulk_load(sbase + Lay::RI0 + st * BT * 8, a.rows + ((int64_t)b * a.H + hq) * a.Lp + qt * BT, BT * 8,
                  bar(KB_QF0 + st));
        issued = i + 1;
      }
      if (*abort) {
        // let the copies already issued land before the CTA's memory goes away
        const long long c0 = clock64();
        while (!mbar_try_wait(bar(KB_KV), 0) && clock64() - c0 < 2000000) {
        }
        for (int i = max(0, issued - 2); i < issued; ++i) {
          const long long c1 = clock64();
          while (!mbar_try_wait(bar(KB_QF0 + (i & 1)), (i >> 1) & 1) && clock64() - c1 < 2000000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (lane == 0 && ntiles > 0) {
      const uint32_t id_s = idesc_f16(BF16, BT, BT / 2, false);  // S^T, dP^T halves: K-major over D
      const uint32_t id_acc = idesc_f16(BF16, BT, D, true);      // dV, dK: B (dO, Q) MN-major
      // S^T and dP^T of half hh (query rows [64 hh, 64 hh + 64)) of tile i
      auto issue_s = [&](int i, int hh) {
        const int st = i & 1;
        const uint32_t qb = sbase + Lay::Q0 + st * NP * kPanel + hh * 8192;
        const uint32_t db = sbase + Lay::DO0 + st * NP * kPanel + hh * 8192;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPanel + (kk & 3) * 32;
          umma_f16_ss(t_s + 64 * hh, sw128_desc(sbase + Lay::K + off, 16, 1024), sw128_desc(qb + off, 16, 1024),
                      id_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPanel + (kk & 3) * 32;
          umma_f16_ss(t_dp + 64 * hh, sw128_desc(sbase + Lay::V + off, 16, 1024), sw128_desc(db + off, 16, 1024),
                      id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(KB_SFA + hh));
      };
      // dV += P^T dO and dK += dS^T Q over half hh's 64 query rows of tile i
      auto issue_acc = [&](int i, int hh) {
        const int st = i & 1;
        const uint32_t qb = sbase + Lay::Q0 + st * NP * kPanel;
        const uint32_t db = sbase + Lay::DO0 + st * NP * kPanel;
#pragma unroll
        for (int k4 = 0; k4 < BT / 32; ++k4) {
          const int kk = hh * (BT / 32) + k4;
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ts(t_dv, t_s + kPackOff + kk * 8, sw128_desc(db + kk * 16 * 128, kPanel, 1024), id_acc, acc);
          umma_f16_ts(t_dk, t_dp + kPackOff + kk * 8, sw128_desc(qb + kk * 16 * 128, kPanel, 1024), id_acc, acc);
        }
      };
      // Software pipeline over tiles: half A of tile i + 1 is issued as soon as
      // half A of tile i has been consumed, so the compute warps of half A
      // work on tile i + 1 while those of half B finish tile i. Every write
      // of a new S^T / dP^T half follows, in issue order, the MMAs that read
      // the packed P^T / dS^T it overwrites (tcgen05.mma runs in issue order).
      bool ok = mbar_wait(bar(KB_KV), 0, abort) && mbar_wait(bar(KB_QF0), 0, abort);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(0, 1);
      }
      for (int i = 0; ok && i < ntiles; ++i) {
        const int st = i & 1;
        const bool more = i + 1 < ntiles;
        if (!mbar_wait(bar(KB_PFA), i & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_acc(i, 0);
        if (more) {
          if (!mbar_wait(bar(KB_QF0 + ((i + 1) & 1)), ((i + 1) >> 1) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(i + 1, 0);
        }
        if (!mbar_wait(bar(KB_PFB), i & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_acc(i, 1);
        umma_commit(bar(KB_QE0 + st));
        if (more) issue_s(i + 1, 1);
      }
      umma_commit(bar(KB_DONE));
      if (!ok) {
        // abort: let the MMAs already issued finish before TMEM is freed
        const long long c0 = clock64();
        while (!mbar_try_wait(bar(KB_DONE), 0) && clock64() - c0 < 4000000) {
        }
      }
    }
   }
  } else {
    setmaxnreg_inc<kRegsCompute>();
    // ------------------------------------------------------------- compute
    const int quad = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = quad * 32 + lane;  // key row == TMEM lane
    const int t = t0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    for (int i = 0; i < ntiles; ++i) {
      const int st = i & 1;
      int g, qt;
      kv_tile(i, per_g, qt0, g, qt);
      const int hq = h * a.G + g;
      const int l0 = qt * BT;
      const int64_t mrow = MASK ? (int64_t)b * a.m_b + (int64_t)hq * a.m_h : 0;
      float* dbrow = DBIAS ? a.dbias + (((int64_t)b * a.H + hq) * a.L) * a.S + t : nullptr;
      // S^T / dP^T of this tile are in TMEM once SF completes; the row pairs
      // were copied with the tile's Q / dO (QF). tcgen05.ld is .sync.aligned:
      // the whole warp takes the same path.
      if (!__all_sync(0xffffffffu, mbar_wait(bar(KB_QF0 + st), (i >> 1) & 1, abort) &&
                                       mbar_wait(bar(KB_SFA + half), i & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float2* ri = reinterpret_cast<const float2*>(sgen + Lay::RI0 + st * BT * 8);
      // both of this warp's 32-column chunks of S^T and dP^T come in one TMEM
      // round trip (half 0: chunks 1 then 0; half 1: chunks 2 then 3), so
      // every packed store below lands on columns already read
      const int c4a = half == 0 ? 1 : 2, c4b = half == 0 ? 0 : 3;
      uint32_t sva[32], dva[32], svb[32], dvb[32];
      __syncwarp();
      tmem_ld32(t_s + lane_off + c4a * 32, sva);
      tmem_ld32(t_dp + lane_off + c4a * 32, dva);
      tmem_ld32(t_s + lane_off + c4b * 32, svb);
      tmem_ld32(t_dp + lane_off + c4b * 32, dvb);
      tmem_wait_ld();
      auto chunk = [&](int c4, const uint32_t(&sv)[32], const uint32_t(&dv)[32]) {
        const int la = l0 + c4 * 32;
        // 0: nothing visible, 1: everything (but padding rows, whose lse is
        // +inf), 2: the causal diagonal crosses the chunk
        const int cls = t >= a.S ? 0 : (!a.causal || t <= la) ? 1 : (t > la + 31 ? 0 : 2);
        uint32_t pk[16], dk[16];
        if (cls == 0) {
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = dk[e] = 0u;
        } else if (!MASK && !DBIAS && cls == 1) {  // every query row sees this key: no per-element test
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float4 rr = *reinterpret_cast<const float4*>(ri + c4 * 32 + 2 * e);  // shared-memory broadcast
            float p0 = __uint_as_float(sv[2 * e]), p1 = __uint_as_float(sv[2 * e + 1]);
            fma2(p0, p1, a.qk_mult, a.qk_mult, -rr.x, -rr.z);
            p0 = exp2_approx(p0);
            p1 = exp2_approx(p1);
            float d0 = __uint_as_float(dv[2 * e]), d1 = __uint_as_float(dv[2 * e + 1]);
            add2(d0, d1, -rr.y, -rr.w);
            mul2(d0, d1, p0, p1);
            pk[e] = pack2<BF16>(p0, p1);
            dk[e] = pack2<BF16>(d0, d1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float pp[2], dd[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int c = c4 * 32 + 2 * e + u;
              const int l = la + 2 * e + u;
              const float2 rw = ri[c];  // shared-memory broadcast
              float x = fmaf(__uint_as_float(sv[2 * e + u]), a.qk_mult, -rw.x);
              bool keep = cls == 1 || t <= l;
              if (MASK) {
                if (l < a.L) {
                  const float mv = bias_value(a.mask, a.mask_dtype, mrow + (int64_t)l * a.m_l + t);
                  if (a.mask_additive) {
                    x = fmaf(mv, kLog2e, x);
                  } else {
                    keep = keep && mv > 0.f;
                  }
                }
              }
              const float p = keep ? exp2_approx(x) : 0.f;  // padding rows: x = -inf, p = 0
              const float ds = keep ? p * (__uint_as_float(dv[2 * e + u]) - rw.y) : 0.f;
              pp[u] = p;
              dd[u] = ds;
              if (DBIAS && l < a.L) dbrow[(int64_t)l * a.S] = ds;
            }
            pk[e] = pack2<BF16>(pp[0], pp[1]);
            dk[e] = pack2<BF16>(dd[0], dd[1]);
          }
        }
        tmem_st16(t_s + lane_off + kPackOff + c4 * 16, pk);
        tmem_st16(t_dp + lane_off + kPackOff + c4 * 16, dk);
      };
      chunk(c4a, sva, dva);
      chunk(c4b, svb, dvb);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(KB_PFA + half));
    }

    // ------------------------------------------------------------ epilogue
    // each of the quadrant's two warps stores half of the D columns
    ok = __all_sync(0xffffffffu, ok);
    if (ok && ntiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(KB_DONE), 0, abort));
    tc_fence_after();
    if (ok) {
      char* dvrow = a.dv ? a.dv + b * a.dv_b + h * a.dv_h + (int64_t)t * a.dv_l : nullptr;
      char* dkrow = a.dk ? a.dk + b * a.dk_b + h * a.dk_h + (int64_t)t * a.dk_l : nullptr;
#pragma unroll 1
      for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
        uint32_t ov[32], ok2[32];
        if (ntiles > 0) {
          __syncwarp();
          tmem_ld32(t_dv + lane_off + c * 32, ov);
          tmem_ld32(t_dk + lane_off + c * 32, ok2);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = ok2[e] = 0u;
        }
        if (t < a.S) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 w, x;
            w.x = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 0]), __uint_as_float(ov[q4 * 8 + 1]));
            w.y = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 2]), __uint_as_float(ov[q4 * 8 + 3]));
            w.z = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 4]), __uint_as_float(ov[q4 * 8 + 5]));
            w.w = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 6]), __uint_as_float(ov[q4 * 8 + 7]));
            x.x = pack2<BF16>(__uint_as_float(ok2[q4 * 8 + 0]) * a.scale, __uint_as_float(ok2[q4 * 8 + 1]) * a.scale);
            x.y = pack2<BF16>(__uint_as_float(ok2[q4 * 8 + 2]) * a.scale, __uint_as_float(ok2[q4 * 8 + 3]) * a.scale);
            x.z = pack2<BF16>(__uint_as_float(ok2[q4 * 8 + 4]) * a.scale, __uint_as_float(ok2[q4 * 8 + 5]) * a.scale);
            x.w = pack2<BF16>(__uint_as_float(ok2[q4 * 8 + 6]) * a.scale, __uint_as_float(ok2[q4 * 8 + 7]) * a.scale);
            if (dvrow) *reinterpret_cast<uint4*>(dvrow + (c * 32 + q4 * 8) * 2) = w;
            if (dkrow) *reinterpret_cast<uint4*>(dkrow + (c * 32 + q4 * 8) * 2) = x;
          }
        }
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
// dQ
// ---------------------------------------------------------------------------
template <int D>
struct QLayout {
  static constexpr int NP = D / 64;
  static constexpr int Q = 0;
  static constexpr int DO = Q + NP * kPanel;
  static constexpr int K0 = DO + NP * kPanel;  // stage s at K0 + s * NP * kPanel
  static constexpr int V0 = K0 + 2 * NP * kPanel;
  static constexpr int BAR = V0 + 2 * NP * kPanel;
  static constexpr int TMEM_SLOT = BAR + 16 * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int TOTAL = ABORT + 8;
  static constexpr int ALLOC = (TOTAL + 1024 > 120 * 1024) ? TOTAL + 1024 : 120 * 1024;
};

// Persistent: one CTA per SM walks the units (query tile, query head, batch)
// in longest-first order (the last query tiles see the most keys under a
// causal mask), dealt to the CTAs in snake order so that every CTA gets a
// near-equal share of key tiles. The K/V ring, the S/dP halves and their
// barriers follow a running count of the CTA's key tiles, so the pipeline
// runs on across units; Q and dO of the next unit are loaded as soon as the
// last S/dP MMAs of the current one have completed (QB_QE). dQ is
// accumulated in two TMEM buffers used by alternate units, so the compute
// warps store one unit's dQ while the tensor cores start the next unit; a
// buffer is reused two units later, after its store (QB_DQE).
enum QBar {
  QB_Q = 0, QB_QE, QB_KF0, QB_KF1, QB_KE0, QB_KE1, QB_SFA, QB_SFB, QB_PFA, QB_PFB,
  QB_DQF0, QB_DQF1, QB_DQE0, QB_DQE1, QB_DONE, QB_COUNT
};

// Unit k of this CTA: false when the CTA has no k-th unit.
__device__ __forceinline__ bool q_unit(const BwdArgs& a, int nqt, int k, int& qt, int& hq, int& b) {
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  const int64_t idx = (int64_t)k * G + ((k & 1) ? G - 1 - c : c);
  const int64_t per = (int64_t)a.H * a.B;
  if (idx >= (int64_t)nqt * per) return false;
  qt = nqt - 1 - (int)(idx / per);
  const int rem = (int)(idx % per);
  hq = rem % a.H;
  b = rem / a.H;
  return true;
}

// Key tiles unit (qt) attends: all of them, or those up to the diagonal.
__device__ __forceinline__ int q_unit_tiles(const BwdArgs& a, int qt) {
  const int nk_all = (a.S + BT - 1) / BT;
  return a.causal ? min(nk_all, qt + 1) : nk_all;
}

template <int D, bool BF16, bool MASK>
__global__ void __launch_bounds__(kBwdThreads, 1)
    sdpa_bwd_q_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                      const BwdArgs a) {
  using Lay = QLayout<D>;
  constexpr int NP = Lay::NP;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  volatile int* abort = reinterpret_cast<volatile int*>(sgen + Lay::ABORT);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + Lay::TMEM_SLOT);
  auto bar = [&](int i) { return sbase + Lay::BAR + 8u * i; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (a.L + BT - 1) / BT;

  if (threadIdx.x == 0) {
    *abort = 0;
    for (int i = 0; i < QB_COUNT; ++i)
      mbar_init(bar(i), (i == QB_PFA || i == QB_PFB) ? (uint32_t)(kComputeWarps / 2)
                        : (i == QB_DQE0 || i == QB_DQE1) ? (uint32_t)kComputeWarps
                                                         : 1u);
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
  const uint32_t t_s = tmem, t_dp = tmem + 128;
  auto t_dq = [&](int x) { return tmem + 256 + x * D; };

  // Each warpgroup changes its register count at the top of its own branch,
  // so the code of the branch is compiled for that count.
  if (warp < 4) {
   setmaxnreg_dec<kRegsCtl>();
   if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      prefetch_tmap(&tm_do);
      int T = 0, uc = 0, issued = 0, q_issued = 0;
      bool ok = true;
      int qt, hq, b;
      for (int k = 0; ok && q_unit(a, nqt, k, qt, hq, b); ++k) {
        const int nk = q_unit_tiles(a, qt), h = hq / a.G;
        if (nk == 0) continue;
        for (int j = 0; j < nk; ++j) {
          const int Tj = T + j, st = Tj & 1;
          if (Tj >= 2 && !mbar_wait(bar(QB_KE0 + st), ((Tj >> 1) - 1) & 1, abort)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(QB_KF0 + st), 2 * NP * kPanel);
          for (int p = 0; p < NP; ++p) {
            tma_load_4d(sbase + Lay::K0 + (st * NP + p) * kPanel, &tm_k, bar(QB_KF0 + st), p * 64, j * BT, h, b);
            tma_load_4d(sbase + Lay::V0 + (st * NP + p) * kPanel, &tm_v, bar(QB_KF0 + st), p * 64, j * BT, h, b);
          }
          issued = Tj + 1;
          if (j == 0) {
            // Q and dO of this unit once the previous unit's last S / dP MMAs
            // are done (its first K/V tile went out before that wait)
            if (uc >= 1 && !mbar_wait(bar(QB_QE), (uc - 1) & 1, abort)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(bar(QB_Q), 2 * NP * kPanel);
            for (int p = 0; p < NP; ++p) {
              tma_load_4d(sbase + Lay::Q + p * kPanel, &tm_q, bar(QB_Q), p * 64, qt * BT, hq, b);
              tma_load_4d(sbase + Lay::DO + p * kPanel, &tm_do, bar(QB_Q), p * 64, qt * BT, hq, b);
            }
            q_issued = uc + 1;
          }
        }
        T += nk;
        ++uc;
      }
      if (*abort) {
        // let the copies in flight land before the CTA exits
        const long long c0 = clock64();
        if (q_issued > 0)
          while (!mbar_try_wait(bar(QB_Q), (q_issued - 1) & 1) && clock64() - c0 < 2000000) {
          }
        for (int j = max(0, issued - 2); j < issued; ++j) {
          const long long c1 = clock64();
          while (!mbar_try_wait(bar(QB_KF0 + (j & 1)), (j >> 1) & 1) && clock64() - c1 < 2000000) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t id_s = idesc_f16(BF16, BT, BT / 2, false);  // S, dP halves (64 keys each)
      const uint32_t id_dq = idesc_f16(BF16, BT, D, true);       // B (K) MN-major
      auto issue_s = [&](int Tj, int hh) {  // S, dP of keys [64 hh, 64 hh + 64) of ring tile Tj
        const int st = Tj & 1;
        const uint32_t kb = sbase + Lay::K0 + st * NP * kPanel + hh * 8192;
        const uint32_t vb = sbase + Lay::V0 + st * NP * kPanel + hh * 8192;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPanel + (kk & 3) * 32;
          umma_f16_ss(t_s + 64 * hh, sw128_desc(sbase + Lay::Q + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                      id_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPanel + (kk & 3) * 32;
          umma_f16_ss(t_dp + 64 * hh, sw128_desc(sbase + Lay::DO + off, 16, 1024), sw128_desc(vb + off, 16, 1024),
                      id_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar(QB_SFA + hh));
      };
      auto issue_dq = [&](int Tj, int j, int hh, int x) {  // dQ_x += dS K over half hh's 64 keys
        const uint32_t kb = sbase + Lay::K0 + (Tj & 1) * NP * kPanel;
#pragma unroll
        for (int k4 = 0; k4 < BT / 32; ++k4) {
          const int kk = hh * (BT / 32) + k4;
          umma_f16_ts(t_dq(x), t_s + kPackOff + kk * 8, sw128_desc(kb + kk * 16 * 128, kPanel, 1024), id_dq,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      int T = 0, uc = 0;
      bool ok = true;
      int qt, hq, b;
      for (int k = 0; ok && q_unit(a, nqt, k, qt, hq, b); ++k) {
        const int nk = q_unit_tiles(a, qt);
        if (nk == 0) continue;
        const int x = uc & 1;
        // dQ buffer x: its store two units ago has completed; Q / dO loaded;
        // the first key tile landed
        if ((uc >= 2 && !mbar_wait(bar(QB_DQE0 + x), ((uc >> 1) - 1) & 1, abort)) ||
            !mbar_wait(bar(QB_Q), uc & 1, abort) || !mbar_wait(bar(QB_KF0 + (T & 1)), (T >> 1) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(T, 0);
        issue_s(T, 1);
        // the same two-half software pipeline as the dK/dV kernel
        for (int j = 0; j < nk; ++j) {
          const int Tj = T + j;
          const bool more = j + 1 < nk;
          if (!mbar_wait(bar(QB_PFA), Tj & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_dq(Tj, j, 0, x);
          if (more) {
            if (!mbar_wait(bar(QB_KF0 + ((Tj + 1) & 1)), ((Tj + 1) >> 1) & 1, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(Tj + 1, 0);
          }
          if (!mbar_wait(bar(QB_PFB), Tj & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_dq(Tj, j, 1, x);
          umma_commit(bar(QB_KE0 + (Tj & 1)));
          if (more) {
            issue_s(Tj + 1, 1);
          } else {
            umma_commit(bar(QB_QE));        // every S / dP of the unit done: Q and dO may be reloaded
            umma_commit(bar(QB_DQF0 + x));  // the unit's dQ is complete
          }
        }
        T += nk;
        ++uc;
      }
      umma_commit(bar(QB_DONE));
      if (!ok) {
        const long long c0 = clock64();
        while (!mbar_try_wait(bar(QB_DONE), 0) && clock64() - c0 < 4000000) {
        }
      }
    }
   }
  } else {
    setmaxnreg_inc<kRegsCompute>();
    // --------------------------------------------------------- compute
    const int quad = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = quad * 32 + lane;  // query row == TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    int T = 0, uc = 0;
    bool ok = true;
    int qt, hq, b;
    for (int k = 0; ok && q_unit(a, nqt, k, qt, hq, b); ++k) {
      const int nk = q_unit_tiles(a, qt);
      if (nk == 0) continue;
      const int l = qt * BT + r;
      const float2 rw = a.rows[((int64_t)b * a.H + hq) * a.Lp + l];  // padding rows: {+inf, 0}
      const int64_t mrow = MASK ? (int64_t)b * a.m_b + (int64_t)hq * a.m_h + (int64_t)min(l, a.L - 1) * a.m_l : 0;
      for (int j = 0; j < nk; ++j) {
        const int Tj = T + j;
        const int kt0 = j * BT;
        if (!__all_sync(0xffffffffu, mbar_wait(bar(QB_SFA + half), Tj & 1, abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // both of this warp's 32-column chunks of S and dP come in one TMEM
        // round trip (half 0: chunks 1 then 0; half 1: chunks 2 then 3), so
        // every packed store below lands on columns already read
        const int c4a = half == 0 ? 1 : 2, c4b = half == 0 ? 0 : 3;
        uint32_t sva[32], dva[32], svb[32], dvb[32];
        __syncwarp();
        tmem_ld32(t_s + lane_off + c4a * 32, sva);
        tmem_ld32(t_dp + lane_off + c4a * 32, dva);
        tmem_ld32(t_s + lane_off + c4b * 32, svb);
        tmem_ld32(t_dp + lane_off + c4b * 32, dvb);
        tmem_wait_ld();
        auto chunk = [&](int c4, const uint32_t(&sv)[32], const uint32_t(&dv)[32]) {
          const int ta = kt0 + c4 * 32;
          // 0: nothing visible, 1: every key (rows past L have lse +inf), 2: per key
          const int cls = (ta >= a.S || (a.causal && ta > l)) ? 0
                          : ((!a.causal || ta + 31 <= l) && ta + 31 < a.S) ? 1 : 2;
          uint32_t dk[16];
          if (cls == 0) {
#pragma unroll
            for (int e = 0; e < 16; ++e) dk[e] = 0u;
          } else if (!MASK && cls == 1) {  // every key visible: no per-key test
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float p0 = __uint_as_float(sv[2 * e]), p1 = __uint_as_float(sv[2 * e + 1]);
              fma2(p0, p1, a.qk_mult, a.qk_mult, -rw.x, -rw.x);
              p0 = exp2_approx(p0);
            p1 = exp2_approx(p1);
              float d0 = __uint_as_float(dv[2 * e]), d1 = __uint_as_float(dv[2 * e + 1]);
              add2(d0, d1, -rw.y, -rw.y);
              mul2(d0, d1, p0, p1);
              dk[e] = pack2<BF16>(d0, d1);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float dd[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int t = ta + 2 * e + u;
                float xs = fmaf(__uint_as_float(sv[2 * e + u]), a.qk_mult, -rw.x);
                bool keep = cls == 1 || (t < a.S && (!a.causal || t <= l));
                if (MASK) {
                  if (keep && l < a.L) {
                    const float mv = bias_value(a.mask, a.mask_dtype, mrow + t);
                    if (a.mask_additive) {
                      xs = fmaf(mv, kLog2e, xs);
                    } else {
                      keep = mv > 0.f;
                    }
                  }
                }
                const float p = keep ? exp2_approx(xs) : 0.f;
                dd[u] = keep ? p * (__uint_as_float(dv[2 * e + u]) - rw.y) : 0.f;
              }
              dk[e] = pack2<BF16>(dd[0], dd[1]);
            }
          }
          tmem_st16(t_s + lane_off + kPackOff + c4 * 16, dk);
        };
        chunk(c4a, sva, dva);
        chunk(c4b, svb, dvb);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(QB_PFA + half));
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      // this unit's dQ: wait for its last MMA, store it, release the buffer
      const int x = uc & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(QB_DQF0 + x), (uc >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (a.dq) {
        char* qrow = a.dq + b * a.dq_b + hq * a.dq_h + (int64_t)l * a.dq_l;
#pragma unroll 1
        for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
          uint32_t ov[32];
          __syncwarp();
          tmem_ld32(t_dq(x) + lane_off + c * 32, ov);
          tmem_wait_ld();
          if (l < a.L) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint4 w;
              w.x = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 0]) * a.scale, __uint_as_float(ov[q4 * 8 + 1]) * a.scale);
              w.y = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 2]) * a.scale, __uint_as_float(ov[q4 * 8 + 3]) * a.scale);
              w.z = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 4]) * a.scale, __uint_as_float(ov[q4 * 8 + 5]) * a.scale);
              w.w = pack2<BF16>(__uint_as_float(ov[q4 * 8 + 6]) * a.scale, __uint_as_float(ov[q4 * 8 + 7]) * a.scale);
              *reinterpret_cast<uint4*>(qrow + (c * 32 + q4 * 8) * 2) = w;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(QB_DQE0 + x));
      T += nk;
      ++uc;
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
// host side
// ---------------------------------------------------------------------------
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t rows_bytes(const rbln_sdpa_bwd_params_t* p) {
  const int64_t Lp = ((int64_t)p->q_len + BT - 1) / BT * BT;
  return (size_t)p->batch * p->num_heads * Lp * sizeof(float2);
}

struct BwdMaps {
  CUtensorMap q, k, v, dout;
};

template <int D, bool BF16, bool MASK, bool DBIAS>
int launch_kv(const BwdMaps& m, const BwdArgs& a, cudaStream_t st) {
  constexpr int sm = KvLayout<D>::ALLOC;
  auto* k = sdpa_bwd_kv_kernel<D, BF16, MASK, DBIAS>;
  static const bool regs_ok = bwd_regs_ok(k);
  if (!regs_ok) return RBLN_ERR_LAUNCH;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) return RBLN_ERR_LAUNCH;
  const int64_t n = (int64_t)((a.S + BT - 1) / BT) * a.Hkv * a.B;
  if (n > 2147483647LL) return RBLN_ERR_UNSUPPORTED;
  k<<<(unsigned)n, kBwdThreads, sm, st>>>(m.q, m.k, m.v, m.dout, a);
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

template <int D, bool BF16, bool MASK>
int launch_q(const BwdMaps& m, const BwdArgs& a, cudaStream_t st) {
  constexpr int sm = QLayout<D>::ALLOC;
  auto* k = sdpa_bwd_q_kernel<D, BF16, MASK>;
  static const bool regs_ok = bwd_regs_ok(k);
  if (!regs_ok) return RBLN_ERR_LAUNCH;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) != cudaSuccess) return RBLN_ERR_LAUNCH;
  // persistent: one CTA per SM (at most one per unit)
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      sms = n;
    if (sms <= 0) sms = 148;
  }
  const int64_t units = (int64_t)((a.L + BT - 1) / BT) * a.H * a.B;
  const int grid = (int)std::min<int64_t>(units, sms);
  k<<<grid, kBwdThreads, sm, st>>>(m.q, m.k, m.v, m.dout, a);
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

template <int D, bool BF16>
int launch_bwd(const rbln_sdpa_bwd_params_t* p, const BwdMaps& m, const BwdArgs& a, cudaStream_t st) {
  const int64_t nrows = (int64_t)a.B * a.H * a.Lp;
  const int64_t threads = nrows * (D / 8);
  sdpa_bwd_rows_kernel<D, BF16><<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      static_cast<const char*>(p->out), p->out_stride[0] * 2, p->out_stride[1] * 2, p->out_stride[2] * 2,
      static_cast<const char*>(p->dout), p->dout_stride[0] * 2, p->dout_stride[1] * 2, p->dout_stride[2] * 2, p->lse,
      p->lse_stride[0], p->lse_stride[1], p->lse_stride[2], const_cast<float2*>(a.rows), a.H, a.L, a.Lp, nrows);
  if (cudaGetLastError() != cudaSuccess) return RBLN_ERR_LAUNCH;
  if (p->dbias && cudaMemsetAsync(p->dbias, 0, (size_t)a.B * a.H * a.L * a.S * sizeof(float), st) != cudaSuccess)
    return RBLN_ERR_LAUNCH;
  if (p->dk || p->dv || p->dbias) {
    const int rc = !a.mask  ? launch_kv<D, BF16, false, false>(m, a, st)
                   : p->dbias ? launch_kv<D, BF16, true, true>(m, a, st)
                              : launch_kv<D, BF16, true, false>(m, a, st);
    if (rc != RBLN_OK) return rc;
  }
  if (p->dq) {
    const int rc = a.mask ? launch_q<D, BF16, true>(m, a, st) : launch_q<D, BF16, false>(m, a, st);
    if (rc != RBLN_OK) return rc;
  }
  return RBLN_OK;
}

static_assert(KvLayout<128>::ALLOC <= 227 * 1024, "kv kernel shared memory");
static_assert(QLayout<128>::ALLOC <= 227 * 1024, "q kernel shared memory");

}  // namespace
}  // namespace rbln

extern "C" {

int rbln_sdpa_bwd_workspace_size(const rbln_sdpa_bwd_params_t* p, size_t* bytes) {
  if (!p || !bytes || p->batch < 0 || p->num_heads < 0 || p->q_len < 0) return RBLN_ERR_INVALID_ARGUMENT;
  *bytes = rbln::rows_bytes(p);
  return RBLN_OK;
}

int rbln_sdpa_bwd(const rbln_sdpa_bwd_params_t* p, cudaStream_t stream) {
  using namespace rbln;
  if (!p || p->batch < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 || p->q_len < 0 || p->kv_len < 0)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->num_heads % p->num_kv_heads) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->head_dim != 64 && p->head_dim != 128) return RBLN_ERR_UNSUPPORTED;
  if (p->dtype != RBLN_DT_BF16 && p->dtype != RBLN_DT_F16) return RBLN_ERR_UNSUPPORTED;
  if (p->batch == 0 || p->q_len == 0 || p->kv_len == 0) return RBLN_OK;
  if (p->num_heads > 65535 || p->num_kv_heads > 65535 || p->batch > 65535) return RBLN_ERR_UNSUPPORTED;
  if (!p->q || !p->k || !p->v || !p->out || !p->dout || !p->lse) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->mask && p->mask_stride[3] != 1) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->dbias && (!p->mask || !p->mask_additive)) return RBLN_ERR_INVALID_ARGUMENT;
  const void* ptrs[8] = {p->q, p->k, p->v, p->out, p->dout, p->dq, p->dk, p->dv};
  for (const void* q : ptrs)
    if (q && !al16(q)) return RBLN_ERR_INVALID_ARGUMENT;
  const int64_t* strides[8] = {p->q_stride, p->k_stride, p->v_stride, p->out_stride,
                               p->dout_stride, p->dq_stride, p->dk_stride, p->dv_stride};
  for (int t = 0; t < 8; ++t)
    for (int i = 0; i < 3; ++i)
      if ((strides[t][i] * 2) % 16) return RBLN_ERR_INVALID_ARGUMENT;
  if (!p->workspace || p->workspace_bytes < rows_bytes(p) || !al16(p->workspace)) return RBLN_ERR_WORKSPACE;

  const int D = p->head_dim, H = p->num_heads, Hkv = p->num_kv_heads, B = p->batch;
  const int L = p->q_len, S = p->kv_len;
  BwdMaps m;
  if (!map_kv(&m.q, p->q, p->dtype, B, H, L, D, p->q_stride[0], p->q_stride[1], p->q_stride[2], BT) ||
      !map_kv(&m.dout, p->dout, p->dtype, B, H, L, D, p->dout_stride[0], p->dout_stride[1], p->dout_stride[2], BT) ||
      !map_kv(&m.k, p->k, p->dtype, B, Hkv, S, D, p->k_stride[0], p->k_stride[1], p->k_stride[2], BT) ||
      !map_kv(&m.v, p->v, p->dtype, B, Hkv, S, D, p->v_stride[0], p->v_stride[1], p->v_stride[2], BT))
    return RBLN_ERR_LAUNCH;
  BwdArgs a{};
  a.B = B;
  a.H = H;
  a.Hkv = Hkv;
  a.G = H / Hkv;
  a.L = L;
  a.S = S;
  a.Lp = (L + BT - 1) / BT * BT;
  a.causal = p->causal ? 1 : 0;
  a.scale = p->scale;
  a.qk_mult = p->scale * kLog2e;
  a.rows = static_cast<const float2*>(p->workspace);
  a.mask = p->mask;
  a.mask_dtype = p->mask_dtype;
  a.mask_additive = p->mask_additive;
  a.m_b = p->mask_stride[0];
  a.m_h = p->mask_stride[1];
  a.m_l = p->mask_stride[2];
  a.dbias = p->dbias;
  a.dq = static_cast<char*>(p->dq);
  a.dq_b = p->dq_stride[0] * 2;
  a.dq_h = p->dq_stride[1] * 2;
  a.dq_l = p->dq_stride[2] * 2;
  a.dk = static_cast<char*>(p->dk);
  a.dk_b = p->dk_stride[0] * 2;
  a.dk_h = p->dk_stride[1] * 2;
  a.dk_l = p->dk_stride[2] * 2;
  a.dv = static_cast<char*>(p->dv);
  a.dv_b = p->dv_stride[0] * 2;
  a.dv_h = p->dv_stride[1] * 2;
  a.dv_l = p->dv_stride[2] * 2;
  a.err = p->error_flags;
  const bool bf = p->dtype == RBLN_DT_BF16;
  if (D == 128) return bf ? launch_bwd<128, true>(p, m, a, stream) : launch_bwd<128, false>(p, m, a, stream);
  return bf ? launch_bwd<64, true>(p, m, a, stream) : launch_bwd<64, false>(p, m, a, stream);
}

}  // extern "C"
