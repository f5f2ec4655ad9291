// Paged-attention decode for sm_100a: one new query token per sequence,
// G query heads per KV head, KV read through a block table.
//
// Semantics follow the reference's CPU definition of
// rbln_custom_ops::paged_causal_attn_decode / paged_attn_decode
// (test/rbln/test_custom_kernel.py:138-216, 388-486): append the new k/v at
// position seq[b] when seq[b] < span, then softmax(q.K^T * scale + mask) . V
// over the span, generalised from the reference's single-block case to a
// real block table (position t lives in block block_table[b, t / bs], row
// t % bs).
//
// Design (bandwidth-bound):
//  * grid = (context splits, Hkv, B); a CTA owns one (sequence, KV head,
//    context split) and all G query heads of that KV head, so every KV byte
//    is read from HBM exactly once.
//  * 4 warps per CTA take 16-token tiles round-robin. A warp loads its tile
//    straight from HBM into MMA fragments with 16-byte coalesced loads: the
//    head dimension of K (and of q) is permuted so that each lane's fragment
//    elements are contiguous in memory, which leaves the dot products
//    unchanged. No shared-memory staging, no barriers in the main loop.
//  * Scores use the tensor cores with tokens as M and heads as N:
//    S^T[16 tok x 8 head] = K[16 x D] . Q^T, then O^T[D x 8] += V^T . P^T. P
//    goes from the accumulator layout to the B-operand layout with two
//    movmatrix transposes. fp32 online softmax, max reduced with shuffles.
//  * fp8-e4m3 caches are converted exactly to f16 in registers
//    (cvt.rn.f16x2.e4m3x2); the per-(block, head) K scale multiplies the
//    scores and the V scale is folded into P before the PV product.
//  * Work is cut into equal chunks across the whole batch ("balanced"
//    split-K): the sequences' lengths, each rounded up to 16 and preceded by
//    seg_cost virtual tokens (the cost of starting a segment), are laid end to
//    end and CTA (c, h) takes list positions [c*W, (c+1)*W) of KV head h,
//    whatever sequences they belong to. Each CTA computes that prefix itself
//    from seq, so no host synchronisation is needed. One wave of CTAs (4 per
//    SM) with equal work leaves no tail of long sequences.
//  * A CTA writes one (O/l, log2-sum-exp) partial per sequence it touches; a
//    merge kernel (launched as a programmatic dependent) combines them. A
//    sequence held by one CTA is written directly by it.
//  * A caller that fixes num_splits (or RBLN_ATTN_DECODE_SCHED=seq) gets the
//    per-sequence grid (splits, Hkv, B) with a.chunk tokens per split.

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

// Fixed device scratch for rbln_paged_causal_attn_decode_noalloc (callers
// that cannot allocate). Host code must not use this name as an address: it
// is a host-side stand-in; the device address comes from
// cudaGetSymbolAddress, looked up once per device below.
static __device__ __align__(256) unsigned char rbln_noalloc_scratch[RBLN_NOALLOC_SCRATCH_BYTES];

namespace rbln {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxDevices = 64;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16;

enum KvKind { KV_BF16 = 0, KV_F16 = 1, KV_FP8 = 2 };

struct DecodeArgs {
  const char* q;
  int64_t qs_b, qs_h, qs_g;  // bytes
  char* out;
  int64_t os_b, os_h, os_g;  // bytes
  const char* k_new;
  const char* v_new;
  int64_t kn_b, kn_h, vn_b, vn_h;  // bytes
  char* kcache;
  char* vcache;
  int64_t cs_block, cs_head, cs_tok;  // elements
  const float* k_scale;
  const float* v_scale;
  int64_t ss_block, ss_head;
  const int32_t* seq;
  int64_t seq_stride;
  const void* bt;
  int bt_dtype;
  int64_t bt_stride;
  const void* mask;
  int mask_dtype;
  int mask_len;
  int64_t mask_stride;
  float scale;
  const float* scale_dev;
  int B, Hkv, G, num_blocks, bs, span;
  int chunk;
  int max_splits;
  int nchunk;       // balanced split: chunks per KV head (grid.x)
  int min_w;        // balanced split: smallest chunk, in tokens
  int seg_cost;     // balanced split: virtual tokens charged to each sequence's start (multiple of 16)
  int* prefix;      // balanced split: [B + 1] padded-length prefix, then W
  // per-sequence split: [B][Hkv][max_splits][G]; balanced: [Hkv][nchunk + B][G]
  float* part_o;    // (.., D) floats per slot
  float* part_lse;  // log2-sum-exp per slot
  uint32_t* err;
  // head-sharded multi-GPU decode: final outputs go to every rank's buffer
  char* const* out_peers;  // nullptr: write `out` only
  int n_peers;
  int head0;  // first head of this rank in the full output
  const float* sinks;  // optional [Hkv * G] sink logits (natural-log units), index h * G + g
  // epoch exchange in the last CTA of the balanced merge kernel (nullptr: none)
  uint32_t* const* peer_flags;
  int peer_rank;
  uint32_t epoch;
  uint64_t wait_ns;
  int* merge_ctr;  // balanced workspace: merge CTAs done (zeroed by the decode kernel)
};

// Sink logit of local query head (h, g) in the log2 domain of the scores,
// or -inf when there are no sinks.
__device__ __forceinline__ float sink_log2(const DecodeArgs& a, int h, int g) {
  return a.sinks ? a.sinks[h * a.G + g] * kLog2e : neg_inf();
}

__device__ __forceinline__ void flag_error(uint32_t* err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

// Every kernel of the decode chain is launched as a programmatic dependent
// of the previous launch on its stream. It first waits until that grid has
// completed and its writes are visible (a no-op when the previous launch
// was not made that way), then lets the next grid on the stream be
// scheduled onto the SMs as this grid's CTAs retire; that grid waits here in
// the same way, so nothing it reads or writes is touched early.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Stores 4 output elements (one 8-byte pair of pairs) of (b, local head h,
// query head g, column d4): to `out`, or to every rank's buffer when the
// heads are sharded over GPUs.
__device__ __forceinline__ void store_out(const DecodeArgs& a, int b, int h, int g, int d4, uint2 v) {
  const int64_t off = b * a.os_b + (int64_t)(a.head0 + h) * a.os_h + (int64_t)g * a.os_g + d4 * 2;
  if (a.out_peers == nullptr) {
    *reinterpret_cast<uint2*>(a.out + off) = v;
  } else {
    for (int r = 0; r < a.n_peers; ++r) *reinterpret_cast<uint2*>(a.out_peers[r] + off) = v;
  }
}

// Context length seen by sequence b, and the number of splits covering it.
__device__ __forceinline__ void decode_extent(const DecodeArgs& a, int b, int& pos, int& L,
                                              int& nsplit) {
  pos = a.seq[b * a.seq_stride];
  if (a.mask) {
    L = min(a.span, a.mask_len);
  } else {
    L = pos < 0 ? 0 : min(pos + 1, a.span);
  }
  nsplit = max(1, (L + a.chunk - 1) / a.chunk);
}

template <int D, int KV>
struct Cfg {
  static constexpr int SZ = (KV == KV_FP8) ? 1 : 2;  // bytes per cache element
  static constexpr int ROW = D * SZ;                  // bytes per token row
  static constexpr int KCH = ROW / 64;                // 16-B K chunks per lane per row
  static constexpr int KR = D / 8;                    // u32 MMA registers per K row
  static constexpr int VSEG = (KV == KV_FP8) ? ((D == 128) ? 16 : 8) : 8;  // contiguous d per seg
  static constexpr int NVE = D / 8;                   // d values per lane per V row
  static constexpr int NSEG = NVE / VSEG;             // 2 for 16-bit D=128, else 1
  static constexpr int NVW = NVE * SZ / 4;            // raw u32 per lane per V row
  static constexpr int MT = D / 16;                   // PV m-tiles
  static constexpr bool MMA_BF16 = (KV == KV_BF16);
};

// d index of a lane's e-th V value (gid = lane/4).
template <int D, int KV>
__device__ __forceinline__ int v_dim(int gid, int e) {
  using C = Cfg<D, KV>;
  return gid * C::VSEG + (e / C::VSEG) * 64 + (e % C::VSEG);
}

// Writes the new token's k/v (bf16/f16 copy, or fp8 quantised with the
// block's scale) at position `pos` of sequence b, KV head h. Threads 0..63
// take K and 64..127 take V, 8 elements each. No barrier inside.
template <int D, int KV, bool Q_BF16>
__device__ __forceinline__ void append_token(const DecodeArgs& a, int b, int h, int pos) {
  using C = Cfg<D, KV>;
  const int tid = threadIdx.x;
  const int64_t blk = load_index(a.bt, a.bt_dtype, b * a.bt_stride + pos / a.bs);
  if (blk < 0 || blk >= a.num_blocks) {
    if (tid == 0) flag_error(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
  } else {
    const int64_t row = (blk * a.cs_block + h * a.cs_head + (pos % a.bs) * a.cs_tok) * C::SZ;
    const int part = tid >> 6;  // 0: K, 1: V
    const int j = tid & 63;     // 8 elements per thread
    if (j < D / 8) {
      const char* src = (part == 0 ? a.k_new + b * a.kn_b + h * a.kn_h
                                   : a.v_new + b * a.vn_b + h * a.vn_h) + j * 16;
      char* dst = (part == 0 ? a.kcache : a.vcache) + row;
      const uint4 x = *reinterpret_cast<const uint4*>(src);
      if constexpr (KV != KV_FP8) {
        *reinterpret_cast<uint4*>(dst + j * 16) = x;
      } else {
        const float sc = (part == 0 ? a.k_scale : a.v_scale)[blk * a.ss_block + h * a.ss_head];
        const uint32_t w[4] = {x.x, x.y, x.z, x.w};
        uint32_t o[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          float f[4];
          float2 lo = unpack2<Q_BF16>(w[2 * k]), hi = unpack2<Q_BF16>(w[2 * k + 1]);
          f[0] = lo.x / sc; f[1] = lo.y / sc; f[2] = hi.x / sc; f[3] = hi.y / sc;
          __nv_fp8x2_storage_t p01 = __nv_cvt_float2_to_fp8x2(make_float2(f[0], f[1]), __NV_SATFINITE, __NV_E4M3);
          __nv_fp8x2_storage_t p23 = __nv_cvt_float2_to_fp8x2(make_float2(f[2], f[3]), __NV_SATFINITE, __NV_E4M3);
          o[k] = uint32_t(p01) | (uint32_t(p23) << 16);
        }
        *reinterpret_cast<uint2*>(dst + j * 8) = make_uint2(o[0], o[1]);
      }
    }
  }
}

// Attention of the G query heads of KV head h of sequence b over the
// context tokens [t0, t1): the CTA's 4 warps take 16-token tiles round-robin;
// their (max, sum, O) are combined in shared memory and written as the final
// output (whole = the CTA saw every token of the sequence) or as the
// (O/l, log2-sum-exp) partial at part_o/part_lse index slot + g.
// Bytes of the CTA combine area: per-warp O [kWarps][8*NT][D] and max/sum.
template <int D, int NT>
__host__ __device__ constexpr int combine_bytes() {
  return (kWarps * 8 * NT * D + 2 * kWarps * 8 * NT) * 4;
}
// Dynamic shared memory of a split CTA (the balanced kernel adds B + 1 ints).
template <int D, int NT>
__host__ __device__ constexpr int segment_smem() {
  return combine_bytes<D, NT>();
}

// LA (block-table lookahead): false = look up each tile's block where it is
// fetched; true = load the next tile's entry into registers one tile early,
// so that the lookup is off the tile's critical path.
template <int D, int KV, bool Q_BF16, int NT, bool LA>
__device__ __forceinline__ void decode_segment(const DecodeArgs& a, unsigned char* dsm, int b, int h, int t0,
                                               int t1, bool append, bool whole, int64_t slot) {
  using C = Cfg<D, KV>;
  constexpr bool MB = C::MMA_BF16;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;

  // ---- append the new token (write-then-read, like the reference) --------
  if (append && a.k_new != nullptr) {
    append_token<D, KV, Q_BF16>(a, b, h, a.seq[b * a.seq_stride]);
    __syncthreads();
  }

  // Block id (-1 when outside [0, num_blocks)) and keep bit of token
  // ts + (lane & 15) (lanes 16..31 repeat it).
  struct TileEntry {
    int blk;
    bool keep;
  };
  auto bt_entry = [&](int ts, TileEntry& e) {
    const int tpos = ts + (lane & 15);
    const bool in = tpos < t1;
    e.keep = in && (a.mask == nullptr || load_keep(a.mask, a.mask_dtype, b * a.mask_stride + tpos));
    const int64_t blk = in ? load_index(a.bt, a.bt_dtype, b * a.bt_stride + tpos / a.bs) : -1;
    e.blk = (blk >= 0 && blk < a.num_blocks) ? (int)blk : -1;
  };
  TileEntry ent;
  if constexpr (LA) bt_entry(t0 + warp * kTile, ent);  // before the query loads: independent of them

  // ---- query fragments: B operand (k = head_dim, n = head) ---------------
  float scale = a.scale_dev ? *a.scale_dev : a.scale;
  uint32_t qf[NT][C::KR];
  float qmax = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int g = gid + 8 * nt;
    const bool live = g < a.G;
    const char* qrow = a.q + b * a.qs_b + h * a.qs_h + (int64_t)g * a.qs_g;
#pragma unroll
    for (int i = 0; i < C::KCH; ++i) {
      if constexpr (KV != KV_FP8) {
        uint4 x = live ? *reinterpret_cast<const uint4*>(qrow + (4 * i + tig) * 16) : make_uint4(0, 0, 0, 0);
        qf[nt][4 * i + 0] = x.x; qf[nt][4 * i + 1] = x.y; qf[nt][4 * i + 2] = x.z; qf[nt][4 * i + 3] = x.w;
      } else {
        // 16 fp8 K elements <-> 16 q elements (32 bytes) at d = 16*(4i+tig)
        const char* src = qrow + (4 * i + tig) * 32;
        uint4 x0 = live ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
        uint4 x1 = live ? *reinterpret_cast<const uint4*>(src + 16) : make_uint4(0, 0, 0, 0);
        const uint32_t w[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          qf[nt][8 * i + k] = w[k];
          float2 f = unpack2<Q_BF16>(w[k]);
          qmax = fmaxf(qmax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    }
  }
  float qk_mult = scale * kLog2e;
  if constexpr (KV == KV_FP8) {
    // q goes to f16 for the f16 MMA. A bf16 q is rescaled by a power of two
    // so its largest magnitude sits in [2^14, 2^15): exact, no overflow.
    float qs = 1.f;
    if constexpr (Q_BF16) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, o));
      if (qmax > 0.f) {
        int ex;
        frexpf(qmax, &ex);
        ex = min(max(15 - ex, -120), 120);
        qs = ldexpf(1.f, ex);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int k = 0; k < C::KR; ++k) {
          float2 f = unpack2<true>(qf[nt][k]);
          qf[nt][k] = pack2<false>(f.x * qs, f.y * qs);
        }
    }
    qk_mult = qk_mult / qs;
  }

  // ---- main loop over this warp's tiles -----------------------------------
  float o_acc[NT][C::MT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int mt = 0; mt < C::MT; ++mt)
#pragma unroll
      for (int k = 0; k < 4; ++k) o_acc[nt][mt][k] = 0.f;
  float m_run[NT][2], l_run[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = neg_inf();
    l_run[nt][0] = l_run[nt][1] = 0.f;
  }

  const char* kc = a.kcache;
  const char* vc = a.vcache;
  const int tv[4] = {2 * tig, 2 * tig + 1, 2 * tig + 8, 2 * tig + 9};

  // One 16-token tile in flight: lane l (mod 16) resolves token ts + l
  // through the block table; the row offsets reach the lanes that load them
  // by shuffles; then the K rows gid / gid+8 and the V rows tv[] are loaded.
  struct Tile {
    uint4 kraw[2][C::KCH];
    uint32_t vraw[4][C::NVW];
    uint32_t vmask;
    float ksc, vsc;
  };
  // The tile's block-table entry and mask byte come from `ent`, loaded one
  // tile earlier (bt_entry) so that the table lookup is off the critical path.
  auto fetch = [&](int ts, Tile& T, const TileEntry& ent) {
    const int tpos = ts + (lane & 15);
    bool valid = ent.keep;
    uint32_t off16 = 0;  // row byte offset / 16
    T.ksc = 1.f;
    T.vsc = 1.f;
    if (valid) {
      const int64_t blk = ent.blk;
      if (blk < 0) {
        valid = false;
        flag_error(a.err, RBLN_DEVERR_BLOCK_ID_RANGE);
      } else {
        off16 = (uint32_t)(((blk * a.cs_block + h * a.cs_head + (tpos % a.bs) * a.cs_tok) * C::SZ) >> 4);
        if constexpr (KV == KV_FP8) {
          T.ksc = a.k_scale[blk * a.ss_block + h * a.ss_head];
          T.vsc = a.v_scale[blk * a.ss_block + h * a.ss_head];
        }
      }
    }
    T.vmask = __ballot_sync(0xffffffffu, valid) & 0xffffu;
    if (T.vmask == 0) return;
    const uint32_t ok0 = __shfl_sync(0xffffffffu, off16, gid);
    const uint32_t ok1 = __shfl_sync(0xffffffffu, off16, gid + 8);
    const bool vk0 = (T.vmask >> gid) & 1, vk1 = (T.vmask >> (gid + 8)) & 1;
#pragma unroll
    for (int i = 0; i < C::KCH; ++i) {
      T.kraw[0][i] = vk0 ? ld_stream_v4(kc + (size_t)ok0 * 16 + (4 * i + tig) * 16) : make_uint4(0, 0, 0, 0);
      T.kraw[1][i] = vk1 ? ld_stream_v4(kc + (size_t)ok1 * 16 + (4 * i + tig) * 16) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t ov = __shfl_sync(0xffffffffu, off16, tv[j]);
      const bool vv = (T.vmask >> tv[j]) & 1;
      const char* rowp = vc + (size_t)ov * 16;
      if constexpr (C::NVW >= 4) {
#pragma unroll
        for (int sg = 0; sg < C::NVW / 4; ++sg) {
          uint4 x = vv ? ld_stream_v4(rowp + (gid * C::VSEG + sg * 64) * C::SZ) : make_uint4(0, 0, 0, 0);
          T.vraw[j][4 * sg + 0] = x.x; T.vraw[j][4 * sg + 1] = x.y;
          T.vraw[j][4 * sg + 2] = x.z; T.vraw[j][4 * sg + 3] = x.w;
        }
      } else {
        uint2 x = vv ? ld_stream_v2(rowp + gid * C::VSEG * C::SZ) : make_uint2(0, 0);
        T.vraw[j][0] = x.x; T.vraw[j][1] = x.y;
      }
    }
  };

  auto consume = [&](const Tile& T) {
    if (T.vmask == 0) return;  // warp-uniform (ballot)
    const bool vk0 = (T.vmask >> gid) & 1, vk1 = (T.vmask >> (gid + 8)) & 1;
    // S^T = K . Q^T
    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    if constexpr (KV != KV_FP8) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int i = kk >> 1, sgl = (kk & 1) * 2;
        const uint32_t* r0 = reinterpret_cast<const uint32_t*>(&T.kraw[0][i]);
        const uint32_t* r1 = reinterpret_cast<const uint32_t*>(&T.kraw[1][i]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          mma16816<MB>(s[nt], r0[sgl], r1[sgl], r0[sgl + 1], r1[sgl + 1], qf[nt][2 * kk], qf[nt][2 * kk + 1]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < C::KCH; ++i) {
        const uint32_t* r0 = reinterpret_cast<const uint32_t*>(&T.kraw[0][i]);
        const uint32_t* r1 = reinterpret_cast<const uint32_t*>(&T.kraw[1][i]);
#pragma unroll
        for (int w = 0; w < 4; ++w) {  // kk = 4i + w uses chunk word w (4 fp8)
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_f16x2x2(r0[w], a0, a2);
          e4m3x4_to_f16x2x2(r1[w], a1, a3);
          const int kk = 4 * i + w;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma16816<false>(s[nt], a0, a1, a2, a3, qf[nt][2 * kk], qf[nt][2 * kk + 1]);
        }
      }
    }

    // online softmax (log2 domain); rows gid / gid+8 are tokens
    float k0m = qk_mult, k1m = qk_mult;
    float vs0 = 1.f, vs1 = 1.f;
    if constexpr (KV == KV_FP8) {
      k0m *= __shfl_sync(0xffffffffu, T.ksc, gid);
      k1m *= __shfl_sync(0xffffffffu, T.ksc, gid + 8);
      vs0 = __shfl_sync(0xffffffffu, T.vsc, gid);
      vs1 = __shfl_sync(0xffffffffu, T.vsc, gid + 8);
    }
    uint32_t pb0[NT], pb1[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float x0 = vk0 ? s[nt][0] * k0m : neg_inf();
      const float x1 = vk0 ? s[nt][1] * k0m : neg_inf();
      const float x2 = vk1 ? s[nt][2] * k1m : neg_inf();
      const float x3 = vk1 ? s[nt][3] * k1m : neg_inf();
      const float mx0 = warp_max_xor_rows(fmaxf(x0, x2));
      const float mx1 = warp_max_xor_rows(fmaxf(x1, x3));
      const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
      const float ms0 = (mn0 == neg_inf()) ? 0.f : mn0;
      const float ms1 = (mn1 == neg_inf()) ? 0.f : mn1;
      const float al0 = exp2_approx(m_run[nt][0] - ms0), al1 = exp2_approx(m_run[nt][1] - ms1);
      const float p0 = exp2_approx(x0 - ms0), p2 = exp2_approx(x2 - ms0);
      const float p1 = exp2_approx(x1 - ms1), p3 = exp2_approx(x3 - ms1);
      l_run[nt][0] = l_run[nt][0] * al0 + p0 + p2;
      l_run[nt][1] = l_run[nt][1] * al1 + p1 + p3;
      m_run[nt][0] = mn0;
      m_run[nt][1] = mn1;
      // once the running maxima settle the factors are exactly 1 (their
      // exponent is exactly 0): the fp8 variant, which spends more issue
      // slots per tile on conversions, skips the rescale for the warp then
      // (measured +0.4 %); for 16-bit caches the vote cost as much as it saved
      if (KV != KV_FP8 || __any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
        for (int mt = 0; mt < C::MT; ++mt) {
          o_acc[nt][mt][0] *= al0; o_acc[nt][mt][2] *= al0;
          o_acc[nt][mt][1] *= al1; o_acc[nt][mt][3] *= al1;
        }
      }
      pb0[nt] = movmatrix_trans(pack2<MB>(p0 * vs0, p1 * vs0));
      pb1[nt] = movmatrix_trans(pack2<MB>(p2 * vs1, p3 * vs1));
    }

    // O^T += V^T . P^T
#pragma unroll
    for (int mt = 0; mt < C::MT; ++mt) {
      uint32_t a0, a1, a2, a3;
      if constexpr (KV != KV_FP8) {
        a0 = prmt(T.vraw[0][mt], T.vraw[1][mt], 0x5410);
        a1 = prmt(T.vraw[0][mt], T.vraw[1][mt], 0x7632);
        a2 = prmt(T.vraw[2][mt], T.vraw[3][mt], 0x5410);
        a3 = prmt(T.vraw[2][mt], T.vraw[3][mt], 0x7632);
      } else {
        const int w = mt >> 1;
        const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;
        const uint32_t x = prmt(T.vraw[0][w], T.vraw[1][w], sel);
        const uint32_t y = prmt(T.vraw[2][w], T.vraw[3][w], sel);
        e4m3x4_to_f16x2x2(x, a0, a1);
        e4m3x4_to_f16x2x2(y, a2, a3);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma16816<MB>(o_acc[nt][mt], a0, a1, a2, a3, pb0[nt], pb1[nt]);
    }
  };

  for (int ts = t0 + warp * kTile; ts < t1; ts += kWarps * kTile) {
    Tile T;
    if constexpr (!LA) bt_entry(ts, ent);
    fetch(ts, T, ent);
    // next tile's lookup overlaps this tile's loads and math
    if constexpr (LA) bt_entry(ts + kWarps * kTile, ent);
    consume(T);
  }

  // ---- combine the 4 warps of this CTA ------------------------------------
  constexpr int GP = 8 * NT;
  auto sO = reinterpret_cast<float(*)[GP][D]>(dsm);
  auto sM = reinterpret_cast<float(*)[GP]>(dsm + kWarps * GP * D * 4);
  auto sL = reinterpret_cast<float(*)[GP]>(dsm + kWarps * GP * D * 4 + kWarps * GP * 4);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const float l0 = warp_sum_xor_rows(l_run[nt][0]);
    const float l1 = warp_sum_xor_rows(l_run[nt][1]);
    const int h0 = 2 * tig + 8 * nt;
    if (gid == 0) {
      sM[warp][h0] = m_run[nt][0]; sM[warp][h0 + 1] = m_run[nt][1];
      sL[warp][h0] = l0; sL[warp][h0 + 1] = l1;
    }
#pragma unroll
    for (int mt = 0; mt < C::MT; ++mt) {
      const int d0 = v_dim<D, KV>(gid, 2 * mt), d1 = v_dim<D, KV>(gid, 2 * mt + 1);
      sO[warp][h0][d0] = o_acc[nt][mt][0];
      sO[warp][h0 + 1][d0] = o_acc[nt][mt][1];
      sO[warp][h0][d1] = o_acc[nt][mt][2];
      sO[warp][h0 + 1][d1] = o_acc[nt][mt][3];
    }
  }
  __syncthreads();

  const bool final_out = whole;
  for (int idx = tid; idx < a.G * (D / 4); idx += kThreads) {
    const int g = idx / (D / 4), d4 = (idx % (D / 4)) * 4;
    float M = neg_inf();
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sM[w][g]);
    float Lsum = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = (sM[w][g] == neg_inf()) ? 0.f : exp2_approx(sM[w][g] - M);
      Lsum += f * sL[w][g];
      const float4 o = *reinterpret_cast<const float4*>(&sO[w][g][d4]);
      acc.x += f * o.x; acc.y += f * o.y; acc.z += f * o.z; acc.w += f * o.w;
    }
    if (final_out) {
      // the sink adds e^{sink - M} to the denominator only; all positions
      // masked (M = -inf) then gives 0, and NaN without a sink
      const float inv = 1.f / (a.sinks ? Lsum + exp2f(sink_log2(a, h, g) - M) : Lsum);
      acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
      store_out(a, b, h, g, d4, make_uint2(pack2<Q_BF16>(acc.x, acc.y), pack2<Q_BF16>(acc.z, acc.w)));
    } else {
      const float inv = 1.f / Lsum;
      acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
      const int64_t ps = slot + g;
      *reinterpret_cast<float4*>(a.part_o + ps * D + d4) = acc;
      if (d4 == 0) a.part_lse[ps] = (M == neg_inf()) ? neg_inf() : M + __log2f(Lsum);
    }
  }
  if (a.out_peers && final_out) __threadfence_system();  // peer stores before the epoch exchange
  __syncthreads();  // the combine area is reused by the CTA's next segment
}



// Context length seen by sequence b (see decode_extent).
__device__ __forceinline__ int seq_len(const DecodeArgs& a, int b, int& pos) {
  pos = a.seq[b * a.seq_stride];
  return a.mask ? min(a.span, a.mask_len) : (pos < 0 ? 0 : min(pos + 1, a.span));
}

// One CTA per (context split, KV head, sequence): each sequence is cut into
// splits of a.chunk tokens.
template <int D, int KV, bool Q_BF16, int NT, bool LA>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 4 : 2) paged_decode_split_kernel(const DecodeArgs a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  pdl_enter();
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  int pos, L, nsplit;
  decode_extent(a, b, pos, L, nsplit);
  if (split >= nsplit) return;
  if (pos < 0 && threadIdx.x == 0 && split == 0) flag_error(a.err, RBLN_DEVERR_SEQ_RANGE);
  const int t0 = split * a.chunk;
  const int t1 = min(t0 + a.chunk, L);
  const bool append = pos >= 0 && pos < a.span && min(pos / a.chunk, nsplit - 1) == split;
  decode_segment<D, KV, Q_BF16, NT, LA>(a, dsm, b, h, t0, t1, append, nsplit == 1,
                                    ((int64_t)(b * a.Hkv + h) * a.max_splits + split) * a.G);
}

// Exclusive prefix P[0..B] of the sequences' lengths rounded up to 16, each
// plus seg_cost virtual tokens ahead of the sequence's real ones, in shared
// memory, and the balanced chunk size W (a multiple of 16). Sequence b's real
// tokens are list positions [P[b] + seg_cost, P[b + 1]). The virtual tokens
// charge each sequence start for its segment's fixed work (query load,
// combine, partial store), so a chunk that covers many short sequences gets
// fewer real tokens. CTA (0, 0) also stores P and W in the workspace for the
// merge kernel.
__device__ __forceinline__ int balanced_prefix(const DecodeArgs& a, int* P) {
  __shared__ int wsum[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (a.B + kThreads - 1) / kThreads;
  const int first = tid * per;
  int sum = 0, pos;
  for (int i = 0; i < per; ++i)
    if (first + i < a.B) sum += ((seq_len(a, first + i, pos) + 15) & ~15) + a.seg_cost;
  int x = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int off = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) off += w < warp ? wsum[w] : 0;
  int run = off + x - sum;
  for (int i = 0; i < per; ++i)
    if (first + i < a.B) {
      P[first + i] = run;
      run += ((seq_len(a, first + i, pos) + 15) & ~15) + a.seg_cost;
    }
  if (tid == kThreads - 1) P[a.B] = off + x;
  __syncthreads();
  const int T = P[a.B];
  const int W = max(a.min_w, ((T + a.nchunk - 1) / a.nchunk + 15) & ~15);
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    for (int i = tid; i <= a.B; i += kThreads) a.prefix[i] = P[i];
    if (tid == 0) {
      a.prefix[a.B + 1] = W;
      a.prefix[a.B + 2] = 0;  // merge CTAs done: counted by the merge kernel
    }
  }
  return W;
}

// Balanced split: the batch's tokens, each sequence padded to a multiple of
// 16 and preceded by seg_cost virtual tokens, are cut into equal chunks of W
// list positions, so every CTA has about the same work however unequal the
// sequences are. CTA (c, h) takes chunk c of KV head h,
// which may cover the end of one sequence and the start of the next ones: one
// segment (and one partial, at slot c + b of head h) per sequence touched.
template <int D, int KV, bool Q_BF16, int NT, bool LA>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 4 : 2) paged_decode_balanced_kernel(const DecodeArgs a) {
  extern __shared__ __align__(16) unsigned char dsm[];
  pdl_enter();
  int* P = reinterpret_cast<int*>(dsm + segment_smem<D, NT>());
  const int c = blockIdx.x, h = blockIdx.y;
  const int W = balanced_prefix(a, P);
  const int T = P[a.B];
  int lo = c * W;
  if (lo >= T) return;
  const int hi = min(lo + W, T);
  // last sequence whose padded range starts at or before lo (it is non-empty)
  int bl = 0, bh = a.B - 1;
  while (bl < bh) {
    const int mid = (bl + bh + 1) >> 1;
    if (P[mid] <= lo) bl = mid; else bh = mid - 1;
  }
  for (int b = bl; b < a.B && lo < hi; ++b) {
    const int pb = P[b] + a.seg_cost, pe = P[b + 1];  // b's real tokens: [pb, pe)
    if (pe <= lo) continue;
    const int seg_hi = min(hi, pe);
    const int seg_lo = max(lo, pb);
    lo = seg_hi;
    if (seg_lo >= seg_hi) continue;  // only b's virtual tokens fall in this chunk
    int pos;
    const int L = seq_len(a, b, pos);
    const int t0 = seg_lo - pb, t1 = min(seg_hi - pb, L);
    const int ap = min(pos, L - 1);
    const bool append = pos >= 0 && pos < a.span && ap >= t0 && ap < t1;
    decode_segment<D, KV, Q_BF16, NT, LA>(a, dsm, b, h, t0, t1, append, seg_lo == pb && seg_hi == pe,
                                      ((int64_t)h * (a.nchunk + a.B) + c + b) * a.G);
  }
}

// Weighted sum of `nsplit` partials (index (base + s) * G + g) of sequence b,
// KV head h into the output, for the query heads [g0, g0 + gn) of this CTA.
// Thread = (query head, 4 dims). Each thread loads the log-sum-exps and its
// 4 output values of 8 partials at once, so a batch costs one L2 round trip,
// and keeps a running maximum across batches (the merge is latency-bound: a
// sequence split over 19 chunks took six dependent round trips with the
// weights computed first). The sink, when given, starts the sum.
template <int D, bool Q_BF16>
__device__ __forceinline__ void merge_partials(const DecodeArgs& a, int b, int h, int64_t base, int nsplit, int g0,
                                               int gn) {
  constexpr int kBatch = 8;
  const int64_t ps = (int64_t)a.G * D;  // floats from one partial slot to the next
  for (int idx = threadIdx.x; idx < gn * (D / 4); idx += kThreads) {
    const int g = g0 + idx / (D / 4), d4 = (idx % (D / 4)) * 4;
    const float* pl = a.part_lse + base * a.G + g;
    const float* po = a.part_o + (base * a.G + g) * D + d4;
    float M = sink_log2(a, h, g);
    float S = (M == neg_inf()) ? 0.f : 1.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < nsplit; s0 += kBatch) {
      float l[kBatch];
      float4 o[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const bool in = s0 + u < nsplit;
        l[u] = in ? pl[(int64_t)(s0 + u) * a.G] : neg_inf();
        o[u] = in ? *reinterpret_cast<const float4*>(po + (s0 + u) * ps) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float mb = M;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) mb = fmaxf(mb, l[u]);
      if (mb != M) {  // M == -inf: S and acc are still 0
        const float c = (M == neg_inf()) ? 0.f : exp2_approx(M - mb);
        S *= c;
        acc.x *= c; acc.y *= c; acc.z *= c; acc.w *= c;
        M = mb;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (l[u] != neg_inf()) {  // a partial with nothing visible carries no weight
          const float w = exp2_approx(l[u] - M);
          S += w;
          acc.x += w * o[u].x; acc.y += w * o[u].y; acc.z += w * o[u].z; acc.w += w * o[u].w;
        }
      }
    }
    // every position masked and no sink: NaN, as softmax of all -inf
    const float inv = (M == neg_inf()) ? pos_nan() : 1.f / S;
    acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
    store_out(a, b, h, g, d4, make_uint2(pack2<Q_BF16>(acc.x, acc.y), pack2<Q_BF16>(acc.z, acc.w)));
  }
  // the per-sequence merge kernel's peer stores are ordered before the epoch
  // exchange by its kernel boundary; the balanced merge kernel orders them
  // through its arrival chain
}

// The merge kernels are programmatic dependents of the decode kernel: they
// wait for it at their start, and let the next launch on the stream be
// scheduled only at the end of their work. Measured on B200: signalling at
// the start let the next decode grid's CTAs wait resident beside a small
// merge grid (32 CTAs of 18 us for 32 sequences x 1 KV head) and slowed the
// call from 101 us to 141 us.
__device__ __forceinline__ void merge_done() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Combines the per-split partials of one (sequence, KV head) of the
// per-sequence split kernel; blockIdx.z takes a slice of the query heads.
template <int D, bool Q_BF16>
__global__ void __launch_bounds__(kThreads) paged_decode_merge_kernel(const DecodeArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int h = blockIdx.x, b = blockIdx.y;
  const int gn = a.G / (int)gridDim.z, g0 = (int)blockIdx.z * gn;
  int pos, L, nsplit;
  decode_extent(a, b, pos, L, nsplit);
  if (nsplit <= 1) return;
  merge_partials<D, Q_BF16>(a, b, h, (int64_t)(b * a.Hkv + h) * a.max_splits, nsplit, g0, gn);
  merge_done();
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Epoch exchange after a head-sharded decode, run by one warp whose stores
// (and all stores it has observed) are done: lane t announces to rank t that
// this rank's outputs are in (release at system scope), then waits until
// rank t has announced this epoch to this rank (acquire). A wait gives up
// after limit_ns of GPU time with RBLN_DEVERR_TIMEOUT.
__device__ __forceinline__ void peer_epoch_exchange(uint32_t* const* flags, int n, int rank, uint32_t epoch,
                                                    uint64_t limit_ns, uint32_t* err) {
  const int t = threadIdx.x & 31;
  if (t >= n) return;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags[t] + rank), "r"(epoch) : "memory");
  const uint32_t* mine = flags[rank] + t;
  const uint64_t t0 = global_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if ((int32_t)(v - epoch) >= 0) break;  // a rank may already be one epoch ahead
    if (global_ns() - t0 > limit_ns) {
      flag_error(err, RBLN_DEVERR_TIMEOUT);
      break;
    }
  }
}

// Merge of the balanced kernel's partials for one (KV head, sequence). Also
// finishes the sequences that no chunk covers (no visible position: the new
// token is still appended and the output is NaN, as softmax of all -inf).
// On the head-sharded path the last merge CTA to finish runs the epoch
// exchange, so the call needs no separate barrier launch.
template <int D, int KV, bool Q_BF16>
__global__ void __launch_bounds__(kThreads) paged_decode_merge_balanced_kernel(const DecodeArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int h = blockIdx.x, b = blockIdx.y;
  const int gn = a.G / (int)gridDim.z, g0 = (int)blockIdx.z * gn;  // this CTA's query heads
  // the chunk size and the sequence's padded range, loaded together with
  // its length (one round trip instead of two)
  const int W = a.prefix[a.B + 1], pb = a.prefix[b], pe = a.prefix[b + 1];
  int pos;
  const int L = seq_len(a, b, pos);
  if (pos < 0 && h == 0 && blockIdx.z == 0 && threadIdx.x == 0) flag_error(a.err, RBLN_DEVERR_SEQ_RANGE);
  if (L == 0) {
    if (a.k_new != nullptr && pos >= 0 && pos < a.span && blockIdx.z == 0) append_token<D, KV, Q_BF16>(a, b, h, pos);
    for (int idx = threadIdx.x; idx < gn * (D / 4); idx += kThreads) {
      const int g = g0 + idx / (D / 4), d4 = (idx % (D / 4)) * 4;
      const float n = a.sinks ? 0.f : pos_nan();  // all softmax mass on the sink
      store_out(a, b, h, g, d4, make_uint2(pack2<Q_BF16>(n, n), pack2<Q_BF16>(n, n)));
    }
  } else {
    const int cf = (pb + a.seg_cost) / W, cl = (pe - 1) / W;
    // cf == cl: one chunk held the whole sequence and wrote the output
    if (cf != cl) {
      merge_partials<D, Q_BF16>(a, b, h, (int64_t)h * (a.nchunk + a.B) + cf + b, cl - cf + 1, g0, gn);
    }
  }
  merge_done();
  if (a.peer_flags == nullptr) return;
  // Ordering of the peer stores before the epoch release: the CTA's stores
  // reach thread 0 through the barrier, its GPU-scope fence orders them
  // before its arrival, the last CTA's fence after its own arrival orders
  // every CTA's stores before the exchange, and the exchange's system-scope
  // release is cumulative over all of them (the decode kernel's stores are
  // ordered before this grid by the dependent launch's wait). One system-
  // scope release per flag instead of a system fence per thread: 10 us less
  // per call on B200.
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(a.merge_ctr, 1) == (int)(gridDim.x * gridDim.y * gridDim.z) - 1;
    __threadfence();
  }
  __syncthreads();
  if (last && threadIdx.x < 32)
    peer_epoch_exchange(a.peer_flags, a.n_peers, a.peer_rank, a.epoch, a.wait_ns, a.err);
}

// The epoch exchange as a kernel of its own (one warp), after the
// per-sequence split grid's kernels.
__global__ void __launch_bounds__(32) peer_epoch_barrier_kernel(uint32_t* const* flags, int n, int rank,
                                                                uint32_t epoch, uint64_t limit_ns, uint32_t* err) {
  peer_epoch_exchange(flags, n, rank, epoch, limit_ns, err);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int dtype_bytes(int dt) {
  switch (dt) {
    case RBLN_DT_F32: case RBLN_DT_I32: return 4;
    case RBLN_DT_F16: case RBLN_DT_BF16: case RBLN_DT_I16: return 2;
    case RBLN_DT_I64: return 8;
    default: return 1;
  }
}

int choose_chunk(const rbln_paged_attn_params_t* p, int span) {
  static const int env_chunk = [] {
    const char* e = std::getenv("RBLN_ATTN_DECODE_CHUNK");
    return e ? std::atoi(e) : 0;
  }();
  if (p->num_splits <= 0 && env_chunk >= 64) return std::min(std::max(64, env_chunk / 64 * 64), std::max(span, 64));
  if (p->num_splits > 0) {
    int c = (span + p->num_splits - 1) / p->num_splits;
    return std::max(64, (c + 63) / 64 * 64);
  }
  // About 24 CTAs per SM if every sequence used the whole span, with splits
  // of 256..2048 tokens: short splits pay the per-CTA start-up and the merge,
  // long ones leave a tail of unequal CTAs (measured on B200 over 256..8192).
  const int64_t target_ctas = 148LL * 24;
  int64_t c = ((int64_t)span * p->batch * p->num_kv_heads + target_ctas - 1) / target_ctas;
  c = (c + 63) / 64 * 64;
  c = std::min<int64_t>(std::max<int64_t>(c, 256), 2048);
  c = std::min<int64_t>(c, std::max(span, 64));
  return (int)((c + 63) / 64 * 64);
}

struct Plan {
  int span, chunk, max_splits;
  bool balanced;
  int nchunk, min_w, seg_cost;
  size_t ws_bytes;
};

// Settings read once from the environment (timing sweeps):
//   RBLN_ATTN_DECODE_SCHED=seq      per-sequence splits instead of balanced
//   RBLN_ATTN_DECODE_WAVES=n        balanced: chunks per KV head fill n waves
//   RBLN_ATTN_DECODE_MINW=t         balanced: smallest chunk in tokens
//   RBLN_ATTN_DECODE_SEGCOST=t      balanced: virtual tokens charged per sequence
//   RBLN_ATTN_DECODE_LOOKAHEAD=0    fp8 caches: no block-table lookahead
struct DecodeEnv {
  bool force_seq = false;
  int lookahead = 1;
  int waves = 0, min_w = 0, seg_cost = -1;
  DecodeEnv() {
    if (const char* e = std::getenv("RBLN_ATTN_DECODE_LOOKAHEAD")) lookahead = std::atoi(e);
    if (const char* e = std::getenv("RBLN_ATTN_DECODE_SCHED")) force_seq = std::string(e) == "seq";
    if (const char* e = std::getenv("RBLN_ATTN_DECODE_WAVES")) waves = std::atoi(e);
    if (const char* e = std::getenv("RBLN_ATTN_DECODE_MINW")) min_w = std::atoi(e);
    if (const char* e = std::getenv("RBLN_ATTN_DECODE_SEGCOST")) seg_cost = std::atoi(e);
  }
};
const DecodeEnv& decode_env() {
  static const DecodeEnv env;
  return env;
}

constexpr int kBalancedMaxBatch = 2048;

// Balanced workspace head: the padded-length prefix [B + 1], the chunk size
// W and the merge kernel's arrival counter, rounded up to 256 bytes.
size_t prefix_bytes(int batch) { return ((size_t)(batch + 3) * sizeof(int) + 255) / 256 * 256; }

int plan_decode(const rbln_paged_attn_params_t* p, Plan* pl) {
  if (!p || p->batch < 0 || p->num_kv_heads <= 0 || p->group <= 0 || p->block_size <= 0 ||
      p->max_blocks <= 0 || p->num_blocks <= 0)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->head_dim != 64 && p->head_dim != 128) return RBLN_ERR_UNSUPPORTED;
  if (p->group > 16) return RBLN_ERR_UNSUPPORTED;
  const int64_t span64 = (int64_t)p->max_blocks * p->block_size;
  if (span64 > (1 << 30)) return RBLN_ERR_UNSUPPORTED;
  pl->span = (int)span64;
  pl->chunk = choose_chunk(p, pl->span);
  pl->max_splits = (pl->span + pl->chunk - 1) / pl->chunk;
  if (pl->max_splits > 2048) return RBLN_ERR_UNSUPPORTED;
  const DecodeEnv& env = decode_env();
  // Balanced chunks unless the caller fixed the number of splits per sequence
  // (num_splits > 0), the batch is too large for the in-CTA prefix, or the
  // padded token total could overflow int32.
  // 128 virtual tokens per sequence start measured best on B200 (0 to 512
  // swept): 94.9 against 98.6 us per call at B=64, L~U[128,4096]; 87.7
  // against 89.5 us at 32 x 32768 tokens on one KV head; 425.7 against 430 us
  // for the B=256 fp8 workload
  const int seg_cost = env.seg_cost >= 0 ? std::min(env.seg_cost, 4096) / 16 * 16 : 128;
  const int64_t padded_total = (int64_t)p->batch * ((span64 + 15) / 16 * 16 + seg_cost);
  pl->balanced = p->num_splits <= 0 && !env.force_seq && p->batch >= 1 && p->batch <= kBalancedMaxBatch &&
                 padded_total < (int64_t(1) << 30);
  pl->nchunk = 0;
  pl->min_w = 0;
  pl->seg_cost = 0;
  pl->ws_bytes = 0;
  if (pl->balanced) {
    // enough chunks per KV head to fill `waves` waves of resident CTAs (4 per
    // SM for up to 8 query heads per KV head, 2 above), each of at least
    // min_w tokens. One wave measured best on B200 (1..4 swept on the ragged
    // B=64 bf16 and B=256 fp8 workloads and on 32 x 32768 tokens).
    const int waves = env.waves > 0 ? env.waves : 1;
    const int per_sm = p->group <= 8 ? 4 : 2;
    // rounded down: a CTA past the resident slots would run as a second
    // wave of its own, a whole chunk long
    pl->nchunk = std::max(1, 148 * per_sm * waves / p->num_kv_heads);
    pl->min_w = env.min_w >= 16 ? env.min_w / 16 * 16 : 256;
    pl->seg_cost = seg_cost;
    const size_t slots = (size_t)p->num_kv_heads * (pl->nchunk + p->batch) * p->group;
    pl->ws_bytes = prefix_bytes(p->batch) + slots * p->head_dim * sizeof(float) +
                   slots * sizeof(float) + 256;
  } else if (pl->max_splits > 1) {
    const size_t slots = (size_t)p->batch * p->num_kv_heads * pl->max_splits * p->group;
    pl->ws_bytes = slots * p->head_dim * sizeof(float) + slots * sizeof(float) + 256;
  }
  return RBLN_OK;
}

// Largest dynamic shared-memory size one kernel has been opted into, per
// device (one instance per kernel instantiation).
struct SmemOptIn {
  std::atomic<int> bytes[kMaxDevices] = {};
};

// Opts `kernel` into `bytes` of dynamic shared memory when that is above
// 48 KB and above what it was opted into before on this device.
bool allow_smem(const void* kernel, int bytes, SmemOptIn& opt) {
  if (bytes <= 48 * 1024) return true;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
  if (opt.bytes[dev].load(std::memory_order_relaxed) >= bytes) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  int cur = opt.bytes[dev].load(std::memory_order_relaxed);
  while (cur < bytes && !opt.bytes[dev].compare_exchange_weak(cur, bytes)) {
  }
  return true;
}

// Launches `kernel` as a programmatic dependent of the previous launch on
// `st`: its CTAs may be scheduled while that grid drains (once all of that
// grid's CTAs have signalled launch_dependents) and wait in-kernel
// (pdl_enter) for its completion.
int launch_dependent(void (*kernel)(DecodeArgs), dim3 grid, size_t smem, cudaStream_t st, const DecodeArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a) == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

// Slices of the query heads per merge CTA: (KV head, sequence) pairs are
// split over heads (halving while G allows) until the merge grid has about
// two CTAs per SM. At 32 sequences x 1 KV head (a long-context decode
// sharded over 8 GPUs) that is 8 CTAs per pair; at 64 x 8 pairs, none.
int merge_head_split(int Hkv, int B, int G) {
  int gz = 1;
  while (G % (2 * gz) == 0 && (int64_t)Hkv * B * gz < 2 * 148) gz *= 2;
  return gz;
}

template <int D, int KV, bool QB, int NT, bool LA>
int launch_typed(const DecodeArgs& a, const Plan& pl, cudaStream_t st, void* const* ev) {
  const int gz = merge_head_split(a.Hkv, a.B, a.G);
  if (ev && ev[0]) cudaEventRecord(static_cast<cudaEvent_t>(ev[0]), st);
  if (pl.balanced) {
    const size_t smem = segment_smem<D, NT>() + (size_t)(a.B + 1) * sizeof(int);
    static SmemOptIn done;
    if (!allow_smem(reinterpret_cast<const void*>(paged_decode_balanced_kernel<D, KV, QB, NT, LA>), (int)smem, done))
      return RBLN_ERR_LAUNCH;
    const int drc =
        launch_dependent(paged_decode_balanced_kernel<D, KV, QB, NT, LA>, dim3(pl.nchunk, a.Hkv), smem, st, a);
    if (drc != RBLN_OK) return drc;
    if (ev && ev[1]) cudaEventRecord(static_cast<cudaEvent_t>(ev[1]), st);
    const int rc = launch_dependent(paged_decode_merge_balanced_kernel<D, KV, QB>, dim3(a.Hkv, a.B, gz), 0, st, a);
    if (rc != RBLN_OK) return rc;
    return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
  }
  static SmemOptIn sdone;
  if (!allow_smem(reinterpret_cast<const void*>(paged_decode_split_kernel<D, KV, QB, NT, LA>), segment_smem<D, NT>(),
                  sdone))
    return RBLN_ERR_LAUNCH;
  const int drc = launch_dependent(paged_decode_split_kernel<D, KV, QB, NT, LA>, dim3(pl.max_splits, a.Hkv, a.B),
                                   segment_smem<D, NT>(), st, a);
  if (drc != RBLN_OK) return drc;
  if (ev && ev[1]) cudaEventRecord(static_cast<cudaEvent_t>(ev[1]), st);
  if (pl.max_splits > 1) {
    const int rc = launch_dependent(paged_decode_merge_kernel<D, QB>, dim3(a.Hkv, a.B, gz), 0, st, a);
    if (rc != RBLN_OK) return rc;
  }
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

template <int D, int KV, bool QB>
int launch_nt(const DecodeArgs& a, const Plan& pl, cudaStream_t st, void* const* ev) {
  // Lookahead only where it fits the 128-register budget of 4 CTAs per SM
  // and measured faster on B200: fp8 caches with up to 8 query heads per KV
  // head (bf16/f16 tiles hold twice the registers and would spill).
  if (a.G > 8) return launch_typed<D, KV, QB, 2, false>(a, pl, st, ev);
  if constexpr (KV == KV_FP8) {
    if (decode_env().lookahead != 0) return launch_typed<D, KV, QB, 1, true>(a, pl, st, ev);
  }
  return launch_typed<D, KV, QB, 1, false>(a, pl, st, ev);
}

template <int D>
int launch_d(const DecodeArgs& a, const Plan& pl, int kv_dt, int q_dt, cudaStream_t st, void* const* ev) {
  if (kv_dt == RBLN_DT_BF16 && q_dt == RBLN_DT_BF16) return launch_nt<D, KV_BF16, true>(a, pl, st, ev);
  if (kv_dt == RBLN_DT_F16 && q_dt == RBLN_DT_F16) return launch_nt<D, KV_F16, false>(a, pl, st, ev);
  if (kv_dt == RBLN_DT_FP8_E4M3 && q_dt == RBLN_DT_BF16) return launch_nt<D, KV_FP8, true>(a, pl, st, ev);
  if (kv_dt == RBLN_DT_FP8_E4M3 && q_dt == RBLN_DT_F16) return launch_nt<D, KV_FP8, false>(a, pl, st, ev);
  return RBLN_ERR_UNSUPPORTED;
}

int run_decode(const rbln_paged_attn_params_t* p, cudaStream_t st, bool require_mask,
               const rbln_peer_out_t* peers = nullptr) {
  Plan pl;
  int rc = plan_decode(p, &pl);
  if (rc != RBLN_OK) return rc;
  if (require_mask && !p->mask) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->batch == 0) return RBLN_OK;
  if (!p->q || !p->out || !p->kcache || !p->vcache || !p->seq || !p->block_table)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->q_len != 1) return RBLN_ERR_INVALID_ARGUMENT;
  if ((p->k_new == nullptr) != (p->v_new == nullptr)) return RBLN_ERR_INVALID_ARGUMENT;
  const int kv_sz = dtype_bytes(p->kv_dtype);
  const int q_sz = dtype_bytes(p->q_dtype);
  if (q_sz != 2) return RBLN_ERR_UNSUPPORTED;
  if (p->kv_dtype == RBLN_DT_FP8_E4M3 && (!p->k_scale || !p->v_scale)) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->block_table_dtype != RBLN_DT_I16 && p->block_table_dtype != RBLN_DT_I32 &&
      p->block_table_dtype != RBLN_DT_I64)
    return RBLN_ERR_UNSUPPORTED;
  // 16-byte rows everywhere
  for (int i = 0; i < 3; ++i)
    if ((p->cache_stride[i] * kv_sz) % 16 != 0) return RBLN_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < 3; ++i)
    if ((p->q_stride[i] * q_sz) % 16 != 0 || (p->out_stride[i] * q_sz) % 8 != 0)
      return RBLN_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->q) || !aligned16(p->kcache) || !aligned16(p->vcache) ||
      (reinterpret_cast<uintptr_t>(p->out) & 7u) != 0)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->k_new) {
    if (!aligned16(p->k_new) || !aligned16(p->v_new)) return RBLN_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 2; ++i)
      if ((p->k_new_stride[i] * q_sz) % 16 != 0 || (p->v_new_stride[i] * q_sz) % 16 != 0)
        return RBLN_ERR_INVALID_ARGUMENT;
  }
  const int64_t cache_bytes_hint = ((int64_t)p->num_blocks * p->cache_stride[0]) * kv_sz;
  if (cache_bytes_hint / 16 > (int64_t)UINT32_MAX) return RBLN_ERR_UNSUPPORTED;
  if (pl.ws_bytes > 0 && (!p->workspace || p->workspace_bytes < pl.ws_bytes)) return RBLN_ERR_WORKSPACE;

  DecodeArgs a{};
  a.q = static_cast<const char*>(p->q);
  a.qs_b = p->q_stride[0] * q_sz; a.qs_h = p->q_stride[1] * q_sz; a.qs_g = p->q_stride[2] * q_sz;
  a.out = static_cast<char*>(p->out);
  a.os_b = p->out_stride[0] * q_sz; a.os_h = p->out_stride[1] * q_sz; a.os_g = p->out_stride[2] * q_sz;
  a.k_new = static_cast<const char*>(p->k_new);
  a.v_new = static_cast<const char*>(p->v_new);
  a.kn_b = p->k_new_stride[0] * q_sz; a.kn_h = p->k_new_stride[1] * q_sz;
  a.vn_b = p->v_new_stride[0] * q_sz; a.vn_h = p->v_new_stride[1] * q_sz;
  a.kcache = static_cast<char*>(p->kcache);
  a.vcache = static_cast<char*>(p->vcache);
  a.cs_block = p->cache_stride[0]; a.cs_head = p->cache_stride[1]; a.cs_tok = p->cache_stride[2];
  a.k_scale = p->k_scale; a.v_scale = p->v_scale;
  a.ss_block = p->scale_stride[0]; a.ss_head = p->scale_stride[1];
  a.seq = p->seq; a.seq_stride = p->seq_stride;
  a.bt = p->block_table; a.bt_dtype = p->block_table_dtype; a.bt_stride = p->block_table_stride;
  a.mask = p->mask; a.mask_dtype = p->mask_dtype; a.mask_len = p->mask_len; a.mask_stride = p->mask_stride[0];
  a.scale = p->scale; a.scale_dev = p->scale_dev;
  a.B = p->batch; a.Hkv = p->num_kv_heads; a.G = p->group; a.num_blocks = p->num_blocks;
  a.bs = p->block_size; a.span = pl.span; a.chunk = pl.chunk; a.max_splits = pl.max_splits;
  a.nchunk = pl.nchunk;
  a.min_w = pl.min_w;
  a.seg_cost = pl.seg_cost;
  if (pl.balanced) {
    uintptr_t w = (reinterpret_cast<uintptr_t>(p->workspace) + 255) & ~uintptr_t(255);
    a.prefix = reinterpret_cast<int*>(w);
    w += prefix_bytes(p->batch);
    const size_t slots = (size_t)p->num_kv_heads * (pl.nchunk + p->batch) * p->group;
    a.part_o = reinterpret_cast<float*>(w);
    a.part_lse = a.part_o + slots * p->head_dim;
  } else if (pl.max_splits > 1) {
    uintptr_t w = (reinterpret_cast<uintptr_t>(p->workspace) + 255) & ~uintptr_t(255);
    const size_t slots = (size_t)p->batch * p->num_kv_heads * pl.max_splits * p->group;
    a.part_o = reinterpret_cast<float*>(w);
    a.part_lse = a.part_o + slots * p->head_dim;
  }
  a.err = p->error_flags;
  a.sinks = p->sinks;
  uint64_t wait_ns = 0;
  if (peers) {
    // the error word is where a timed-out exchange is reported: required
    if (peers->n < 1 || peers->n > 32 || peers->rank < 0 || peers->rank >= peers->n || peers->head0 < 0 ||
        !peers->out || !peers->flags || !p->error_flags)
      return RBLN_ERR_INVALID_ARGUMENT;
    a.out_peers = reinterpret_cast<char* const*>(peers->out);
    a.n_peers = peers->n;
    a.head0 = peers->head0;
    wait_ns = (uint64_t)(peers->wait_limit_us ? peers->wait_limit_us : 2000000u) * 1000u;
    if (pl.balanced) {  // the merge kernel's last CTA runs the exchange
      a.peer_flags = peers->flags;
      a.peer_rank = peers->rank;
      a.epoch = peers->epoch;
      a.wait_ns = wait_ns;
      a.merge_ctr = a.prefix + p->batch + 2;
    }
  }
  const int lrc = p->head_dim == 128 ? launch_d<128>(a, pl, p->kv_dtype, p->q_dtype, st, p->prof_events)
                                     : launch_d<64>(a, pl, p->kv_dtype, p->q_dtype, st, p->prof_events);
  if (lrc != RBLN_OK || !peers || pl.balanced) return lrc;
  peer_epoch_barrier_kernel<<<1, 32, 0, st>>>(peers->flags, peers->n, peers->rank, peers->epoch, wait_ns,
                                              p->error_flags);
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

}  // namespace
}  // namespace rbln

extern "C" {

int rbln_attn_abi_version(void) { return RBLN_ATTN_ABI_VERSION; }

size_t rbln_paged_attn_params_sizeof(void) { return sizeof(rbln_paged_attn_params_t); }

size_t rbln_peer_out_sizeof(void) { return sizeof(rbln_peer_out_t); }

int rbln_paged_decode_workspace_size(const rbln_paged_attn_params_t* p, size_t* bytes) {
  if (!bytes) return RBLN_ERR_INVALID_ARGUMENT;
  rbln::Plan pl;
  const int rc = rbln::plan_decode(p, &pl);
  if (rc != RBLN_OK) return rc;
  *bytes = pl.ws_bytes;
  return RBLN_OK;
}

int rbln_paged_causal_attn_decode(const rbln_paged_attn_params_t* p, cudaStream_t stream) {
  return rbln::run_decode(p, stream, /*require_mask=*/false);
}

int rbln_paged_attn_decode(const rbln_paged_attn_params_t* p, cudaStream_t stream) {
  return rbln::run_decode(p, stream, /*require_mask=*/true);
}

int rbln_paged_causal_attn_decode_peers(const rbln_paged_attn_params_t* p, const rbln_peer_out_t* peers,
                                        cudaStream_t stream) {
  if (!peers) return RBLN_ERR_INVALID_ARGUMENT;
  return rbln::run_decode(p, stream, /*require_mask=*/false, peers);
}

int rbln_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return RBLN_ERR_INVALID_ARGUMENT;
  void* d = nullptr;
  if (cudaMalloc(&d, bytes) != cudaSuccess) return RBLN_ERR_LAUNCH;
  cudaIpcMemHandle_t h;
  if (cudaMemset(d, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, d) != cudaSuccess) {
    cudaFree(d);
    return RBLN_ERR_LAUNCH;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == RBLN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = d;
  return RBLN_OK;
}

int rbln_ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH; }

int rbln_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return RBLN_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

int rbln_ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH; }

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu[kNoallocMaxDevices];
std::atomic<void*> g_noalloc_addr[kNoallocMaxDevices];

// Device address of the fixed scratch on the current device, looked up with
// that device current. Only a successful lookup is kept: a failed one (for
// example a first call made while a stream is being captured) is tried
// again on the next call.
int noalloc_scratch(void** addr) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) return RBLN_ERR_NO_DEVICE;
  void* a = g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (a == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu[dev]);
    a = g_noalloc_addr[dev].load(std::memory_order_relaxed);
    if (a == nullptr) {
      void* found = nullptr;
      if (cudaGetSymbolAddress(&found, rbln_noalloc_scratch) != cudaSuccess || found == nullptr) {
        cudaGetLastError();  // the failed lookup leaves no sticky error behind
        return RBLN_ERR_LAUNCH;
      }
      g_noalloc_addr[dev].store(found, std::memory_order_release);
      a = found;
    }
  }
  *addr = a;
  return RBLN_OK;
}
}  // namespace

int rbln_paged_causal_attn_decode_noalloc(const rbln_paged_attn_params_t* p, cudaStream_t stream) {
  if (!p) return RBLN_ERR_INVALID_ARGUMENT;
  rbln::Plan pl;
  int rc = rbln::plan_decode(p, &pl);
  if (rc != RBLN_OK) return rc;
  if (pl.ws_bytes > RBLN_NOALLOC_SCRATCH_BYTES) return RBLN_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != RBLN_OK) return rc;
  rbln_paged_attn_params_t q = *p;
  q.workspace = scratch;
  q.workspace_bytes = RBLN_NOALLOC_SCRATCH_BYTES;
  return rbln::run_decode(&q, stream, /*require_mask=*/false);
}

}  // extern "C"
