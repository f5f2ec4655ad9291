// Scaled dot-product attention forward (aten::_scaled_dot_product_fused_
// attention_overrideable on CUDA), reference semantics from
// torch_rbln/_internal/kernels/sdpa.py:244-289 (_sdpa_cpu_fallback): GQA by
// head ratio (query head h reads KV head h / (Hq / Hkv)), optional bool
// keep-mask or additive float mask, top-left causal mask.
//
// bf16 / f16 run on the tcgen05 flash-attention kernel (attn_prefill.cu).
// f32 runs on an exact-fp32 SIMT flash kernel: the tensor cores have no fp32
// mode that meets a 1e-5 relative bound, and the f32 shapes this path serves
// (1x32x512x64, ~1 GFLOP) are latency-sized.

#include "common.cuh"

namespace rbln {
int attn_tc_dense(const void* q, const int64_t* qs, void* out, const int64_t* os, float* lse, const int64_t* ls,
                  const void* k, const void* v, const int64_t* ks, const int64_t* vs, int dtype, int B, int Hkv,
                  int G, int L, int S, int D, int causal, const void* mask, int mask_dtype, int mask_additive,
                  const int64_t* ms, float scale, uint32_t* err, cudaStream_t st);

namespace {

constexpr int FQ = 64;   // query rows per CTA
constexpr int FK = 64;   // keys per tile
constexpr int FT = 256;  // threads (16 x 16)

struct F32Args {
  const float* q;
  int64_t qs_b, qs_h, qs_l;
  const float* k;
  int64_t ks_b, ks_h, ks_l;
  const float* v;
  int64_t vs_b, vs_h, vs_l;
  float* out;
  int64_t os_b, os_h, os_l;
  float* lse;
  int64_t ls_b, ls_h, ls_l;
  const void* mask;
  int mask_dtype, mask_additive;
  int64_t m_b, m_h, m_l, m_s;
  int B, Hq, Hkv, L, S, causal;
  float scale;
};

__device__ __forceinline__ float f32_mask(const void* base, int dt, int64_t i) {
  switch (dt) {
    case RBLN_DT_F32: return static_cast<const float*>(base)[i];
    case RBLN_DT_F16: return __half2float(static_cast<const __half*>(base)[i]);
    case RBLN_DT_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
    default: return static_cast<const uint8_t*>(base)[i] ? 1.f : 0.f;
  }
}

// Thread (ty, tx) owns query rows 4ty..4ty+3; for scores the keys
// tx + 16j (j < 4) of the tile, for the output the head-dim columns
// 4tx + 64c .. 4tx + 64c + 3 (c < D / 64). Shared-memory rows are padded to
// D + 4 floats: 16-byte aligned, so every operand is read as a float4 (one
// load per 8 FMAs; scalar reads made the kernel load-bound at one per two),
// and rows tx + 16j of consecutive tx start 4 banks apart, so the K reads
// of a warp are conflict-free. Every dot product and every output column
// accumulates in the same order as a scalar loop over d or over the keys.
template <int D>
__global__ void __launch_bounds__(FT) sdpa_f32_kernel(const F32Args a) {
  constexpr int DP = D + 4;
  constexpr int PP = FK + 4;
  constexpr int DC = D / 64;  // float4 output columns per thread
  extern __shared__ __align__(16) float fsm[];
  float* Qs = fsm;           // [FQ][DP]
  float* Ks = Qs + FQ * DP;  // [FK][DP]
  float* Vs = Ks + FK * DP;  // [FK][DP]
  float* Ps = Vs + FK * DP;  // [FQ][PP]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  // grid (head, query tile, batch), query tiles in reverse: CTAs are
  // dispatched head-fastest, so every head's longest causal tiles start first
  const int qb = (int)gridDim.y - 1 - (int)blockIdx.y, hq = blockIdx.x, b = blockIdx.z;
  const int hk = hq / (a.Hq / a.Hkv);
  const int l0 = qb * FQ;

  for (int idx = tid; idx < FQ * D; idx += FT) {
    const int r = idx / D, d = idx % D;
    const int l = l0 + r;
    Qs[r * DP + d] = (l < a.L) ? a.q[b * a.qs_b + hq * a.qs_h + (int64_t)l * a.qs_l + d] : 0.f;
  }
  float m_run[4], l_run[4];
  float4 o[4][DC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = neg_inf();
    l_run[i] = 0.f;
#pragma unroll
    for (int c = 0; c < DC; ++c) o[i][c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int kend = a.S;
  if (a.causal) kend = min(kend, l0 + FQ);
  const int ntiles = (kend + FK - 1) / FK;

  for (int t = 0; t < ntiles; ++t) {
    const int k0 = t * FK;
    __syncthreads();
    for (int idx = tid; idx < FK * D; idx += FT) {
      const int r = idx / D, d = idx % D;
      const int kk = k0 + r;
      const bool in = kk < a.S;
      Ks[r * DP + d] = in ? a.k[b * a.ks_b + hk * a.ks_h + (int64_t)kk * a.ks_l + d] : 0.f;
      Vs[r * DP + d] = in ? a.v[b * a.vs_b + hk * a.vs_h + (int64_t)kk * a.vs_l + d] : 0.f;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; d += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(&Qs[(4 * ty + i) * DP + d]);
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(&Ks[(tx + 16 * j) * DP + d]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
          s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
          s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
          s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int l = l0 + 4 * ty + i;
      float mx = neg_inf();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kk = k0 + tx + 16 * j;
        bool keep = (l < a.L) && (kk < a.S) && (!a.causal || kk <= l);
        float x = s[i][j] * a.scale;
        if (keep && a.mask) {
          const float mv = f32_mask(a.mask, a.mask_dtype, b * a.m_b + hq * a.m_h + (int64_t)l * a.m_l + kk * a.m_s);
          if (a.mask_additive) x += mv;
          else keep = mv > 0.f;
        }
        s[i][j] = keep ? x : neg_inf();
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m_run[i], mx);
      const float mu = (mn == neg_inf()) ? 0.f : mn;
      const float alpha = expf(m_run[i] - mu);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - mu);
        Ps[(4 * ty + i) * PP + tx + 16 * j] = p;
        sum += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      l_run[i] = l_run[i] * alpha + sum;
      m_run[i] = mn;
#pragma unroll
      for (int c = 0; c < DC; ++c) {
        o[i][c].x *= alpha; o[i][c].y *= alpha; o[i][c].z *= alpha; o[i][c].w *= alpha;
      }
    }
    __syncthreads();
#pragma unroll 2
    for (int kk = 0; kk < FK; kk += 4) {
      float4 pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4*>(&Ps[(4 * ty + i) * PP + kk]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int c = 0; c < DC; ++c) {
          const float4 vv = *reinterpret_cast<const float4*>(&Vs[(kk + u) * DP + 4 * tx + 64 * c]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float pw = u == 0 ? pv[i].x : u == 1 ? pv[i].y : u == 2 ? pv[i].z : pv[i].w;
            o[i][c].x = fmaf(pw, vv.x, o[i][c].x);
            o[i][c].y = fmaf(pw, vv.y, o[i][c].y);
            o[i][c].z = fmaf(pw, vv.z, o[i][c].z);
            o[i][c].w = fmaf(pw, vv.w, o[i][c].w);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + 4 * ty + i;
    if (l >= a.L) continue;
    const float inv = 1.f / l_run[i];
    float* orow = a.out + b * a.os_b + hq * a.os_h + (int64_t)l * a.os_l;
#pragma unroll
    for (int c = 0; c < DC; ++c) {
      const int d = 4 * tx + 64 * c;
      orow[d] = o[i][c].x * inv;
      orow[d + 1] = o[i][c].y * inv;
      orow[d + 2] = o[i][c].z * inv;
      orow[d + 3] = o[i][c].w * inv;
    }
    if (a.lse && tx == 0)
      a.lse[b * a.ls_b + hq * a.ls_h + (int64_t)l * a.ls_l] =
          (m_run[i] == neg_inf()) ? neg_inf() : m_run[i] + logf(l_run[i]);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int D>
int launch_f32(const F32Args& a, int L, int H, int B, cudaStream_t stream) {
  const size_t sm = (size_t)(3 * 64 * (D + 4) + 64 * (FK + 4)) * sizeof(float);
  if (cudaFuncSetAttribute(sdpa_f32_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
    return RBLN_ERR_LAUNCH;
  if ((L + FQ - 1) / FQ > 65535) return RBLN_ERR_UNSUPPORTED;
  dim3 grid(H, (L + FQ - 1) / FQ, B);
  sdpa_f32_kernel<D><<<grid, FT, sm, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? RBLN_OK : RBLN_ERR_LAUNCH;
}

}  // namespace
}  // namespace rbln

extern "C" int rbln_sdpa_fwd(const rbln_sdpa_params_t* p, cudaStream_t stream) {
  using namespace rbln;
  if (!p || p->batch < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 || p->q_len < 0 || p->kv_len < 0)
    return RBLN_ERR_INVALID_ARGUMENT;
  if (p->num_heads % p->num_kv_heads) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->head_dim != 64 && p->head_dim != 128) return RBLN_ERR_UNSUPPORTED;
  if (p->batch == 0 || p->q_len == 0) return RBLN_OK;
  if (!p->q || !p->k || !p->v || !p->out) return RBLN_ERR_INVALID_ARGUMENT;
  if (p->num_heads > 65535 || p->batch > 65535) return RBLN_ERR_UNSUPPORTED;
  const int G = p->num_heads / p->num_kv_heads;
  if (p->dtype == RBLN_DT_BF16 || p->dtype == RBLN_DT_F16) {
    if (p->kv_len == 0) return RBLN_ERR_UNSUPPORTED;
    if (p->mask && p->mask_stride[3] != 1) return RBLN_ERR_INVALID_ARGUMENT;
    if (!al16(p->q) || !al16(p->k) || !al16(p->v) || !al16(p->out)) return RBLN_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 3; ++i)
      if ((p->q_stride[i] * 2) % 16 || (p->k_stride[i] * 2) % 16 || (p->v_stride[i] * 2) % 16 ||
          (p->out_stride[i] * 2) % 16)
        return RBLN_ERR_INVALID_ARGUMENT;
    const int64_t qs[4] = {p->q_stride[0], p->q_stride[1] * G, p->q_stride[1], p->q_stride[2]};
    const int64_t os[4] = {p->out_stride[0], p->out_stride[1] * G, p->out_stride[1], p->out_stride[2]};
    const int64_t ls[4] = {p->lse_stride[0], p->lse_stride[1] * G, p->lse_stride[1], p->lse_stride[2]};
    const int64_t ks[3] = {p->k_stride[0], p->k_stride[1], p->k_stride[2]};
    const int64_t vs[3] = {p->v_stride[0], p->v_stride[1], p->v_stride[2]};
    const int64_t ms[3] = {p->mask_stride[0], p->mask_stride[1], p->mask_stride[2]};
    return attn_tc_dense(p->q, qs, p->out, os, p->lse, ls, p->k, p->v, ks, vs, p->dtype, p->batch, p->num_kv_heads, G,
                         p->q_len, p->kv_len, p->head_dim, p->causal, p->mask, p->mask_dtype, p->mask_additive, ms,
                         p->scale, p->error_flags, stream);
  }
  if (p->dtype != RBLN_DT_F32) return RBLN_ERR_UNSUPPORTED;
  F32Args a{};
  a.q = static_cast<const float*>(p->q);
  a.qs_b = p->q_stride[0];
  a.qs_h = p->q_stride[1];
  a.qs_l = p->q_stride[2];
  a.k = static_cast<const float*>(p->k);
  a.ks_b = p->k_stride[0];
  a.ks_h = p->k_stride[1];
  a.ks_l = p->k_stride[2];
  a.v = static_cast<const float*>(p->v);
  a.vs_b = p->v_stride[0];
  a.vs_h = p->v_stride[1];
  a.vs_l = p->v_stride[2];
  a.out = static_cast<float*>(p->out);
  a.os_b = p->out_stride[0];
  a.os_h = p->out_stride[1];
  a.os_l = p->out_stride[2];
  a.lse = p->lse;
  a.ls_b = p->lse_stride[0];
  a.ls_h = p->lse_stride[1];
  a.ls_l = p->lse_stride[2];
  a.mask = p->mask;
  a.mask_dtype = p->mask_dtype;
  a.mask_additive = p->mask_additive;
  a.m_b = p->mask_stride[0];
  a.m_h = p->mask_stride[1];
  a.m_l = p->mask_stride[2];
  a.m_s = p->mask_stride[3];
  a.B = p->batch;
  a.Hq = p->num_heads;
  a.Hkv = p->num_kv_heads;
  a.L = p->q_len;
  a.S = p->kv_len;
  a.causal = p->causal;
  a.scale = p->scale;
  return p->head_dim == 64 ? launch_f32<64>(a, p->q_len, p->num_heads, p->batch, stream)
                           : launch_f32<128>(a, p->q_len, p->num_heads, p->batch, stream);
}
