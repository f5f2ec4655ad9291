// PyTorch operator layer: defines the rbln_custom_ops schemas (identical to
// the ones the reference's torch.library.custom_op definitions generate,
// test/rbln/test_custom_kernel.py:31-486, 576-645) and registers CUDA kernels that
// validate the tensors, allocate the output and scratch from the PyTorch
// caching allocator, and call the C-ABI entry points of librbln_attn.
//
// Argument checks follow the reference frontends
// (torch_rbln/_internal/register_custom_ops.py:175-450): the cache's last
// dimension must be a multiple of 64, inputs are made contiguous. Departures,
// on purpose: the output dtype is q.dtype (not forced fp16), the caller's
// scale is honoured, batch > 1 prefill is allowed.
#include <ATen/ATen.h>
#include <ATen/Context.h>
#include <ATen/SDPBackend.h>
#include <ATen/cuda/CUDAContext.h>
#include <ATen/ops/_fused_sdp_choice_native.h>
#include <c10/core/GradMode.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <string>

#include "rbln_attn.h"

namespace {

int to_rbln_dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return RBLN_DT_F32;
    case at::kHalf: return RBLN_DT_F16;
    case at::kBFloat16: return RBLN_DT_BF16;
    case at::kFloat8_e4m3fn: return RBLN_DT_FP8_E4M3;
    case at::kShort: return RBLN_DT_I16;
    case at::kInt: return RBLN_DT_I32;
    case at::kLong: return RBLN_DT_I64;
    case at::kBool: return RBLN_DT_BOOL;
    case at::kByte: return RBLN_DT_BOOL;
    default: return -1;
  }
}

const char* status_name(int rc) {
  switch (rc) {
    case RBLN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RBLN_ERR_UNSUPPORTED: return "unsupported configuration";
    case RBLN_ERR_WORKSPACE: return "workspace too small";
    case RBLN_ERR_LAUNCH: return "kernel launch failed";
    case RBLN_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown error";
  }
}

bool debug_checks() {
  static const bool on = [] {
    const char* e = std::getenv("RBLN_ATTN_CHECK");
    return e && std::string(e) != "0";
  }();
  return on;
}

// Moves an index/mask tensor to q's device (callers may keep small tensors on
// the host, as the reference's tests do for `scale`).
at::Tensor on_device(const at::Tensor& t, const at::Tensor& like) {
  return t.device() == like.device() ? t : t.to(like.device());
}

struct Common {
  at::Tensor q, k, v, seq, bt, mask, scale_dev, out, err, sinks;
  rbln_paged_attn_params_t p{};
};

// Shared validation and parameter fill for the four paged ops.
void fill_paged(Common& c, const char* op, const at::Tensor& q_in, const at::Tensor& k_in,
                const at::Tensor& v_in, at::Tensor& kcache, at::Tensor& vcache, const at::Tensor& seq_in,
                const at::Tensor& scale, const at::Tensor& block_table_in, int64_t block_size,
                const std::optional<at::Tensor>& mask_in, bool decode) {
  TORCH_CHECK(q_in.is_cuda(), op, ": expected CUDA tensors, q is on ", q_in.device());
  TORCH_CHECK(q_in.dim() == 5 && k_in.dim() == 5 && v_in.dim() == 5, op,
              ": q/k/v must be 5-D [B, Hkv, G, S, D] / [B, Hkv, 1, S, D]");
  TORCH_CHECK(kcache.dim() == 5 && vcache.dim() == 5, op,
              ": kcache/vcache must be 5-D [num_blocks, Hkv, 1, block_size, D]");
  TORCH_CHECK(kcache.size(-1) % 64 == 0, op,
              ": the last dimension of K-cache must be a multiple of 64, but got shape ", kcache.sizes());
  TORCH_CHECK(vcache.size(-1) % 64 == 0, op,
              ": the last dimension of V-cache must be a multiple of 64, but got shape ", vcache.sizes());
  TORCH_CHECK(kcache.sizes() == vcache.sizes() && kcache.strides() == vcache.strides() &&
                  kcache.scalar_type() == vcache.scalar_type(),
              op, ": kcache and vcache must match in shape, strides and dtype");
  TORCH_CHECK(kcache.is_cuda() && kcache.device() == q_in.device(), op, ": caches must be on q's device");
  TORCH_CHECK(kcache.stride(-1) == 1 && kcache.size(2) == 1, op,
              ": caches must be [num_blocks, Hkv, 1, block_size, D] with a contiguous last dim");
  const auto dt = q_in.scalar_type();
  TORCH_CHECK(dt == at::kBFloat16 || dt == at::kHalf, op, ": q must be bfloat16 or float16, got ", dt);
  TORCH_CHECK(k_in.scalar_type() == dt && v_in.scalar_type() == dt, op, ": q, k, v must share a dtype");

  c.q = q_in.contiguous();
  c.k = k_in.contiguous();
  c.v = v_in.contiguous();
  const int64_t B = c.q.size(0), Hkv = c.q.size(1), G = c.q.size(2), S = c.q.size(3), D = c.q.size(4);
  TORCH_CHECK(c.k.size(0) == B && c.k.size(1) == Hkv && c.k.size(2) == 1 && c.k.size(3) == S &&
                  c.k.size(4) == D && c.v.sizes() == c.k.sizes(),
              op, ": k/v must be [B, Hkv, 1, S, D] matching q ", c.q.sizes(), ", got ", c.k.sizes());
  TORCH_CHECK(kcache.size(1) == Hkv, op, ": caches hold ", kcache.size(1), " KV heads, q has ", Hkv);
  TORCH_CHECK(D <= kcache.size(-1), op, ": head_dim ", D, " exceeds the cache's last dim ", kcache.size(-1));
  TORCH_CHECK(kcache.size(3) == block_size, op, ": block_size ", block_size,
              " does not match the cache's block dimension ", kcache.size(3));
  if (decode) TORCH_CHECK(S == 1, op, ": decode takes one query token per sequence, got S = ", S);

  c.seq = on_device(seq_in, c.q);
  TORCH_CHECK(c.seq.numel() == B, op, ": seq must hold one entry per sequence, got ", c.seq.sizes());
  if (c.seq.scalar_type() != at::kInt) c.seq = c.seq.to(at::kInt);
  c.seq = c.seq.contiguous();

  c.bt = on_device(block_table_in, c.q);
  if (c.bt.dim() == 1) c.bt = c.bt.unsqueeze(0).expand({B, c.bt.size(0)});
  TORCH_CHECK(c.bt.dim() == 2 && (c.bt.size(0) == B || c.bt.size(0) == 1), op,
              ": block_table must be [B, max_blocks], got ", c.bt.sizes());
  const auto btt = c.bt.scalar_type();
  TORCH_CHECK(btt == at::kShort || btt == at::kInt || btt == at::kLong, op,
              ": block_table must be int16/int32/int64");
  if (c.bt.stride(1) != 1) c.bt = c.bt.contiguous();

  auto& p = c.p;
  p.batch = (int32_t)B;
  p.num_kv_heads = (int32_t)Hkv;
  p.group = (int32_t)G;
  p.q_len = (int32_t)S;
  p.head_dim = (int32_t)D;
  p.num_blocks = (int32_t)kcache.size(0);
  p.block_size = (int32_t)block_size;
  p.max_blocks = (int32_t)c.bt.size(1);
  p.q = c.q.data_ptr();
  for (int i = 0; i < 4; ++i) p.q_stride[i] = c.q.stride(i);
  p.q_dtype = to_rbln_dtype(dt);
  c.out = at::empty_like(c.q, at::MemoryFormat::Contiguous);
  p.out = c.out.data_ptr();
  for (int i = 0; i < 4; ++i) p.out_stride[i] = c.out.stride(i);
  p.k_new = c.k.data_ptr();
  p.v_new = c.v.data_ptr();
  p.k_new_stride[0] = c.k.stride(0); p.k_new_stride[1] = c.k.stride(1); p.k_new_stride[2] = c.k.stride(3);
  p.v_new_stride[0] = c.v.stride(0); p.v_new_stride[1] = c.v.stride(1); p.v_new_stride[2] = c.v.stride(3);
  p.kcache = kcache.data_ptr();
  p.vcache = vcache.data_ptr();
  p.kv_dtype = to_rbln_dtype(kcache.scalar_type());
  p.cache_stride[0] = kcache.stride(0);
  p.cache_stride[1] = kcache.stride(1);
  p.cache_stride[2] = kcache.stride(3);
  p.seq = c.seq.data_ptr<int32_t>();
  p.seq_stride = 1;
  p.block_table = c.bt.data_ptr();
  p.block_table_dtype = to_rbln_dtype(btt);
  p.block_table_stride = c.bt.size(0) == 1 ? 0 : c.bt.stride(0);

  if (mask_in.has_value() && mask_in->defined()) {
    c.mask = on_device(*mask_in, c.q);
    TORCH_CHECK(c.mask.scalar_type() == at::kFloat || c.mask.scalar_type() == at::kHalf ||
                    c.mask.scalar_type() == at::kBFloat16 || c.mask.scalar_type() == at::kBool,
                op, ": mask must be floating point or bool");
    if (c.mask.stride(-1) != 1) c.mask = c.mask.contiguous();
    p.mask = c.mask.data_ptr();
    p.mask_dtype = to_rbln_dtype(c.mask.scalar_type());
    p.mask_len = (int32_t)std::min<int64_t>(c.mask.size(-1), (int64_t)p.max_blocks * block_size);
    // batch stride: the mask's leading dim is the batch (or broadcast 1)
    p.mask_stride[0] = c.mask.size(0) == 1 ? 0 : c.mask.stride(0);
    // query-row stride for prefill keep-masks [B, 1, 1, S_q, L]
    p.mask_stride[1] = (c.mask.dim() >= 2 && c.mask.size(-2) == S) ? c.mask.stride(-2) : 0;
  }

  if (scale.is_cuda()) {
    c.scale_dev = scale.scalar_type() == at::kFloat ? scale : scale.to(at::kFloat);
    p.scale_dev = c.scale_dev.data_ptr<float>();
  } else {
    p.scale = scale.item<float>();
  }
  if (debug_checks()) {
    c.err = at::zeros({1}, c.q.options().dtype(at::kInt));
    p.error_flags = reinterpret_cast<uint32_t*>(c.err.data_ptr<int32_t>());
  }
}

void check_rc(int rc, const char* op) {
  TORCH_CHECK(rc == RBLN_OK, op, ": ", status_name(rc), " (status ", rc, ")");
}

void check_device_flags(const Common& c, const char* op) {
  if (!c.err.defined()) return;
  const int flags = c.err.item<int>();
  TORCH_CHECK(flags == 0, op, ": device-side input check failed (flags 0x", std::hex, flags,
              "): block_table entry out of range or seq out of range");
}

at::Tensor run_decode(Common& c, at::Tensor& kcache, const char* op, bool require_mask) {
  c10::cuda::CUDAGuard guard(c.q.device());
  size_t ws = 0;
  check_rc(rbln_paged_decode_workspace_size(&c.p, &ws), op);
  at::Tensor wst;
  if (ws > 0) {
    wst = at::empty({(int64_t)ws}, c.q.options().dtype(at::kByte));
    c.p.workspace = wst.data_ptr();
    c.p.workspace_bytes = ws;
  }
  auto stream = at::cuda::getCurrentCUDAStream(c.q.device().index());
  const int rc = require_mask ? rbln_paged_attn_decode(&c.p, stream.stream())
                              : rbln_paged_causal_attn_decode(&c.p, stream.stream());
  check_rc(rc, op);
  check_device_flags(c, op);
  return c.out;
}

// rbln_custom_ops::paged_attn_decode (register_custom_ops.py:253-293)
at::Tensor paged_attn_decode_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                  const at::Tensor& mask, at::Tensor& kcache, at::Tensor& vcache,
                                  const at::Tensor& seq, const at::Tensor& scale,
                                  const at::Tensor& block_table, int64_t block_size) {
  Common c;
  TORCH_CHECK(kcache.scalar_type() == q.scalar_type(), "paged_attn_decode: cache dtype must equal q dtype");
  fill_paged(c, "paged_attn_decode", q, k, v, kcache, vcache, seq, scale, block_table, block_size, mask, true);
  return run_decode(c, kcache, "paged_attn_decode", true);
}

// rbln_custom_ops::paged_causal_attn_decode (register_custom_ops.py:409-450)
at::Tensor paged_causal_attn_decode_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                         at::Tensor& kcache, at::Tensor& vcache, const at::Tensor& seq,
                                         const at::Tensor& scale, const at::Tensor& block_table,
                                         int64_t block_size, const std::optional<at::Tensor>& mask) {
  Common c;
  TORCH_CHECK(kcache.scalar_type() == q.scalar_type(),
              "paged_causal_attn_decode: cache dtype must equal q dtype (use the _kvfp8 op for fp8 caches)");
  fill_paged(c, "paged_causal_attn_decode", q, k, v, kcache, vcache, seq, scale, block_table, block_size,
             mask, true);
  return run_decode(c, kcache, "paged_causal_attn_decode", false);
}

// fp8-e4m3 KV cache with one fp32 dequant scale per (block, KV head). No
// counterpart in the reference's op set; same contract as
// paged_causal_attn_decode plus the two scale tensors [num_blocks, Hkv].
at::Tensor paged_causal_attn_decode_kvfp8_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                               at::Tensor& kcache, at::Tensor& vcache,
                                               const at::Tensor& k_scale, const at::Tensor& v_scale,
                                               const at::Tensor& seq, const at::Tensor& scale,
                                               const at::Tensor& block_table, int64_t block_size,
                                               const std::optional<at::Tensor>& mask) {
  const char* op = "paged_causal_attn_decode_kvfp8";
  TORCH_CHECK(kcache.scalar_type() == at::kFloat8_e4m3fn, op, ": caches must be float8_e4m3fn");
  TORCH_CHECK(k_scale.scalar_type() == at::kFloat && v_scale.scalar_type() == at::kFloat, op,
              ": k_scale/v_scale must be float32 [num_blocks, Hkv]");
  TORCH_CHECK(k_scale.dim() == 2 && k_scale.size(0) == kcache.size(0) && k_scale.size(1) == kcache.size(1) &&
                  v_scale.sizes() == k_scale.sizes() && v_scale.strides() == k_scale.strides(),
              op, ": k_scale/v_scale must be [num_blocks, Hkv]");
  TORCH_CHECK(k_scale.device() == q.device() && v_scale.device() == q.device(), op,
              ": scales must be on q's device");
  Common c;
  fill_paged(c, op, q, k, v, kcache, vcache, seq, scale, block_table, block_size, mask, true);
  c.p.k_scale = k_scale.data_ptr<float>();
  c.p.v_scale = v_scale.data_ptr<float>();
  c.p.scale_stride[0] = k_scale.stride(0);
  c.p.scale_stride[1] = k_scale.stride(1);
  return run_decode(c, kcache, op, false);
}

at::Tensor run_prefill(Common& c, const char* op, bool keep_mask) {
  c10::cuda::CUDAGuard guard(c.q.device());
  size_t ws = 0;
  check_rc(rbln_paged_prefill_workspace_size(&c.p, &ws), op);
  at::Tensor wst;
  if (ws > 0) {
    wst = at::empty({(int64_t)ws}, c.q.options().dtype(at::kByte));
    c.p.workspace = wst.data_ptr();
    c.p.workspace_bytes = ws;
  }
  auto stream = at::cuda::getCurrentCUDAStream(c.q.device().index());
  const int rc = keep_mask ? rbln_paged_attn_prefill(&c.p, stream.stream())
                           : rbln_paged_causal_attn_prefill(&c.p, stream.stream());
  check_rc(rc, op);
  check_device_flags(c, op);
  return c.out;
}

// rbln_custom_ops::paged_attn_prefill (register_custom_ops.py:175-229)
at::Tensor paged_attn_prefill_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                   const at::Tensor& mask, at::Tensor& kcache, at::Tensor& vcache,
                                   const at::Tensor& seq, const at::Tensor& scale, const at::Tensor& block_table,
                                   int64_t block_size) {
  const char* op = "paged_attn_prefill";
  TORCH_CHECK(kcache.scalar_type() == q.scalar_type(), op, ": cache dtype must equal q dtype");
  Common c;
  fill_paged(c, op, q, k, v, kcache, vcache, seq, scale, block_table, block_size, mask, false);
  return run_prefill(c, op, true);
}

// rbln_custom_ops::paged_causal_attn_prefill (register_custom_ops.py:324-379)
at::Tensor paged_causal_attn_prefill_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                          at::Tensor& kcache, at::Tensor& vcache, const at::Tensor& seq,
                                          const at::Tensor& scale, const at::Tensor& block_table, int64_t block_size,
                                          bool is_bidirectional, const std::optional<at::Tensor>& mask) {
  const char* op = "paged_causal_attn_prefill";
  TORCH_CHECK(kcache.scalar_type() == q.scalar_type(), op, ": cache dtype must equal q dtype");
  Common c;
  fill_paged(c, op, q, k, v, kcache, vcache, seq, scale, block_table, block_size, mask, false);
  c.p.causal = is_bidirectional ? 0 : 1;
  return run_prefill(c, op, false);
}

// rbln_attn::paged_kv_write: the paged ops' append step on its own (k, v
// [B, Hkv, 1, S, D] at positions [seq[b], seq[b] + S)); fp8 caches take
// k_scale / v_scale [num_blocks, Hkv] and get per-(block, head) scales
// recomputed (rbln_paged_kv_write, kv_write.cu).
void paged_kv_write_cuda(const at::Tensor& k_in, const at::Tensor& v_in, at::Tensor& kcache, at::Tensor& vcache,
                         const at::Tensor& seq_in, const at::Tensor& block_table_in, int64_t block_size,
                         const std::optional<at::Tensor>& k_scale, const std::optional<at::Tensor>& v_scale) {
  const char* op = "paged_kv_write";
  TORCH_CHECK(k_in.is_cuda() && k_in.dim() == 5 && v_in.sizes() == k_in.sizes() && k_in.size(2) == 1, op,
              ": k/v must be CUDA [B, Hkv, 1, S, D]");
  TORCH_CHECK(kcache.dim() == 5 && kcache.sizes() == vcache.sizes() && kcache.strides() == vcache.strides() &&
                  kcache.stride(-1) == 1 && kcache.size(3) == block_size && kcache.device() == k_in.device(),
              op, ": caches must be [num_blocks, Hkv, 1, block_size, D] on k's device, alike");
  const auto dt = k_in.scalar_type();
  TORCH_CHECK((dt == at::kBFloat16 || dt == at::kHalf) && v_in.scalar_type() == dt, op, ": k/v bf16 or f16");
  const bool fp8 = kcache.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || kcache.scalar_type() == dt, op, ": cache dtype must be k's or float8_e4m3fn");
  TORCH_CHECK(vcache.scalar_type() == kcache.scalar_type(), op, ": kcache and vcache dtypes differ");
  at::Tensor k = k_in.contiguous(), v = v_in.contiguous();
  const int64_t B = k.size(0), Hkv = k.size(1), S = k.size(3), D = k.size(4);
  TORCH_CHECK(kcache.size(1) == Hkv && kcache.size(-1) == D, op, ": cache heads / head_dim differ from k's");
  at::Tensor seq = on_device(seq_in, k).reshape({-1}).to(at::kInt).contiguous();
  TORCH_CHECK(seq.numel() == B, op, ": seq must hold one entry per sequence");
  at::Tensor bt = on_device(block_table_in, k);
  if (bt.dim() == 1) bt = bt.unsqueeze(0);
  TORCH_CHECK(bt.dim() == 2 && (bt.size(0) == B || bt.size(0) == 1), op, ": block_table must be [B, max_blocks]");
  if (bt.stride(1) != 1) bt = bt.contiguous();
  rbln_paged_attn_params_t p{};
  p.batch = (int32_t)B;
  p.num_kv_heads = (int32_t)Hkv;
  p.group = 1;
  p.q_len = (int32_t)S;
  p.head_dim = (int32_t)D;
  p.num_blocks = (int32_t)kcache.size(0);
  p.block_size = (int32_t)block_size;
  p.max_blocks = (int32_t)bt.size(1);
  p.q_dtype = to_rbln_dtype(dt);
  p.k_new = k.data_ptr();
  p.v_new = v.data_ptr();
  p.k_new_stride[0] = k.stride(0); p.k_new_stride[1] = k.stride(1); p.k_new_stride[2] = k.stride(3);
  p.v_new_stride[0] = v.stride(0); p.v_new_stride[1] = v.stride(1); p.v_new_stride[2] = v.stride(3);
  p.kcache = kcache.data_ptr();
  p.vcache = vcache.data_ptr();
  p.kv_dtype = to_rbln_dtype(kcache.scalar_type());
  p.cache_stride[0] = kcache.stride(0); p.cache_stride[1] = kcache.stride(1); p.cache_stride[2] = kcache.stride(3);
  if (fp8) {
    TORCH_CHECK(k_scale.has_value() && v_scale.has_value() && k_scale->scalar_type() == at::kFloat &&
                    v_scale->scalar_type() == at::kFloat && k_scale->dim() == 2 &&
                    k_scale->size(0) == kcache.size(0) && k_scale->size(1) == Hkv &&
                    v_scale->sizes() == k_scale->sizes() && v_scale->strides() == k_scale->strides() &&
                    k_scale->device() == k.device() && v_scale->device() == k.device(),
                op, ": fp8 caches need float32 k_scale / v_scale [num_blocks, Hkv] on the caches' device");
    p.k_scale = k_scale->data_ptr<float>();
    p.v_scale = v_scale->data_ptr<float>();
    p.scale_stride[0] = k_scale->stride(0);
    p.scale_stride[1] = k_scale->stride(1);
  }
  p.seq = seq.data_ptr<int32_t>();
  p.seq_stride = 1;
  p.block_table = bt.data_ptr();
  p.block_table_dtype = to_rbln_dtype(bt.scalar_type());
  p.block_table_stride = bt.size(0) == 1 ? 0 : bt.stride(0);
  at::Tensor err;
  if (debug_checks()) {
    err = at::zeros({1}, k.options().dtype(at::kInt));
    p.error_flags = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  }
  c10::cuda::CUDAGuard guard(k.device());
  check_rc(rbln_paged_kv_write(&p, at::cuda::getCurrentCUDAStream(k.device().index()).stream()), op);
  if (err.defined()) {
    const int flags = err.item<int>();
    TORCH_CHECK(flags == 0, op, ": device-side input check failed (flags 0x", std::hex, flags, ")");
  }
}

// ---------------------------------------------------------------------------
// flash_attention_naive_{prefill,decode}: the unified-cache form of the paged
// ops (torch_rbln/_internal/register_custom_ops.py:453-560; CPU semantics in
// test/rbln/test_custom_kernel.py:546-573). kv_cache [2, num_blocks, Hkv, 1,
// P, D] stacks the K pool (index 0) and the V pool (index 1), each block one
// partition of P tokens; block_tables lists a sequence's partitions (1-D for
// prefill, [B, NP] for decode); seq_idx [B, 1] is the position of the first
// new token; mask is a keep-mask over partition positions. The new rows are
// written at seq_idx through the block table and attention runs over the
// mask's positions: the keep-mask paged path on kv_cache[0] / kv_cache[1].
// slot_mapping is accepted for the schema and not read (the positions follow
// from seq_idx and block_tables, as in the reference's CPU semantics).
// sinks [Hkv * G] (any float dtype) are per-query-head sink logits.
// ---------------------------------------------------------------------------
at::Tensor flash_attention_naive(const char* op, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                 at::Tensor& kv_cache, const at::Tensor& mask, const at::Tensor& scale,
                                 const at::Tensor& seq_idx, const at::Tensor& block_tables,
                                 const at::Tensor& slot_mapping, const std::optional<at::Tensor>& sinks,
                                 bool decode) {
  TORCH_CHECK(kv_cache.dim() == 6 && kv_cache.size(0) == 2, op,
              ": kv_cache must be [2, num_blocks, Hkv, 1, partition, D], got ", kv_cache.sizes());
  TORCH_CHECK(kv_cache.size(-1) % 64 == 0, op,
              ": The last dimension of kv_cache must be a multiple of 64, but got shape ", kv_cache.sizes());
  TORCH_CHECK(kv_cache.scalar_type() == q.scalar_type(), op, ": kv_cache dtype must equal q dtype");
  if (!decode)
    for (const at::Tensor* t : {&q, &k, &v})
      TORCH_CHECK(t->dim() >= 1 && t->size(0) == 1, op, " batch size of q/k/v must be 1, but got shape ",
                  t->sizes());
  TORCH_CHECK(slot_mapping.defined(), op, ": slot_mapping is required");
  at::Tensor kcache = kv_cache.select(0, 0);
  at::Tensor vcache = kv_cache.select(0, 1);
  // seq_idx [B, 1] (or [B]): one start position per sequence
  const at::Tensor seq = seq_idx.dim() == 2 ? seq_idx.select(1, 0) : seq_idx;
  Common c;
  fill_paged(c, op, q, k, v, kcache, vcache, seq, scale, block_tables, kv_cache.size(-2), mask, decode);
  if (sinks.has_value() && sinks->defined()) {
    TORCH_CHECK(at::isFloatingType(sinks->scalar_type()), op, ": sinks must be floating point");
    TORCH_CHECK(sinks->numel() == (int64_t)c.p.num_kv_heads * c.p.group, op, ": sinks must hold one logit per ",
                "query head (", c.p.num_kv_heads * c.p.group, "), got ", sinks->sizes());
    c.sinks = on_device(*sinks, c.q).to(at::kFloat).contiguous();
    c.p.sinks = c.sinks.data_ptr<float>();
  }
  return decode ? run_decode(c, kcache, op, true) : run_prefill(c, op, true);
}

at::Tensor flash_attention_naive_prefill_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                              at::Tensor& kv_cache, const at::Tensor& mask, const at::Tensor& scale,
                                              const at::Tensor& seq_idx, const at::Tensor& block_tables,
                                              const at::Tensor& slot_mapping,
                                              const std::optional<at::Tensor>& sinks) {
  return flash_attention_naive("flash_attention_naive_prefill", q, k, v, kv_cache, mask, scale, seq_idx,
                               block_tables, slot_mapping, sinks, false);
}

at::Tensor flash_attention_naive_decode_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                             at::Tensor& kv_cache, const at::Tensor& mask, const at::Tensor& scale,
                                             const at::Tensor& seq_idx, const at::Tensor& block_tables,
                                             const at::Tensor& slot_mapping,
                                             const std::optional<at::Tensor>& sinks) {
  return flash_attention_naive("flash_attention_naive_decode", q, k, v, kv_cache, mask, scale, seq_idx,
                               block_tables, slot_mapping, sinks, true);
}

// ---------------------------------------------------------------------------
// SDPA: aten::_scaled_dot_product_fused_attention_overrideable on CUDA, and
// the backend choice that routes F.scaled_dot_product_attention to it
// (mirrors _fused_sdp_choice_privateuse1, aten/src/ATen/native/
// RBLNRegisterOps.cpp:89-102, which picks "overrideable" for 4-D inputs).
// ---------------------------------------------------------------------------
std::atomic<bool> g_sdpa_route{[] {
  const char* e = std::getenv("RBLN_ATTN_SDPA");
  return !(e && std::string(e) == "0");
}()};

bool sm100_device(const at::Tensor& t) {
  if (!t.is_cuda()) return false;
  const auto* prop = at::cuda::getDeviceProperties(t.device().index());
  return prop->major == 10;
}

// The inputs the CUDA kernels here take; anything else goes to torch's own
// CUDA backends.
bool sdpa_supported(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                    const std::optional<at::Tensor>& mask, double dropout_p) {
  if (q.dim() != 4 || k.dim() != 4 || v.dim() != 4) return false;
  if (q.is_nested() || k.is_nested() || v.is_nested()) return false;
  const auto dt = q.scalar_type();
  if (dt != at::kBFloat16 && dt != at::kHalf && dt != at::kFloat) return false;
  if (k.scalar_type() != dt || v.scalar_type() != dt) return false;
  if (k.device() != q.device() || v.device() != q.device() || !sm100_device(q)) return false;
  const int64_t D = q.size(3);
  if ((D != 64 && D != 128) || k.size(3) != D || v.size(3) != D) return false;
  if (k.size(0) != q.size(0) || v.size(0) != q.size(0) || k.size(1) != v.size(1) || k.size(2) != v.size(2))
    return false;
  if (k.size(1) == 0 || q.size(1) % k.size(1) != 0) return false;
  if (q.numel() == 0 || k.numel() == 0) return false;
  if (dropout_p > 0.0) return false;
  // the backward (sdpa_bwd.cu) runs on the tensor cores: bf16 / f16 only
  const bool grad = c10::GradMode::is_enabled() &&
                    (q.requires_grad() || k.requires_grad() || v.requires_grad() ||
                     (mask.has_value() && mask->defined() && mask->requires_grad()));
  if (grad && dt == at::kFloat) return false;
  if (mask.has_value() && mask->defined()) {
    const auto& m = *mask;
    if (m.dim() < 2 || m.dim() > 4 || m.device() != q.device()) return false;
    if (m.scalar_type() != at::kBool && !at::isFloatingType(m.scalar_type())) return false;
  }
  return true;
}

int64_t fused_sdp_choice_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                              const std::optional<at::Tensor>& mask, double dropout_p, bool is_causal,
                              std::optional<double> scale, bool enable_gqa) {
  if (g_sdpa_route.load() && at::globalContext().userEnabledOverrideableSDP() &&
      sdpa_supported(q, k, v, mask, dropout_p))
    return static_cast<int64_t>(at::SDPBackend::overrideable);
  return at::native::_fused_sdp_choice_cuda(q, k, v, mask, dropout_p, is_causal, scale, enable_gqa);
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, c10::SymInt, c10::SymInt, at::Tensor, at::Tensor,
           at::Tensor>
sdpa_overrideable_cuda(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                       const std::optional<at::Tensor>& attn_bias, double dropout_p, bool is_causal,
                       bool return_debug_mask, std::optional<double> scale) {
  // input validation as in the reference (sdpa.py:85-119): ValueError
  TORCH_CHECK_VALUE(query.scalar_type() == key.scalar_type() && query.scalar_type() == value.scalar_type(),
                    "Expected query, key, and value to have the same dtype, but got query.dtype: ",
                    query.scalar_type(), ", key.dtype: ", key.scalar_type(), ", and value.dtype: ",
                    value.scalar_type(), " instead.");
  TORCH_CHECK_VALUE(query.device() == key.device() && query.device() == value.device(),
                    "Expected query, key, and value to have the same device type, but got query.device: ",
                    query.device(), ", key.device: ", key.device(), ", and value.device: ", value.device(),
                    " instead.");
  if (attn_bias.has_value() && attn_bias->defined()) {
    TORCH_CHECK_VALUE(attn_bias->scalar_type() == at::kBool || at::isFloatingType(attn_bias->scalar_type()),
                      "Expected attn_mask to have dtype bool or floating point, but got attn_mask.dtype: ",
                      attn_bias->scalar_type(), " instead.");
    TORCH_CHECK_VALUE(attn_bias->device() == query.device(),
                      "Expected attn_mask to have the same device as query, but got attn_mask.device: ",
                      attn_bias->device(), " and query.device: ", query.device(), " instead.");
  }
  TORCH_CHECK(sdpa_supported(query, key, value, attn_bias, dropout_p),
              "_scaled_dot_product_fused_attention_overrideable (CUDA, sm_100a): unsupported inputs "
              "(need 4-D bf16/f16/f32 q/k/v with head_dim 64 or 128, Hq % Hkv == 0, no dropout; "
              "bf16/f16 when a gradient is needed)");
  c10::cuda::CUDAGuard guard(query.device());
  auto inner = [](const at::Tensor& t) { return t.stride(-1) == 1 ? t : t.contiguous(); };
  at::Tensor q = inner(query), k = inner(key), v = inner(value);
  const int64_t B = q.size(0), H = q.size(1), L = q.size(2), D = q.size(3);
  const int64_t Hkv = k.size(1), S = k.size(2);
  at::Tensor out = at::empty({B, H, L, D}, q.options());
  at::Tensor lse = at::empty({B, H, L}, q.options().dtype(at::kFloat));
  rbln_sdpa_params_t p{};
  p.batch = (int32_t)B;
  p.num_heads = (int32_t)H;
  p.num_kv_heads = (int32_t)Hkv;
  p.q_len = (int32_t)L;
  p.kv_len = (int32_t)S;
  p.head_dim = (int32_t)D;
  p.dtype = to_rbln_dtype(q.scalar_type());
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.out = out.data_ptr();
  for (int i = 0; i < 3; ++i) {
    p.q_stride[i] = q.stride(i);
    p.k_stride[i] = k.stride(i);
    p.v_stride[i] = v.stride(i);
    p.out_stride[i] = out.stride(i);
    p.lse_stride[i] = lse.stride(i);
  }
  p.lse = lse.data_ptr<float>();
  at::Tensor m;
  if (attn_bias.has_value() && attn_bias->defined()) {
    m = *attn_bias;
    if (m.scalar_type() != at::kBool && m.scalar_type() != at::kFloat && m.scalar_type() != at::kHalf &&
        m.scalar_type() != at::kBFloat16)
      m = m.to(at::kFloat);
    while (m.dim() < 4) m = m.unsqueeze(0);
    m = m.expand({B, H, L, S});
    if (m.stride(3) != 1 && q.scalar_type() != at::kFloat) m = m.contiguous();
    p.mask = m.data_ptr();
    p.mask_dtype = to_rbln_dtype(m.scalar_type());
    p.mask_additive = m.scalar_type() == at::kBool ? 0 : 1;
    for (int i = 0; i < 4; ++i) p.mask_stride[i] = m.stride(i);
  }
  p.causal = is_causal ? 1 : 0;
  p.scale = (float)(scale.has_value() ? *scale : 1.0 / std::sqrt((double)D));
  at::Tensor err;
  if (debug_checks()) {
    err = at::zeros({1}, q.options().dtype(at::kInt));
    p.error_flags = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  }
  auto stream = at::cuda::getCurrentCUDAStream(q.device().index());
  check_rc(rbln_sdpa_fwd(&p, stream.stream()), "_scaled_dot_product_fused_attention_overrideable");
  if (err.defined()) {
    const int flags = err.item<int>();
    TORCH_CHECK(flags == 0, "_scaled_dot_product_fused_attention_overrideable: device error flags 0x", std::hex,
                flags);
  }
  at::Tensor debug = return_debug_mask ? at::empty({B, H, L, S}, q.options().dtype(at::kFloat))
                                       : at::empty({0}, q.options().dtype(at::kFloat));
  at::Tensor cum_q = at::empty({0}, q.options().dtype(at::kLong));
  at::Tensor cum_k = at::empty({0}, q.options().dtype(at::kLong));
  at::Tensor seed = at::empty({}, at::TensorOptions().dtype(at::kLong).device(at::kCPU));
  at::Tensor offset = at::empty({}, at::TensorOptions().dtype(at::kLong).device(at::kCPU));
  return {out, lse, cum_q, cum_k, c10::SymInt(L), c10::SymInt(S), seed, offset, debug};
}

// aten::_scaled_dot_product_fused_attention_overrideable_backward on CUDA
// (reference sdpa.py:754-821): dq, dk, dv as grad_input_mask asks, and
// grad_attn_bias for a floating-point mask (full [B, H, L, S], in the mask's
// dtype; autograd sums it down to the mask's broadcast shape). P is
// recomputed from q, k and the forward's logsumexp.
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> sdpa_overrideable_backward_cuda(
    const at::Tensor& grad_out, const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
    const at::Tensor& attn_bias, std::array<bool, 4> grad_input_mask, const at::Tensor& out,
    const at::Tensor& logsumexp, const at::Tensor& cum_seq_q, const at::Tensor& cum_seq_k, c10::SymInt max_q,
    c10::SymInt max_k, double dropout_p, bool is_causal, const at::Tensor& philox_seed,
    const at::Tensor& philox_offset, std::optional<double> scale) {
  const char* op = "_scaled_dot_product_fused_attention_overrideable_backward";
  TORCH_CHECK(dropout_p == 0.0, op, ": dropout is not supported");
  TORCH_CHECK(query.dim() == 4 && key.dim() == 4 && value.dim() == 4 && grad_out.dim() == 4 && out.dim() == 4, op,
              ": expected 4-D tensors");
  const auto dt = query.scalar_type();
  TORCH_CHECK(dt == at::kBFloat16 || dt == at::kHalf, op, ": bf16 / f16 only, got ", dt);
  TORCH_CHECK(key.scalar_type() == dt && value.scalar_type() == dt && grad_out.scalar_type() == dt &&
                  out.scalar_type() == dt,
              op, ": q, k, v, out and grad_out must share a dtype");
  c10::cuda::CUDAGuard guard(query.device());
  // last dim contiguous and 16-byte aligned rows
  auto rows16 = [](const at::Tensor& t) {
    const bool ok = t.stride(-1) == 1 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0 &&
                    (t.stride(0) * 2) % 16 == 0 && (t.stride(1) * 2) % 16 == 0 && (t.stride(2) * 2) % 16 == 0;
    return ok ? t : t.contiguous();
  };
  at::Tensor q = rows16(query), k = rows16(key), v = rows16(value), o = rows16(out), dout = rows16(grad_out);
  const int64_t B = q.size(0), H = q.size(1), L = q.size(2), D = q.size(3);
  const int64_t Hkv = k.size(1), S = k.size(2);
  TORCH_CHECK(logsumexp.defined() && logsumexp.dim() == 3 && logsumexp.size(0) == B && logsumexp.size(1) == H &&
                  logsumexp.size(2) == L && logsumexp.scalar_type() == at::kFloat,
              op, ": logsumexp must be the forward's fp32 [B, H, L]");
  at::Tensor lse = logsumexp;
  at::Tensor dq = grad_input_mask[0] ? at::empty_like(q, at::MemoryFormat::Contiguous) : at::Tensor();
  at::Tensor dk = grad_input_mask[1] ? at::empty_like(k, at::MemoryFormat::Contiguous) : at::Tensor();
  at::Tensor dv = grad_input_mask[2] ? at::empty_like(v, at::MemoryFormat::Contiguous) : at::Tensor();
  rbln_sdpa_bwd_params_t p{};
  p.batch = (int32_t)B;
  p.num_heads = (int32_t)H;
  p.num_kv_heads = (int32_t)Hkv;
  p.q_len = (int32_t)L;
  p.kv_len = (int32_t)S;
  p.head_dim = (int32_t)D;
  p.dtype = to_rbln_dtype(dt);
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.out = o.data_ptr();
  p.dout = dout.data_ptr();
  p.lse = lse.data_ptr<float>();
  for (int i = 0; i < 3; ++i) {
    p.q_stride[i] = q.stride(i);
    p.k_stride[i] = k.stride(i);
    p.v_stride[i] = v.stride(i);
    p.out_stride[i] = o.stride(i);
    p.dout_stride[i] = dout.stride(i);
    p.lse_stride[i] = lse.stride(i);
    if (dq.defined()) p.dq_stride[i] = dq.stride(i);
    if (dk.defined()) p.dk_stride[i] = dk.stride(i);
    if (dv.defined()) p.dv_stride[i] = dv.stride(i);
  }
  p.dq = dq.defined() ? dq.data_ptr() : nullptr;
  p.dk = dk.defined() ? dk.data_ptr() : nullptr;
  p.dv = dv.defined() ? dv.data_ptr() : nullptr;
  at::Tensor m, dbias;
  if (attn_bias.defined() && attn_bias.numel() > 0) {  // an empty tensor means no mask (sdpa.py:800)
    m = attn_bias;
    TORCH_CHECK(m.scalar_type() == at::kBool || at::isFloatingType(m.scalar_type()), op,
                ": attn_bias must be bool or floating point");
    if (m.scalar_type() != at::kBool && m.scalar_type() != at::kFloat && m.scalar_type() != at::kHalf &&
        m.scalar_type() != at::kBFloat16)
      m = m.to(at::kFloat);
    while (m.dim() < 4) m = m.unsqueeze(0);
    m = m.expand({B, H, L, S});
    if (m.stride(3) != 1) m = m.contiguous();
    p.mask = m.data_ptr();
    p.mask_dtype = to_rbln_dtype(m.scalar_type());
    p.mask_additive = m.scalar_type() == at::kBool ? 0 : 1;
    for (int i = 0; i < 4; ++i) p.mask_stride[i] = m.stride(i);
    if (grad_input_mask[3] && m.scalar_type() != at::kBool) {
      dbias = at::empty({B, H, L, S}, q.options().dtype(at::kFloat));
      p.dbias = dbias.data_ptr<float>();
    }
  }
  p.causal = is_causal ? 1 : 0;
  p.scale = (float)(scale.has_value() ? *scale : 1.0 / std::sqrt((double)D));
  size_t ws = 0;
  check_rc(rbln_sdpa_bwd_workspace_size(&p, &ws), op);
  at::Tensor wst = at::empty({(int64_t)std::max<size_t>(ws, 16)}, q.options().dtype(at::kByte));
  p.workspace = wst.data_ptr();
  p.workspace_bytes = ws;
  at::Tensor err;
  if (debug_checks()) {
    err = at::zeros({1}, q.options().dtype(at::kInt));
    p.error_flags = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  }
  auto stream = at::cuda::getCurrentCUDAStream(q.device().index());
  check_rc(rbln_sdpa_bwd(&p, stream.stream()), op);
  if (err.defined()) {
    const int flags = err.item<int>();
    TORCH_CHECK(flags == 0, op, ": device error flags 0x", std::hex, flags);
  }
  at::Tensor gbias;
  if (dbias.defined()) gbias = dbias.to(attn_bias.scalar_type());
  return {dq, dk, dv, gbias};
}

void set_sdpa_route(bool enabled) { g_sdpa_route.store(enabled); }
bool sdpa_route_enabled() { return g_sdpa_route.load(); }

}  // namespace

TORCH_LIBRARY(rbln_attn, m) {
  m.def("set_sdpa_route(bool enabled) -> ()");
  m.def("sdpa_route_enabled() -> bool");
  m.def(
      "paged_kv_write(Tensor k, Tensor v, Tensor(a!) kcache, Tensor(b!) vcache, Tensor seq, Tensor block_table, "
      "SymInt block_size, Tensor(c!)? k_scale=None, Tensor(d!)? v_scale=None) -> ()");
}

TORCH_LIBRARY_IMPL(rbln_attn, CUDA, m) { m.impl("paged_kv_write", &paged_kv_write_cuda); }

TORCH_LIBRARY_IMPL(rbln_attn, CompositeExplicitAutograd, m) {
  m.impl("set_sdpa_route", &set_sdpa_route);
  m.impl("sdpa_route_enabled", &sdpa_route_enabled);
}

TORCH_LIBRARY_IMPL(aten, CUDA, m) {
  m.impl("_fused_sdp_choice", &fused_sdp_choice_cuda);
  m.impl("_scaled_dot_product_fused_attention_overrideable", &sdpa_overrideable_cuda);
  m.impl("_scaled_dot_product_fused_attention_overrideable_backward", &sdpa_overrideable_backward_cuda);
}

TORCH_LIBRARY(rbln_custom_ops, m) {
  m.def(
      "paged_attn_prefill(Tensor q, Tensor k, Tensor v, Tensor mask, Tensor(a4!) kcache, Tensor(a5!) vcache, "
      "Tensor seq, Tensor scale, Tensor block_table, SymInt block_size) -> Tensor");
  m.def(
      "paged_attn_decode(Tensor q, Tensor k, Tensor v, Tensor mask, Tensor(a4!) kcache, Tensor(a5!) vcache, "
      "Tensor seq, Tensor scale, Tensor block_table, SymInt block_size) -> Tensor");
  m.def(
      "paged_causal_attn_prefill(Tensor q, Tensor k, Tensor v, Tensor(a3!) kcache, Tensor(a4!) vcache, "
      "Tensor seq, Tensor scale, Tensor block_table, SymInt block_size, bool is_bidirectional, "
      "Tensor? mask=None) -> Tensor");
  m.def(
      "paged_causal_attn_decode(Tensor q, Tensor k, Tensor v, Tensor(a3!) kcache, Tensor(a4!) vcache, "
      "Tensor seq, Tensor scale, Tensor block_table, SymInt block_size, Tensor? mask=None) -> Tensor");
  m.def(
      "paged_causal_attn_decode_kvfp8(Tensor q, Tensor k, Tensor v, Tensor(a3!) kcache, Tensor(a4!) vcache, "
      "Tensor k_scale, Tensor v_scale, Tensor seq, Tensor scale, Tensor block_table, SymInt block_size, "
      "Tensor? mask=None) -> Tensor");
  m.def(
      "flash_attention_naive_prefill(Tensor q, Tensor k, Tensor v, Tensor(a3!) kv_cache, Tensor mask, "
      "Tensor scale, Tensor seq_idx, Tensor block_tables, Tensor slot_mapping, Tensor? sinks=None) -> Tensor");
  m.def(
      "flash_attention_naive_decode(Tensor q, Tensor k, Tensor v, Tensor(a3!) kv_cache, Tensor mask, "
      "Tensor scale, Tensor seq_idx, Tensor block_tables, Tensor slot_mapping, Tensor? sinks=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(rbln_custom_ops, CUDA, m) {
  m.impl("paged_attn_prefill", &paged_attn_prefill_cuda);
  m.impl("paged_causal_attn_prefill", &paged_causal_attn_prefill_cuda);
  m.impl("paged_attn_decode", &paged_attn_decode_cuda);
  m.impl("paged_causal_attn_decode", &paged_causal_attn_decode_cuda);
  m.impl("paged_causal_attn_decode_kvfp8", &paged_causal_attn_decode_kvfp8_cuda);
  m.impl("flash_attention_naive_prefill", &flash_attention_naive_prefill_cuda);
  m.impl("flash_attention_naive_decode", &flash_attention_naive_decode_cuda);
}
