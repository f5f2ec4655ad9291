/*
 * rbln_attn.h — C-ABI of the B200 (sm_100a) attention kernels behind the
 * torch-rbln attention hot path.
 *
 * Every entry point takes a plain-old-data parameter struct (device pointers,
 * element strides, shapes, dtype codes) and a cudaStream_t, launches its
 * kernels on that stream without any host synchronisation, allocates nothing
 * (scratch memory is passed in by the caller; ask the *_workspace_size query
 * for its size), throws nothing, and returns an rbln_status_t.
 *
 * Tensor layouts follow the reference's custom-op contract
 * (test/rbln/test_custom_kernel.py:31-486, torch_rbln/_internal/
 * register_custom_ops.py:154-450):
 *   q, out        [B, Hkv, G, S_q, D]     (S_q = 1 for decode)
 *   k, v (new)    [B, Hkv, 1, S_q, D]
 *   kcache,vcache [num_blocks, Hkv, 1, block_size, D_cache >= D]
 *   seq           [B, 1] int32   decode: position of the new token
 *                                prefill: start offset of the chunk
 *   block_table   [B, max_blocks] int16/int32/int64
 * The innermost dimension of every tensor must be contiguous and every row
 * must start on a 16-byte boundary.
 */
#ifndef RBLN_ATTN_H_
#define RBLN_ATTN_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RBLN_ATTN_ABI_VERSION 3

typedef enum {
  RBLN_OK = 0,
  RBLN_ERR_INVALID_ARGUMENT = -1, /* null pointer, bad shape/stride/alignment */
  RBLN_ERR_UNSUPPORTED = -2,      /* valid, but not a configuration built here */
  RBLN_ERR_WORKSPACE = -3,        /* workspace missing or too small */
  RBLN_ERR_LAUNCH = -4,           /* cudaLaunch* reported an error */
  RBLN_ERR_NO_DEVICE = -5,        /* no sm_100 device current */
  RBLN_ERR_SCRATCH_LIMIT = -6     /* needs more than the fixed no-allocation scratch */
} rbln_status_t;

typedef enum {
  RBLN_DT_F32 = 0,
  RBLN_DT_F16 = 1,
  RBLN_DT_BF16 = 2,
  RBLN_DT_FP8_E4M3 = 3,
  RBLN_DT_I16 = 4,
  RBLN_DT_I32 = 5,
  RBLN_DT_I64 = 6,
  RBLN_DT_BOOL = 7 /* one byte, non-zero = keep */
} rbln_dtype_t;

/* Device-side error bits, OR-ed into *error_flags when a kernel meets an
 * input it must not dereference. The access is skipped (the position is
 * treated as masked) and the kernel carries on. */
#define RBLN_DEVERR_BLOCK_ID_RANGE 0x1u /* block_table entry outside [0, num_blocks) */
#define RBLN_DEVERR_SEQ_RANGE 0x2u      /* seq < 0, or a write past the table's span */
#define RBLN_DEVERR_TIMEOUT 0x4u        /* a pipeline wait gave up (the CTA returned early) */

/* Paged attention over a block-table-indexed KV cache: one parameter block
 * serves decode (S_q = 1) and chunked prefill (S_q >= 1). */
typedef struct {
  /* shapes */
  int32_t batch;        /* B */
  int32_t num_kv_heads; /* Hkv */
  int32_t group;        /* G = query heads per KV head */
  int32_t q_len;        /* S_q (1 for decode) */
  int32_t head_dim;     /* D: 64 or 128 */
  int32_t num_blocks;   /* physical blocks in the pool (kcache.size(0)) */
  int32_t block_size;   /* tokens per block */
  int32_t max_blocks;   /* block_table.size(1); span = max_blocks*block_size */

  /* query / output, dtype q_dtype (F16 or BF16), strides in elements */
  const void* q;
  int64_t q_stride[4]; /* b, h, g, s */
  void* out;
  int64_t out_stride[4];
  int32_t q_dtype;

  /* new keys/values to append (same dtype as q); NULL = no append */
  const void* k_new;
  const void* v_new;
  int64_t k_new_stride[3]; /* b, h, s */
  int64_t v_new_stride[3];

  /* paged caches: dtype kv_dtype (F16, BF16 or FP8_E4M3) */
  void* kcache;
  void* vcache;
  int32_t kv_dtype;
  int64_t cache_stride[3]; /* block, head, token (same for K and V) */
  /* fp8 only: one fp32 dequant scale per (block, head), K and V separately
   * (read-only for attention; rbln_paged_kv_write rewrites the touched ones) */
  const float* k_scale;
  const float* v_scale;
  int64_t scale_stride[2]; /* block, head */

  const int32_t* seq;
  int64_t seq_stride;
  const void* block_table;
  int32_t block_table_dtype; /* I16, I32 or I64 */
  int64_t block_table_stride;

  /* optional keep-mask (value > 0 keeps the position); NULL = causal/length.
   * decode:  [B, mask_len]          (mask_stride[0] = batch stride)
   * prefill: [B, S_q, mask_len]     (mask_stride = batch, query row) */
  const void* mask;
  int32_t mask_dtype;
  int32_t mask_len;
  int64_t mask_stride[2];
  int32_t causal;        /* prefill: 1 = causal offset by seq[b], 0 = bidirectional */

  float scale;            /* softmax scale, used when scale_dev == NULL */
  const float* scale_dev; /* optional device pointer to an fp32 scale */

  void* workspace;        /* caller-allocated scratch (see *_workspace_size) */
  size_t workspace_bytes;
  uint32_t* error_flags;  /* optional device word, see RBLN_DEVERR_* */
  int32_t num_splits;     /* 0 = heuristic; else context splits per sequence */
  /* optional cudaEvent_t pair recorded on `stream` right before and right
   * after the main attention kernel (measurement hook; NULL = none) */
  void* prof_events[2];
  /* optional attention-sink logits, fp32 [num_kv_heads * group] (index
   * h * group + g), in the units of scale * q.k: each query head's softmax
   * gets one extra term exp(sink) that carries no value row, so
   * out = sum_i e^{s_i} v_i / (sum_i e^{s_i} + e^{sink}). NULL = none.
   * Schema argument `sinks` of flash_attention_naive_{prefill,decode}
   * (torch_rbln/_internal/register_custom_ops.py:453-560). */
  const float* sinks;
} rbln_paged_attn_params_t;

/* ABI checks for foreign-function bindings. */
int rbln_attn_abi_version(void);
size_t rbln_paged_attn_params_sizeof(void);

/* Scratch needed by the decode entry points for these parameters. */
int rbln_paged_decode_workspace_size(const rbln_paged_attn_params_t* p, size_t* bytes);

/* rbln_custom_ops::paged_causal_attn_decode
 * (reference frontend torch_rbln/_internal/register_custom_ops.py:409-450,
 *  CPU semantics test/rbln/test_custom_kernel.py:388-486).
 * Appends k_new/v_new at position seq[b] (when seq[b] < span), then attends
 * the G query heads of every KV head over positions [0, min(seq[b]+1, span)),
 * or over the positions whose mask value is > 0 when p->mask is set. */
int rbln_paged_causal_attn_decode(const rbln_paged_attn_params_t* p, cudaStream_t stream);

/* rbln_custom_ops::paged_attn_decode
 * (reference frontend register_custom_ops.py:253-293,
 *  CPU semantics test_custom_kernel.py:138-216).
 * Same append; attention over the positions whose mask value is > 0.
 * p->mask is required. */
int rbln_paged_attn_decode(const rbln_paged_attn_params_t* p, cudaStream_t stream);

/* Optional scratch for the prefill entry points: when p->workspace holds
 * this many bytes, a pre-pass orders the (sequence, query-tile) work items
 * longest first before the attention kernel runs; without it the kernel
 * uses a fixed order. 0 when no pre-pass applies. */
int rbln_paged_prefill_workspace_size(const rbln_paged_attn_params_t* p, size_t* bytes);

/* rbln_custom_ops::paged_causal_attn_prefill
 * (reference frontend register_custom_ops.py:324-379,
 *  CPU semantics test_custom_kernel.py:262-343).
 * Writes k_new/v_new at positions [seq[b], seq[b] + S_q), then attends query
 * row s (absolute position seq[b] + s) over keys t <= seq[b] + s
 * (p->causal = 1) or t < seq[b] + S_q (p->causal = 0, "is_bidirectional");
 * p->mask, when set, is an extra [B, L] keep-mask over keys.
 * bf16/f16 only, q and caches of one dtype, D in {64, 128}, block_size in
 * {8, 16, 32, 64, 128} or a multiple of 128. No workspace. */
int rbln_paged_causal_attn_prefill(const rbln_paged_attn_params_t* p, cudaStream_t stream);

/* rbln_custom_ops::paged_attn_prefill
 * (reference frontend register_custom_ops.py:175-229,
 *  CPU semantics test_custom_kernel.py:31-92).
 * Same write; attention keeps key t for query row s when
 * mask[b, s, t] > 0 (p->mask required, mask_stride = {batch, query row}). */
int rbln_paged_attn_prefill(const rbln_paged_attn_params_t* p, cudaStream_t stream);

/* Paged KV-cache write on its own: k_new/v_new [B, Hkv, S = q_len, D]
 * (strides b, h, s in k_new_stride / v_new_stride) written at positions
 * [seq[b], seq[b] + S) through the block table -- the append step of the
 * decode and prefill ops (reference CPU semantics test_custom_kernel.py:63-79,
 * 182-186), for a cache filled without attending in the same call. q_dtype
 * is the dtype of k_new / v_new (BF16 / F16). kv_dtype equal to it: a copy.
 * kv_dtype FP8_E4M3 with k_scale / v_scale [num_blocks, Hkv]: every touched
 * (block, head) gets scale = max(amax, 1e-6) / 448 over its valid rows (those
 * the sequence already holds before seq[b], and the new ones); held rows are
 * re-quantized to the new scale, new rows quantized as x * (1 / scale) in
 * float32 (round to nearest even, saturated). Rows past the write are left
 * as they are.
 * No reference counterpart as a separate entry point. */
int rbln_paged_kv_write(const rbln_paged_attn_params_t* p, cudaStream_t stream);

/* Dense scaled dot-product attention, forward. */
typedef struct {
  int32_t batch, num_heads, num_kv_heads, q_len, kv_len, head_dim; /* GQA: num_heads % num_kv_heads == 0 */
  int32_t dtype;          /* F32, F16 or BF16, shared by q, k, v and out */
  const void* q;          /* [B, Hq, L, D]; strides in elements: b, h, l (d contiguous) */
  int64_t q_stride[3];
  const void* k;          /* [B, Hkv, S, D] */
  int64_t k_stride[3];
  const void* v;
  int64_t v_stride[3];
  void* out;              /* [B, Hq, L, D] */
  int64_t out_stride[3];
  float* lse;             /* optional [B, Hq, L] fp32 natural-log logsumexp */
  int64_t lse_stride[3];
  const void* mask;       /* optional [B|1, Hq|1, L, S] */
  int32_t mask_dtype;     /* BOOL (keep) or F32/F16/BF16 */
  int32_t mask_additive;  /* 1: float mask added to the scores; 0: value > 0 keeps */
  int64_t mask_stride[4]; /* b, h, l, s (s stride must be 1 for F16/BF16 inputs) */
  int32_t causal;         /* top-left: query l sees keys s <= l */
  float scale;
  uint32_t* error_flags;
} rbln_sdpa_params_t;

/* aten::_scaled_dot_product_fused_attention_overrideable, forward
 * (reference torch_rbln/_internal/kernels/sdpa.py:670-751; math of
 * _sdpa_cpu_fallback, sdpa.py:244-289). bf16/f16 on the tensor cores,
 * f32 exactly in fp32. D in {64, 128}. */
int rbln_sdpa_fwd(const rbln_sdpa_params_t* p, cudaStream_t stream);

/* Dense scaled dot-product attention, backward. Shapes and strides as for
 * the forward; every tensor's last dim contiguous, rows 16-byte aligned. */
typedef struct {
  int32_t batch, num_heads, num_kv_heads, q_len, kv_len, head_dim;
  int32_t dtype;          /* F16 or BF16, shared by every tensor below except lse / dbias */
  const void* q;          /* [B, Hq, L, D] */
  int64_t q_stride[3];
  const void* k;          /* [B, Hkv, S, D] */
  int64_t k_stride[3];
  const void* v;
  int64_t v_stride[3];
  const void* out;        /* forward output [B, Hq, L, D] */
  int64_t out_stride[3];
  const void* dout;       /* gradient of the output [B, Hq, L, D] */
  int64_t dout_stride[3];
  const float* lse;       /* forward logsumexp [B, Hq, L] (natural log; -inf for a row with no key) */
  int64_t lse_stride[3];
  void* dq;               /* [B, Hq, L, D]; NULL: not computed */
  int64_t dq_stride[3];
  void* dk;               /* [B, Hkv, S, D] (summed over the query heads of each KV head); NULL: not computed */
  int64_t dk_stride[3];
  void* dv;               /* [B, Hkv, S, D]; NULL: not computed */
  int64_t dv_stride[3];
  const void* mask;       /* as in rbln_sdpa_params_t */
  int32_t mask_dtype;
  int32_t mask_additive;
  int64_t mask_stride[4];
  float* dbias;           /* optional fp32 [B, Hq, L, S] contiguous: gradient of the additive mask (needs mask) */
  int32_t causal;
  float scale;
  void* workspace;        /* rbln_sdpa_bwd_workspace_size bytes */
  size_t workspace_bytes;
  uint32_t* error_flags;
} rbln_sdpa_bwd_params_t;

/* Scratch for rbln_sdpa_bwd: one {lse, rowsum(dout * out)} pair per query row. */
int rbln_sdpa_bwd_workspace_size(const rbln_sdpa_bwd_params_t* p, size_t* bytes);

/* aten::_scaled_dot_product_fused_attention_overrideable_backward
 * (reference torch_rbln/_internal/kernels/sdpa.py:754-821 with the math of
 * _sdpa_backward_fallback, sdpa.py:614-667, and grad_attn_bias at :800-818):
 * with P the forward's attention weights (recomputed from q, k and lse),
 *   dv = P^T dout, dS = P * (dout v^T - rowsum(dout * out)),
 *   dq = scale * dS k, dk = scale * dS^T q, dbias = dS,
 * GQA gradients summed over each KV head's query heads. bf16/f16 on the
 * tensor cores, D in {64, 128}. */
int rbln_sdpa_bwd(const rbln_sdpa_bwd_params_t* p, cudaStream_t stream);

/* No counterpart in the reference: a variant of rbln_paged_causal_attn_decode
 * for callers that cannot allocate device memory -- for example a runtime
 * that has handed all device memory to its own pool at start-up, or a
 * plugin whose host framework forbids allocation while work is enqueued
 * (cudaMalloc may also synchronise the device, which a latency-bound decode
 * loop cannot afford). Same semantics and parameters; p->workspace and
 * p->workspace_bytes are ignored. Its split-K scratch is a fixed array of
 * RBLN_NOALLOC_SCRATCH_BYTES in device memory, owned by this library and held
 * on every GPU that loads it until the process exits. Requests that need
 * more return RBLN_ERR_SCRATCH_LIMIT and launch nothing.
 * The first call on each device looks up the array's device address (with
 * that device current); make that first call before any stream capture. A
 * lookup that fails returns RBLN_ERR_LAUNCH and is tried again on the next
 * call; a successful one is kept for the life of the process, so do not call
 * this entry point after cudaDeviceReset (the kept address belongs to the
 * context that the reset destroyed).
 * All calls share the one array: calls that overlap on the GPU (other
 * streams, other threads) race on it and must be serialised by the caller.
 * Nothing in it needs to start at zero: every partial the merge step reads
 * is written earlier in the same call. Allocates nothing. */
#define RBLN_NOALLOC_SCRATCH_BYTES (16u << 20)
int rbln_paged_causal_attn_decode_noalloc(const rbln_paged_attn_params_t* p, cudaStream_t stream);

/* ---- KV-head-sharded decode with the head outputs written over NVLink ----
 * No counterpart in the reference's C++ (its only collective is an
 * all-gather through ProcessGroupRBLN, torch_rbln/csrc/distributed/c10d/rbln/
 * ProcessGroupRBLN.cpp:754-830): one process per GPU owns a slice of the KV
 * heads, and the decode kernels store each final head output straight into
 * every rank's full output buffer (peer memory mapped with CUDA IPC), then
 * the last CTA of the merge kernel (or, on the per-sequence split grid, a
 * one-warp kernel) exchanges a per-call epoch through every rank's flag
 * array and waits until all ranks' writes are in. The wait is bounded by
 * wait_limit_us: on expiry it ORs RBLN_DEVERR_TIMEOUT into p->error_flags
 * and returns, and the remote heads of that call's output are not valid.
 * This replaces the decode + all-gather + re-layout copy. */
#define RBLN_IPC_HANDLE_BYTES 64
typedef struct rbln_peer_out {
  void* const* out;       /* device array [n]: every rank's full output buffer, mapped on this GPU */
  uint32_t* const* flags; /* device array [n]: every rank's flag array (n uint32), mapped on this GPU */
  int32_t n;              /* ranks */
  int32_t rank;           /* this rank */
  int32_t head0;          /* first KV head of this rank in the full output */
  uint32_t epoch;         /* this call's epoch; strictly increasing over calls (flags start at 0) */
  uint32_t wait_limit_us; /* longest wait for the peers' epochs, in microseconds of GPU time;
                             0 = 2,000,000 (2 s). ABI version 3 added this field. */
} rbln_peer_out_t;

size_t rbln_peer_out_sizeof(void);

/* Device memory that other processes can map: cudaMalloc of `bytes` (zeroed)
 * and its IPC handle (RBLN_IPC_HANDLE_BYTES bytes). Free with rbln_ipc_free. */
int rbln_ipc_alloc(size_t bytes, void** ptr, void* handle);
int rbln_ipc_free(void* ptr);
/* Maps another process's rbln_ipc_alloc buffer into this process (current
 * device; peer access enabled lazily). Unmap with rbln_ipc_close. */
int rbln_ipc_open(const void* handle, void** ptr);
int rbln_ipc_close(void* ptr);

/* rbln_paged_causal_attn_decode on this rank's KV heads (p describes the
 * local heads: num_kv_heads, q, k/v, caches), with the output of local head
 * h written to head peers->head0 + h of every rank's full output buffer;
 * p->out must be this rank's own full buffer and p->out_stride its strides
 * (all ranks' buffers have the same layout). When the stream reaches the end
 * of this call, every rank's buffer holds all heads of this epoch (no host
 * synchronisation). Buffers reused across calls must alternate (at least two
 * per rank): a rank may run one call ahead of the others. */
int rbln_paged_causal_attn_decode_peers(const rbln_paged_attn_params_t* p, const rbln_peer_out_t* peers,
                                        cudaStream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* RBLN_ATTN_H_ */
