"""CPU oracle for the paged-attention custom ops. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only to check or time against it. No product code path imports
it.

It restates, in torch CPU ops, the reference's own CPU definition of the four
rbln_custom_ops paged ops (test/rbln/test_custom_kernel.py, the "simplified
mock implementations" of optimum-rbln's operators):

  paged_attn_prefill         test_custom_kernel.py:31-92
  paged_attn_decode          test_custom_kernel.py:138-216
  paged_causal_attn_prefill  test_custom_kernel.py:262-343
  paged_causal_attn_decode   test_custom_kernel.py:388-486
  flash_attention_naive_{prefill,decode}
                             test_custom_kernel.py:546-645 (unified cache
                             kv_cache[0] = K pool, kv_cache[1] = V pool)

The reference's CPU definitions only cover one physical block per sequence
(prefill always uses block 0, decode uses kcache[b]; block_table and
block_size are ignored). This restatement generalises them to a real block
table, which is what the CUDA kernels implement:

  * position t of sequence b lives in block block_table[b, t // block_size],
    row t % block_size; the addressable span is max_blocks * block_size;
  * new k/v rows are written first (decode: at seq[b] when seq[b] < span,
    like test_custom_kernel.py:182-186; prefill: at [seq[b], seq[b] + S_q)),
    then read back (write-then-read);
  * causal prefill masks key t for query i when t > seq[b] + i (the
    reference's tril at :326-331 has no seq offset and is only right for
    seq[b] == 0); bidirectional prefill attends [0, seq[b] + S_q);
  * an fp8-e4m3 cache holds x / scale[block, head] (saturated to +-448);
    it is read as float(e4m3) * scale[block, head];
  * a block_table entry outside [0, num_blocks) makes its positions masked
    (the CUDA kernels skip such reads and raise a device error flag).

Two arithmetic modes:
  mode="mock": the op sequence of the reference (scores in q.dtype, fp32
      softmax, probabilities rounded to q.dtype, P.V in q.dtype). On the
      reference's own single-block configurations this equals the reference
      bit for bit (tests/test_oracle_golden.py pins it).
  mode="fp32": every product in float32 with no intermediate rounding; the
      tolerance reference for the CUDA kernels.
"""

from __future__ import annotations

from typing import Optional

import torch

FP8_MAX = 448.0


def span_of(block_table: torch.Tensor, block_size: int) -> int:
    return int(block_table.shape[-1]) * int(block_size)


def _bt_row(block_table: torch.Tensor, b: int) -> torch.Tensor:
    bt = block_table if block_table.dim() == 2 else block_table.reshape(1, -1)
    return bt[b if bt.shape[0] > 1 else 0].to(torch.int64)


def _locate(block_table: torch.Tensor, b: int, pos: torch.Tensor, block_size: int, num_blocks: int):
    """Physical (block, row, valid) of logical positions `pos` of sequence b."""
    row = _bt_row(block_table, b)
    blk = row[pos // block_size]
    valid = (blk >= 0) & (blk < num_blocks)
    return blk.clamp(0, max(num_blocks - 1, 0)), pos % block_size, valid


def quantize_fp8(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """x / scale, saturated to the e4m3 range, rounded to nearest even."""
    return (x.float() / scale.float()).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def _write_rows(cache, new, block_table, b, positions, block_size, scale=None):
    """Writes new[:, i, :D] (per KV head) at logical positions[i] of sequence b."""
    num_blocks = cache.shape[0]
    span = span_of(block_table, block_size)
    D = new.shape[-1]
    for i, t in enumerate(positions.tolist()):
        if t < 0 or t >= span:
            continue
        blk, off, ok = _locate(block_table, b, torch.tensor([t]), block_size, num_blocks)
        if not bool(ok[0]):
            continue
        blk, off = int(blk[0]), int(off[0])
        rows = new[:, i, :D]  # [Hkv, D]
        if cache.dtype == torch.float8_e4m3fn:
            rows = quantize_fp8(rows, scale[blk].reshape(-1, 1))
        cache[blk, :, 0, off, :D] = rows.to(cache.dtype)


def _gather(cache, block_table, b, span, block_size, D, scale=None):
    """Per-sequence view [Hkv, span, D] of the paged cache (+ validity)."""
    pos = torch.arange(span)
    blk, off, ok = _locate(block_table, b, pos, block_size, cache.shape[0])
    rows = cache[blk, :, 0, off, :D]  # [span, Hkv, D]
    if cache.dtype == torch.float8_e4m3fn:
        rows = rows.float() * scale[blk].float().unsqueeze(-1)
    return rows.permute(1, 0, 2), ok


def _attend(q, K, V, keep, scale, mode, sinks=None):
    """softmax(q.K^T * scale | keep) . V for one sequence.

    q [Hkv, G, S, D], K/V [Hkv, T, D], keep [S, T] bool -> [Hkv, G, S, D].
    sinks [Hkv * G] (fp32 mode only): one extra logit per query head that
    joins the softmax and carries no value row (the attention-sink form,
    out = sum_t e^{w_t} V_t / (sum_t e^{w_t} + e^{sink})).
    """
    if mode == "mock":
        # the reference's CPU definitions take `sinks` but do not read it
        # (test_custom_kernel.py:589-594)
        assert sinks is None, "mode='mock' follows the reference, which ignores sinks"
        dt = q.dtype
        Kc, Vc = K.to(dt), V.to(dt)
        # matmul in q.dtype, then `* scale` (test_custom_kernel.py:87,199)
        w = torch.matmul(q, Kc.unsqueeze(1).transpose(-1, -2)) * scale
        add = torch.where(keep, 0.0, -float("inf"))  # float32, like :88,204
        w = w + add
        p = torch.nn.functional.softmax(w, dim=-1, dtype=torch.float32).to(dt)
        return torch.matmul(p, Vc.unsqueeze(1))
    qf, Kf, Vf = q.float(), K.float(), V.float()
    w = torch.matmul(qf, Kf.unsqueeze(1).transpose(-1, -2)) * float(scale)
    w = w.masked_fill(~keep, -float("inf"))
    if sinks is not None:
        Hkv, G, S = w.shape[:3]
        sk = sinks.float().reshape(Hkv, G, 1, 1).expand(Hkv, G, S, 1)
        p = torch.softmax(torch.cat([w, sk], dim=-1), dim=-1)[..., :-1]
    else:
        p = torch.softmax(w, dim=-1)
    return torch.matmul(p, Vf.unsqueeze(1))


def paged_decode(q, k, v, kcache, vcache, seq, scale, block_table, block_size,
                 mask: Optional[torch.Tensor] = None, *, k_scale=None, v_scale=None,
                 mode: str = "fp32", sinks: Optional[torch.Tensor] = None) -> torch.Tensor:
    """paged_causal_attn_decode (mask=None or [B, L]) / paged_attn_decode (mask [B,1,1,1,L]).

    Mutates kcache/vcache. Returns [B, Hkv, G, 1, D] in q.dtype (mode="mock")
    or float32 (mode="fp32").
    """
    B, Hkv, G, S, D = q.shape
    assert S == 1
    span = span_of(block_table, block_size)
    seqv = seq.reshape(-1).to(torch.int64)
    outs = []
    for b in range(B):
        p = int(seqv[b])
        if p >= 0:
            _write_rows(kcache, k[b, :, 0], block_table, b, torch.tensor([p]), block_size, k_scale)
            _write_rows(vcache, v[b, :, 0], block_table, b, torch.tensor([p]), block_size, v_scale)
        K, okk = _gather(kcache, block_table, b, span, block_size, D, k_scale)
        V, _ = _gather(vcache, block_table, b, span, block_size, D, v_scale)
        t = torch.arange(span)
        if mask is not None:
            mrow = mask[b if mask.shape[0] > 1 else 0].reshape(-1)
            L = min(span, mrow.numel())
            keep = torch.zeros(span, dtype=torch.bool)
            keep[:L] = mrow[:L] > 0
        else:
            L = min(p + 1, span) if p >= 0 else 0
            keep = t < L
        keep = (keep & okk).reshape(1, span)
        outs.append(_attend(q[b], K, V, keep, scale, mode, sinks))
    out = torch.stack(outs, 0)
    return out if mode == "mock" else out.float()


def paged_prefill(q, k, v, kcache, vcache, seq, scale, block_table, block_size,
                  mask: Optional[torch.Tensor] = None, *, causal: bool = True,
                  position_mask: Optional[torch.Tensor] = None, mode: str = "fp32",
                  sinks: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Chunked prefill over a paged cache.

    paged_attn_prefill:        mask = keep-mask [B|1, 1, 1, S_q, L], causal ignored.
    paged_causal_attn_prefill: mask=None, causal = not is_bidirectional,
                               position_mask = optional [B|1, L] keep-mask.
    Mutates kcache/vcache. Returns [B, Hkv, G, S_q, D].
    """
    B, Hkv, G, S, D = q.shape
    span = span_of(block_table, block_size)
    seqv = seq.reshape(-1).to(torch.int64)
    outs = []
    for b in range(B):
        s0 = int(seqv[b if seqv.numel() > 1 else 0])
        pos = torch.arange(S) + s0
        _write_rows(kcache, k[b, :, 0], block_table, b, pos, block_size)
        _write_rows(vcache, v[b, :, 0], block_table, b, pos, block_size)
        K, okk = _gather(kcache, block_table, b, span, block_size, D)
        V, _ = _gather(vcache, block_table, b, span, block_size, D)
        t = torch.arange(span).reshape(1, span)
        qi = pos.reshape(S, 1)
        if mask is not None:
            m = mask[b if mask.shape[0] > 1 else 0].reshape(-1, mask.shape[-1])[-S:]  # [S, L]
            L = min(span, m.shape[-1])
            keep = torch.zeros(S, span, dtype=torch.bool)
            keep[:, :L] = m[:, :L] > 0
        elif causal:
            keep = t <= qi
        else:
            keep = (t < s0 + S).expand(S, span)
        if position_mask is not None:
            pm = position_mask[b if position_mask.shape[0] > 1 else 0].reshape(-1)
            L = min(span, pm.numel())
            pk = torch.zeros(span, dtype=torch.bool)
            pk[:L] = pm[:L] > 0
            keep = keep & pk.reshape(1, span)
        keep = keep & okk.reshape(1, span)
        outs.append(_attend(q[b], K, V, keep, scale, mode, sinks))
    out = torch.stack(outs, 0)
    return out if mode == "mock" else out.float()


def flash_attention_naive(q, k, v, kv_cache, mask, scale, seq_idx, block_tables,
                          sinks: Optional[torch.Tensor] = None, *, decode: bool,
                          mode: str = "fp32") -> torch.Tensor:
    """flash_attention_naive_prefill (decode=False) / _decode (decode=True).

    The reference's CPU definition (test_custom_kernel.py:546-573) handles a
    single partition: it writes k/v into block block_tables[0] at offset
    seq_idx[0][0] of both halves of kv_cache, then attends over the
    partition's positions under `mask[..., :partition] > 0` (fp32 softmax,
    probabilities rounded to q.dtype). The general form is the keep-mask
    paged op over kv_cache[0] / kv_cache[1] with block_size = partition and
    seq = seq_idx[:, 0]; on a single partition the two coincide op for op.
    Mutates kv_cache.
    """
    block_size = kv_cache.shape[-2]
    seq = seq_idx.reshape(seq_idx.shape[0], -1)[:, 0] if seq_idx.dim() > 0 else seq_idx.reshape(1)
    kc, vc = kv_cache[0], kv_cache[1]
    if decode:
        return paged_decode(q, k, v, kc, vc, seq, scale, block_tables, block_size, mask=mask,
                            mode=mode, sinks=sinks)
    return paged_prefill(q, k, v, kc, vc, seq, scale, block_tables, block_size, mask=mask,
                         mode=mode, sinks=sinks)


def contiguous_cache(kcache, block_table, block_size, b, D, scale=None):
    """Gathers sequence b of a paged cache into the reference's per-sequence
    layout [1, Hkv, 1, span, D] (used to feed the CPU baseline)."""
    span = span_of(block_table, block_size)
    K, _ = _gather(kcache, block_table, b, span, block_size, D, scale)
    return K.unsqueeze(0).unsqueeze(2)


def mock_decode_contiguous(q, k, v, kcache, vcache, seq, scale, mask=None):
    """The reference's CPU decode on its own layout, op for op
    (test_custom_kernel.py:431-486 for mask=None or [B, L];
    :178-216 when `mask` is [B, 1, 1, 1, L]).

    kcache/vcache: [B, Hkv, 1, max_seq, D] contiguous per-sequence caches
    (cache b belongs to sequence b). Mutates the caches; returns q.dtype.
    This is the CPU path the benchmark times as the baseline.
    """
    B, Hkv, G, _, D = q.shape
    max_seq = kcache.shape[-2]
    outs = []
    for b in range(B):
        p = int(seq[b, 0])
        if p < max_seq:
            kcache[b, :, :, p, :] = k[b].squeeze(-2)
            vcache[b, :, :, p, :] = v[b].squeeze(-2)
        ks = kcache[b].unsqueeze(0)[..., :D].unsqueeze(2)
        vs = vcache[b].unsqueeze(0)[..., :D].unsqueeze(2)
        qi = q[b].view(Hkv, 1, G, 1, D)
        w = torch.matmul(qi, ks.transpose(-1, -2)) * scale
        if mask is not None and mask.dim() == 5:
            add = torch.where(mask[b, :, :, :, :max_seq] > 0, 0.0, -float("inf"))
        elif mask is not None:
            add = torch.where(mask[b:b + 1].view(1, 1, 1, 1, -1)[..., :max_seq] > 0, 0.0, -float("inf"))
        else:
            n = min(p + 1, max_seq)
            add = torch.full((1, max_seq), -float("inf"), dtype=q.dtype)
            add[:, :n] = 0.0
            add = add.view(1, 1, 1, 1, max_seq)
        w = torch.softmax(w + add, dim=-1, dtype=torch.float32).to(q.dtype)
        outs.append(torch.matmul(w, vs).view(Hkv, G, 1, D))
    return torch.stack(outs, 0)


def mock_prefill_contiguous(q, k, v, kcache, vcache, s, scale, keep_mask):
    """The reference's CPU prefill on its own layout, op for op
    (test_custom_kernel.py:72-92): one sequence, caches [1, Hkv, 1, max_seq, D],
    new rows written at [s, s + S_q), keep_mask [1, 1, 1, S_q, max_seq].
    Mutates the caches; returns q.dtype. This is the CPU path the benchmark
    times as the prefill baseline."""
    partition = kcache.size(-2)
    S = q.size(-2)
    D = k.size(-1)
    kcache[0].unsqueeze(0)[:, :, :, s:s + S, :D].copy_(k[:, :, :, :, :D])
    vcache[0].unsqueeze(0)[:, :, :, s:s + S, :D].copy_(v[:, :, :, :, :D])
    ks = kcache[0].unsqueeze(0)[..., :D]
    vs = vcache[0].unsqueeze(0)[..., :D]
    w = torch.matmul(q, ks.transpose(3, 4)) * scale
    w = w + torch.where(keep_mask[:, :, :, :, :partition] > 0, 0.0, -float("inf"))
    w = torch.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(w, vs)


def kv_write(k_new, v_new, kcache, vcache, seq, block_table, block_size, k_scale=None, v_scale=None):
    """The paged ops' append step on its own (what rbln_paged_kv_write does).

    k_new / v_new [B, Hkv, 1, S, D] go to positions [seq[b], seq[b] + S) of
    each sequence through the block table (test_custom_kernel.py:63-79 writes
    the same rows into the reference's single block). A bf16 / f16 cache
    takes the values as they are. An fp8-e4m3 cache with scales
    [num_blocks, Hkv]: for every (block, head) the write touches,
      amax  = max(|float(e4m3) * old_scale| over the rows the sequence holds
                  in the block before seq[b], |new values|)
      scale = max(amax, 1e-6) / 448
    held rows become e4m3(float(e4m3) * old_scale * inv), new rows
    e4m3(x * inv), inv = 1 / scale rounded once to float32 (round to nearest
    even after saturating to +-448). Rows past the write stay as they are.
    Mutates the caches (and scales).
    """
    B, Hkv, _, S, D = k_new.shape
    seqv = seq.reshape(-1).to(torch.int64)
    fp8 = kcache.dtype == torch.float8_e4m3fn
    for b in range(B):
        s0 = int(seqv[b])
        row = _bt_row(block_table, b)
        for bi in range(s0 // block_size, (s0 + S - 1) // block_size + 1):
            phys = int(row[bi])
            base = bi * block_size
            lo, hi = max(s0, base) - base, min(s0 + S, base + block_size) - base
            held = lo if s0 > base else 0
            for cache, new, scales in ((kcache, k_new, k_scale), (vcache, v_new, v_scale)):
                rows_new = new[b, :, 0, base + lo - s0: base + hi - s0, :D]  # [Hkv, n, D]
                if not fp8:
                    cache[phys, :, 0, lo:hi, :D] = rows_new.to(cache.dtype)
                    continue
                for h in range(Hkv):
                    old = scales[phys, h].float()
                    deq = cache[phys, h, 0, :held, :D].float() * old
                    nv = rows_new[h].float()
                    amax = torch.cat([deq.abs().reshape(-1), nv.abs().reshape(-1)]).max()
                    sc = torch.clamp(amax, min=1e-6) / FP8_MAX
                    inv = 1.0 / sc

                    def q8(x):
                        return (x * inv).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)

                    if held > 0 and bool(sc != old):
                        cache[phys, h, 0, :held, :D] = q8(deq)
                    cache[phys, h, 0, lo:hi, :D] = q8(nv)
                    scales[phys, h] = sc
