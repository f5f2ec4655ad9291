"""CPU oracle for scaled_dot_product_attention. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.

`sdpa_reference` restates the reference's CPU path for
aten::_scaled_dot_product_fused_attention_overrideable,
`_sdpa_cpu_fallback` (torch_rbln/_internal/kernels/sdpa.py:244-289):
  1. GQA: K/V heads are repeated n_rep = Hq / Hkv times, each KV head's
     copies adjacent (`_repeat_kv`, sdpa.py:180-189);
  2. a bool mask becomes additive (True -> 0, False -> -inf) in q's dtype
     (`_convert_bool_mask_to_float`, sdpa.py:192-206);
  3. float16 is upcast to float32 (other dtypes compute in their own);
  4. torch's CPU scaled_dot_product_attention, then cast back.
Causal masking is top-left aligned (query i sees keys j <= i), as in
torch's CPU kernel and the reference's `_create_causal_mask` (sdpa.py:209-225).

`sdpa_math` is an explicit float64 softmax(Q K^T * scale + mask) V with the
same conventions, used to cross-check the reference path and as the
tolerance reference for float32 inputs.
"""

from __future__ import annotations

import math
from typing import Optional

import torch


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1 or x.dim() != 4:
        return x
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, n_rep, s, d).reshape(b, h * n_rep, s, d)


def bool_mask_to_additive(mask: Optional[torch.Tensor], dtype: torch.dtype) -> Optional[torch.Tensor]:
    if mask is None or mask.dtype != torch.bool:
        return mask
    return torch.where(mask, torch.zeros((), dtype=dtype), torch.full((), float("-inf"), dtype=dtype))


def sdpa_reference(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None):
    q, k, v = query.cpu(), key.cpu(), value.cpu()
    if q.dim() == 4 and k.dim() == 4 and q.size(1) != k.size(1) and q.size(1) % k.size(1) == 0:
        n = q.size(1) // k.size(1)
        k, v = repeat_kv(k, n), repeat_kv(v, n)
    m = bool_mask_to_additive(attn_mask.cpu() if attn_mask is not None else None, q.dtype)
    dt = q.dtype
    cd = torch.float32 if dt == torch.float16 else dt
    out = torch._C._nn.scaled_dot_product_attention(
        q.to(cd), k.to(cd), v.to(cd), attn_mask=m.to(cd) if m is not None else None,
        dropout_p=dropout_p, is_causal=is_causal, scale=scale, enable_gqa=False)
    return out.to(dt)


def sdpa_math(query, key, value, attn_mask=None, is_causal=False, scale=None, dtype=torch.float64,
              return_lse=False):
    q, k, v = query.to(dtype), key.to(dtype), value.to(dtype)
    if q.dim() == 4 and q.size(1) != k.size(1):
        n = q.size(1) // k.size(1)
        k, v = repeat_kv(k, n), repeat_kv(v, n)
    L, S = q.size(-2), k.size(-2)
    s = scale if scale is not None else 1.0 / math.sqrt(q.size(-1))
    w = torch.matmul(q, k.transpose(-1, -2)) * s
    if is_causal:
        keep = torch.ones(L, S, dtype=torch.bool).tril()
        w = w.masked_fill(~keep, float("-inf"))
    if attn_mask is not None:
        if attn_mask.dtype == torch.bool:
            w = w.masked_fill(~attn_mask, float("-inf"))
        else:
            w = w + attn_mask.to(dtype)
    lse = torch.logsumexp(w, dim=-1)
    out = torch.matmul(torch.softmax(w, dim=-1), v)
    return (out, lse) if return_lse else out


def sdpa_backward_reference(grad_out, query, key, value, attn_mask=None, is_causal=False, scale=None,
                            grad_bias=False, upcast_f16=True):
    """aten::_scaled_dot_product_fused_attention_overrideable_backward as the
    reference computes it on the CPU (torch_rbln/_internal/kernels/sdpa.py):

      * attention weights recomputed by `_sdpa_attn_weights_fallback`
        (:393-431): float16 upcast to float32 (others stay in their dtype),
        GQA by `_repeat_kv`, scores * scale, a top-left causal -inf triangle
        added, the mask added (in the compute dtype), softmax, then cast back
        to the input dtype;
      * gradients by `_sdpa_backward_fallback` (:614-667), in the same
        compute dtype: dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(dP * P))
        * scale, dQ = dS K, dK = dS^T Q, GQA sums over each KV head's query
        heads, cast back;
      * grad_attn_bias (:800-818) = P * (dP - rowsum(dP * P)) in the input
        dtype (no upcast) from the cast-back weights, when asked for and a
        mask is given.

    upcast_f16=False runs the same op sequence in the input dtype for float16
    too: the arithmetic of a half-precision backward, used by the tests as
    the error yardstick for the tensor-core kernels.
    Returns (dq, dk, dv, dbias or None).
    """
    dt = query.dtype
    cd = torch.float32 if (dt == torch.float16 and upcast_f16) else dt
    q, k, v, go = query.cpu().to(cd), key.cpu().to(cd), value.cpu().to(cd), grad_out.cpu().to(cd)
    L, S = q.size(-2), k.size(-2)
    s = scale if scale is not None else 1.0 / math.sqrt(q.size(-1))
    n_rep = q.size(1) // k.size(1) if q.dim() == 4 else 1
    kx, vx = repeat_kv(k, n_rep), repeat_kv(v, n_rep)
    # _sdpa_attn_weights_fallback: the mask arrives already additive (the
    # forward converted a bool mask, sdpa.py:192-206)
    m = bool_mask_to_additive(attn_mask.cpu(), dt) if attn_mask is not None else None
    w = torch.matmul(q, kx.transpose(-2, -1)) * s
    if is_causal:
        w = w + torch.triu(torch.full((L, S), float("-inf"), dtype=cd), diagonal=1)
    if m is not None:
        w = w + m.to(cd)
    p = torch.softmax(w, dim=-1).to(dt).to(cd)
    # _sdpa_backward_fallback
    dv = torch.matmul(p.transpose(-2, -1), go)
    dp = torch.matmul(go, vx.transpose(-2, -1))
    sum_term = (dp * p).sum(dim=-1, keepdim=True)
    ds = p * (dp - sum_term) * s
    dq = torch.matmul(ds, kx)
    dk = torch.matmul(ds.transpose(-2, -1), q)
    if n_rep > 1:
        B, Hkv, D = k.size(0), k.size(1), k.size(-1)
        dk = dk.view(B, Hkv, n_rep, S, D).sum(dim=2)
        dv = dv.view(B, Hkv, n_rep, S, D).sum(dim=2)
    dbias = None
    if grad_bias and attn_mask is not None:
        pw, gv = p.to(dt), repeat_kv(value.cpu(), n_rep)
        gw = torch.matmul(grad_out.cpu(), gv.transpose(-2, -1))
        dbias = pw * (gw - (gw * pw).sum(dim=-1, keepdim=True))
    return dq.to(dt), dk.to(dt), dv.to(dt), dbias


def sdpa_backward_math(grad_out, query, key, value, attn_mask=None, is_causal=False, scale=None,
                       dtype=torch.float64):
    """The same gradients evaluated exactly (float64, no intermediate
    rounding): the tolerance reference. Returns (dq, dk, dv, dbias)."""
    q = query.cpu().to(dtype).requires_grad_(True)
    k = key.cpu().to(dtype).requires_grad_(True)
    v = value.cpu().to(dtype).requires_grad_(True)
    m = None
    if attn_mask is not None:
        m = attn_mask.cpu()
        m = m if m.dtype == torch.bool else m.to(dtype).requires_grad_(True)
    with torch.enable_grad():
        out = sdpa_math(q, k, v, m, is_causal=is_causal, scale=scale, dtype=dtype)
        out.backward(grad_out.cpu().to(dtype))
    dbias = m.grad if (m is not None and m.dtype != torch.bool) else None
    return q.grad, k.grad, v.grad, dbias
