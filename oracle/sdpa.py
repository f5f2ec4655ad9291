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
