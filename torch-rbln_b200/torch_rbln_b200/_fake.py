"""Fake (meta) kernels: output metadata equals q's, as in the reference's
register_fake functions (test/rbln/test_custom_kernel.py:95-135, 219-259,
346-385, 489-526, 597-645)."""

from __future__ import annotations

import torch

_NAMES = (
    "paged_attn_prefill",
    "paged_attn_decode",
    "paged_causal_attn_prefill",
    "paged_causal_attn_decode",
    "paged_causal_attn_decode_kvfp8",
    "flash_attention_naive_prefill",
    "flash_attention_naive_decode",
)


def _like_q(q, *args, **kwargs):
    return torch.empty_like(q)


for _name in _NAMES:
    if hasattr(torch.ops.rbln_custom_ops, _name):
        torch.library.register_fake(f"rbln_custom_ops::{_name}", _like_q)


def _writes_only(*args, **kwargs):
    """paged_kv_write mutates its caches (and scales) and returns nothing."""
    return None


torch.library.register_fake("rbln_attn::paged_kv_write", _writes_only)
