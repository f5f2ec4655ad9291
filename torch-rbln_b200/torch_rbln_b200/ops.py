"""Python entry points for the rbln_custom_ops paged-attention ops.

Thin wrappers over torch.ops.rbln_custom_ops.* that keep the reference
frontends' argument-count contract (torch_rbln/_internal/
register_custom_ops.py:175-560: "takes 10 inputs" / "takes 9 or 10 inputs"
RuntimeErrors). Model code may call either these or torch.ops directly.
"""

from __future__ import annotations

import torch

_ops = torch.ops.rbln_custom_ops


def _count(name: str, args: tuple, lo: int, hi: int) -> None:
    if not (lo <= len(args) <= hi):
        want = f"{lo}" if lo == hi else f"{lo} or {hi}"
        raise RuntimeError(f"{name} takes {want} inputs, but got {len(args)}.")


def paged_attn_prefill(*args):
    _count("paged_attn_prefill", args, 10, 10)
    return _ops.paged_attn_prefill(*args)


def paged_attn_decode(*args):
    _count("paged_attn_decode", args, 10, 10)
    return _ops.paged_attn_decode(*args)


def paged_causal_attn_prefill(*args):
    _count("paged_causal_attn_prefill", args, 10, 11)
    return _ops.paged_causal_attn_prefill(*args)


def paged_causal_attn_decode(*args):
    _count("paged_causal_attn_decode", args, 9, 10)
    return _ops.paged_causal_attn_decode(*args)


def paged_causal_attn_decode_kvfp8(*args):
    _count("paged_causal_attn_decode_kvfp8", args, 11, 12)
    return _ops.paged_causal_attn_decode_kvfp8(*args)


def flash_attention_naive_prefill(*args):
    _count("flash_attention_naive_prefill", args, 9, 10)
    return _ops.flash_attention_naive_prefill(*args)


def flash_attention_naive_decode(*args):
    _count("flash_attention_naive_decode", args, 9, 10)
    return _ops.flash_attention_naive_decode(*args)
