"""Seeded synthetic inputs for the paged-attention ops (shared by tests and bench).

Every tensor is drawn from a torch.Generator on the CPU, so the oracle and
the GPU see the same bits. Shapes follow the reference's op contract
(test/rbln/test_custom_kernel.py): q [B, Hkv, G, S, D], k/v [B, Hkv, 1, S, D],
caches [num_blocks, Hkv, 1, block_size, D], seq [B, 1] int32,
block_table [B, max_blocks].
"""

from __future__ import annotations

import math

import torch


def quantize_pool_fp8(pool: torch.Tensor):
    """Per-(block, head) scale = amax / 448, e4m3 values = x / scale."""
    amax = pool.float().abs().amax(dim=(2, 3, 4)).clamp_min(1e-6)
    scale = (amax / 448.0).contiguous()
    q = (pool.float() / scale[:, :, None, None, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q, scale


def make_decode(B, Hkv, G, D, block_size, lens, num_blocks=None, dtype=torch.bfloat16, seed=0,
                kv_std=0.5, fp8=False, bt_dtype=torch.int32, extra_blocks=1):
    """lens[b] = context length including the new token (seq[b] = lens[b] - 1)."""
    g = torch.Generator().manual_seed(seed)
    max_blocks = max(1, math.ceil(max(lens) / block_size)) + extra_blocks
    if num_blocks is None:
        num_blocks = B * max_blocks + 3
    assert num_blocks >= B * max_blocks
    perm = torch.randperm(num_blocks, generator=g)[: B * max_blocks].reshape(B, max_blocks).to(bt_dtype)
    q = torch.randn([B, Hkv, G, 1, D], generator=g).to(dtype)
    k = (torch.randn([B, Hkv, 1, 1, D], generator=g) * kv_std).to(dtype)
    v = (torch.randn([B, Hkv, 1, 1, D], generator=g) * kv_std).to(dtype)
    kpool = torch.randn([num_blocks, Hkv, 1, block_size, D], generator=g) * kv_std
    vpool = torch.randn([num_blocks, Hkv, 1, block_size, D], generator=g) * kv_std
    seq = (torch.tensor(lens, dtype=torch.int32) - 1).reshape(B, 1)
    out = dict(q=q, k=k, v=v, seq=seq, block_table=perm, block_size=block_size,
               scale=torch.tensor(1.0 / math.sqrt(D)))
    if fp8:
        out["kcache"], out["k_scale"] = quantize_pool_fp8(kpool)
        out["vcache"], out["v_scale"] = quantize_pool_fp8(vpool)
    else:
        out["kcache"], out["vcache"] = kpool.to(dtype), vpool.to(dtype)
    return out


def to_device(d: dict, device) -> dict:
    return {k: (v.to(device) if isinstance(v, torch.Tensor) and k != "scale" else v) for k, v in d.items()}


def clone_caches(d: dict) -> dict:
    e = dict(d)
    e["kcache"], e["vcache"] = d["kcache"].clone(), d["vcache"].clone()
    return e
