"""Parity at the benchmarked configurations' full sizes, on one GPU.

The inputs are built by the benchmark's own builders (bench.py), so these
are exactly the shapes and seeded value distributions that bench.py times:

  * chunked prefill: batch 8, 32 query / 8 KV heads, head_dim 128, 512 new
    tokens per sequence on cached context ~U[0, 8192], block_size 16,
    causal; every sequence checked;
  * long-context decode: batch 32, 64 query / 8 KV heads, context 32768,
    bf16, a 65,536-block pool; 4 seeded sequences checked (all heads);
  * fp8-e4m3 KV decode: batch 256, 32 / 8 heads, context ~U[512, 8192],
    per-(block, head) scales; 16 seeded sequences checked;
  * bf16 decode: batch 64, context ~U[128, 4096], a 20,000-block pool;
    every sequence checked.

The GPU runs the whole batch through the public torch ops; the oracle
(oracle/paged_attention.py, fp32) runs on the checked sequences with their
blocks copied from the GPU's pool. Tolerance: rtol 1e-3, atol 1.2e-2, the
reference's (test/rbln/test_custom_kernel.py:654-655). Appended cache rows
are compared bit for bit.
"""

import math

import pytest
import torch

import bench
from torch_rbln_b200 import sharding

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1.2e-2
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch_rbln_b200  # noqa: F401


def _check_decode(d, out, idx):
    from oracle import paged_attention as opa

    blocks, table = sharding.shard_batch(d["seq"], d["bt"], d["bs"], idx)
    dv = d["kcache"].device
    kc, vc = d["kcache"][blocks.to(dv)].cpu(), d["vcache"][blocks.to(dv)].cpu()
    ks = d["k_scale"][blocks.to(dv)].cpu() if d["fp8"] else None
    vs = d["v_scale"][blocks.to(dv)].cpu() if d["fp8"] else None
    kc_ref, vc_ref = kc.clone(), vc.clone()
    ref = opa.paged_decode(d["q"][idx], d["k"][idx], d["v"][idx], kc_ref, vc_ref, d["seq"][idx], d["scale"], table,
                           d["bs"], k_scale=ks, v_scale=vs, mode="fp32")
    got = out[idx.to(out.device)].cpu().float()
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, ref, rtol=RTOL, atol=ATOL)
    # the GPU appended the new rows before this copy; the oracle's append of
    # the same rows must leave the bytes unchanged
    assert torch.equal(kc_ref.view(torch.uint8), kc.view(torch.uint8))
    assert torch.equal(vc_ref.view(torch.uint8), vc.view(torch.uint8))


def _run_decode(d):
    ops = torch.ops.rbln_custom_ops
    x = {n: d[n].to(DEV) for n in ("q", "k", "v", "seq", "bt")}
    scale = torch.tensor(d["scale"])
    if d["fp8"]:
        out = ops.paged_causal_attn_decode_kvfp8(x["q"], x["k"], x["v"], d["kcache"], d["vcache"], d["k_scale"],
                                                 d["v_scale"], x["seq"], scale, x["bt"], d["bs"])
    else:
        out = ops.paged_causal_attn_decode(x["q"], x["k"], x["v"], d["kcache"], d["vcache"], x["seq"], scale,
                                           x["bt"], d["bs"])
    torch.cuda.synchronize()
    return out


def _subset(B, n, seed):
    return torch.randperm(B, generator=torch.Generator().manual_seed(seed))[:n].sort().values


def test_decode_bf16_full_batch():
    d = bench.build_decode(bench.WORKLOADS["decode"], torch.device(DEV), seed=0)
    out = _run_decode(d)
    _check_decode(d, out, torch.arange(d["B"]))


def test_long_context_decode_full_size():
    d = bench.build_decode(bench.WORKLOADS["decode_long"], torch.device(DEV), seed=0)
    assert d["B"] == 32 and int(d["lens"].min()) == 32768 and d["G"] == 8
    out = _run_decode(d)
    _check_decode(d, out, _subset(d["B"], 4, 11))


def test_fp8_decode_full_size():
    d = bench.build_decode_sharded(bench.WORKLOADS["decode_fp8"], "batch", 0, 1, torch.device(DEV))
    assert d["B"] == 256 and d["fp8"]
    out = _run_decode(d)
    _check_decode(d, out, _subset(d["B"], 16, 12))


def test_chunked_prefill_full_size():
    from oracle import paged_attention as opa

    d = bench.build_prefill(bench.COMPUTE["prefill"], torch.device(DEV), seed=0)
    x = {n: d[n].to(DEV) for n in ("q", "k", "v", "seq", "bt")}
    out = torch.ops.rbln_custom_ops.paged_causal_attn_prefill(x["q"], x["k"], x["v"], d["kcache"], d["vcache"],
                                                              x["seq"], torch.tensor(d["scale"]), x["bt"], d["bs"],
                                                              False)
    torch.cuda.synchronize()
    assert d["B"] == 8 and d["S"] == 512
    for b in range(d["B"]):
        nb = int(math.ceil((int(d["ctx"][b]) + d["S"]) / d["bs"]))
        blocks = d["bt"][b, :nb].long().to(DEV)
        kc, vc = d["kcache"][blocks].cpu(), d["vcache"][blocks].cpu()
        kc_ref, vc_ref = kc.clone(), vc.clone()
        table = torch.arange(nb, dtype=torch.int32).reshape(1, nb)
        ref = opa.paged_prefill(d["q"][b:b + 1], d["k"][b:b + 1], d["v"][b:b + 1], kc_ref, vc_ref,
                                d["seq"][b:b + 1], d["scale"], table, d["bs"], causal=True, mode="fp32")
        got = out[b:b + 1].cpu().float()
        assert torch.isfinite(got).all()
        torch.testing.assert_close(got, ref, rtol=RTOL, atol=ATOL, msg=lambda m: f"sequence {b}: {m}")
        assert torch.equal(kc_ref, kc) and torch.equal(vc_ref, vc), f"sequence {b}: appended rows differ"
