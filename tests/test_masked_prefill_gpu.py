"""Masked chunked prefill on the 128-key tcgen05 kernel.

paged_attn_prefill (keep-mask), paged_causal_attn_prefill with a position
mask, and flash_attention_naive_prefill run a mask pre-pass (keep bits per
query row and 128-key tile; tiles with no kept key skipped, fully kept tiles
unmasked) when the call has its workspace, which the torch ops always pass.
Checked against the fp32 oracle with the reference's tolerance (rtol 1e-3,
atol 1.2e-2, test/rbln/test_custom_kernel.py:654-655); a row with no kept
key is NaN on both sides (softmax over nothing), or 0 with an attention sink.
"""

import math

import pytest
import torch

from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1.2e-2
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch_rbln_b200  # noqa: F401


def make(B, Hkv, G, D, bs, S, starts, seed, extra_blocks=2, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    max_blocks = math.ceil((max(starts) + S) / bs) + extra_blocks
    nblk = B * max_blocks + 3
    bt = torch.randperm(nblk, generator=g)[: B * max_blocks].reshape(B, max_blocks).to(torch.int32)
    d = dict(q=torch.randn([B, Hkv, G, S, D], generator=g).to(dtype),
             k=torch.randn([B, Hkv, 1, S, D], generator=g).to(dtype),
             v=torch.randn([B, Hkv, 1, S, D], generator=g).to(dtype),
             kcache=torch.randn([nblk, Hkv, 1, bs, D], generator=g).to(dtype),
             vcache=torch.randn([nblk, Hkv, 1, bs, D], generator=g).to(dtype),
             seq=torch.tensor(starts, dtype=torch.int32).reshape(B, 1), block_table=bt, block_size=bs,
             scale=torch.tensor(1.0 / math.sqrt(D)))
    return d, max_blocks * bs


def to_dev(d):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) and k != "scale" else v) for k, v in d.items()}


def gpu_keep(d, mask):
    x = to_dev(d)
    out = torch.ops.rbln_custom_ops.paged_attn_prefill(x["q"], x["k"], x["v"], mask.to(DEV), x["kcache"], x["vcache"],
                                                       x["seq"], x["scale"], x["block_table"], x["block_size"])
    torch.cuda.synchronize()
    return out.cpu(), x["kcache"].cpu(), x["vcache"].cpu()


def oracle_keep(d, mask, sinks=None):
    kc, vc = d["kcache"].clone(), d["vcache"].clone()
    out = opa.paged_prefill(d["q"], d["k"], d["v"], kc, vc, d["seq"], d["scale"], d["block_table"], d["block_size"],
                            mask=mask, sinks=sinks)
    return out, kc, vc


def check(got, ref):
    torch.testing.assert_close(got[0].float(), ref[0], rtol=RTOL, atol=ATOL, equal_nan=True)
    assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2])


def tile_pattern_mask(B, S, span, seed):
    """A keep-mask [B, 1, 1, S, span] whose 128-key tiles are, per 64-row
    band, all dropped, all kept, random, or an offset-causal staircase."""
    g = torch.Generator().manual_seed(seed)
    m = torch.zeros(B, S, span)
    for b in range(B):
        for r0 in range(0, S, 64):
            for t0 in range(0, span, 128):
                kind = int(torch.randint(0, 4, (1,), generator=g))
                blk = m[b, r0:r0 + 64, t0:t0 + 128]
                if kind == 1:
                    blk.fill_(1.0)
                elif kind == 2:
                    blk.copy_((torch.rand(blk.shape, generator=g) > 0.5).float())
                elif kind == 3:
                    rr = torch.arange(blk.shape[0]).reshape(-1, 1)
                    tt = torch.arange(blk.shape[1]).reshape(1, -1)
                    blk.copy_((tt <= rr + int(torch.randint(0, 128, (1,), generator=g))).float())
    return m.reshape(B, 1, 1, S, span)


@pytest.mark.parametrize("G,D,bs", [(4, 128, 16), (8, 64, 32), (1, 128, 128), (2, 64, 8)])
def test_keep_mask_tile_classes(G, D, bs):
    """Skipped, fully kept and partly kept tiles in one call, over kept keys
    anywhere in the span (before, inside and after the chunk)."""
    B, Hkv, S, starts = 3, 2, 200, [0, 300, 777]
    d, span = make(B, Hkv, G, D, bs, S, starts, seed=G * 100 + D + bs)
    mask = tile_pattern_mask(B, S, span, seed=5 + G).to(torch.bfloat16)
    check(gpu_keep(d, mask), oracle_keep(d, mask))


@pytest.mark.parametrize("mdtype", [torch.float32, torch.float16, torch.bool])
def test_keep_mask_random_and_empty_rows(mdtype):
    """Random keep bits, a mask shorter than the span, and rows with no kept
    key (NaN, as the reference's softmax over -inf everywhere)."""
    B, Hkv, G, D, bs, S, starts = 2, 2, 4, 128, 16, 150, [40, 500]
    d, span = make(B, Hkv, G, D, bs, S, starts, seed=21)
    g = torch.Generator().manual_seed(22)
    L = span - 37
    m = torch.rand(B, 1, 1, S, L, generator=g) > 0.3
    m[:, :, :, 5] = False   # query row 5: nothing kept
    m[1, :, :, 77] = False  # one more, in one sequence only
    mask = m if mdtype == torch.bool else m.to(mdtype)
    got = gpu_keep(d, mask)
    check(got, oracle_keep(d, mask))
    assert torch.isnan(got[0][:, :, :, 5]).all() and torch.isnan(got[0][1, :, :, 77]).all()
    assert torch.isfinite(got[0][0, :, :, 77]).all()


def test_offset_causal_keep_mask_equals_causal_op_bitwise():
    """An offset-causal keep-mask visits the same key tiles and masks the
    same keys as the causal op on the same kernel: bit-identical output."""
    B, Hkv, G, D, bs, S, starts = 2, 2, 4, 128, 16, 256, [130, 1000]
    d, span = make(B, Hkv, G, D, bs, S, starts, seed=31)
    t = torch.arange(span).reshape(1, 1, span)
    qi = torch.arange(S).reshape(1, S, 1) + torch.tensor(starts).reshape(B, 1, 1)
    keep = (t <= qi).to(torch.bfloat16).reshape(B, 1, 1, S, span)
    got_keep = gpu_keep(d, keep)
    x = to_dev(d)
    causal = torch.ops.rbln_custom_ops.paged_causal_attn_prefill(x["q"], x["k"], x["v"], x["kcache"], x["vcache"],
                                                                 x["seq"], x["scale"], x["block_table"], bs, False)
    torch.cuda.synchronize()
    assert torch.equal(got_keep[0], causal.cpu())
    check(got_keep, oracle_keep(d, keep))


def test_masked_kernel_matches_the_one_tile_fallback():
    """Without its workspace a keep-mask call runs on the one-tile kernel;
    both agree within the stated tolerance (different tilings)."""
    from torch_rbln_b200 import cabi

    B, Hkv, G, D, bs, S, starts = 2, 2, 4, 128, 16, 180, [64, 900]
    d, span = make(B, Hkv, G, D, bs, S, starts, seed=41)
    mask = tile_pattern_mask(B, S, span, seed=42).to(torch.bfloat16)
    outs = []
    for use_ws in (False, True):
        x = to_dev(d)
        md = mask.to(DEV)
        p, keep = cabi.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"], bs,
                                    float(x["scale"]), mask=md)
        if use_ws:
            cabi.attach_workspace(p, DEV, keep, prefill=True)
            assert p.workspace_bytes > 0
        assert cabi.call("rbln_paged_attn_prefill", p) == cabi.OK
        torch.cuda.synchronize()
        outs.append(keep["out"].cpu().float())
    torch.testing.assert_close(outs[1], outs[0], rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(outs[1], oracle_keep(d, mask)[0], rtol=RTOL, atol=ATOL)


def test_position_mask_with_empty_tiles():
    """paged_causal_attn_prefill with a position mask that drops whole 128-key
    tiles of the cached context."""
    B, Hkv, G, D, bs, S, starts = 2, 2, 4, 128, 16, 100, [700, 260]
    d, span = make(B, Hkv, G, D, bs, S, starts, seed=51)
    pm = torch.ones(B, span, dtype=torch.bfloat16)
    pm[:, 128:384] = 0      # two whole tiles dropped
    pm[0, 10:20] = 0        # part of a tile
    x = to_dev(d)
    out = torch.ops.rbln_custom_ops.paged_causal_attn_prefill(x["q"], x["k"], x["v"], x["kcache"], x["vcache"],
                                                              x["seq"], x["scale"], x["block_table"], bs, False,
                                                              pm.to(DEV))
    torch.cuda.synchronize()
    kc, vc = d["kcache"].clone(), d["vcache"].clone()
    ref = opa.paged_prefill(d["q"], d["k"], d["v"], kc, vc, d["seq"], d["scale"], d["block_table"], bs, causal=True,
                            position_mask=pm)
    check((out.cpu(), x["kcache"].cpu(), x["vcache"].cpu()), (ref, kc, vc))


@pytest.mark.parametrize("masked", [False, True])
def test_sinks_on_the_128_key_kernel(masked):
    """Attention sinks in the 128-key kernel's epilogue: the mask-free causal
    path (C-ABI, sinks set) and the keep-mask path, with rows that see no key
    giving 0 instead of NaN."""
    from torch_rbln_b200 import cabi

    B, Hkv, G, D, bs, S, starts = 2, 2, 4, 128, 16, 140, [0, 333]
    d, span = make(B, Hkv, G, D, bs, S, starts, seed=61)
    sinks = torch.randn(Hkv * G, generator=torch.Generator().manual_seed(62)) * 2.0
    x = to_dev(d)
    mask = None
    if masked:
        mask = tile_pattern_mask(B, S, span, seed=63).to(torch.bfloat16)
        mask[:, :, :, 9] = 0  # a row with no kept key
    p, keep = cabi.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"], bs,
                                float(x["scale"]), mask=None if mask is None else mask.to(DEV))
    cabi.attach_workspace(p, DEV, keep, prefill=True)
    sk = sinks.to(DEV)
    p.sinks = sk.data_ptr()
    assert cabi.call("rbln_paged_attn_prefill" if masked else "rbln_paged_causal_attn_prefill", p) == cabi.OK
    torch.cuda.synchronize()
    kc, vc = d["kcache"].clone(), d["vcache"].clone()
    ref = opa.paged_prefill(d["q"], d["k"], d["v"], kc, vc, d["seq"], d["scale"], d["block_table"], bs,
                            mask=mask, causal=True, sinks=sinks)
    got = keep["out"].cpu()
    torch.testing.assert_close(got.float(), ref, rtol=RTOL, atol=ATOL)
    if masked:
        assert (got[:, :, :, 9] == 0).all()
