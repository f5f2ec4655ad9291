"""Pins the CPU oracle to the reference's own outputs (tests/golden/*.pt).

The fixtures were produced by running the reference's CPU definitions
(test/rbln/test_custom_kernel.py:31-486 and sdpa.py:_sdpa_cpu_fallback) in
tests/golden/make_golden.py. The oracle's mode="mock" must match them bit
for bit on the reference's single-block configurations; mode="fp32" must
match within the reference's own tolerance (test_custom_kernel.py:654-655).
"""

import hashlib
import math
import os

import pytest
import torch

from oracle import paged_attention as opa
from oracle import sdpa as osd

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
RTOL, ATOL = 1e-3, 1.2e-2


def _tol(dtype):
    """The reference's tolerance (test_custom_kernel.py:654-655, float16). The
    reference's bfloat16 path rounds the scores to bfloat16 (8-bit mantissa),
    so its distance from an exact fp32 evaluation is wider."""
    return dict(rtol=1.6e-2, atol=3e-2) if dtype == torch.bfloat16 else dict(rtol=RTOL, atol=ATOL)


def _load(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _full(pre, max_seq):
    B, H, one, P, D = pre.shape
    c = torch.zeros([B, H, one, max_seq, D], dtype=pre.dtype)
    c[:, :, :, :P] = pre
    return c


DECODE = _load("paged_decode.pt")
PREFILL = _load("paged_prefill.pt")


@pytest.mark.parametrize("idx", range(len(DECODE)))
@pytest.mark.parametrize("op", ["paged_attn_decode", "paged_causal_attn_decode", "paged_causal_attn_decode_pmask"])
def test_decode_oracle_matches_reference(idx, op):
    c = DECODE[idx]
    exp = c["results"][op]
    scale = torch.tensor(1.0 / math.sqrt(c["D"]))
    bt = torch.tensor([[0], [1]], dtype=torch.int16)
    mask = {"paged_attn_decode": c["mask"], "paged_causal_attn_decode": None,
            "paged_causal_attn_decode_pmask": c["pmask"]}[op]
    for mode in ("mock", "fp32"):
        kc, vc = _full(c["kpre"], c["max_seq"]), _full(c["vpre"], c["max_seq"])
        out = opa.paged_decode(c["q"], c["k"], c["v"], kc, vc, c["ctx"], scale, bt, c["max_seq"], mask, mode=mode)
        if mode == "mock":
            assert out.dtype == exp["out"].dtype and out.shape == exp["out"].shape
            assert torch.equal(out, exp["out"]), f"max diff {(out.float() - exp['out'].float()).abs().max()}"
        else:
            torch.testing.assert_close(out, exp["out"].float(), **_tol(c["dtype"]))
        rows_k = torch.stack([kc[b, :, 0, int(c["ctx"][b, 0])] for b in range(c["B"])])
        rows_v = torch.stack([vc[b, :, 0, int(c["ctx"][b, 0])] for b in range(c["B"])])
        assert torch.equal(rows_k, exp["krow"]) and torch.equal(rows_v, exp["vrow"])


@pytest.mark.parametrize("idx", range(len(PREFILL)))
@pytest.mark.parametrize("op", ["paged_attn_prefill_s0", "paged_attn_prefill_s1", "paged_causal_attn_prefill",
                                "paged_causal_attn_prefill_bidir"])
def test_prefill_oracle_matches_reference(idx, op):
    c = PREFILL[idx]
    exp = c["results"][op]
    D, S, ms, dt = c["D"], c["S"], c["max_seq"], c["dtype"]
    scale = torch.tensor(1.0 / math.sqrt(D))
    bt = torch.tensor([0], dtype=torch.int16)
    for mode in ("mock", "fp32"):
        kc = torch.zeros([1, c["Hkv"], 1, ms, D], dtype=dt)
        vc = torch.zeros_like(kc)
        kw = {}
        if op == "paged_attn_prefill_s0":
            kw["mask"] = torch.ones([1, S, ms], dtype=dt).tril().view(1, 1, 1, S, ms)
        elif op == "paged_attn_prefill_s1":
            s1 = c["s1"]
            kc[:, :, :, :s1] = c["kpre"]
            vc[:, :, :, :s1] = c["vpre"]
            kw["mask"] = torch.ones([1, S, ms], dtype=dt).tril(diagonal=s1).view(1, 1, 1, S, ms)
        elif op == "paged_causal_attn_prefill":
            kw["causal"] = True
        else:
            pm = torch.zeros([1, ms], dtype=dt)
            pm[:, :S] = 1
            kw["causal"] = False
            kw["position_mask"] = pm
        seq = torch.tensor([[exp["seq"]]], dtype=torch.int32)
        out = opa.paged_prefill(c["q"], c["k"], c["v"], kc, vc, seq, scale, bt, ms, mode=mode, **kw)
        if mode == "mock":
            assert torch.equal(out, exp["out"]), f"max diff {(out.float() - exp['out'].float()).abs().max()}"
        else:
            torch.testing.assert_close(out, exp["out"].float(), **_tol(dt))
        assert _sha(kc) == exp["kc"] and _sha(vc) == exp["vc"]


def test_offset_causal_equals_explicit_mask():
    """paged_causal_attn_prefill's offset-causal rule (the generalisation) equals
    the reference's paged_attn_prefill driven by an offset tril keep-mask."""
    c = PREFILL[0]
    D, S, ms, dt, s1 = c["D"], c["S"], c["max_seq"], c["dtype"], c["s1"]
    scale = torch.tensor(1.0 / math.sqrt(D))
    bt = torch.tensor([0], dtype=torch.int16)
    seq = torch.tensor([[s1]], dtype=torch.int32)
    kc = torch.zeros([1, c["Hkv"], 1, ms, D], dtype=dt)
    vc = torch.zeros_like(kc)
    kc[:, :, :, :s1], vc[:, :, :, :s1] = c["kpre"], c["vpre"]
    out = opa.paged_prefill(c["q"], c["k"], c["v"], kc.clone(), vc.clone(), seq, scale, bt, ms, causal=True,
                            mode="mock")
    assert torch.equal(out, c["results"]["paged_attn_prefill_s1"]["out"])


SDPA = _load("sdpa_small.pt")


@pytest.mark.parametrize("idx", range(len(SDPA)))
def test_sdpa_oracle_matches_reference(idx):
    c = SDPA[idx]
    out = osd.sdpa_reference(c["q"], c["k"], c["v"], c["mask"], 0.0, c["causal"], None)
    assert torch.equal(out, c["out"])
    ref = osd.sdpa_math(c["q"], c["k"], c["v"], c["mask"], c["causal"])
    tol = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-2}[c["dtype"]]
    assert (out.double() - ref).abs().max() / ref.abs().max() < tol


def sdpa_config1_inputs():
    g = torch.Generator().manual_seed(0)
    q = torch.randn([1, 32, 512, 64], generator=g)
    k = torch.randn([1, 8, 512, 64], generator=g)
    v = torch.randn([1, 8, 512, 64], generator=g)
    return q, k, v


def test_sdpa_config1_oracle_matches_reference():
    fx = _load("sdpa_config1.pt")
    q, k, v = sdpa_config1_inputs()
    assert (_sha(q), _sha(k), _sha(v)) == (fx["sha_q"], fx["sha_k"], fx["sha_v"])
    out = osd.sdpa_reference(q, k, v, None, 0.0, True, 1.0 / 8.0)
    assert torch.equal(out[0][fx["heads"]][:, fx["rows"]], fx["out_sample"])
    assert out.double().sum().item() == fx["out_sum"].item()
    ref = osd.sdpa_math(q, k, v, None, True, 1.0 / 8.0)
    assert ((out.double() - ref).abs().max() / ref.abs().max()).item() < 1e-5


def test_paged_block_table_gather_is_a_permutation():
    """Scattering a contiguous cache through a random block table and reading it
    back through the oracle reproduces the contiguous result exactly."""
    g = torch.Generator().manual_seed(3)
    B, Hkv, G, D, bs, nblk = 3, 2, 4, 64, 16, 40
    max_blocks = 8
    q = torch.randn([B, Hkv, G, 1, D], generator=g)
    k = torch.randn([B, Hkv, 1, 1, D], generator=g)
    v = torch.randn([B, Hkv, 1, 1, D], generator=g)
    seq = torch.tensor([[5], [77], [127]], dtype=torch.int32)
    perm = torch.randperm(nblk, generator=g)[: B * max_blocks].reshape(B, max_blocks).to(torch.int32)
    kp = torch.randn([nblk, Hkv, 1, bs, D], generator=g)
    vp = torch.randn([nblk, Hkv, 1, bs, D], generator=g)
    out_paged = opa.paged_decode(q, k, v, kp.clone(), vp.clone(), seq, 0.125, perm, bs)
    # same data laid out contiguously, one block per sequence
    kc = torch.stack([opa.contiguous_cache(kp, perm, bs, b, D)[0] for b in range(B)])
    vc = torch.stack([opa.contiguous_cache(vp, perm, bs, b, D)[0] for b in range(B)])
    bt = torch.arange(B, dtype=torch.int32).reshape(B, 1)
    out_contig = opa.paged_decode(q, k, v, kc, vc, seq, 0.125, bt, max_blocks * bs)
    assert torch.equal(out_paged, out_contig)


@pytest.mark.parametrize("idx", range(len(DECODE)))
@pytest.mark.parametrize("op", ["paged_attn_decode", "paged_causal_attn_decode", "paged_causal_attn_decode_pmask"])
def test_contiguous_mock_restatement_matches_reference(idx, op):
    """The CPU-baseline restatement (reference layout) equals the reference bit for bit."""
    c = DECODE[idx]
    exp = c["results"][op]
    mask = {"paged_attn_decode": c["mask"], "paged_causal_attn_decode": None,
            "paged_causal_attn_decode_pmask": c["pmask"]}[op]
    kc, vc = _full(c["kpre"], c["max_seq"]), _full(c["vpre"], c["max_seq"])
    out = opa.mock_decode_contiguous(c["q"], c["k"], c["v"], kc, vc, c["ctx"], torch.tensor(1.0 / math.sqrt(c["D"])),
                                     mask)
    assert torch.equal(out, exp["out"])


@pytest.mark.parametrize("idx", range(len(PREFILL)))
def test_contiguous_prefill_restatement_matches_reference(idx):
    """The prefill CPU-baseline restatement equals the reference bit for bit."""
    c = PREFILL[idx]
    exp = c["results"]["paged_attn_prefill_s1"]
    D, S, ms, dt, s1 = c["D"], c["S"], c["max_seq"], c["dtype"], c["s1"]
    kc = torch.zeros([1, c["Hkv"], 1, ms, D], dtype=dt)
    vc = torch.zeros_like(kc)
    kc[:, :, :, :s1], vc[:, :, :, :s1] = c["kpre"], c["vpre"]
    mask = torch.ones([1, S, ms], dtype=dt).tril(diagonal=s1).view(1, 1, 1, S, ms)
    out = opa.mock_prefill_contiguous(c["q"], c["k"], c["v"], kc, vc, s1, torch.tensor(1.0 / math.sqrt(D)), mask)
    assert torch.equal(out, exp["out"])
    assert _sha(kc) == exp["kc"] and _sha(vc) == exp["vc"]


NAIVE = _load("flash_attention_naive.pt")


@pytest.mark.parametrize("idx", range(len(NAIVE)))
def test_flash_attention_naive_oracle_matches_reference(idx):
    """flash_attention_naive_{prefill,decode} (test_custom_kernel.py:546-645):
    the keep-mask paged restatement over kv_cache[0] / kv_cache[1] equals the
    reference's single-partition definition, output and mutated cache."""
    c = NAIVE[idx]
    exp = c["results"]
    scale = torch.tensor(1.0 / math.sqrt(c["D"]))
    seq_idx = torch.tensor([[c["s0"]]], dtype=torch.int32)
    bt = torch.tensor([[0]], dtype=torch.int16) if c["decode"] else torch.tensor([0], dtype=torch.int16)
    for mode in ("mock", "fp32"):
        kv = c["kv_cache"].clone()
        out = opa.flash_attention_naive(c["q"], c["k"], c["v"], kv, c["mask"], scale, seq_idx, bt,
                                        decode=c["decode"], mode=mode)
        if mode == "mock":
            assert out.dtype == exp["out"].dtype and out.shape == exp["out"].shape
            assert torch.equal(out, exp["out"]), f"max diff {(out.float() - exp['out'].float()).abs().max()}"
        else:
            torch.testing.assert_close(out, exp["out"].float(), **_tol(c["dtype"]))
        assert _sha(kv) == exp["kv_cache"]


def test_sinks_oracle_properties():
    """Attention-sink restatement: a sink of -inf is no sink; a sink is the
    softmax over the scores plus one extra logit whose column is dropped, so
    out(sink) = out(no sink) * Z / (Z + e^sink) per query head, Z the sum of
    e^score over the kept positions."""
    c = NAIVE[0]
    scale = 1.0 / math.sqrt(c["D"])
    seq_idx = torch.tensor([[c["s0"]]], dtype=torch.int32)
    bt = torch.tensor([0], dtype=torch.int16)
    H = c["Hkv"] * c["G"]
    gen = torch.Generator().manual_seed(7)
    sinks = torch.randn(H, generator=gen) * 2

    def run(s):
        kv = c["kv_cache"].clone()
        return opa.flash_attention_naive(c["q"], c["k"], c["v"], kv, c["mask"], scale, seq_idx, bt, s,
                                         decode=False)

    base = run(None)
    assert torch.equal(run(torch.full([H], -float("inf"))), base)
    with_sink = run(sinks)
    # Z per (head, query row): recompute the scores of the written cache
    kv = c["kv_cache"].clone()
    run_kv = opa.flash_attention_naive(c["q"], c["k"], c["v"], kv, c["mask"], scale, seq_idx, bt, decode=False)
    assert torch.equal(run_kv, base)
    K = kv[0, 0, :, 0].float()  # [Hkv, P, D]
    w = torch.matmul(c["q"][0].float(), K.unsqueeze(1).transpose(-1, -2)) * scale  # [Hkv, G, S, P]
    keep = c["mask"][0, 0, 0] > 0
    Z = torch.where(keep, w.exp(), torch.zeros_like(w)).sum(-1, keepdim=True)  # [Hkv, G, S, 1]
    e = sinks.reshape(c["Hkv"], c["G"], 1, 1).exp()
    torch.testing.assert_close(with_sink[0], base[0] * Z / (Z + e), rtol=1e-5, atol=1e-6)


SDPA_BWD = _load("sdpa_bwd.pt")


@pytest.mark.parametrize("idx", range(len(SDPA_BWD)))
def test_sdpa_backward_oracle_matches_reference(idx):
    """The backward restatement equals the reference's own backward entry
    point (sdpa.py:754-821, run on CPU tensors) bit for bit: dq, dk, dv and
    grad_attn_bias. For float32 the exact float64 evaluation agrees to 1e-4."""
    c = SDPA_BWD[idx]
    got = osd.sdpa_backward_reference(c["grad_out"], c["q"], c["k"], c["v"], c["mask"], c["causal"], None,
                                      grad_bias=c["mask"] is not None)
    for name, g in zip(("dq", "dk", "dv", "dbias"), got):
        if c[name] is None:
            assert g is None
            continue
        assert g.dtype == c[name].dtype and torch.equal(g, c[name]), name
    if c["dtype"] == torch.float32:
        ex = osd.sdpa_backward_math(c["grad_out"], c["q"], c["k"], c["v"], c["mask"], c["causal"], None)
        for name, e in zip(("dq", "dk", "dv", "dbias"), ex):
            if c[name] is not None:
                torch.testing.assert_close(c[name].double(), e.expand_as(c[name]), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("idx", range(len(PREFILL)))
def test_kv_write_matches_reference_prefill_writes(idx):
    """The standalone write (oracle.kv_write) leaves the caches exactly as the
    reference's paged_attn_prefill leaves them (fixture digests), at seq 0 and
    at seq s1 over a cache already holding s1 rows."""
    c = PREFILL[idx]
    D, ms, dt, s1 = c["D"], c["max_seq"], c["dtype"], c["s1"]
    bt = torch.tensor([0], dtype=torch.int16)
    for key, s0 in (("paged_attn_prefill_s0", 0), ("paged_attn_prefill_s1", s1)):
        kc = torch.zeros([1, c["Hkv"], 1, ms, D], dtype=dt)
        vc = torch.zeros_like(kc)
        if s0:
            kc[:, :, :, :s1], vc[:, :, :, :s1] = c["kpre"], c["vpre"]
        opa.kv_write(c["k"], c["v"], kc, vc, torch.tensor([[s0]], dtype=torch.int32), bt, ms)
        assert _sha(kc) == c["results"][key]["kc"] and _sha(vc) == c["results"][key]["vc"]


def test_kv_write_fp8_oracle_properties():
    """The fp8 write rule (oracle.kv_write; the reference has no fp8 cache, so
    it is checked by its defining properties): every touched (block, head)
    scale is max(amax of its valid rows, 1e-6) / 448; the new rows dequantize
    to within e4m3 rounding (relative 2^-4, absolute 2^-9 * scale near 0);
    rows past the write are untouched; repeating a write changes nothing."""
    g = torch.Generator().manual_seed(11)
    B, Hkv, D, bs, S = 2, 2, 64, 16, 21
    nblk, mb = 12, 5
    bt = torch.randperm(nblk, generator=g)[: B * mb].reshape(B, mb).to(torch.int32)
    kc = opa.quantize_fp8(torch.randn(nblk, Hkv, 1, bs, D, generator=g), torch.ones(1))
    vc, ks, vs = kc.clone(), torch.ones(nblk, Hkv), torch.ones(nblk, Hkv)
    seq = torch.tensor([3, 16], dtype=torch.int32)  # mid-block start with held rows; block-aligned start
    k = torch.randn(B, Hkv, 1, S, D, generator=g).to(torch.bfloat16) * 3
    v = torch.randn(B, Hkv, 1, S, D, generator=g).to(torch.bfloat16)
    before = kc.clone()
    held_deq = {}
    for b in range(B):
        s0 = int(seq[b])
        blk = int(bt[b, s0 // bs])
        held_deq[b] = kc[blk, :, 0, : s0 % bs].float() * ks[blk].reshape(Hkv, 1, 1)
    opa.kv_write(k, v, kc, vc, seq, bt, bs, ks, vs)
    for b in range(B):
        s0 = int(seq[b])
        for i in range(S):
            p = s0 + i
            blk, row = int(bt[b, p // bs]), p % bs
            deq = kc[blk, :, 0, row].float() * ks[blk].reshape(Hkv, 1)
            x = k[b, :, 0, i].float()
            tol = 2.0 ** -4 * x.abs() + 2.0 ** -9 * ks[blk].reshape(Hkv, 1)
            assert bool(((deq - x).abs() <= tol).all())
        for bi in range(s0 // bs, (s0 + S - 1) // bs + 1):
            blk = int(bt[b, bi])
            lo, hi = max(s0, bi * bs) - bi * bs, min(s0 + S, (bi + 1) * bs) - bi * bs
            new = k[b, :, 0, bi * bs + lo - s0: bi * bs + hi - s0].float().abs().amax(dim=(1, 2))
            if bi == s0 // bs and s0 % bs:
                new = torch.maximum(new, held_deq[b].abs().amax(dim=(1, 2)))
            assert torch.equal(ks[blk], torch.clamp(new, min=1e-6) / opa.FP8_MAX)
            assert torch.equal(kc[blk, :, 0, hi:].view(torch.uint8), before[blk, :, 0, hi:].view(torch.uint8))
    snap = (kc.clone(), vc.clone(), ks.clone(), vs.clone())
    opa.kv_write(k, v, kc, vc, seq, bt, bs, ks, vs)
    assert torch.equal(kc.view(torch.uint8), snap[0].view(torch.uint8))
    assert torch.equal(vc.view(torch.uint8), snap[1].view(torch.uint8))
    assert torch.equal(ks, snap[2]) and torch.equal(vs, snap[3])


def test_sinks_decode_oracle_fully_masked_and_limits():
    """Decode with sinks: a sequence with no visible position gives 0 (all
    softmax mass on the sink) where it gives NaN without sinks; a sink of
    -inf changes nothing; a very large sink drives every output to 0."""
    c = NAIVE[2]  # a decode case
    assert c["decode"]
    scale = 1.0 / math.sqrt(c["D"])
    seq_idx = torch.tensor([[c["s0"]]], dtype=torch.int32)
    bt = torch.tensor([[0]], dtype=torch.int16)
    H = c["Hkv"] * c["G"]

    def run(mask, s):
        kv = c["kv_cache"].clone()
        return opa.flash_attention_naive(c["q"], c["k"], c["v"], kv, mask, scale, seq_idx, bt, s, decode=True)

    none = torch.zeros_like(c["mask"])
    assert torch.isnan(run(none, None)).all()
    assert torch.count_nonzero(run(none, torch.zeros(H))) == 0
    base = run(c["mask"], None)
    assert torch.equal(run(c["mask"], torch.full([H], -float("inf"))), base)
    assert run(c["mask"], torch.full([H], 1e4)).abs().max() < 1e-30
