"""Parity of the sm_100a paged-decode kernels with the oracle and the reference.

Tolerance (stated): the reference's own, rtol = 1e-3 and atol = 1.2e-2
(test/rbln/test_custom_kernel.py:654-655), against the oracle's exact fp32
evaluation of the same inputs. Cache writes (the appended row) must be
bit-exact; the block-table known-answer test must be exact.
"""

import ctypes
import math
import os

import pytest
import torch

from oracle import paged_attention as opa
from tests.paged_inputs import clone_caches, make_decode, to_device

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1.2e-2
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch_rbln_b200  # noqa: F401  (fails loudly if the extension is missing)


def cabi():
    from torch_rbln_b200 import cabi as c

    return c


def run_op(d, mask=None, op="paged_causal_attn_decode"):
    x = to_device(d, DEV)
    ops = torch.ops.rbln_custom_ops
    if op == "paged_attn_decode":
        out = ops.paged_attn_decode(x["q"], x["k"], x["v"], mask.to(DEV), x["kcache"], x["vcache"], x["seq"],
                                    x["scale"], x["block_table"], x["block_size"])
    elif "k_scale" in x:
        out = ops.paged_causal_attn_decode_kvfp8(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["k_scale"],
                                                 x["v_scale"], x["seq"], x["scale"], x["block_table"],
                                                 x["block_size"], None if mask is None else mask.to(DEV))
    else:
        out = ops.paged_causal_attn_decode(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["scale"],
                                           x["block_table"], x["block_size"],
                                           None if mask is None else mask.to(DEV))
    torch.cuda.synchronize()
    return out.cpu(), x["kcache"].cpu(), x["vcache"].cpu()


def run_cabi(d, mask=None, num_splits=0, entry="rbln_paged_causal_attn_decode", err=None):
    c = cabi()
    x = to_device(d, DEV)
    p, keep = c.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"],
                             x["block_size"], float(x["scale"]), mask=None if mask is None else mask.to(DEV),
                             k_scale=x.get("k_scale"), v_scale=x.get("v_scale"), num_splits=num_splits)
    c.attach_workspace(p, DEV, keep)
    if err is not None:
        p.error_flags = err.data_ptr()
    rc = c.call(entry, p)
    assert rc == c.OK, f"{entry} returned {rc}"
    torch.cuda.synchronize()
    return keep["out"].cpu(), x["kcache"].cpu(), x["vcache"].cpu()


def oracle(d, mask=None, op="causal"):
    e = clone_caches(d)
    out = opa.paged_decode(e["q"], e["k"], e["v"], e["kcache"], e["vcache"], e["seq"], e["scale"],
                           e["block_table"], e["block_size"], mask, k_scale=e.get("k_scale"),
                           v_scale=e.get("v_scale"), mode="fp32")
    return out, e["kcache"], e["vcache"]


def check(got, ref, rtol=RTOL, atol=ATOL):
    go, gk, gv = got
    ro, rk, rv = ref
    assert torch.isfinite(go.float()).all()
    torch.testing.assert_close(go.float(), ro, rtol=rtol, atol=atol)
    assert torch.equal(gk.view(torch.uint8), rk.view(torch.uint8)), "kcache differs after the append"
    assert torch.equal(gv.view(torch.uint8), rv.view(torch.uint8)), "vcache differs after the append"


# --- the reference's own configurations (golden fixtures) -------------------
GOLDEN = torch.load(os.path.join(os.path.dirname(__file__), "golden", "paged_decode.pt"), weights_only=False)


@pytest.mark.parametrize("idx", [i for i, c in enumerate(GOLDEN) if c["dtype"] != torch.float32])
@pytest.mark.parametrize("op", ["paged_attn_decode", "paged_causal_attn_decode", "paged_causal_attn_decode_pmask"])
def test_decode_matches_reference_fixtures(idx, op):
    c = GOLDEN[idx]
    exp = c["results"][op]
    full = lambda pre: torch.cat([pre, torch.zeros(pre.shape[:3] + (c["max_seq"] - pre.shape[3], pre.shape[4]),
                                                   dtype=pre.dtype)], dim=3)
    d = dict(q=c["q"], k=c["k"], v=c["v"], kcache=full(c["kpre"]), vcache=full(c["vpre"]), seq=c["ctx"],
             block_table=torch.tensor([[0], [1]], dtype=torch.int16), block_size=c["max_seq"],
             scale=torch.tensor(1.0 / math.sqrt(c["D"])))
    mask = {"paged_attn_decode": c["mask"], "paged_causal_attn_decode": None,
            "paged_causal_attn_decode_pmask": c["pmask"]}[op]
    out, kc, vc = run_op(d, mask, "paged_attn_decode" if op == "paged_attn_decode" else "causal")
    assert out.dtype == exp["out"].dtype and out.shape == exp["out"].shape
    ref_o, _, _ = oracle(d, mask)
    torch.testing.assert_close(out.float(), ref_o, rtol=RTOL, atol=ATOL)
    tol = dict(rtol=1.6e-2, atol=3e-2) if c["dtype"] == torch.bfloat16 else dict(rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(out.float(), exp["out"].float(), **tol)
    rows_k = torch.stack([kc[b, :, 0, int(c["ctx"][b, 0])] for b in range(c["B"])])
    rows_v = torch.stack([vc[b, :, 0, int(c["ctx"][b, 0])] for b in range(c["B"])])
    assert torch.equal(rows_k, exp["krow"]) and torch.equal(rows_v, exp["vrow"])


# --- real block tables -------------------------------------------------------
CASES = [
    # B, Hkv, G, D, bs, lens
    (3, 2, 4, 128, 16, [1, 17, 300]),
    (4, 8, 4, 128, 16, [128, 1000, 4096, 77]),
    (2, 2, 8, 128, 16, [2048, 33]),
    (2, 1, 1, 64, 16, [64, 65]),
    (3, 2, 4, 64, 32, [31, 32, 700]),
    (2, 2, 16, 128, 16, [500, 90]),
    (2, 2, 6, 64, 8, [7, 123]),
    (2, 2, 4, 128, 64, [1, 640]),
    (2, 2, 12, 64, 16, [257, 1030]),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", CASES)
def test_decode_random_block_table(case, dtype):
    B, Hkv, G, D, bs, lens = case
    d = make_decode(B, Hkv, G, D, bs, lens, dtype=dtype, seed=sum(case[5]) + case[0] * case[3])
    ref = oracle(d)
    check(run_op(d), ref)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 64])
def test_decode_split_counts_via_cabi(splits):
    d = make_decode(3, 2, 4, 128, 16, [900, 1, 4000], seed=splits)
    ref = oracle(d)
    check(run_cabi(d, num_splits=splits), ref)


@pytest.mark.parametrize("bt_dtype", [torch.int16, torch.int32, torch.int64])
def test_decode_block_table_dtypes(bt_dtype):
    d = make_decode(2, 2, 4, 128, 16, [333, 1200], bt_dtype=bt_dtype, seed=5)
    check(run_op(d), oracle(d))


@pytest.mark.parametrize("mdt", [torch.float32, torch.bfloat16, torch.bool])
def test_decode_explicit_mask(mdt):
    """paged_attn_decode keeps exactly the positions with mask > 0, including
    positions past seq[b]; causal decode with a mask does the same."""
    B, lens = 3, [100, 700, 31]
    d = make_decode(B, 2, 4, 128, 16, lens, seed=9, extra_blocks=2)
    span = d["block_table"].shape[1] * 16
    g = torch.Generator().manual_seed(4)
    keep = torch.rand([B, span], generator=g) > 0.5
    keep[:, 0] = True
    keep[1, 690:] = True   # beyond seq: the reference's mask rule still keeps them
    keep[2] = False        # fully masked row -> NaN, like softmax over all -inf
    mask = keep.to(mdt) if mdt != torch.bool else keep
    m5 = mask.reshape(B, 1, 1, 1, span)
    ref = oracle(d, m5)
    got = run_op(d, m5, "paged_attn_decode")
    assert torch.isnan(got[0][2].float()).all() and torch.isnan(ref[0][2]).all()
    check(tuple(t[:2] if i == 0 else t for i, t in enumerate(got)), (ref[0][:2], ref[1], ref[2]))
    got2 = run_op(d, mask.reshape(B, span))
    torch.testing.assert_close(got2[0][:2].float(), ref[0][:2], rtol=RTOL, atol=ATOL)


def test_decode_block_table_known_answer():
    """Exact-indexing check: V rows encode their logical position, one K row
    dominates the softmax, so the output must be that row's V exactly."""
    B, Hkv, G, D, bs = 4, 2, 4, 128, 16
    lens = [50, 1000, 16, 4097]
    d = make_decode(B, Hkv, G, D, bs, lens, seed=11)
    bt = d["block_table"].long()
    target = [13, 777, 15, 4096]  # 4096 is the appended token of sequence 3
    d["q"] = torch.ones_like(d["q"])
    d["kcache"].zero_()
    d["k"].zero_()
    vp = torch.zeros(d["vcache"].shape, dtype=torch.float32)
    for b in range(B):
        for t in range(lens[b]):
            blk, off = int(bt[b, t // bs]), t % bs
            vp[blk, :, 0, off, 0] = t // 256
            vp[blk, :, 0, off, 1] = t % 256
            vp[blk, :, 0, off, 2] = b
        tt = target[b]
        if tt == lens[b] - 1:
            d["k"][b, :, 0, 0, :] = 64.0
        else:
            d["kcache"][int(bt[b, tt // bs]), :, 0, tt % bs, :] = 64.0
    d["vcache"] = vp.to(d["vcache"].dtype)
    # the appended token of every sequence encodes its own position too
    d["v"].zero_()
    for b in range(B):
        t = lens[b] - 1
        d["v"][b, :, 0, 0, 0] = t // 256
        d["v"][b, :, 0, 0, 1] = t % 256
        d["v"][b, :, 0, 0, 2] = b
    out, _, _ = run_op(d)
    for b in range(B):
        exp = torch.tensor([target[b] // 256, target[b] % 256, b], dtype=out.dtype)
        for h in range(Hkv):
            for g in range(G):
                assert torch.equal(out[b, h, g, 0, :3], exp), (b, h, g, out[b, h, g, 0, :4])


@pytest.mark.parametrize("qdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
def test_decode_fp8_kv(qdt, D):
    d = make_decode(4, 2, 4, D, 16, [300, 1, 2000, 64], dtype=qdt, fp8=True, seed=D)
    ref = oracle(d)
    check(run_op(d), ref)
    check(run_cabi(d, num_splits=3), ref)


def test_decode_invalid_block_id_sets_flag():
    """An out-of-range block id inside the attended span is skipped (treated
    as masked) and reported in the device error word."""
    d = make_decode(2, 2, 4, 128, 16, [200, 200], seed=2)
    d["block_table"][1, 3] = 10 ** 6
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = run_cabi(d, err=err)
    assert int(err.item()) & cabi().DEVERR_BLOCK_ID_RANGE
    ref = oracle(d)  # the oracle masks invalid blocks the same way
    torch.testing.assert_close(got[0].float(), ref[0], rtol=RTOL, atol=ATOL)


def test_decode_full_size_config_properties():
    """Paged decode bf16 at full size (B=64, 32/8 heads, D=128, bs=16,
    L ~ U[128, 4096], 20k-block pool): parity on every sequence with the
    oracle, and bit-identical output after a consistent relabelling of the
    physical blocks (pool and table permuted together)."""
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(128, 4097, (64,), generator=g).tolist()
    d = make_decode(64, 8, 4, 128, 16, lens, num_blocks=20000, seed=0)
    ref = oracle(d)
    got = run_op(d)
    check(got, ref)
    pi = torch.randperm(20000, generator=g)
    inv = torch.empty_like(pi)
    inv[pi] = torch.arange(20000)
    e = dict(d)
    e["kcache"], e["vcache"] = d["kcache"][pi].contiguous(), d["vcache"][pi].contiguous()
    e["block_table"] = inv[d["block_table"].long()].to(torch.int32)
    got2 = run_op(e)
    assert torch.equal(got2[0], got[0])


def test_decode_error_contract():
    c = cabi()
    d = make_decode(1, 1, 4, 128, 16, [10], seed=1)
    x = to_device(d, DEV)
    p, keep = c.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"], 16, 0.1)
    p.head_dim = 96
    assert c.call("rbln_paged_causal_attn_decode", p) == c.ERR_UNSUPPORTED
    p.head_dim = 128
    assert c.call("rbln_paged_attn_decode", p) == c.ERR_INVALID_ARGUMENT  # mask required
    with pytest.raises(RuntimeError, match="multiple of 64"):
        bad = torch.zeros([4, 1, 1, 16, 96], dtype=torch.bfloat16, device=DEV)
        torch.ops.rbln_custom_ops.paged_causal_attn_decode(x["q"][..., :96].contiguous(), x["k"][..., :96].contiguous(),
                                                           x["v"][..., :96].contiguous(), bad, bad.clone(), x["seq"],
                                                           x["scale"], x["block_table"], 16)


# --- balanced chunks (the default schedule) ----------------------------------
def test_decode_balanced_chunks_span_many_sequences():
    """Many short sequences: one chunk of the balanced schedule covers the end
    of one sequence and several whole ones (one partial or one final output
    per sequence it touches)."""
    g = torch.Generator().manual_seed(21)
    lens = torch.randint(1, 60, (300,), generator=g).tolist()
    d = make_decode(300, 2, 4, 128, 16, lens, seed=21)
    check(run_op(d), oracle(d))


def test_decode_balanced_single_token_sequences():
    """512 one-token sequences: the balanced split charges each sequence start
    a run of virtual tokens, so most chunks cover only virtual tokens of some
    sequences and must skip them; every sequence still gets its output."""
    d = make_decode(512, 2, 4, 128, 16, [1] * 512, seed=24)
    check(run_op(d), oracle(d))


@pytest.mark.parametrize("G", [4, 16])
def test_decode_balanced_one_long_sequence(G):
    """One sequence spread over many chunks, next to short ones."""
    d = make_decode(3, 2, G, 128, 16, [20000, 5, 300], seed=22)
    check(run_op(d), oracle(d))


def test_decode_negative_seq_sets_flag():
    """seq[b] < 0: no visible position and nothing appended for that sequence,
    its output is NaN and the device error word has DEVERR_SEQ_RANGE; the
    other sequences are unaffected."""
    d = make_decode(3, 2, 4, 128, 16, [100, 50, 700], seed=23)
    d["seq"][1, 0] = -1
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = run_cabi(d, err=err)
    assert int(err.item()) & cabi().DEVERR_SEQ_RANGE
    assert torch.isnan(got[0][1].float()).all()
    keep = torch.tensor([0, 2])
    sub = dict(d, q=d["q"][keep], k=d["k"][keep], v=d["v"][keep], seq=d["seq"][keep],
               block_table=d["block_table"][keep])
    ref = oracle(sub)
    check((got[0][keep], got[1], got[2]), ref)
