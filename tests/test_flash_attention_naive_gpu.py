"""Parity of flash_attention_naive_{prefill,decode} on the sm_100a kernels.

The ops are the keep-mask paged kernels over the two halves of the unified
cache kv_cache [2, num_blocks, Hkv, 1, P, D]. Checks:
  * the reference's single-partition configurations (golden fixtures from
    its CPU definition, test/rbln/test_custom_kernel.py:546-645): output
    against the oracle's exact fp32 evaluation and against the reference's
    output, the mutated cache bit-exact (same SHA-256 as the reference's);
  * several partitions per sequence through a shuffled block table, batch
    > 1 decode, a chunk that starts mid-partition;
  * attention sinks (per query head logits) on the decode whole-sequence,
    balanced-merge and per-sequence-split paths and on the prefill kernel,
    including a fully masked sequence (all mass on the sink: output 0).

Tolerance (stated): rtol 1e-3, atol 1.2e-2 (test_custom_kernel.py:654-655)
against the oracle's fp32 evaluation; bfloat16 against the reference's own
output uses rtol 1.6e-2, atol 3e-2 (its scores are rounded to bfloat16).
"""

import hashlib
import math
import os

import pytest
import torch

from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1.2e-2
DEV = "cuda"
NAIVE = torch.load(os.path.join(os.path.dirname(__file__), "golden", "flash_attention_naive.pt"),
                   weights_only=False)


@pytest.fixture(scope="module", autouse=True)
def _ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch_rbln_b200  # noqa: F401  (fails loudly if the extension is missing)


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def run_op(x, decode, sinks=None):
    """Calls the op on device copies of x; returns (out, kv_cache) on the CPU."""
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) and k != "scale" else v) for k, v in x.items()}
    op = (torch.ops.rbln_custom_ops.flash_attention_naive_decode if decode
          else torch.ops.rbln_custom_ops.flash_attention_naive_prefill)
    args = [d["q"], d["k"], d["v"], d["kv_cache"], d["mask"], d["scale"], d["seq_idx"], d["block_tables"],
            d["slot_mapping"]]
    if sinks is not None:
        args.append(sinks.to(DEV))
    out = op(*args)
    torch.cuda.synchronize()
    return out.cpu(), d["kv_cache"].cpu()


def run_oracle(x, decode, sinks=None):
    kv = x["kv_cache"].clone()
    out = opa.flash_attention_naive(x["q"], x["k"], x["v"], kv, x["mask"], x["scale"], x["seq_idx"],
                                    x["block_tables"], sinks, decode=decode, mode="fp32")
    return out, kv


def check(got, ref, finite=True):
    go, gkv = got
    ro, rkv = ref
    if finite:
        assert torch.isfinite(go.float()).all()
    torch.testing.assert_close(go.float(), ro, rtol=RTOL, atol=ATOL, equal_nan=not finite)
    assert torch.equal(gkv.view(torch.uint8), rkv.view(torch.uint8)), "kv_cache differs after the write"


# --- the reference's configurations ------------------------------------------
@pytest.mark.parametrize("idx", range(len(NAIVE)))
def test_reference_configurations(idx):
    c = NAIVE[idx]
    x = dict(q=c["q"], k=c["k"], v=c["v"], kv_cache=c["kv_cache"].clone(), mask=c["mask"],
             scale=torch.tensor(1.0 / math.sqrt(c["D"])), seq_idx=torch.tensor([[c["s0"]]], dtype=torch.int32),
             block_tables=(torch.tensor([[0]], dtype=torch.int16) if c["decode"]
                           else torch.tensor([0], dtype=torch.int16)),
             slot_mapping=torch.arange(c["S"], dtype=torch.int32))
    if c["dtype"] == torch.float32:
        # the kernels take bfloat16 / float16 (the reference device op returns float16)
        with pytest.raises(RuntimeError, match="bfloat16 or float16"):
            run_op(x, c["decode"])
        return
    got = run_op(x, c["decode"])
    check(got, run_oracle(x, c["decode"]))
    tol = dict(rtol=1.6e-2, atol=3e-2) if c["dtype"] == torch.bfloat16 else dict(rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(got[0].float(), c["results"]["out"].float(), **tol)
    assert _sha(got[1]) == c["results"]["kv_cache"], "kv_cache differs from the reference's"


# --- several partitions, batch > 1 --------------------------------------------
def make_case(B, Hkv, G, D, P, NP, starts, S, dtype=torch.float16, seed=0, causal=True, holes=False):
    g = torch.Generator().manual_seed(seed)
    nblk = B * NP + 3
    bt = torch.randperm(nblk, generator=g)[: B * NP].reshape(B, NP).to(torch.int32)
    L = NP * P
    mask = torch.zeros([B, 1, 1, S, L], dtype=dtype)
    for b, s0 in enumerate(starts):
        if causal:
            mask[b, 0, 0] = torch.ones([S, L], dtype=dtype).tril(diagonal=s0)
        else:
            mask[b, 0, 0, :, : s0 + S] = 1
        if holes:
            mask[b, 0, 0, :, torch.randperm(max(s0, 1), generator=g)[: s0 // 3]] = 0
    return dict(q=torch.randn([B, Hkv, G, S, D], generator=g).to(dtype),
                k=torch.randn([B, Hkv, 1, S, D], generator=g).to(dtype),
                v=torch.randn([B, Hkv, 1, S, D], generator=g).to(dtype),
                kv_cache=torch.randn([2, nblk, Hkv, 1, P, D], generator=g).to(dtype) * 0.7,
                mask=mask, scale=torch.tensor(1.0 / math.sqrt(D)),
                seq_idx=torch.tensor(starts, dtype=torch.int32).reshape(B, 1),
                block_tables=bt if B > 1 or S == 1 else bt.reshape(-1),
                slot_mapping=torch.arange(S, dtype=torch.int32))


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_several_partitions(D, dtype):
    x = make_case(3, 2, 4, D, 64, 6, [70, 5, 300], 1, dtype=dtype, seed=D, holes=True)
    check(run_op(x, True), run_oracle(x, True))


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_chunk_across_partitions(D):
    x = make_case(1, 2, 4, D, 128, 4, [100], 150, seed=3 + D)
    check(run_op(x, False), run_oracle(x, False))


# --- attention sinks ----------------------------------------------------------
def sinks_for(x, seed=11):
    H = x["q"].shape[1] * x["q"].shape[2]
    return torch.randn(H, generator=torch.Generator().manual_seed(seed)) * 2 + 1


@pytest.mark.parametrize("short_mask", [False, True])
@pytest.mark.parametrize("D", [64, 128])
def test_decode_sinks(D, short_mask):
    """Full 384-position masks split each sequence over chunks (merge path);
    128-position masks keep each sequence in one chunk (whole-sequence path)."""
    x = make_case(3, 2, 4, D, 64, 6, [70, 5, 300], 1, seed=21 + D)
    if short_mask:
        x["mask"] = x["mask"][..., :128].contiguous()
    x["mask"][1] = 0  # sequence 1 sees nothing: all softmax mass on the sink
    s = sinks_for(x)
    got, ref = run_op(x, True, s), run_oracle(x, True, s)
    check(got, ref)
    assert torch.count_nonzero(got[0][1]) == 0
    # without sinks the fully masked sequence is NaN, as softmax of all -inf
    x["kv_cache"] = make_case(3, 2, 4, D, 64, 6, [70, 5, 300], 1, seed=21 + D)["kv_cache"]
    nos, _ = run_op(x, True)
    assert torch.isnan(nos[1]).all()
    assert torch.isfinite(nos[0].float()).all() and torch.isfinite(nos[2].float()).all()


def test_decode_sinks_long_context_merge():
    """4000 visible positions: the balanced kernel cuts the sequence into
    chunks whose partials the merge kernel combines with the sink."""
    x = make_case(2, 2, 4, 128, 128, 32, [3999, 99], 1, seed=5)
    x["mask"][:] = 0
    x["mask"][0, ..., :4000] = 1
    x["mask"][1, ..., :100] = 1
    s = sinks_for(x, 3) + 4  # comparable to the largest scores
    check(run_op(x, True, s), run_oracle(x, True, s))


def test_decode_sinks_split_path_cabi():
    """The per-sequence split kernel and its merge (num_splits > 0) through the
    C-ABI, with the sinks pointer set in the parameter struct."""
    from torch_rbln_b200 import cabi as c

    x = make_case(2, 2, 4, 128, 128, 16, [2000, 700], 1, seed=9)
    x["mask"][:] = 0
    x["mask"][0, ..., :2001] = 1
    x["mask"][1, ..., :701] = 1
    s = sinks_for(x, 4) + 3
    ref = run_oracle(x, True, s)
    d = {k: (v.to(DEV) if isinstance(v, torch.Tensor) and k != "scale" else v) for k, v in x.items()}
    kv = d["kv_cache"]
    p, keep = c.paged_params(d["q"], d["k"], d["v"], kv[0], kv[1], d["seq_idx"].reshape(-1).contiguous(),
                             d["block_tables"], 128, float(x["scale"]), mask=d["mask"], num_splits=4)
    sk = s.to(DEV)
    p.sinks = sk.data_ptr()
    c.attach_workspace(p, DEV, keep)
    rc = c.call("rbln_paged_attn_decode", p)
    assert rc == c.OK
    torch.cuda.synchronize()
    check((keep["out"].cpu(), kv.cpu()), ref)


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_sinks(D):
    x = make_case(1, 2, 4, D, 128, 4, [100], 150, seed=31 + D)
    x["mask"][0, 0, 0, 7] = 0  # one query row sees nothing: output 0
    s = sinks_for(x, 5)
    got, ref = run_op(x, False, s), run_oracle(x, False, s)
    check(got, ref)
    assert torch.count_nonzero(got[0][0, :, :, 7]) == 0


def test_sinks_shape_is_checked():
    x = make_case(1, 2, 4, 64, 64, 2, [10], 1)
    with pytest.raises(RuntimeError, match="one logit per query head"):
        run_op(x, True, torch.zeros(3))


def test_prefill_batch_must_be_one():
    """register_custom_ops.py:478-482: prefill q / k / v batch must be 1."""
    x = make_case(2, 2, 4, 64, 64, 2, [0, 0], 16)
    with pytest.raises(RuntimeError, match="batch size"):
        run_op(x, False)
