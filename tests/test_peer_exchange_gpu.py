"""The head-sharded decode's epoch exchange on one GPU, through the C-ABI.

rbln_paged_causal_attn_decode_peers is called as rank 0 of 2, with both
"ranks'" output buffers and flag arrays in this GPU's own memory. Nothing
plays rank 1, so its announcement never arrives: the wait must give up after
the 1 ms limit with RBLN_DEVERR_TIMEOUT in the error word (which the Python
layer turns into ShardedDecodeError), after the local heads were stored into
both buffers and this rank's epoch was announced to both flag arrays. The
control case pre-sets rank 1's announcement, and the same call must pass
without an error. Both schedules are covered: the balanced one (the merge
kernel's last CTA runs the exchange) and the per-sequence split grid (a
separate one-warp kernel runs it).
"""

import ctypes

import pytest
import torch

from tests.paged_inputs import make_decode, to_device

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from torch_rbln_b200 import cabi as c

    c.lib()
    return c


def _call(cabi, d, num_splits, peer_already_announced):
    x = to_device(d, "cuda")
    B, Hkv, G, _, D = x["q"].shape
    outs = [torch.zeros([B, 2 * Hkv, G, 1, D], dtype=x["q"].dtype, device="cuda") for _ in range(2)]
    flags = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(2)]
    if peer_already_announced:
        flags[0][1] = 1  # rank 1 has announced epoch 1 to rank 0
    out_ptrs = torch.tensor([o.data_ptr() for o in outs], dtype=torch.int64, device="cuda")
    flag_ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    p, keep = cabi.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"],
                                x["block_size"], float(x["scale"]), out=outs[0], num_splits=num_splits)
    cabi.attach_workspace(p, "cuda", keep)
    p.error_flags = err.data_ptr()
    po = cabi.PeerOut()
    po.out, po.flags = out_ptrs.data_ptr(), flag_ptrs.data_ptr()
    po.n, po.rank, po.head0, po.epoch, po.wait_limit_us = 2, 0, 0, 1, 1000
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    rc = cabi.lib().rbln_paged_causal_attn_decode_peers(ctypes.byref(p), ctypes.byref(po),
                                                          ctypes.c_void_p(stream.cuda_stream))
    e1.record(stream)
    assert rc == cabi.OK, rc
    torch.cuda.synchronize()
    return outs, flags, int(err.item()), e0.elapsed_time(e1), keep


def _reference(cabi, d, num_splits):
    """The plain entry point with the same schedule (bit-identical results)."""
    x = to_device(d, "cuda")
    p, keep = cabi.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"],
                                x["block_size"], float(x["scale"]), num_splits=num_splits)
    cabi.attach_workspace(p, "cuda", keep)
    assert cabi.call("rbln_paged_causal_attn_decode", p) == cabi.OK
    torch.cuda.synchronize()
    return keep["out"]


@pytest.mark.parametrize("num_splits", [0, 5])
def test_exchange_wait_runs_out_and_reports_timeout(cabi, num_splits):
    from torch_rbln_b200 import sharding

    d = make_decode(3, 2, 4, 128, 16, [300, 1500, 40], seed=41)
    ref = _reference(cabi, d, num_splits)
    outs, flags, err, ms, _ = _call(cabi, d, num_splits, peer_already_announced=False)
    assert err & cabi.DEVERR_TIMEOUT, err
    assert ms < 1000.0, ms                         # the 1 ms limit ended the wait, not the 2 s default
    assert flags[0].tolist() == [1, 0] and flags[1].tolist() == [1, 0]  # announced to self and to rank 1
    for o in outs:                                 # local heads stored into both ranks' buffers
        assert torch.equal(o[:, :2], ref)
        assert not o[:, 2:].any()                  # rank 1's heads never arrived
    with pytest.raises(sharding.ShardedDecodeError, match="timed out"):
        sharding.raise_on_device_error(err, 0, 2, 1)


@pytest.mark.parametrize("num_splits", [0, 5])
def test_exchange_passes_when_the_peer_has_announced(cabi, num_splits):
    d = make_decode(3, 2, 4, 128, 16, [300, 1500, 40], seed=42)
    ref = _reference(cabi, d, num_splits)
    outs, flags, err, _, _ = _call(cabi, d, num_splits, peer_already_announced=True)
    assert err == 0
    assert flags[1].tolist() == [1, 0]
    for o in outs:
        assert torch.equal(o[:, :2], ref)


def test_peers_entry_requires_an_error_word(cabi):
    d = make_decode(1, 2, 4, 128, 16, [64], seed=43)
    x = to_device(d, "cuda")
    p, keep = cabi.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"],
                                16, 0.1)
    cabi.attach_workspace(p, "cuda", keep)  # everything valid but the missing error word
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_ptrs = torch.tensor([keep["out"].data_ptr()], dtype=torch.int64, device="cuda")
    flag_ptrs = torch.tensor([flags.data_ptr()], dtype=torch.int64, device="cuda")
    po = cabi.PeerOut()
    po.out, po.flags, po.n, po.rank, po.epoch = out_ptrs.data_ptr(), flag_ptrs.data_ptr(), 1, 0, 1
    rc = cabi.lib().rbln_paged_causal_attn_decode_peers(ctypes.byref(p), ctypes.byref(po),
                                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == cabi.ERR_INVALID_ARGUMENT  # rejected before any launch
