"""rbln_paged_causal_attn_decode_noalloc, the decode entry point for callers
that cannot allocate device memory (a runtime whose memory is all handed to
its own pool, or a host framework that forbids allocation while work is
enqueued). It keeps its split-K scratch in a fixed device array owned by
the library, so the caller passes only inputs and outputs.

Checked through the C-ABI against the allocating entry point
(rbln_paged_causal_attn_decode with a caller-supplied workspace), with the
decode tests' tolerance, on two calls in a row: the second call runs over
scratch that still holds the first call's partials. This file is named so
that pytest collects it last.
"""

import ctypes

import pytest
import torch

from tests.paged_inputs import make_decode, to_device

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1.2e-2  # same as the decode parity tests


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from torch_rbln_b200 import cabi

    L = cabi.lib()
    fn = L.rbln_paged_causal_attn_decode_noalloc
    fn.argtypes = [ctypes.POINTER(cabi.PagedAttnParams), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return cabi, L


def _run(cabi, L, d, noalloc, num_splits=0):
    x = to_device(d, "cuda")
    p, keep = cabi.paged_params(x["q"], x["k"], x["v"], x["kcache"], x["vcache"], x["seq"], x["block_table"],
                                x["block_size"], float(x["scale"]), k_scale=x.get("k_scale"),
                                v_scale=x.get("v_scale"), num_splits=num_splits)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = L.rbln_paged_causal_attn_decode_noalloc(ctypes.byref(p), stream)
    else:
        cabi.attach_workspace(p, "cuda", keep)
        rc = L.rbln_paged_causal_attn_decode(ctypes.byref(p), stream)
    assert rc == cabi.OK, rc
    torch.cuda.synchronize()
    return keep["out"].cpu(), x["kcache"].cpu(), x["vcache"].cpu()


def _check(cabi, L, d, num_splits):
    ref = _run(cabi, L, d, noalloc=False, num_splits=num_splits)
    got = _run(cabi, L, d, noalloc=True, num_splits=num_splits)
    torch.testing.assert_close(got[0].float(), ref[0].float(), rtol=RTOL, atol=ATOL)
    assert torch.equal(got[1].view(torch.uint8), ref[1].view(torch.uint8))
    assert torch.equal(got[2].view(torch.uint8), ref[2].view(torch.uint8))


def test_noalloc_decode_matches_allocating_entry_point(lib):
    cabi, L = lib
    workloads = [
        make_decode(4, 2, 4, 128, 16, [3000, 17, 1500, 4000], seed=21),                     # many splits
        make_decode(3, 8, 8, 128, 16, [900, 2500, 64], seed=22, fp8=True),                   # fp8, G = 8
    ]
    for d in workloads:  # two calls in a row share the fixed scratch
        _check(cabi, L, d, num_splits=9)


def test_noalloc_balanced_schedule_over_stale_scratch(lib):
    """The default schedule (num_splits = 0: equal token chunks over the
    batch) keeps a length prefix and [Hkv, chunks + B, G, D] partials in the
    scratch, laid out unlike the per-sequence grid. Run it right after a
    per-sequence call, so that it starts over that call's leftovers, then
    twice more in a row."""
    cabi, L = lib
    _check(cabi, L, make_decode(4, 2, 4, 128, 16, [3000, 17, 1500, 4000], seed=23), num_splits=9)
    lens = [129, 4096, 1, 2000, 37, 3333, 640, 16]
    _check(cabi, L, make_decode(8, 8, 4, 128, 16, lens, seed=24), num_splits=0)
    _check(cabi, L, make_decode(8, 8, 4, 128, 16, lens[::-1], seed=25, fp8=True), num_splits=0)


def test_noalloc_rejects_requests_over_the_scratch_limit(lib):
    cabi, L = lib
    B, Hkv, G, D = 64, 8, 16, 128
    q = torch.zeros([B, Hkv, G, 1, D], dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros([B, Hkv, 1, 1, D], dtype=torch.bfloat16, device="cuda")
    cache = torch.zeros([4, Hkv, 1, 16, D], dtype=torch.bfloat16, device="cuda")
    seq = torch.full([B, 1], 4000, dtype=torch.int32, device="cuda")
    bt = torch.zeros([B, 251], dtype=torch.int32, device="cuda")
    p, keep = cabi.paged_params(q, kv, kv, cache, cache.clone(), seq, bt, 16, 0.1, num_splits=2048)
    # 64 * 8 * 63 splits * 16 * 129 * 4 bytes = 266 MB, far above 16 MiB: rejected, nothing launched
    rc = L.rbln_paged_causal_attn_decode_noalloc(ctypes.byref(p),
                                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == cabi.ERR_SCRATCH_LIMIT
