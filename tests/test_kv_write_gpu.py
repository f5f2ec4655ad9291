"""The standalone paged KV-cache write (rbln_paged_kv_write, op
rbln_attn::paged_kv_write) against the oracle (oracle.paged_attention.kv_write,
pinned to the reference's own prefill writes in test_oracle_golden.py).

Bar: bit-exact caches for bf16 / f16 (a copy) and for fp8-e4m3 (same
float32 arithmetic, IEEE division, round to nearest even with saturation),
bit-exact recomputed scales; then the fp8 decode kernel reading the written
cache agrees with the oracle's decode of the oracle's cache within the
reference's tolerance (rtol 1e-3, atol 1.2e-2, test_custom_kernel.py:654-655).
"""

import pytest
import torch

from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch_rbln_b200  # noqa: F401


def setup(B, Hkv, D, bs, max_blocks, dtype, cache_dtype, seed):
    g = torch.Generator().manual_seed(seed)
    nblk = B * max_blocks + 3
    bt = torch.randperm(nblk, generator=g)[: B * max_blocks].reshape(B, max_blocks).to(torch.int32)
    if cache_dtype == torch.float8_e4m3fn:
        pool = torch.randn([nblk, Hkv, 1, bs, D], generator=g)
        kc, ks = opa.quantize_fp8(pool, torch.ones(1)), torch.ones(nblk, Hkv)
        vc, vs = kc.clone(), ks.clone()
    else:
        kc = torch.randn([nblk, Hkv, 1, bs, D], generator=g).to(cache_dtype)
        vc, ks, vs = kc.clone(), None, None
    return g, bt, kc, vc, ks, vs


def write_both(k, v, kc, vc, seq, bt, bs, ks, vs):
    """(GPU result, oracle result) of one write; the GPU copies of the caches
    are passed in and updated."""
    ops = torch.ops.rbln_attn
    ops.paged_kv_write(k.to(DEV), v.to(DEV), kc[0], vc[0], seq.to(DEV), bt.to(DEV), bs,
                       None if ks is None else ks[0], None if vs is None else vs[0])
    opa.kv_write(k, v, kc[1], vc[1], seq, bt, bs, None if ks is None else ks[1], None if vs is None else vs[1])
    torch.cuda.synchronize()


def assert_same(dev_t, cpu_t, what):
    assert torch.equal(dev_t.cpu().view(torch.uint8), cpu_t.view(torch.uint8)), what


@pytest.mark.parametrize("cache", [torch.bfloat16, torch.float16, torch.float8_e4m3fn])
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_then_decode_writes(cache, D):
    """A prefill chunk that starts mid-block, then single-token writes that
    land in partly filled blocks (held rows re-quantized for fp8)."""
    B, Hkv, bs, mb = 3, 2, 16, 8
    dt = torch.float16 if cache == torch.float16 else torch.bfloat16
    g, bt, kc0, vc0, ks0, vs0 = setup(B, Hkv, D, bs, mb, dt, cache, seed=D)
    kc, vc = [kc0.to(DEV), kc0.clone()], [vc0.to(DEV), vc0.clone()]
    ks = None if ks0 is None else [ks0.to(DEV), ks0.clone()]
    vs = None if vs0 is None else [vs0.to(DEV), vs0.clone()]
    starts = torch.tensor([0, 5, 30], dtype=torch.int32)
    S = 41
    k = (torch.randn([B, Hkv, 1, S, D], generator=g) * 0.5).to(dt)
    v = (torch.randn([B, Hkv, 1, S, D], generator=g) * 0.5).to(dt)
    write_both(k, v, kc, vc, starts, bt, bs, ks, vs)
    pos = starts + S
    for step in range(3):
        k1 = (torch.randn([B, Hkv, 1, 1, D], generator=g) * (1 + step)).to(dt)  # growing amax: scales change
        v1 = (torch.randn([B, Hkv, 1, 1, D], generator=g) * (1 + step)).to(dt)
        write_both(k1, v1, kc, vc, pos, bt, bs, ks, vs)
        pos = pos + 1
    assert_same(kc[0], kc[1], "kcache")
    assert_same(vc[0], vc[1], "vcache")
    if ks is not None:
        assert_same(ks[0], ks[1], "k_scale")
        assert_same(vs[0], vs[1], "v_scale")
        # the fp8 decode kernel reads what the writer wrote
        q = torch.randn([B, Hkv, 4, 1, D], generator=g).to(dt)
        k2 = torch.randn([B, Hkv, 1, 1, D], generator=g).to(dt) * 0.1
        v2 = torch.randn([B, Hkv, 1, 1, D], generator=g).to(dt) * 0.1
        scale = torch.tensor(D ** -0.5)
        out = torch.ops.rbln_custom_ops.paged_causal_attn_decode_kvfp8(
            q.to(DEV), k2.to(DEV), v2.to(DEV), kc[0], vc[0], ks[0], vs[0], pos.reshape(B, 1).to(DEV), scale,
            bt.to(DEV), bs)
        ref = opa.paged_decode(q, k2, v2, kc[1], vc[1], pos.reshape(B, 1), scale, bt, bs, None, k_scale=ks[1],
                               v_scale=vs[1], mode="fp32")
        torch.testing.assert_close(out.cpu().float(), ref, rtol=1e-3, atol=1.2e-2)


@pytest.mark.parametrize("D", [64, 128])
def test_f16_rows_into_fp8_cache(D):
    """f16 rows into an fp8 cache (the amax taken on packed f16 pairs): a
    chunk that starts and ends inside blocks, over held rows that are
    re-quantized; caches and scales bit-exact."""
    B, Hkv, bs, mb = 3, 2, 16, 8
    g, bt, kc0, vc0, ks0, vs0 = setup(B, Hkv, D, bs, mb, torch.float16, torch.float8_e4m3fn, seed=100 + D)
    kc, vc = [kc0.to(DEV), kc0.clone()], [vc0.to(DEV), vc0.clone()]
    ks, vs = [ks0.to(DEV), ks0.clone()], [vs0.to(DEV), vs0.clone()]
    starts = torch.tensor([0, 5, 30], dtype=torch.int32)
    k = (torch.randn([B, Hkv, 1, 37, D], generator=g) * 2).to(torch.float16)
    v = (torch.randn([B, Hkv, 1, 37, D], generator=g) * 2).to(torch.float16)
    write_both(k, v, kc, vc, starts, bt, bs, ks, vs)
    assert_same(kc[0], kc[1], "kcache")
    assert_same(vc[0], vc[1], "vcache")
    assert_same(ks[0], ks[1], "k_scale")
    assert_same(vs[0], vs[1], "v_scale")


def test_invalid_block_id_sets_the_flag():
    from torch_rbln_b200 import cabi

    B, Hkv, D, bs = 1, 1, 64, 16
    kc = torch.zeros([4, Hkv, 1, bs, D], dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    k = torch.ones([B, Hkv, 1, 8, D], dtype=torch.bfloat16, device=DEV)
    bt = torch.tensor([[9]], dtype=torch.int32, device=DEV)  # outside the 4-block pool
    seq = torch.zeros([B], dtype=torch.int32, device=DEV)
    q = torch.empty([B, Hkv, 1, 8, D], dtype=torch.bfloat16, device=DEV)
    p, keep = cabi.paged_params(q, k, k, kc, vc, seq, bt, bs, 1.0)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    p.error_flags = err.data_ptr()
    assert cabi.call("rbln_paged_kv_write", p) == cabi.OK
    torch.cuda.synchronize()
    assert int(err.item()) & cabi.DEVERR_BLOCK_ID_RANGE
    assert torch.count_nonzero(kc) == 0


@pytest.mark.parametrize("cache", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("bs,D", [(8, 128), (16, 128), (32, 64), (32, 128), (64, 64), (128, 128)])
def test_block_sizes_both_kernels(cache, bs, D):
    """Block sizes on both sides of the register kernel's limit (bs * D <=
    2048 keeps a block's new rows in registers; larger blocks take the
    two-pass kernel), with writes that start and end inside blocks, span
    several blocks, and fill a block exactly: caches and scales bit-exact."""
    B, Hkv, mb = 4, 2, 6
    dt = torch.bfloat16
    g, bt, kc0, vc0, ks0, vs0 = setup(B, Hkv, D, bs, mb, dt, cache, seed=bs * 1000 + D)
    kc, vc = (kc0.to(DEV), kc0.clone()), (vc0.to(DEV), vc0.clone())
    ks = None if ks0 is None else (ks0.to(DEV), ks0.clone())
    vs = None if vs0 is None else (vs0.to(DEV), vs0.clone())
    S = bs + bs // 2 + 3
    starts = torch.tensor([0, bs // 2 + 1, bs, 2 * bs - 1], dtype=torch.int32)
    k = (torch.randn([B, Hkv, 1, S, D], generator=g) * 3).to(dt)
    v = (torch.randn([B, Hkv, 1, S, D], generator=g) * 0.25).to(dt)
    write_both(k, v, kc, vc, starts, bt, bs, ks, vs)
    assert_same(kc[0], kc[1], "k cache")
    assert_same(vc[0], vc[1], "v cache")
    if ks is not None:
        assert_same(ks[0], ks[1], "k scales")
        assert_same(vs[0], vs[1], "v scales")
