"""SDPA backward through the reference's boundary on CUDA.

loss.backward() through F.scaled_dot_product_attention -> (autograd of)
aten::_scaled_dot_product_fused_attention_overrideable ->
aten::_scaled_dot_product_fused_attention_overrideable_backward (CUDA kernel
here, sdpa_bwd.cu), the op the reference implements at sdpa.py:754-821.

Tolerance (stated): the tensor-core kernels round P and dS to the input
dtype before their matrix products, as any half-precision backward does.
Each gradient's max-abs error against the exact float64 evaluation must be
at most 3x the error of the reference's own backward arithmetic run in the
input dtype (oracle.sdpa.sdpa_backward_reference, upcast_f16=False), or
2e-3 x the gradient's max magnitude, whichever is larger.
"""

import os

import pytest
import torch
import torch.nn.functional as F

from oracle import sdpa as osd

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ext():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import torch_rbln_b200  # noqa: F401


def grads_cuda(q, k, v, go, mask=None, causal=False, mask_grad=False, need=(True, True, True)):
    qd = q.to(DEV).requires_grad_(need[0])
    kd = k.to(DEV).requires_grad_(need[1])
    vd = v.to(DEV).requires_grad_(need[2])
    md = None
    if mask is not None:
        md = mask.to(DEV)
        if mask_grad:
            md.requires_grad_(True)
    assert torch._fused_sdp_choice(qd, kd, vd, attn_mask=md, is_causal=causal,
                                   enable_gqa=q.shape[1] != k.shape[1]) == 4  # overrideable: the route here
    out = F.scaled_dot_product_attention(qd, kd, vd, attn_mask=md, is_causal=causal,
                                         enable_gqa=q.shape[1] != k.shape[1])
    out.backward(go.to(DEV))
    torch.cuda.synchronize()
    g = [t.grad.cpu() if t.grad is not None else None for t in (qd, kd, vd)]
    g.append(md.grad.cpu() if (md is not None and mask_grad) else None)
    return g


def check(got, q, k, v, go, mask, causal, names=("dq", "dk", "dv", "dbias")):
    exact = osd.sdpa_backward_math(go, q, k, v, mask, causal)
    lowp = osd.sdpa_backward_reference(go, q, k, v, mask, causal, grad_bias=mask is not None, upcast_f16=False)
    for name, g, e, r in zip(names, got, exact, lowp):
        if g is None:
            continue
        assert g.dtype == q.dtype or name == "dbias"
        assert g.shape == e.shape, (name, g.shape, e.shape)
        assert torch.isfinite(g.float()).all(), name
        err = (g.double() - e).abs().max().item()
        if r is not None and r.shape != e.shape:  # a broadcast mask's gradient is summed down to its shape
            r = r.double().sum_to_size(e.shape)
        base = (r.double() - e).abs().max().item() if r is not None else 0.0
        bound = max(3 * base, 2e-3 * e.abs().max().item())
        assert err <= bound, f"{name}: max err {err:.3e} > bound {bound:.3e} (half-precision reference {base:.3e})"


def rand(shape, dtype, g, s=1.0):
    return (torch.randn(shape, generator=g) * s).to(dtype)


def test_route_and_fp32_grad_goes_elsewhere():
    q = torch.randn(1, 4, 64, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    assert torch._fused_sdp_choice(q, q, q) == 4
    q32 = torch.randn(1, 4, 64, 64, device=DEV, dtype=torch.float32, requires_grad=True)
    assert torch._fused_sdp_choice(q32, q32, q32) != 4  # no fp32 backward kernel: torch's own backends
    with torch.no_grad():
        assert torch._fused_sdp_choice(q32, q32, q32) == 4


FIX = torch.load(os.path.join(os.path.dirname(__file__), "golden", "sdpa_bwd.pt"), weights_only=False)


def grads_aten(q, k, v, go, mask, causal):
    """The forward and backward aten ops called directly (F.scaled_dot_product_attention
    refuses an explicit mask together with is_causal=True; the ops take both)."""
    qd, kd, vd, god = q.to(DEV), k.to(DEV), v.to(DEV), go.to(DEV)
    md = None if mask is None else mask.to(DEV)
    res = torch.ops.aten._scaled_dot_product_fused_attention_overrideable(qd, kd, vd, md, 0.0, causal, False)
    e = torch.empty(0, device=DEV)
    g = torch.ops.aten._scaled_dot_product_fused_attention_overrideable_backward(
        god, qd, kd, vd, md if md is not None else e, [True, True, True, md is not None], res[0], res[1], res[2],
        res[3], res[4], res[5], 0.0, causal, res[6], res[7])
    torch.cuda.synchronize()
    return [t.cpu() if t is not None else None for t in g]


@pytest.mark.parametrize("idx", [i for i, c in enumerate(FIX) if c["dtype"] != torch.float32])
def test_reference_fixtures(idx):
    c = FIX[idx]
    if c["causal"] and c["mask"] is not None:
        got = grads_aten(c["q"], c["k"], c["v"], c["grad_out"], c["mask"], True)
    else:
        got = grads_cuda(c["q"], c["k"], c["v"], c["grad_out"], c["mask"], c["causal"],
                         mask_grad=c["mask"] is not None)
    for name, gv in zip(("dq", "dk", "dv"), got):
        assert gv.shape == c[name].shape and gv.dtype == c[name].dtype
    check(got, c["q"], c["k"], c["v"], c["grad_out"], c["mask"], c["causal"])


CASES = [
    # B, H, Hkv, L, S, D, causal, mask, dtype
    (2, 8, 2, 256, 256, 128, True, None, torch.bfloat16),
    (1, 4, 4, 200, 333, 64, False, None, torch.float16),
    (1, 8, 1, 130, 130, 128, True, None, torch.bfloat16),
    (2, 4, 2, 96, 160, 64, False, "float", torch.bfloat16),
    (1, 4, 2, 128, 128, 128, True, "bool", torch.float16),
    (1, 2, 2, 300, 100, 64, True, None, torch.bfloat16),
    (1, 2, 2, 100, 300, 64, True, None, torch.float16),
    (1, 16, 4, 1024, 1024, 128, True, None, torch.bfloat16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(str(x) for x in c[:6]) + f"-{c[6]}-{c[7]}-{c[8]}")
def test_backward_matches_exact(case):
    B, H, Hkv, L, S, D, causal, mk, dt = case
    g = torch.Generator().manual_seed(B * 1000 + L + S + D)
    q, k, v = rand((B, H, L, D), dt, g), rand((B, Hkv, S, D), dt, g), rand((B, Hkv, S, D), dt, g)
    go = rand((B, H, L, D), dt, g)
    mask = None
    if mk == "float":
        mask = rand((1, H, L, S), dt, g, 2.0)
    elif mk == "bool":
        mask = torch.rand((L, S), generator=g) > 0.3
        mask[:, 0] = True  # every row keeps a key
    if causal and mask is not None:
        got = grads_aten(q, k, v, go, mask, True)
    else:
        got = grads_cuda(q, k, v, go, mask, causal, mask_grad=mk == "float")
    check(got, q, k, v, go, mask, causal)
    if causal and S > L:
        # top-left causal: keys past the last query are seen by nobody
        assert torch.count_nonzero(got[1][:, :, L:]) == 0 and torch.count_nonzero(got[2][:, :, L:]) == 0


def test_partial_grad_input_mask():
    """Only q needs a gradient: the dK/dV kernel is skipped, dq is unchanged."""
    g = torch.Generator().manual_seed(3)
    dt = torch.bfloat16
    q, k, v, go = (rand((1, 4, 192, 64), dt, g), rand((1, 2, 192, 64), dt, g), rand((1, 2, 192, 64), dt, g),
                   rand((1, 4, 192, 64), dt, g))
    only_q = grads_cuda(q, k, v, go, causal=True, need=(True, False, False))
    full = grads_cuda(q, k, v, go, causal=True)
    assert only_q[1] is None and only_q[2] is None
    assert torch.equal(only_q[0], full[0])


def test_aten_backward_op_directly():
    """The op with grad_input_mask [F, T, T, F] returns no dq and the same dk /
    dv, bit for bit, as with [T, T, T, F] after the same forward (each output
    element has one writer: no atomics, deterministic); both match the exact
    gradients."""
    g = torch.Generator().manual_seed(5)
    dt = torch.float16
    q, k, v, go = (rand((1, 4, 160, 128), dt, g), rand((1, 4, 160, 128), dt, g), rand((1, 4, 160, 128), dt, g),
                   rand((1, 4, 160, 128), dt, g))
    qd, kd, vd, god = q.to(DEV), k.to(DEV), v.to(DEV), go.to(DEV)
    res = torch.ops.aten._scaled_dot_product_fused_attention_overrideable(qd, kd, vd, None, 0.0, True, False)
    e = torch.empty(0, device=DEV)

    def bwd(mask4):
        return torch.ops.aten._scaled_dot_product_fused_attention_overrideable_backward(
            god, qd, kd, vd, e, mask4, res[0], res[1], res[2], res[3], res[4], res[5], 0.0, True, res[6], res[7])

    dq1, dk1, dv1, _ = bwd([True, True, True, False])
    dq2, dk2, dv2, db2 = bwd([False, True, True, False])
    torch.cuda.synchronize()
    assert dq2 is None and db2 is None
    assert torch.equal(dk1, dk2) and torch.equal(dv1, dv2)
    check([dq1.cpu(), dk1.cpu(), dv1.cpu(), None], q, k, v, go, None, True)
