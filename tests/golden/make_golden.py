"""Generates the golden fixtures in this folder from the reference's own CPU code.

Run where a checkout of RBLN-SW/torch-rbln is available (it is not needed to
run the tests), naming its root with --reference or TORCH_RBLN_REFERENCE:

    python tests/golden/make_golden.py --reference <torch-rbln checkout>

Sources executed:
  * the reference's CPU definitions of the paged ops and of
    flash_attention_naive_{prefill,decode},
    test/rbln/test_custom_kernel.py lines 1-646 (the module-level
    torch.library.custom_op definitions), executed without their
    `torch.testing._internal` import (it needs `expecttest`, absent here);
  * torch_rbln._internal.kernels.sdpa._sdpa_cpu_fallback (sdpa.py:244-289)
    and scaled_dot_product_fused_attention_overrideable_backward_rbln
    (sdpa.py:754-821) on CPU tensors, imported with TORCH_RBLN_DIAGNOSE=1 so
    that the package skips loading the NPU runtime (its CPU-fallback log hook,
    which needs that runtime, is replaced by a no-op).

The configurations are the reference tests' (test_custom_kernel.py:660-1001:
num_kv_heads 8, q heads per KV head 4, head_dim 64, seq 256, block_size ==
max_seq, seq = 0 for prefill) scaled down in max_seq / heads so the
fixtures stay small, in the reference's dtype (float16) plus bfloat16 and
float32. Caches are stored as their written prefix (the rest is zero, as in
the reference tests); caches after a prefill are stored as SHA-256 digests.
"""

from __future__ import annotations

import argparse
import hashlib
import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref: str):
    """Returns (_sdpa_cpu_fallback, the backward entry point)."""
    sys.path.insert(0, ref)
    path = os.path.join(ref, "test", "rbln", "test_custom_kernel.py")
    lines = open(path).read().split("\n")[:646]
    lines = [l for l in lines if "torch.testing._internal" not in l]
    ns: dict = {}
    exec(compile("\n".join(lines), path, "exec"), ns)
    os.environ["TORCH_RBLN_DIAGNOSE"] = "1"
    from torch_rbln._internal.kernels import sdpa as ref_sdpa  # noqa: E402

    # the CPU-fallback log line needs the NPU runtime's extension module;
    # only that logging hook is replaced
    ref_sdpa.rbln_log_cpu_fallback = lambda *a, **k: None
    return ref_sdpa._sdpa_cpu_fallback, ref_sdpa.scaled_dot_product_fused_attention_overrideable_backward_rbln


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def decode_cases(gen):
    out = []
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        for D in (64, 128):
            B, Hkv, G, max_seq = 2, 2, 4, 128
            ctx = torch.tensor([[60], [37]], dtype=torch.int32)
            q = torch.randn([B, Hkv, G, 1, D], generator=gen).to(dtype)
            k = torch.randn([B, Hkv, 1, 1, D], generator=gen).to(dtype)
            v = torch.randn([B, Hkv, 1, 1, D], generator=gen).to(dtype)
            prefix = 64
            kpre = torch.zeros([B, Hkv, 1, prefix, D], dtype=dtype)
            vpre = torch.zeros([B, Hkv, 1, prefix, D], dtype=dtype)
            for b in range(B):
                n = int(ctx[b, 0])
                kpre[b, :, :, :n] = torch.randn([Hkv, 1, n, D], generator=gen).to(dtype)
                vpre[b, :, :, :n] = torch.randn([Hkv, 1, n, D], generator=gen).to(dtype)
            mask = torch.zeros([B, 1, 1, 1, max_seq], dtype=dtype)
            for b in range(B):
                mask[b, 0, 0, 0, : int(ctx[b, 0]) + 1] = 1.0
            # an irregular keep-mask for the optional-mask path of causal decode
            pmask = (torch.rand([B, max_seq], generator=gen) > 0.3).to(dtype)
            pmask[:, 0] = 1
            out.append(dict(dtype=dtype, D=D, B=B, Hkv=Hkv, G=G, max_seq=max_seq, ctx=ctx, q=q, k=k, v=v,
                            kpre=kpre, vpre=vpre, mask=mask, pmask=pmask))
    return out


def full_cache(pre, max_seq):
    B, H, one, P, D = pre.shape
    c = torch.zeros([B, H, one, max_seq, D], dtype=pre.dtype)
    c[:, :, :, :P] = pre
    return c


def run_decode(case):
    ops = torch.ops.rbln_custom_ops
    scale = torch.tensor(1.0 / math.sqrt(case["D"]))
    bt = torch.tensor([[0], [1]], dtype=torch.int16)
    res = {}
    for name in ("paged_attn_decode", "paged_causal_attn_decode", "paged_causal_attn_decode_pmask"):
        kc = full_cache(case["kpre"], case["max_seq"])
        vc = full_cache(case["vpre"], case["max_seq"])
        if name == "paged_attn_decode":
            o = ops.paged_attn_decode(case["q"], case["k"], case["v"], case["mask"], kc, vc, case["ctx"], scale,
                                      bt, case["max_seq"])
        elif name == "paged_causal_attn_decode":
            o = ops.paged_causal_attn_decode(case["q"], case["k"], case["v"], kc, vc, case["ctx"], scale, bt,
                                             case["max_seq"])
        else:
            o = ops.paged_causal_attn_decode(case["q"], case["k"], case["v"], kc, vc, case["ctx"], scale, bt,
                                             case["max_seq"], case["pmask"])
        # the op writes one row per sequence (at ctx[b]); keep just those rows
        rows_k = torch.stack([kc[b, :, 0, int(case["ctx"][b, 0])] for b in range(case["B"])])
        rows_v = torch.stack([vc[b, :, 0, int(case["ctx"][b, 0])] for b in range(case["B"])])
        assert torch.equal(kc[:, :, :, 64:], torch.zeros_like(kc[:, :, :, 64:]))
        res[name] = dict(out=o, krow=rows_k, vrow=rows_v)
    return res


def prefill_cases(gen):
    out = []
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        for D in (64, 128):
            Hkv, G, S, max_seq = 1, 4, 32, 128
            q = torch.randn([1, Hkv, G, S, D], generator=gen).to(dtype)
            k = torch.randn([1, Hkv, 1, S, D], generator=gen).to(dtype)
            v = torch.randn([1, Hkv, 1, S, D], generator=gen).to(dtype)
            # context already in block 0 before the chunk (used by the s > 0 case)
            s1 = 24
            kpre = torch.zeros([1, Hkv, 1, s1, D], dtype=dtype)
            vpre = torch.zeros([1, Hkv, 1, s1, D], dtype=dtype)
            kpre[:] = torch.randn([1, Hkv, 1, s1, D], generator=gen).to(dtype)
            vpre[:] = torch.randn([1, Hkv, 1, s1, D], generator=gen).to(dtype)
            out.append(dict(dtype=dtype, D=D, Hkv=Hkv, G=G, S=S, max_seq=max_seq, s1=s1, q=q, k=k, v=v,
                            kpre=kpre, vpre=vpre))
    return out


def run_prefill(case):
    ops = torch.ops.rbln_custom_ops
    D, S, ms, dt = case["D"], case["S"], case["max_seq"], case["dtype"]
    scale = torch.tensor(1.0 / math.sqrt(D))
    bt = torch.tensor([0], dtype=torch.int16)
    res = {}
    # (1) paged_attn_prefill, seq = 0, causal keep-mask (test_custom_kernel.py:682-684)
    kc = torch.zeros([1, case["Hkv"], 1, ms, D], dtype=dt)
    vc = torch.zeros_like(kc)
    mask0 = torch.ones([1, S, ms], dtype=dt).tril().view(1, 1, 1, S, ms)
    o = ops.paged_attn_prefill(case["q"], case["k"], case["v"], mask0, kc, vc,
                               torch.tensor([[0]], dtype=torch.int32), scale, bt, ms)
    res["paged_attn_prefill_s0"] = dict(out=o, seq=0, kc=sha(kc), vc=sha(vc))
    # (2) paged_attn_prefill, seq = s1 > 0, keep-mask offset by s1 (chunked prefill)
    s1 = case["s1"]
    kc = torch.zeros([1, case["Hkv"], 1, ms, D], dtype=dt)
    vc = torch.zeros_like(kc)
    kc[:, :, :, :s1] = case["kpre"]
    vc[:, :, :, :s1] = case["vpre"]
    mask1 = torch.ones([1, S, ms], dtype=dt).tril(diagonal=s1).view(1, 1, 1, S, ms)
    o = ops.paged_attn_prefill(case["q"], case["k"], case["v"], mask1, kc, vc,
                               torch.tensor([[s1]], dtype=torch.int32), scale, bt, ms)
    res["paged_attn_prefill_s1"] = dict(out=o, seq=s1, kc=sha(kc), vc=sha(vc))
    # (3) paged_causal_attn_prefill, causal, seq = 0 (test_custom_kernel.py:837-918)
    kc = torch.zeros([1, case["Hkv"], 1, ms, D], dtype=dt)
    vc = torch.zeros_like(kc)
    o = ops.paged_causal_attn_prefill(case["q"], case["k"], case["v"], kc, vc,
                                      torch.tensor([[0]], dtype=torch.int32), scale, bt, ms, False)
    res["paged_causal_attn_prefill"] = dict(out=o, seq=0, kc=sha(kc), vc=sha(vc))
    # (4) bidirectional with a position mask covering the written span
    kc = torch.zeros([1, case["Hkv"], 1, ms, D], dtype=dt)
    vc = torch.zeros_like(kc)
    pm = torch.zeros([1, ms], dtype=dt)
    pm[:, :S] = 1
    o = ops.paged_causal_attn_prefill(case["q"], case["k"], case["v"], kc, vc,
                                      torch.tensor([[0]], dtype=torch.int32), scale, bt, ms, True, pm)
    res["paged_causal_attn_prefill_bidir"] = dict(out=o, seq=0, kc=sha(kc), vc=sha(vc))
    return res


def naive_cases(gen):
    """flash_attention_naive_{prefill,decode} on one partition, as
    test_custom_kernel.py:1003-1093 runs them (kv_cache [2, 1, Hkv, 1, P, D]
    of random values, keep-mask over [0, valid_len)), with the heads and the
    partition scaled down, plus a chunk at a nonzero offset with a causal
    keep-mask (prefill) and a longer history (decode)."""
    out = []
    Hkv, G, P = 1, 4, 64
    for dtype, D in ((torch.float16, 64), (torch.float16, 128), (torch.bfloat16, 64), (torch.float32, 64)):
        for name, decode, S, s0, causal in (("prefill", False, P, 0, False),
                                            ("prefill_offset", False, 40, 24, True),
                                            ("decode", True, 1, 32, False),
                                            ("decode_long", True, 1, 50, False)):
            q = torch.randn([1, Hkv, G, S, D], generator=gen).to(dtype)
            k = torch.randn([1, Hkv, 1, S, D], generator=gen).to(dtype)
            v = torch.randn([1, Hkv, 1, S, D], generator=gen).to(dtype)
            kv = torch.randn([2, 1, Hkv, 1, P, D], generator=gen).to(dtype)
            mask = torch.zeros([1, 1, 1, S, P], dtype=dtype)
            if causal:
                mask[0, 0, 0] = torch.ones([S, P], dtype=dtype).tril(diagonal=s0)
            else:
                mask[..., : s0 + S] = 1
            out.append(dict(name=name, decode=decode, dtype=dtype, D=D, Hkv=Hkv, G=G, P=P, S=S, s0=s0,
                            q=q, k=k, v=v, kv_cache=kv, mask=mask))
    return out


def run_naive(case):
    ops = torch.ops.rbln_custom_ops
    kv = case["kv_cache"].clone()
    scale = torch.tensor(1.0 / math.sqrt(case["D"]))
    seq_idx = torch.tensor([[case["s0"]]], dtype=torch.int32)
    bt = torch.tensor([[0]], dtype=torch.int16) if case["decode"] else torch.tensor([0], dtype=torch.int16)
    slots = torch.arange(case["S"], dtype=torch.int32)
    op = ops.flash_attention_naive_decode if case["decode"] else ops.flash_attention_naive_prefill
    o = op(case["q"], case["k"], case["v"], kv, case["mask"], scale, seq_idx, bt, slots)
    return dict(out=o, kv_cache=sha(kv))


def sdpa_bwd_cases(gen, backward):
    """The reference's SDPA backward on CPU tensors (sdpa.py:754-821: the
    attention-weight cache misses, so it runs _sdpa_attn_weights_fallback and
    _sdpa_backward_fallback, plus grad_attn_bias): GQA 4 query heads over 2
    KV heads, L = 24 queries over S = 40 keys, causal or not, with or without
    an additive float mask."""
    cases = []
    B, H, Hkv, L, S = 1, 4, 2, 24, 40
    for dtype, D in ((torch.float16, 64), (torch.float16, 128), (torch.bfloat16, 64), (torch.float32, 64)):
        for causal in (False, True):
            for masked in (False, True):
                q = torch.randn(B, H, L, D, generator=gen).to(dtype)
                k = torch.randn(B, Hkv, S, D, generator=gen).to(dtype)
                v = torch.randn(B, Hkv, S, D, generator=gen).to(dtype)
                go = torch.randn(B, H, L, D, generator=gen).to(dtype)
                mask = (torch.randn(1, H, L, S, generator=gen) * 2).to(dtype) if masked else None
                out = torch.empty(B, H, L, D, dtype=dtype)  # read only by the attention-weight cache
                e = torch.empty(0)
                dq, dk, dv, db = backward(go, q, k, v, mask, [True, True, True, masked], out, e, e, e, L, S, 0.0,
                                          causal, torch.empty(()), torch.empty(()), None)
                cases.append(dict(dtype=dtype, D=D, causal=causal, q=q, k=k, v=v, grad_out=go, mask=mask,
                                  dq=dq, dk=dk, dv=dv, dbias=db if masked else None))
    return cases


def sdpa_cases(gen, fallback):
    cases = []
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        for causal, L, S, mask_kind in ((True, 48, 48, None), (False, 32, 48, "float"), (False, 32, 48, "bool"),
                                        (True, 32, 48, None)):
            q = torch.randn([1, 4, L, 64], generator=gen).to(dtype)
            k = torch.randn([1, 2, S, 64], generator=gen).to(dtype)
            v = torch.randn([1, 2, S, 64], generator=gen).to(dtype)
            mask = None
            if mask_kind == "float":
                mask = (torch.randn([1, 1, L, S], generator=gen) * 0.5).to(dtype)
            elif mask_kind == "bool":
                mask = torch.rand([1, 4, L, S], generator=gen) > 0.2
                mask[..., 0] = True
            out = fallback(q, k, v, mask, 0.0, causal, None, enable_gqa=False)
            cases.append(dict(dtype=dtype, causal=causal, q=q, k=k, v=v, mask=mask, out=out))
    return cases


def sdpa_config1(fallback):
    """Causal GQA fp32, Llama-3.2-1B attention shape: q [1,32,512,64], k/v [1,8,512,64], N(0,1) from seed 0."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn([1, 32, 512, 64], generator=g)
    k = torch.randn([1, 8, 512, 64], generator=g)
    v = torch.randn([1, 8, 512, 64], generator=g)
    out = fallback(q, k, v, None, 0.0, True, 1.0 / 8.0, enable_gqa=False)
    rows = torch.arange(0, 512, 7)
    return dict(sha_q=sha(q), sha_k=sha(k), sha_v=sha(v), rows=rows, heads=torch.tensor([0, 5, 17, 31]),
                out_sample=out[0][[0, 5, 17, 31]][:, rows].clone(), out_sum=out.double().sum(),
                out_sumsq=(out.double() ** 2).sum())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TORCH_RBLN_REFERENCE"),
                    help="root of a RBLN-SW/torch-rbln checkout (default: $TORCH_RBLN_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or TORCH_RBLN_REFERENCE")
    fallback, backward = load_reference(args.reference)
    torch.manual_seed(0)
    gen = torch.Generator().manual_seed(1234)
    dec = decode_cases(gen)
    for c in dec:
        c["results"] = run_decode(c)
    torch.save(dec, os.path.join(HERE, "paged_decode.pt"))
    pre = prefill_cases(gen)
    for c in pre:
        c["results"] = run_prefill(c)
    torch.save(pre, os.path.join(HERE, "paged_prefill.pt"))
    torch.save(sdpa_cases(gen, fallback), os.path.join(HERE, "sdpa_small.pt"))
    torch.save(sdpa_config1(fallback), os.path.join(HERE, "sdpa_config1.pt"))
    naive = naive_cases(torch.Generator().manual_seed(4321))
    for c in naive:
        c["results"] = run_naive(c)
    torch.save(naive, os.path.join(HERE, "flash_attention_naive.pt"))
    torch.save(sdpa_bwd_cases(torch.Generator().manual_seed(987), backward), os.path.join(HERE, "sdpa_bwd.pt"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
