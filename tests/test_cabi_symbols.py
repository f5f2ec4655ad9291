"""CPU checks of the C-ABI boundary: the library loads, exports every entry
point include/*.h declares, and the ctypes struct matches the C layout."""

import ctypes
import glob
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:int|size_t|void|const char\s*\*)\s+(rbln_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_functions()
    assert "rbln_paged_causal_attn_decode" in names and "rbln_paged_attn_decode" in names


def test_library_exports_every_declared_symbol():
    from torch_rbln_b200 import cabi

    lib = ctypes.CDLL(cabi._LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(cabi.ENTRY_POINTS) <= set(declared_functions())


def test_abi_version_and_struct_size():
    from torch_rbln_b200 import cabi

    L = cabi.lib()
    assert L.rbln_attn_abi_version() == 3
    assert L.rbln_paged_attn_params_sizeof() == ctypes.sizeof(cabi.PagedAttnParams)
    assert L.rbln_peer_out_sizeof() == ctypes.sizeof(cabi.PeerOut)


@pytest.mark.parametrize("cname,pyname", [("rbln_paged_attn_params_t", "PagedAttnParams"),
                                          ("rbln_sdpa_params_t", "SdpaParams"),
                                          ("rbln_sdpa_bwd_params_t", "SdpaBwdParams"),
                                          ("rbln_peer_out_t", "PeerOut")])
def test_struct_field_offsets_match_c(cname, pyname):
    from torch_rbln_b200 import cabi

    cls = getattr(cabi, pyname)
    fields = [f for f, _ in cls._fields_]
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"rbln_attn.h\"\nint main(void){\n"
    for f in fields:
        src += f'  printf("%zu\\n", offsetof({cname}, {f}));\n'
    src += f'  printf("%zu\\n", sizeof({cname}));\n  return 0;\n}}\n'
    with tempfile.TemporaryDirectory() as td:
        c = os.path.join(td, "off.c")
        exe = os.path.join(td, "off")
        open(c, "w").write(src)
        cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
        r = subprocess.run(["gcc", c, "-o", exe, "-I", os.path.join(ROOT, "include"), "-I", cuda_inc],
                           capture_output=True, text=True)
        if r.returncode != 0:
            pytest.skip("gcc or CUDA headers unavailable: " + r.stderr[-200:])
        offs = [int(x) for x in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    got = [getattr(cls, f).offset for f in fields] + [ctypes.sizeof(cls)]
    assert offs == got


def test_torch_ops_registered_with_reference_schemas():
    import torch
    import torch_rbln_b200  # noqa: F401

    ops = torch.ops.rbln_custom_ops
    assert str(ops.paged_attn_decode.default._schema) == (
        "rbln_custom_ops::paged_attn_decode(Tensor q, Tensor k, Tensor v, Tensor mask, Tensor(a4!) kcache, "
        "Tensor(a5!) vcache, Tensor seq, Tensor scale, Tensor block_table, SymInt block_size) -> Tensor")
    assert str(ops.paged_causal_attn_decode.default._schema) == (
        "rbln_custom_ops::paged_causal_attn_decode(Tensor q, Tensor k, Tensor v, Tensor(a3!) kcache, "
        "Tensor(a4!) vcache, Tensor seq, Tensor scale, Tensor block_table, SymInt block_size, "
        "Tensor? mask=None) -> Tensor")
    assert str(ops.paged_causal_attn_prefill.default._schema) == (
        "rbln_custom_ops::paged_causal_attn_prefill(Tensor q, Tensor k, Tensor v, Tensor(a3!) kcache, "
        "Tensor(a4!) vcache, Tensor seq, Tensor scale, Tensor block_table, SymInt block_size, "
        "bool is_bidirectional, Tensor? mask=None) -> Tensor")
    assert str(ops.paged_attn_prefill.default._schema) == (
        "rbln_custom_ops::paged_attn_prefill(Tensor q, Tensor k, Tensor v, Tensor mask, Tensor(a4!) kcache, "
        "Tensor(a5!) vcache, Tensor seq, Tensor scale, Tensor block_table, SymInt block_size) -> Tensor")
    # test_custom_kernel.py:576-645
    for name in ("flash_attention_naive_prefill", "flash_attention_naive_decode"):
        assert str(getattr(ops, name).default._schema) == (
            f"rbln_custom_ops::{name}(Tensor q, Tensor k, Tensor v, Tensor(a3!) kv_cache, Tensor mask, "
            "Tensor scale, Tensor seq_idx, Tensor block_tables, Tensor slot_mapping, Tensor? sinks=None) -> Tensor")


def test_naive_wrappers_keep_the_argument_count_contract():
    """register_custom_ops.py:476,534: 9 or 10 inputs, else RuntimeError."""
    import torch_rbln_b200 as tr

    for fn in (tr.flash_attention_naive_prefill, tr.flash_attention_naive_decode):
        with pytest.raises(RuntimeError, match="takes 9 or 10 inputs"):
            fn(*([None] * 8))


def test_fake_kernels_give_q_metadata():
    import torch
    import torch_rbln_b200  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(2, 8, 4, 1, 64, dtype=torch.float16)
        k = torch.empty(2, 8, 1, 1, 64, dtype=torch.float16)
        kc = torch.empty(4, 8, 1, 16, 64, dtype=torch.float16)
        out = torch.ops.rbln_custom_ops.paged_causal_attn_decode(
            q, k, k, kc, kc, torch.empty(2, 1, dtype=torch.int32), torch.empty(()), torch.empty(2, 2, dtype=torch.int32), 16)
        assert out.shape == q.shape and out.dtype == q.dtype


def test_fake_kernel_of_the_kv_write():
    """rbln_attn::paged_kv_write traces under fake tensors (it returns nothing)."""
    import torch
    import torch_rbln_b200  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        k = torch.empty(2, 8, 1, 4, 64, dtype=torch.bfloat16)
        kc = torch.empty(16, 8, 1, 16, 64, dtype=torch.float8_e4m3fn)
        sc = torch.empty(16, 8)
        assert torch.ops.rbln_attn.paged_kv_write(k, k, kc, kc, torch.empty(2, dtype=torch.int32),
                                                  torch.empty(2, 4, dtype=torch.int32), 16, sc, sc) is None


def test_cpu_tensors_are_rejected_no_fallback():
    """No CPU fallback: the ops have no CPU kernel."""
    import torch
    import torch_rbln_b200  # noqa: F401

    q = torch.zeros(1, 1, 4, 1, 64, dtype=torch.bfloat16)
    k = torch.zeros(1, 1, 1, 1, 64, dtype=torch.bfloat16)
    kc = torch.zeros(2, 1, 1, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        torch.ops.rbln_custom_ops.paged_causal_attn_decode(
            q, k, k, kc, kc, torch.zeros(1, 1, dtype=torch.int32), torch.tensor(0.125),
            torch.zeros(1, 2, dtype=torch.int32), 16)


def test_new_entry_points_reject_bad_parameters_before_any_launch():
    """Argument checks of rbln_sdpa_bwd and rbln_paged_kv_write return their
    status codes on the host (no device work), so they run without a GPU."""
    import torch

    from torch_rbln_b200 import cabi

    L = cabi.lib()
    assert L.rbln_sdpa_bwd(None, None) == cabi.ERR_INVALID_ARGUMENT
    assert L.rbln_paged_kv_write(None, None) == cabi.ERR_INVALID_ARGUMENT
    q = torch.zeros(1, 4, 64, 64, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 64, 64, dtype=torch.bfloat16)
    lse = torch.zeros(1, 4, 64)
    p = cabi.sdpa_bwd_params(q, k, k, q, q, lse, q, k, k)
    n = ctypes.c_size_t(0)
    assert L.rbln_sdpa_bwd_workspace_size(ctypes.byref(p), ctypes.byref(n)) == cabi.OK
    assert n.value == 1 * 4 * 128 * 8  # one {lse, delta} pair per row, rows padded to 128
    p.head_dim = 96
    assert L.rbln_sdpa_bwd(ctypes.byref(p), None) == cabi.ERR_UNSUPPORTED
    p.head_dim = 64
    p.dtype = cabi.DT_F32
    assert L.rbln_sdpa_bwd(ctypes.byref(p), None) == cabi.ERR_UNSUPPORTED
    p.dtype = cabi.DT_BF16
    p.num_heads = 3  # not a multiple of the KV heads
    assert L.rbln_sdpa_bwd(ctypes.byref(p), None) == cabi.ERR_INVALID_ARGUMENT
    p.num_heads = 4
    p.q_stride[2] = 65  # rows not 16-byte aligned
    p.workspace = 0
    assert L.rbln_sdpa_bwd(ctypes.byref(p), None) == cabi.ERR_INVALID_ARGUMENT
    p.q_stride[2] = 64
    assert L.rbln_sdpa_bwd(ctypes.byref(p), None) == cabi.ERR_WORKSPACE  # no workspace given
    p.dbias = 16  # dbias without an additive mask
    assert L.rbln_sdpa_bwd(ctypes.byref(p), None) == cabi.ERR_INVALID_ARGUMENT

    kn = torch.zeros(2, 2, 1, 8, 64, dtype=torch.bfloat16)
    kc = torch.zeros(8, 2, 1, 16, 64, dtype=torch.float8_e4m3fn)
    seq = torch.zeros(2, dtype=torch.int32)
    bt = torch.zeros(2, 4, dtype=torch.int32)
    w, _ = cabi.paged_params(kn, kn, kn, kc, kc, seq, bt, 16, 1.0)
    assert L.rbln_paged_kv_write(ctypes.byref(w), None) == cabi.ERR_INVALID_ARGUMENT  # fp8 without scales
    w.head_dim = 80
    assert L.rbln_paged_kv_write(ctypes.byref(w), None) == cabi.ERR_UNSUPPORTED
    w.head_dim = 64
    w.q_dtype = cabi.DT_F32
    assert L.rbln_paged_kv_write(ctypes.byref(w), None) == cabi.ERR_UNSUPPORTED
    w.q_dtype = cabi.DT_BF16
    scales = torch.ones(8, 2)
    w.k_scale = w.v_scale = scales.data_ptr()
    w.block_table_dtype = cabi.DT_F32
    assert L.rbln_paged_kv_write(ctypes.byref(w), None) == cabi.ERR_UNSUPPORTED
