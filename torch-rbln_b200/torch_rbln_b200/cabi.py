"""ctypes binding of the C-ABI in include/rbln_attn.h (librbln_attn.so).

This is the foreign-function view of the kernels, independent of PyTorch's
dispatcher: a caller fills `PagedAttnParams` with device pointers, strides
and dtype codes and calls an entry point with a CUDA stream handle. The
helpers at the bottom fill the struct from torch tensors, for the tests and
the benchmark.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "librbln_attn.so")

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_WORKSPACE = -3
ERR_LAUNCH = -4
ERR_NO_DEVICE = -5
ERR_SCRATCH_LIMIT = -6

DT_F32, DT_F16, DT_BF16, DT_FP8_E4M3, DT_I16, DT_I32, DT_I64, DT_BOOL = range(8)
DEVERR_BLOCK_ID_RANGE = 0x1
DEVERR_SEQ_RANGE = 0x2
DEVERR_TIMEOUT = 0x4

_DT = {
    torch.float32: DT_F32,
    torch.float16: DT_F16,
    torch.bfloat16: DT_BF16,
    torch.float8_e4m3fn: DT_FP8_E4M3,
    torch.int16: DT_I16,
    torch.int32: DT_I32,
    torch.int64: DT_I64,
    torch.bool: DT_BOOL,
    torch.uint8: DT_BOOL,
}

c_i32, c_i64, c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p


class PagedAttnParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i32), ("num_kv_heads", c_i32), ("group", c_i32), ("q_len", c_i32),
        ("head_dim", c_i32), ("num_blocks", c_i32), ("block_size", c_i32), ("max_blocks", c_i32),
        ("q", c_vp), ("q_stride", c_i64 * 4),
        ("out", c_vp), ("out_stride", c_i64 * 4),
        ("q_dtype", c_i32),
        ("k_new", c_vp), ("v_new", c_vp), ("k_new_stride", c_i64 * 3), ("v_new_stride", c_i64 * 3),
        ("kcache", c_vp), ("vcache", c_vp), ("kv_dtype", c_i32), ("cache_stride", c_i64 * 3),
        ("k_scale", c_vp), ("v_scale", c_vp), ("scale_stride", c_i64 * 2),
        ("seq", c_vp), ("seq_stride", c_i64),
        ("block_table", c_vp), ("block_table_dtype", c_i32), ("block_table_stride", c_i64),
        ("mask", c_vp), ("mask_dtype", c_i32), ("mask_len", c_i32), ("mask_stride", c_i64 * 2),
        ("causal", c_i32),
        ("scale", ctypes.c_float), ("scale_dev", c_vp),
        ("workspace", c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("error_flags", c_vp),
        ("num_splits", c_i32),
        ("prof_events", c_vp * 2),
        ("sinks", c_vp),
    ]


class SdpaParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i32), ("num_heads", c_i32), ("num_kv_heads", c_i32), ("q_len", c_i32), ("kv_len", c_i32),
        ("head_dim", c_i32), ("dtype", c_i32),
        ("q", c_vp), ("q_stride", c_i64 * 3),
        ("k", c_vp), ("k_stride", c_i64 * 3),
        ("v", c_vp), ("v_stride", c_i64 * 3),
        ("out", c_vp), ("out_stride", c_i64 * 3),
        ("lse", c_vp), ("lse_stride", c_i64 * 3),
        ("mask", c_vp), ("mask_dtype", c_i32), ("mask_additive", c_i32), ("mask_stride", c_i64 * 4),
        ("causal", c_i32), ("scale", ctypes.c_float),
        ("error_flags", c_vp),
    ]


class SdpaBwdParams(ctypes.Structure):
    _fields_ = [
        ("batch", c_i32), ("num_heads", c_i32), ("num_kv_heads", c_i32), ("q_len", c_i32), ("kv_len", c_i32),
        ("head_dim", c_i32), ("dtype", c_i32),
        ("q", c_vp), ("q_stride", c_i64 * 3),
        ("k", c_vp), ("k_stride", c_i64 * 3),
        ("v", c_vp), ("v_stride", c_i64 * 3),
        ("out", c_vp), ("out_stride", c_i64 * 3),
        ("dout", c_vp), ("dout_stride", c_i64 * 3),
        ("lse", c_vp), ("lse_stride", c_i64 * 3),
        ("dq", c_vp), ("dq_stride", c_i64 * 3),
        ("dk", c_vp), ("dk_stride", c_i64 * 3),
        ("dv", c_vp), ("dv_stride", c_i64 * 3),
        ("mask", c_vp), ("mask_dtype", c_i32), ("mask_additive", c_i32), ("mask_stride", c_i64 * 4),
        ("dbias", c_vp),
        ("causal", c_i32), ("scale", ctypes.c_float),
        ("workspace", c_vp), ("workspace_bytes", ctypes.c_size_t),
        ("error_flags", c_vp),
    ]


class PeerOut(ctypes.Structure):
    """rbln_peer_out_t: every rank's output buffer and flag array, as mapped on this GPU."""
    _fields_ = [("out", c_vp), ("flags", c_vp), ("n", c_i32), ("rank", c_i32), ("head0", c_i32),
                ("epoch", ctypes.c_uint32), ("wait_limit_us", ctypes.c_uint32)]


IPC_HANDLE_BYTES = 64

# entry points: (name, restype, argtypes)
ENTRY_POINTS = {
    "rbln_attn_abi_version": (ctypes.c_int, []),
    "rbln_paged_attn_params_sizeof": (ctypes.c_size_t, []),
    "rbln_peer_out_sizeof": (ctypes.c_size_t, []),
    "rbln_paged_decode_workspace_size": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams),
                                                        ctypes.POINTER(ctypes.c_size_t)]),
    "rbln_paged_causal_attn_decode": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams), c_vp]),
    "rbln_paged_attn_decode": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams), c_vp]),
    "rbln_paged_prefill_workspace_size": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams),
                                                         ctypes.POINTER(ctypes.c_size_t)]),
    "rbln_paged_causal_attn_prefill": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams), c_vp]),
    "rbln_paged_attn_prefill": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams), c_vp]),
    "rbln_paged_kv_write": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams), c_vp]),
    "rbln_sdpa_fwd": (ctypes.c_int, [ctypes.POINTER(SdpaParams), c_vp]),
    "rbln_sdpa_bwd_workspace_size": (ctypes.c_int, [ctypes.POINTER(SdpaBwdParams), ctypes.POINTER(ctypes.c_size_t)]),
    "rbln_sdpa_bwd": (ctypes.c_int, [ctypes.POINTER(SdpaBwdParams), c_vp]),
    "rbln_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(c_vp), c_vp]),
    "rbln_ipc_free": (ctypes.c_int, [c_vp]),
    "rbln_ipc_open": (ctypes.c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "rbln_ipc_close": (ctypes.c_int, [c_vp]),
    "rbln_paged_causal_attn_decode_peers": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams),
                                                           ctypes.POINTER(PeerOut), c_vp]),
    "rbln_paged_causal_attn_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(PagedAttnParams), c_vp]),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"{_LIB_PATH} is missing; build with "
                               "`python torch-rbln_b200/torch_rbln_b200/_build.py`")
        L = ctypes.CDLL(_LIB_PATH)
        for name, (res, args) in ENTRY_POINTS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.rbln_paged_attn_params_sizeof() != ctypes.sizeof(PagedAttnParams):
            raise RuntimeError("rbln_paged_attn_params_t layout mismatch between ctypes and the library")
        if L.rbln_peer_out_sizeof() != ctypes.sizeof(PeerOut):
            raise RuntimeError("rbln_peer_out_t layout mismatch between ctypes and the library")
        _lib = L
    return _lib


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def paged_params(q, k_new, v_new, kcache, vcache, seq, block_table, block_size, scale,
                 mask=None, k_scale=None, v_scale=None, out=None, causal=1, num_splits=0):
    """Fills PagedAttnParams from tensors laid out as the reference's ops take them.

    Returns (params, keepalive) where keepalive holds tensors that must
    outlive the call (the output among them, keepalive["out"]).
    """
    B, Hkv, G, S, D = q.shape
    out = torch.empty_like(q) if out is None else out
    bt = block_table if block_table.dim() == 2 else block_table.reshape(1, -1)
    p = PagedAttnParams()
    p.batch, p.num_kv_heads, p.group, p.q_len, p.head_dim = B, Hkv, G, S, D
    p.num_blocks, p.block_size, p.max_blocks = kcache.shape[0], block_size, bt.shape[1]
    p.q = q.data_ptr()
    for i in range(4):
        p.q_stride[i] = q.stride(i)
        p.out_stride[i] = out.stride(i)
    p.out = out.data_ptr()
    p.q_dtype = _DT[q.dtype]
    if k_new is not None:
        p.k_new, p.v_new = k_new.data_ptr(), v_new.data_ptr()
        for i, d in enumerate((0, 1, 3)):
            p.k_new_stride[i] = k_new.stride(d)
            p.v_new_stride[i] = v_new.stride(d)
    p.kcache, p.vcache = kcache.data_ptr(), vcache.data_ptr()
    p.kv_dtype = _DT[kcache.dtype]
    for i, d in enumerate((0, 1, 3)):
        p.cache_stride[i] = kcache.stride(d)
    if k_scale is not None:
        p.k_scale, p.v_scale = k_scale.data_ptr(), v_scale.data_ptr()
        p.scale_stride[0], p.scale_stride[1] = k_scale.stride(0), k_scale.stride(1)
    p.seq = seq.data_ptr()
    p.seq_stride = 1
    p.block_table = bt.data_ptr()
    p.block_table_dtype = _DT[bt.dtype]
    p.block_table_stride = 0 if bt.shape[0] == 1 else bt.stride(0)
    if mask is not None:
        p.mask = mask.data_ptr()
        p.mask_dtype = _DT[mask.dtype]
        p.mask_len = min(mask.shape[-1], p.max_blocks * block_size)
        p.mask_stride[0] = 0 if mask.shape[0] == 1 else mask.stride(0)
        p.mask_stride[1] = mask.stride(-2) if (mask.dim() >= 2 and S > 1 and mask.shape[-2] == S) else 0
    p.causal = causal
    if isinstance(scale, torch.Tensor) and scale.is_cuda:
        p.scale_dev = scale.data_ptr()
    else:
        p.scale = float(scale)
    p.num_splits = num_splits
    return p, {"out": out}


def attach_workspace(p: PagedAttnParams, device, keep: dict, prefill: bool = False) -> None:
    n = ctypes.c_size_t(0)
    query = lib().rbln_paged_prefill_workspace_size if prefill else lib().rbln_paged_decode_workspace_size
    rc = query(ctypes.byref(p), ctypes.byref(n))
    if rc != OK:
        raise RuntimeError(f"rbln_paged_decode_workspace_size failed: {rc}")
    if n.value:
        ws = torch.empty(n.value, dtype=torch.uint8, device=device)
        keep["ws"] = ws
        p.workspace, p.workspace_bytes = ws.data_ptr(), n.value


def sdpa_params(q, k, v, out, lse=None, causal=True, scale=None):
    """Fills SdpaParams for q [B, Hq, L, D], k/v [B, Hkv, S, D] (inner dim contiguous)."""
    p = SdpaParams()
    p.batch, p.num_heads, p.q_len, p.head_dim = q.shape
    p.num_kv_heads, p.kv_len = k.shape[1], k.shape[2]
    p.dtype = _DT[q.dtype]
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        setattr(p, name, t.data_ptr())
        st = getattr(p, name + "_stride")
        for i in range(3):
            st[i] = t.stride(i)
    if lse is not None:
        p.lse = lse.data_ptr()
        for i in range(3):
            p.lse_stride[i] = lse.stride(i)
    p.causal = 1 if causal else 0
    p.scale = scale if scale is not None else 1.0 / (q.shape[-1] ** 0.5)
    return p


def sdpa_bwd_params(q, k, v, out, dout, lse, dq=None, dk=None, dv=None, causal=True, scale=None):
    """Fills SdpaBwdParams (no mask); dq / dk / dv None are not computed."""
    p = SdpaBwdParams()
    p.batch, p.num_heads, p.q_len, p.head_dim = q.shape
    p.num_kv_heads, p.kv_len = k.shape[1], k.shape[2]
    p.dtype = _DT[q.dtype]
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out), ("dout", dout), ("lse", lse), ("dq", dq),
                    ("dk", dk), ("dv", dv)):
        if t is None:
            continue
        setattr(p, name, t.data_ptr())
        st = getattr(p, name + "_stride")
        for i in range(3):
            st[i] = t.stride(i)
    p.causal = 1 if causal else 0
    p.scale = scale if scale is not None else 1.0 / (q.shape[-1] ** 0.5)
    return p


def call(name: str, p: PagedAttnParams, stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return getattr(lib(), name)(ctypes.byref(p), ctypes.c_void_p(s.cuda_stream))
