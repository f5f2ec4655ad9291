"""B200 (sm_100a) attention hot path for torch-rbln's operator interface.

Importing this package:
  * loads librbln_attn_torch.so, which defines the rbln_custom_ops schemas
    (identical to the reference's, test/rbln/test_custom_kernel.py:31-486) and
    registers their CUDA kernels; those call the C-ABI in librbln_attn.so
    (include/rbln_attn.h). The same library registers the SDPA route: CUDA
    kernels for aten::_scaled_dot_product_fused_attention_overrideable and
    its backward, and a CUDA _fused_sdp_choice that selects them, mirroring
    the reference's registration (aten/src/ATen/native/RBLNRegisterOps.cpp:
    89-105);
  * registers shape-only (fake) implementations for tracing, as the
    reference does with `register_fake` (test_custom_kernel.py:95-135 ...).

There is no CPU fallback: the ops have CUDA kernels only, and importing
fails if the native libraries have not been built (run
`python torch-rbln_b200/torch_rbln_b200/_build.py` or `__graft_entry__.build()`).
"""

from __future__ import annotations

import os

import torch

_LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
CABI_LIBRARY = os.path.join(_LIB_DIR, "librbln_attn.so")
TORCH_LIBRARY = os.path.join(_LIB_DIR, "librbln_attn_torch.so")

if not (os.path.exists(CABI_LIBRARY) and os.path.exists(TORCH_LIBRARY)):
    raise ImportError(
        "torch_rbln_b200: native libraries are missing from "
        f"{_LIB_DIR}; build them with `python torch-rbln_b200/torch_rbln_b200/_build.py`")

torch.ops.load_library(TORCH_LIBRARY)

from . import _fake  # noqa: E402,F401  (registers fake kernels)
from .ops import (  # noqa: E402,F401
    flash_attention_naive_decode,
    flash_attention_naive_prefill,
    paged_attn_decode,
    paged_attn_prefill,
    paged_causal_attn_decode,
    paged_causal_attn_decode_kvfp8,
    paged_causal_attn_prefill,
)

__all__ = [
    "flash_attention_naive_decode",
    "flash_attention_naive_prefill",
    "paged_attn_decode",
    "paged_attn_prefill",
    "paged_causal_attn_decode",
    "paged_causal_attn_decode_kvfp8",
    "paged_causal_attn_prefill",
    "CABI_LIBRARY",
    "TORCH_LIBRARY",
]
