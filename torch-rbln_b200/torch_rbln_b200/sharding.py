"""KV-head sharding of paged decode across the GPUs of one node.

The reference has no model-parallel attention of its own: its only
collective is an all-gather through ProcessGroupRBLN
(torch_rbln/csrc/distributed/c10d/rbln/ProcessGroupRBLN.cpp:754-830), used
by tests that shard tensors by hand (test/distributed/test_tp_pp.py:268).
Here one process drives one GPU: rank r owns a contiguous slice of the KV
heads (its slice of the paged KV pool and the matching query heads), runs
rbln_custom_ops.paged_causal_attn_decode on it, and one all-gather of the
per-rank head outputs rebuilds [B, Hkv, G, 1, D] on every rank. The block
table and sequence lengths are replicated. That all-gather is the only
exchange (NCCL over NVLink / NVSwitch on GPUs, gloo on CPU).
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [h0, h1) slice of KV heads owned by `rank`."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def shard_heads(t: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    """The rank's slice of a [.., Hkv, ..] tensor along `dim` (a view)."""
    h0, h1 = kv_head_range(t.shape[dim], rank, world)
    return t.narrow(dim, h0, h1 - h0)


def all_gather_heads(out_local: torch.Tensor, world: int, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """[B, Hkv/world, G, S, D] per rank -> [B, Hkv, G, S, D] on every rank,
    heads in rank order."""
    if world == 1:
        return out_local
    x = out_local.contiguous()
    buf = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, x, group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), x, group=group)
    B, h, G, S, D = x.shape
    return buf.permute(1, 0, 2, 3, 4, 5).reshape(B, world * h, G, S, D)


def head_sharded_paged_decode(q, k, v, kcache_local, vcache_local, seq, scale, block_table, block_size,
                              mask=None, *, rank: int, world: int, group=None):
    """paged_causal_attn_decode with the KV heads split over `world` ranks.

    q, k, v hold all heads ([B, Hkv, G|1, 1, D], replicated); the caches hold
    only this rank's heads. Returns the full [B, Hkv, G, 1, D] output on
    every rank (one all-gather)."""
    ql, kl, vl = (shard_heads(t, rank, world) for t in (q, k, v))
    out_local = torch.ops.rbln_custom_ops.paged_causal_attn_decode(
        ql.contiguous(), kl.contiguous(), vl.contiguous(), kcache_local, vcache_local, seq, scale, block_table,
        block_size, mask)
    return all_gather_heads(out_local, world, group)


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2, "strides": None}


class PeerHeadOutput:
    """Output buffers of a KV-head-sharded decode that every rank writes into.

    Each rank allocates `nbuf` full-size output buffers [B, Hkv, G, 1, D] and
    a flag array of `world` uint32 with rbln_ipc_alloc, the CUDA IPC handles
    are exchanged over `group`, and every rank maps the others' buffers
    (plain peer mappings over NVLink, no multicast). The decode kernels then
    store each head's output into all ranks' buffers, and a one-warp kernel
    exchanges a per-call epoch through the flag arrays
    (rbln_paged_causal_attn_decode_peers). Calls cycle through the `nbuf`
    buffers: a rank may run one call ahead of the others, so the output of a
    call stays valid until `nbuf` calls later on this rank.
    """

    def __init__(self, shape, dtype: torch.dtype, rank: int, world: int, group=None, nbuf: int = 2):
        from . import cabi

        self._lib = cabi.lib()
        self.rank, self.world, self.nbuf = rank, world, nbuf
        self.shape, self.dtype = tuple(shape), dtype
        self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = 1
        for n in shape:
            nbytes *= n
        nbytes *= torch.empty((), dtype=dtype).element_size()
        self._local: List[int] = []
        handles = []
        for size in [nbytes] * nbuf + [4 * world]:
            ptr, h = ctypes.c_void_p(), (ctypes.c_char * cabi.IPC_HANDLE_BYTES)()
            if self._lib.rbln_ipc_alloc(size, ctypes.byref(ptr), h) != cabi.OK:
                raise RuntimeError("rbln_ipc_alloc failed")
            self._local.append(ptr.value)
            handles.append(bytes(h))
        gathered = [None] * world
        dist.all_gather_object(gathered, handles, group=group)
        self._opened: List[int] = []
        table = []  # table[i][r]: address on this GPU of rank r's i-th buffer (i == nbuf: flags)
        for i in range(nbuf + 1):
            row = []
            for r in range(world):
                if r == rank:
                    row.append(self._local[i])
                    continue
                h = (ctypes.c_char * cabi.IPC_HANDLE_BYTES).from_buffer_copy(gathered[r][i])
                ptr = ctypes.c_void_p()
                if self._lib.rbln_ipc_open(h, ctypes.byref(ptr)) != cabi.OK:
                    raise RuntimeError(f"rbln_ipc_open failed for rank {r}")
                self._opened.append(ptr.value)
                row.append(ptr.value)
            table.append(row)
        self._dev_out = [torch.tensor(table[i], dtype=torch.int64, device=self.device) for i in range(nbuf)]
        self._dev_flags = torch.tensor(table[nbuf], dtype=torch.int64, device=self.device)
        el = torch.empty((), dtype=dtype).element_size()
        self.outputs = [torch.as_tensor(_DeviceArray(self._local[i], self.shape, f"<i{el}"), device=self.device)
                        .view(dtype) for i in range(nbuf)]
        self.epoch = 0

    def next(self, head0: int):
        """(output tensor, rbln_peer_out_t) for the next call."""
        from . import cabi

        self.epoch += 1
        i = self.epoch % self.nbuf
        po = cabi.PeerOut()
        po.out, po.flags = self._dev_out[i].data_ptr(), self._dev_flags.data_ptr()
        po.n, po.rank, po.head0, po.epoch = self.world, self.rank, head0, self.epoch
        return self.outputs[i], po

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a device sync)."""
        torch.cuda.synchronize(self.device)
        for ptr in self._opened:
            self._lib.rbln_ipc_close(ctypes.c_void_p(ptr))
        for ptr in self._local:
            self._lib.rbln_ipc_free(ctypes.c_void_p(ptr))
        self._opened, self._local, self.outputs = [], [], []


def head_sharded_paged_decode_p2p(q, k, v, kcache_local, vcache_local, seq, scale, block_table, block_size,
                                  peer: PeerHeadOutput, *, workspace: Optional[dict] = None,
                                  q_is_local: bool = False):
    """head_sharded_paged_decode with the all-gather fused into the kernels:
    the local heads' outputs are stored straight into every rank's buffer in
    `peer` (NVLink peer stores) and the ranks exchange a per-call epoch
    (rbln_paged_causal_attn_decode_peers). Returns this rank's full output
    [B, Hkv, G, 1, D], valid until `peer.nbuf` calls later. With
    q_is_local, q/k/v are this rank's heads only (as in a model whose
    projections are already sharded)."""
    from . import cabi

    rank, world = peer.rank, peer.world
    if q_is_local:  # q, k, v already hold only this rank's heads
        ql, kl, vl = q, k, v
        h0 = rank * q.shape[1]
    else:
        ql, kl, vl = (shard_heads(t, rank, world).contiguous() for t in (q, k, v))
        h0, _ = kv_head_range(q.shape[1], rank, world)
    out, po = peer.next(h0)
    p, keep = cabi.paged_params(ql, kl, vl, kcache_local, vcache_local, seq, block_table, block_size, scale,
                                out=out)
    # split-K scratch: cached in `workspace` across calls when given
    cache = workspace if workspace is not None else keep
    n = ctypes.c_size_t(0)
    if cabi.lib().rbln_paged_decode_workspace_size(ctypes.byref(p), ctypes.byref(n)) != cabi.OK:
        raise RuntimeError("rbln_paged_decode_workspace_size failed")
    if n.value:
        ws = cache.get("ws")
        if ws is None or ws.numel() < n.value:
            ws = cache["ws"] = torch.empty(n.value, dtype=torch.uint8, device=q.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = cabi.lib().rbln_paged_causal_attn_decode_peers(ctypes.byref(p), ctypes.byref(po), ctypes.c_void_p(stream))
    if rc != cabi.OK:
        raise RuntimeError(f"rbln_paged_causal_attn_decode_peers failed: {rc}")
    return out
