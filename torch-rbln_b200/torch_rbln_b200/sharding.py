"""Sharding of paged decode across the GPUs of one node.

The reference has no model-parallel attention of its own: its only
collective is an all-gather through ProcessGroupRBLN
(torch_rbln/csrc/distributed/c10d/rbln/ProcessGroupRBLN.cpp:754-830), used
by tests that shard tensors by hand (test/distributed/test_tp_pp.py:268).
Here one process drives one GPU, and a batch is split one of two ways:

  * by KV head: rank r owns a contiguous slice of the KV heads (its slice of
    the paged KV pool and the matching query heads), runs
    rbln_custom_ops.paged_causal_attn_decode on it, and one all-gather of
    the per-rank head outputs rebuilds [B, Hkv, G, 1, D] on every rank. The
    block table and sequence lengths are replicated. That all-gather is the
    only exchange (NCCL over NVLink / NVSwitch on GPUs, gloo on CPU), or it
    is fused into the decode kernels as NVLink peer stores (PeerHeadOutput).
  * by sequence: the sequences of a decode batch are independent (the
    reference's CPU definition loops over them, test/rbln/test_custom_kernel.py:
    437-482), so rank r holds B / N of them with its own pool of their blocks
    and its own block table, and no collective is needed at all.

A rank that fails before a collective (an exception, or a process that
never joins) surfaces on the others as ShardedDecodeError once the process
group's timeout expires, the analogue of the reference's process-group
timeout (ProcessGroupRBLN.hpp:46).
"""

from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist


class ShardedDecodeError(RuntimeError):
    """A sharded decode step could not complete on this rank: a peer rank
    failed or never joined the exchange (its collective timed out or its
    connection closed), or a device-side wait for a peer's outputs gave up."""


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
    try:
        if dist.get_backend(group) == "nccl":
            dist.all_gather_into_tensor(buf, x, group=group)
        else:
            dist.all_gather(list(buf.unbind(0)), x, group=group)
    except (RuntimeError, dist.DistError) as e:
        raise ShardedDecodeError(
            f"rank {dist.get_rank(group)} of {world}: the head-output all-gather failed; a peer rank "
            f"failed or did not join before the process group's timeout ({type(e).__name__}: {e})") from e
    B, h, G, S, D = x.shape
    return buf.permute(1, 0, 2, 3, 4, 5).reshape(B, world * h, G, S, D)


def batch_partition(lengths: torch.Tensor, world: int, balanced: bool = True) -> List[torch.Tensor]:
    """Sequence indices each of `world` ranks holds when a decode batch is
    split by sequence. Every rank gets len(lengths) // world sequences (the
    first len % world ranks one more).

    balanced=False: contiguous ranges [r * B / world, (r + 1) * B / world).
    balanced=True: sequences sorted by length, longest first, dealt out in
    snake order (0, 1, .., N-1, N-1, .., 0, 0, ..), which keeps the counts
    equal and the ranks' token totals close, so that no rank holds the
    step up (each rank's time is its own tokens). Indices within a rank are
    ascending."""
    if world <= 0:
        raise ValueError(f"bad world size {world}")
    B = int(lengths.numel())
    if not balanced:
        out, start = [], 0
        for r in range(world):
            n = B // world + (1 if r < B % world else 0)
            out.append(torch.arange(start, start + n, dtype=torch.int64))
            start += n
        return out
    order = torch.argsort(lengths.reshape(-1).to(torch.int64), descending=True, stable=True).tolist()
    parts: List[List[int]] = [[] for _ in range(world)]
    for i, b in enumerate(order):
        lap, k = divmod(i, world)
        parts[k if lap % 2 == 0 else world - 1 - k].append(b)
    return [torch.tensor(sorted(p), dtype=torch.int64) for p in parts]


def shard_batch(seq: torch.Tensor, block_table: torch.Tensor, block_size: int,
                indices: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """One rank's part of a batch split by sequence.

    For the sequences `indices` (decode: seq[b] is the new token's position,
    so blocks [0, ceil((seq[b] + 1) / block_size)) are in use) returns
    (blocks, local_table): the global physical ids of the blocks they use,
    each once, in order of first use, and their rows of the block table
    renumbered into positions of `blocks`. The rank's pools are
    pool[blocks] (K, V and fp8 scales alike), so it holds only its own
    sequences' blocks. Table entries past a sequence's blocks are 0 (never
    read). A block shared by sequences of two ranks is copied into both."""
    bt = block_table if block_table.dim() == 2 else block_table.reshape(1, -1)
    seqv = seq.reshape(-1).to(torch.int64)
    idx = indices.to(torch.int64)
    local = torch.zeros((idx.numel(), bt.shape[1]), dtype=bt.dtype)
    remap = {}
    blocks: List[int] = []
    for i, b in enumerate(idx.tolist()):
        row = bt[b if bt.shape[0] > 1 else 0].tolist()
        used = min(len(row), max(0, int(math.ceil((int(seqv[b]) + 1) / block_size))))
        for j in range(used):
            g = int(row[j])
            if g not in remap:
                remap[g] = len(blocks)
                blocks.append(g)
            local[i, j] = remap[g]
    return torch.tensor(blocks, dtype=torch.int64), local


def scatter_batch(outputs: Sequence[torch.Tensor], parts: Sequence[torch.Tensor]) -> torch.Tensor:
    """Reassembles per-rank decode outputs [len(parts[r]), ...] into batch
    order (for checks; the decode itself needs no exchange)."""
    B = sum(int(p.numel()) for p in parts)
    first = outputs[0]
    full = torch.empty((B,) + tuple(first.shape[1:]), dtype=first.dtype, device=first.device)
    for o, p in zip(outputs, parts):
        full[p.to(full.device)] = o
    return full


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


def raise_on_device_error(bits: int, rank: int, world: int, epoch: int) -> None:
    """Turns a head-sharded decode's device error word (RBLN_DEVERR_* bits)
    into ShardedDecodeError; 0 passes."""
    from . import cabi

    if not bits:
        return
    what = ("timed out waiting for a peer rank's outputs" if bits & cabi.DEVERR_TIMEOUT
            else "met an invalid block id or position")
    raise ShardedDecodeError(f"rank {rank} of {world}: head-sharded decode {what} "
                             f"(error bits 0x{bits:x}, by epoch {epoch}); remote heads may be stale")


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

    The wait for the other ranks' epochs is bounded by `wait_limit_us` of GPU
    time. When it runs out (a rank died or never launched its part), the
    kernel sets RBLN_DEVERR_TIMEOUT in this object's device error word and
    returns, leaving that call's remote heads stale; check() (a host sync)
    raises ShardedDecodeError from then on. The word is never cleared: the
    exchange cannot be trusted again without a new process group.
    """

    def __init__(self, shape, dtype: torch.dtype, rank: int, world: int, group=None, nbuf: int = 2,
                 wait_limit_us: int = 2_000_000):
        from . import cabi

        self._lib = cabi.lib()
        self.rank, self.world, self.nbuf = rank, world, nbuf
        self.wait_limit_us = int(wait_limit_us)
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
        self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0

    def next(self, head0: int):
        """(output tensor, rbln_peer_out_t) for the next call. The call must
        pass error_word (its data_ptr) as the parameter block's error_flags."""
        from . import cabi

        self.epoch += 1
        i = self.epoch % self.nbuf
        po = cabi.PeerOut()
        po.out, po.flags = self._dev_out[i].data_ptr(), self._dev_flags.data_ptr()
        po.n, po.rank, po.head0, po.epoch = self.world, self.rank, head0, self.epoch
        po.wait_limit_us = self.wait_limit_us
        return self.outputs[i], po

    def check(self) -> None:
        """Waits for this rank's calls so far and raises ShardedDecodeError if
        any of them saw a device-side error (a timed-out epoch exchange)."""
        torch.cuda.synchronize(self.device)
        raise_on_device_error(int(self.error_word.item()), self.rank, self.world, self.epoch)

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
                                  q_is_local: bool = False, check: bool = False):
    """head_sharded_paged_decode with the all-gather fused into the kernels:
    the local heads' outputs are stored straight into every rank's buffer in
    `peer` (NVLink peer stores) and the ranks exchange a per-call epoch
    (rbln_paged_causal_attn_decode_peers). Returns this rank's full output
    [B, Hkv, G, 1, D], valid until `peer.nbuf` calls later. With
    q_is_local, q/k/v are this rank's heads only (as in a model whose
    projections are already sharded). A timed-out exchange is recorded in
    peer.error_word; check=True synchronises and raises ShardedDecodeError
    on it at once (otherwise peer.check() does, at a point of the caller's
    choosing)."""
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
    p.error_flags = peer.error_word.data_ptr()
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
    if check:
        peer.check()
    return out
