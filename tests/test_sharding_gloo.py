"""Host-side logic of KV-head sharding, on CPU with world_size-2 gloo ranks."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from torch_rbln_b200 import sharding


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_kv_head_range():
    assert sharding.kv_head_range(8, 0, 2) == (0, 4)
    assert sharding.kv_head_range(8, 3, 4) == (6, 8)
    with pytest.raises(ValueError):
        sharding.kv_head_range(8, 0, 3)
    with pytest.raises(ValueError):
        sharding.kv_head_range(8, 2, 2)


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import paged_attention as opa
        from tests.paged_inputs import make_decode

        # (1) all-gather assembly: heads come back in rank order
        full = torch.arange(2 * 8 * 4 * 1 * 16, dtype=torch.float32).reshape(2, 8, 4, 1, 16)
        got = sharding.all_gather_heads(sharding.shard_heads(full, rank, world).contiguous(), world)
        ok1 = torch.equal(got, full)
        # (2) the oracle's decode sharded by heads + all-gather == unsharded
        d = make_decode(3, 8, 4, 64, 16, [40, 300, 129], seed=5)
        ref = opa.paged_decode(d["q"], d["k"], d["v"], d["kcache"].clone(), d["vcache"].clone(), d["seq"],
                               d["scale"], d["block_table"], 16)
        sl = lambda t: sharding.shard_heads(t, rank, world)
        local = opa.paged_decode(sl(d["q"]), sl(d["k"]), sl(d["v"]), sl(d["kcache"]).clone(),
                                 sl(d["vcache"]).clone(), d["seq"], d["scale"], d["block_table"], 16)
        got2 = sharding.all_gather_heads(local, world)
        ok2 = torch.equal(got2, ref)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok1, ok2, None))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, False, repr(e)))


def test_head_sharded_decode_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok1, ok2, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert ok1 and ok2, (rank, ok1, ok2)
