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


# ---------------------------------------------------------------------------
# batch split by sequence (the fp8 decode workload's partitioning)
# ---------------------------------------------------------------------------
def test_batch_partition_counts_and_balance():
    g = torch.Generator().manual_seed(3)
    lens = torch.randint(512, 8193, (256,), generator=g)
    for world in (1, 2, 4, 8):
        for balanced in (False, True):
            parts = sharding.batch_partition(lens, world, balanced=balanced)
            allidx = torch.cat(parts).sort().values
            assert torch.equal(allidx, torch.arange(256))            # every sequence exactly once
            assert {int(p.numel()) for p in parts} == {256 // world}  # equal counts
        # snake order keeps the ranks' token totals within a few percent
        tot = [int(lens[p].sum()) for p in sharding.batch_partition(lens, world)]
        assert max(tot) / (sum(tot) / world) < 1.02
    # contiguous ranges when not balanced, uneven B
    parts = sharding.batch_partition(torch.ones(10), 4, balanced=False)
    assert [p.tolist() for p in parts] == [[0, 1, 2], [3, 4, 5], [6, 7], [8, 9]]


def test_shard_batch_renumbers_blocks():
    bt = torch.tensor([[7, 3, 9, 0], [2, 5, 0, 0], [4, 8, 6, 1]], dtype=torch.int32)
    seq = torch.tensor([[40], [17], [3]], dtype=torch.int32)  # 3, 2 and 1 blocks in use (bs = 16)
    blocks, local = sharding.shard_batch(seq, bt, 16, torch.tensor([0, 2]))
    assert blocks.tolist() == [7, 3, 9, 4]
    assert local.tolist() == [[0, 1, 2, 0], [3, 0, 0, 0]]
    assert local.dtype == bt.dtype


def _batch_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        from oracle import paged_attention as opa
        from tests.paged_inputs import make_decode

        lens = [700, 33, 1300, 512, 90, 2049, 16, 640]
        d = make_decode(8, 2, 4, 64, 16, lens, seed=9, fp8=True)
        full = opa.paged_decode(d["q"], d["k"], d["v"], d["kcache"].clone(), d["vcache"].clone(), d["seq"],
                                d["scale"], d["block_table"], 16, k_scale=d["k_scale"].clone(),
                                v_scale=d["v_scale"].clone())
        parts = sharding.batch_partition(torch.tensor(lens), world)
        idx = parts[rank]
        blocks, table = sharding.shard_batch(d["seq"], d["block_table"], 16, idx)
        # this rank holds only its sequences' blocks, renumbered
        local = opa.paged_decode(d["q"][idx], d["k"][idx], d["v"][idx], d["kcache"][blocks].clone(),
                                 d["vcache"][blocks].clone(), d["seq"][idx], d["scale"], table, 16,
                                 k_scale=d["k_scale"][blocks].clone(), v_scale=d["v_scale"][blocks].clone())
        # the check gathers the outputs (the split decode itself needs no exchange)
        outs = [None] * world
        dist.all_gather_object(outs, local)
        got = sharding.scatter_batch(outs, parts)
        ok = torch.equal(got, full) and blocks.numel() < d["kcache"].shape[0]
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, None))
    except Exception as e:
        q.put((rank, False, repr(e)))


def test_batch_sharded_decode_gloo_matches_unsharded_bitwise():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert ok, rank


# ---------------------------------------------------------------------------
# failure detection: a rank that fails before the head all-gather
# ---------------------------------------------------------------------------
def _failing_worker(rank, world, port, q, mode, release):
    """Rank 1 raises before the all-gather and then either stays alive
    without joining (mode "stall") or exits its process (mode "exit").
    Rank 0 must get ShardedDecodeError within the process group's timeout."""
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    x = torch.full((2, 4, 4, 1, 16), float(rank))
    if rank == 1:
        try:
            raise RuntimeError("injected failure on rank 1 before the head all-gather")
        except RuntimeError as e:
            q.put((rank, "raised", repr(e), 0.0))
        q.close()
        q.join_thread()  # flush the message before the process ends abruptly
        if mode == "exit":
            os._exit(1)
        release.wait(30)  # alive, never joins the collective
        os._exit(0)
    t0 = time.monotonic()
    try:
        sharding.all_gather_heads(x, world)
        q.put((rank, "no error", None, time.monotonic() - t0))
    except sharding.ShardedDecodeError as e:
        q.put((rank, "ShardedDecodeError", str(e)[:300], time.monotonic() - t0))
    except Exception as e:  # any other type is a failure of the contract
        q.put((rank, type(e).__name__, str(e)[:300], time.monotonic() - t0))
    q.close()
    q.join_thread()
    os._exit(0)  # the group is broken: leave without a collective teardown


@pytest.mark.parametrize("mode", ["stall", "exit"])
def test_rank_failure_before_all_gather_raises_on_the_others(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    release = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q, mode, release)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = {r: (what, msg, dt) for r, what, msg, dt in (q.get(timeout=120) for _ in procs)}
    finally:
        release.set()
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[1][0] == "raised"
    what, msg, dt = res[0]
    assert what == "ShardedDecodeError", (what, msg)
    assert "rank 0 of 2" in msg
    assert dt < 60, dt  # bounded by the 3 s process-group timeout, not a hang
