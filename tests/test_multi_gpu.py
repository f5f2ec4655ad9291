"""Head-sharded paged decode on 2 GPUs.

Skipped unless two or more GPUs are visible. Each rank owns half of the KV
heads of the pool; the full output must match the oracle within the decode
tolerance (rtol 1e-3, atol 1.2e-2) on every rank, both with an NCCL
all-gather of the head outputs and with the outputs stored straight into
every rank's buffer by the decode kernels (NVLink peer stores + epoch
barrier). NVLS is off (NCCL_NVLS_ENABLE=0), no multicast is used, and the
process group has a short timeout.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import sys
        from datetime import timedelta

        import torch.distributed as dist

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        for pth in (root, os.path.join(root, "torch-rbln_b200")):
            sys.path.insert(0, pth)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        import torch_rbln_b200  # noqa: F401
        from torch_rbln_b200 import sharding
        from oracle import paged_attention as opa
        from tests.paged_inputs import make_decode

        d = make_decode(4, 8, 8, 128, 16, [3000, 17, 1500, 4096], seed=31)
        ref = opa.paged_decode(d["q"], d["k"], d["v"], d["kcache"].clone(), d["vcache"].clone(), d["seq"],
                               d["scale"], d["block_table"], 16)
        kc = sharding.shard_heads(d["kcache"], rank, world).contiguous().to(dev)
        vc = sharding.shard_heads(d["vcache"], rank, world).contiguous().to(dev)
        out = sharding.head_sharded_paged_decode(d["q"].to(dev), d["k"].to(dev), d["v"].to(dev), kc, vc,
                                                 d["seq"].to(dev), d["scale"], d["block_table"].to(dev), 16,
                                                 rank=rank, world=world)
        torch.cuda.synchronize()
        err = None
        try:
            torch.testing.assert_close(out.cpu().float(), ref, rtol=1e-3, atol=1.2e-2)
        except AssertionError as e:
            err = str(e)[:300]
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, err))
    except Exception as e:
        q.put((rank, repr(e)))


def test_head_sharded_decode_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err in res:
        assert err is None, f"rank {rank}: {err}"


def _worker_p2p(rank, world, port, q):
    try:
        import sys
        from datetime import timedelta

        import torch.distributed as dist

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        for pth in (root, os.path.join(root, "torch-rbln_b200")):
            sys.path.insert(0, pth)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        import torch_rbln_b200  # noqa: F401
        from torch_rbln_b200 import cabi, sharding
        from oracle import paged_attention as opa
        from tests.paged_inputs import make_decode

        d = make_decode(4, 8, 8, 128, 16, [3000, 17, 1500, 4096], seed=32)
        kc = sharding.shard_heads(d["kcache"], rank, world).contiguous().to(dev)
        vc = sharding.shard_heads(d["vcache"], rank, world).contiguous().to(dev)
        peer = sharding.PeerHeadOutput(tuple(d["q"].shape), d["q"].dtype, rank, world)
        err = None
        # three calls in a row with different queries: epochs advance and the
        # two output buffers alternate
        for it in range(3):
            qi = (d["q"].float() * (1.0 + 0.25 * it)).to(d["q"].dtype)
            ref = opa.paged_decode(qi, d["k"], d["v"], d["kcache"].clone(), d["vcache"].clone(), d["seq"],
                                   d["scale"], d["block_table"], 16)
            out = sharding.head_sharded_paged_decode_p2p(qi.to(dev), d["k"].to(dev), d["v"].to(dev), kc, vc,
                                                         d["seq"].to(dev), d["scale"], d["block_table"].to(dev),
                                                         16, peer)
            torch.cuda.synchronize()
            try:
                torch.testing.assert_close(out.cpu().float(), ref, rtol=1e-3, atol=1.2e-2)
            except AssertionError as e:
                err = f"call {it}: " + str(e)[:300]
                break
        if err is None:
            try:
                peer.check()  # no exchange timed out
            except sharding.ShardedDecodeError as e:
                err = str(e)
        dist.barrier()
        peer.close()
        dist.destroy_process_group()
        q.put((rank, err))
    except Exception as e:
        q.put((rank, repr(e)))


def test_head_sharded_decode_p2p_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_p2p, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err in res:
        assert err is None, f"rank {rank}: {err}"
