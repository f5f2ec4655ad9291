"""CPU checks of bench.py's input construction and record layout (no GPU).

- Weak scaling: every replica rank runs the one-GPU decode workload itself
  (the same lengths and block table, so the same bytes per rank) over its own
  KV pool data.
- Both arms build a compute record's `config` with the same function, and it
  names the workload, the parallelism, the L2 treatment and the work per step.
"""

import torch

import bench


def _tiny_decode():
    # the headline workload's shape rules at a size that builds in milliseconds
    return dict(bench.WORKLOADS["decode"], B=6, Hkv=2, G=4, D=64, lmin=16, lmax=200, pool=120)


def test_replicas_share_lengths_and_block_table():
    wl = _tiny_decode()
    cpu = torch.device("cpu")
    r0 = bench.build_decode_sharded(wl, "replicas", 0, 2, cpu)
    r1 = bench.build_decode_sharded(wl, "replicas", 1, 2, cpu)
    one = bench.build_decode(wl, cpu, seed=0)
    assert torch.equal(r0["lens"], r1["lens"]) and torch.equal(r0["lens"], one["lens"])
    assert torch.equal(r0["bt"], r1["bt"]) and torch.equal(r0["seq"], r1["seq"])
    assert bench.decode_bytes(r0) == bench.decode_bytes(r1)
    assert not torch.equal(r0["kcache"], r1["kcache"])  # each rank its own KV data
    assert torch.equal(r0["kcache"], one["kcache"])     # rank 0 is the one-GPU workload


def test_compute_config_fields():
    wl = bench.COMPUTE["sdpa"]
    d = {"flops": 123}
    cfg = bench.compute_config(wl, d, 1)
    assert cfg == {"workload": wl["desc"], "parallelism": "single GPU", "l2": bench.L2_FLUSH_NOTE,
                   "flops_per_step": 123}
    assert bench.compute_config(wl, d, 4)["parallelism"] == "replicas x4"
    kv = bench.kv_write_config(bench.KVWRITE["kv_write_fp8"], {"bytes": 7}, 1)
    assert kv["bytes_per_step"] == 7 and kv["l2"] == bench.L2_FLUSH_NOTE
