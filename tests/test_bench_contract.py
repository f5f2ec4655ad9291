"""CPU checks of bench.py's input construction and record layout (no GPU).

- Weak scaling: every replica rank runs the one-GPU decode workload itself
  (the same lengths and block table, so the same bytes per rank) over its own
  KV pool data.
- Both arms build a compute record's `config` with the same function, and it
  names the workload, the parallelism, the L2 treatment and the work per step.
- The KV-write record's parity check compares caches and scales bit for bit
  and fails on a wrong write.
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


def test_kv_write_parity_catches_a_wrong_cache(monkeypatch):
    # the oracle stands in for the kernel on the CPU; a step that flips one
    # bit of every cache byte after writing must fail the check
    from oracle import paged_attention as opa

    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    wl = dict(bench.KVWRITE["kv_write_fp8_small"], B=6, Hkv=2, S=40, cmax=100)
    d = bench.build_kv_write(wl, seed=3)
    kc = torch.zeros([d["nblk"], d["Hkv"], 1, d["bs"], d["D"]], dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ks, vs = torch.ones(d["nblk"], d["Hkv"]), torch.ones(d["nblk"], d["Hkv"])

    def step():
        opa.kv_write(d["k"], d["v"], kc, vc, d["seq"], d["bt"], d["bs"], ks, vs)

    def wrong_step():
        step()
        kc.view(torch.uint8).bitwise_xor_(1)

    step()
    good = bench.kv_write_parity(d, kc, vc, ks, vs, step, n=3)
    assert good["ok"] and good["n_checked"] == 3 and good["tolerance"] == "bit-exact"
    assert not bench.kv_write_parity(d, kc, vc, ks, vs, wrong_step, n=3)["ok"]
