#!/usr/bin/env python
"""Benchmark of the B200 attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload suite|decode|decode_fp8|decode_long|prefill|sdpa|sdpa_bf16|sdpa_bwd|...]

Default (`--workload suite`): one JSON line whose headline is the paged
decode (bf16, batch 64, 32 query / 8 KV heads, head_dim 128, block_size 16,
context length per sequence uniform in [128, 4096], block table = seeded
random permutation of a 20,000-block KV pool, K/V ~ N(0,1)*0.5, one new
token per sequence; metric: algorithmic HBM bytes per step / time, GB/s),
and whose `workloads` object carries one record per other workload of the
metric, each with its own value, roofline, e2e, clocks, parity and (rank 0,
one GPU) CPU baseline:

  long_context_decode  batch 32, 64 query / 8 KV heads, context 32768, bf16;
                       KV heads sharded over the ranks, the head outputs
                       stored into every rank's buffer by the decode kernels
                       (strong scaling; run at every N)
  fp8_decode           fp8-e4m3 KV with per-(block, head) scales, batch 256,
                       context ~U[512, 8192]; the batch split by sequence
                       over the ranks, each with its own pool and block
                       table (strong scaling, global batch 256 at every N)
  chunked_prefill      batch 8 x 512 new tokens, cached context ~U[0, 8192],
                       32 / 8 heads, head_dim 128, causal (TFLOP/s; N = 1)
  sdpa_f32             causal GQA SDPA fp32, 1 x 32 / 8 heads x 512 x 64 (N = 1)
  sdpa_backward        causal GQA SDPA backward bf16, 2 x 32 / 8 x 4096 x 128 (N = 1)
  kv_write_fp8         the standalone fp8 KV-cache write (N = 1)

A decode step is one call of the op over the batch (append + attention).
`value` times K steps with inputs resident in HBM (CUDA events around the
whole loop, no events inside it); `roofline` times the main kernel alone in
a separate loop, with CUDA events that the C-ABI records on the launch
stream around that kernel; `e2e` times the public torch API with the step's
inputs copied from pinned host memory (for decode, packed into one staging
buffer and one copy per step) and the result copied back inside the timed
region. Decode pools are far larger than the 126 MB L2; the compute
workloads flush L2 (a 256 MB write) before each timed iteration.

Under torchrun (N > 1) the headline runs N replicas of the decode batch
(sequences are independent; no collective on the data path): every rank the
one-GPU workload's lengths and block table over its own KV data, so the
per-GPU work is fixed; every number is whole-job work over the
max-over-ranks device time.

`parity` in each record compares the output of the last timed call with the
CPU oracle (oracle/paged_attention.py, oracle/sdpa.py) on a seeded subset of
the sequences, on every rank; for the head-sharded decode every rank's full
output buffer must also be bit-identical to every other rank's.

--impl reference times the reference's CPU algorithm for the same workloads
on this host's cores (the oracle's restatement of the reference CPU ops, on
bounded samples), rank 0 only.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "torch-rbln_b200"))

import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
RTOL, ATOL = 1e-3, 1.2e-2  # the reference's tolerance, test/rbln/test_custom_kernel.py:654-655


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
# shard: how a workload is split over N > 1 ranks ("replicas": every rank its
# own batch; "heads": KV heads sharded; "batch": sequences split)
WORKLOADS = {
    "decode": dict(desc="paged decode bf16 B=64 Hq=32 Hkv=8 D=128 bs=16 L~U[128,4096] pool=20000",
                   B=64, Hkv=8, G=4, D=128, bs=16, lmin=128, lmax=4096, pool=20000, fp8=False, shard="replicas"),
    "decode_fp8": dict(desc="paged decode fp8-e4m3 KV B=256 Hq=32 Hkv=8 D=128 bs=16 L~U[512,8192]",
                       B=256, Hkv=8, G=4, D=128, bs=16, lmin=512, lmax=8192, pool=None, fp8=True, shard="batch"),
    "decode_long": dict(desc="paged decode bf16 B=32 Hq=64 Hkv=8 D=128 bs=16 L=32768 pool=65536",
                        B=32, Hkv=8, G=8, D=128, bs=16, lmin=32768, lmax=32768, pool=65536, fp8=False,
                        shard="heads"),
    # profiling cases for ncu --set full: inputs still larger than L2, well under 1 GB on the device
    "decode_small": dict(desc="paged decode bf16 B=16 Hq=32 Hkv=8 D=128 bs=16 L~U[128,4096] pool=5000",
                         B=16, Hkv=8, G=4, D=128, bs=16, lmin=128, lmax=4096, pool=5000, fp8=False,
                         shard="replicas"),
    "decode_fp8_small": dict(desc="paged decode fp8-e4m3 KV B=64 Hq=32 Hkv=8 D=128 bs=16 L~U[512,8192]",
                             B=64, Hkv=8, G=4, D=128, bs=16, lmin=512, lmax=8192, pool=None, fp8=True,
                             shard="replicas"),
}

COMPUTE = {
    "prefill": dict(kind="prefill", B=8, Hkv=8, G=4, D=128, bs=16, S=512, cmin=0, cmax=8192,
                    desc="paged chunked prefill bf16 B=8 Hq=32 Hkv=8 D=128 S_q=512 new tokens, "
                         "cached ctx~U[0,8192], bs=16, causal"),
    "prefill_small": dict(kind="prefill", B=2, Hkv=8, G=4, D=128, bs=16, S=512, cmin=2048, cmax=6144,
                          desc="paged chunked prefill bf16 B=2 Hq=32 Hkv=8 D=128 S_q=512 ctx~U[2048,6144]"),
    # the same chunks through paged_attn_prefill with an offset-causal keep-mask [B, 1, 1, S_q, span]
    # (key t kept for query row s when t <= ctx_b + s), as the reference's tests drive that op
    "prefill_mask": dict(kind="prefill", keep_mask=True, B=8, Hkv=8, G=4, D=128, bs=16, S=512, cmin=0, cmax=8192,
                         desc="paged chunked prefill with a keep-mask (paged_attn_prefill) bf16 B=8 Hq=32 Hkv=8 "
                              "D=128 S_q=512 new tokens, cached ctx~U[0,8192], bs=16, offset-causal bf16 mask"),
    "prefill_mask_small": dict(kind="prefill", keep_mask=True, B=2, Hkv=8, G=4, D=128, bs=16, S=512, cmin=2048,
                               cmax=6144, desc="paged chunked prefill with a keep-mask bf16 B=2 Hq=32 Hkv=8 D=128 "
                                               "S_q=512 ctx~U[2048,6144]"),
    "sdpa": dict(kind="sdpa", B=1, Hq=32, Hkv=8, L=512, D=64, dtype=torch.float32,
                 desc="SDPA causal GQA fp32 B=1 Hq=32 Hkv=8 L=S=512 D=64 (Llama-3.2-1B attention shape)"),
    "sdpa_bf16": dict(kind="sdpa", B=4, Hq=32, Hkv=8, L=4096, D=128, dtype=torch.bfloat16,
                      desc="SDPA causal GQA bf16 B=4 Hq=32 Hkv=8 L=S=4096 D=128"),
    "sdpa_bwd": dict(kind="sdpa_bwd", B=2, Hq=32, Hkv=8, L=4096, D=128, dtype=torch.bfloat16,
                     desc="SDPA backward causal GQA bf16 B=2 Hq=32 Hkv=8 L=S=4096 D=128 (dq, dk, dv)"),
    "sdpa_bwd_small": dict(kind="sdpa_bwd", B=1, Hq=32, Hkv=8, L=2048, D=128, dtype=torch.bfloat16,
                           desc="SDPA backward causal GQA bf16 B=1 Hq=32 Hkv=8 L=S=2048 D=128 (dq, dk, dv)"),
}

KVWRITE = {
    "kv_write_fp8": dict(B=64, Hkv=8, D=128, bs=16, S=512, cmax=4096,
                         desc="paged KV write bf16 -> fp8-e4m3 cache, per-(block, head) scale recompute: B=64 "
                              "sequences x 512 new rows, Hkv=8, D=128, bs=16, start ~U[0,4096]"),
    "kv_write_fp8_small": dict(B=16, Hkv=8, D=128, bs=16, S=512, cmax=4096,
                               desc="paged KV write bf16 -> fp8-e4m3 cache: B=16 sequences x 512 new rows, Hkv=8, "
                                    "D=128, bs=16"),
}

# the default line: headline workload, then the records of `workloads`
# (name in the line -> workload, and whether it runs at N > 1)
SUITE_HEADLINE = "decode"
SUITE = [("long_context_decode", "decode_long", True), ("fp8_decode", "decode_fp8", True),
         ("chunked_prefill", "prefill", False), ("chunked_prefill_keep_mask", "prefill_mask", False),
         ("sdpa_f32", "sdpa", False),
         ("sdpa_backward", "sdpa_bwd", False), ("kv_write_fp8", "kv_write_fp8", False)]


# ---------------------------------------------------------------------------
# run context (one process per GPU)
# ---------------------------------------------------------------------------
class Ctx:
    def __init__(self, with_gpu: bool = True):
        self.ws = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = None
        self.stream = None
        self.pg = False
        if with_gpu:
            torch.cuda.set_device(self.local)
            self.dev = torch.device("cuda", self.local)
            self.stream = torch.cuda.current_stream(self.dev)
            if self.ws > 1:
                import torch.distributed as dist
                from datetime import timedelta

                dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.dev)
                self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def reduce(self, values, op="max"):
        """Element-wise max / min / sum of a list of floats over the ranks."""
        if not self.pg:
            return list(values)
        import torch.distributed as dist

        t = torch.tensor([float(x) for x in values], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
        return t.tolist()

    def close(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _traffic_from_profiles(wl_name):
    """DRAM bytes per launch of the main kernel, from the committed ncu summary
    (a `traffic_bytes_per_launch[<workload>]: N` line), if one exists."""
    import glob
    import re

    key = f"traffic_bytes_per_launch[{wl_name}]:"
    for p in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        for line in open(p):
            if line.startswith(key):
                m = re.search(r"(\d+)", line[len(key):])
                if m:
                    return int(m.group(1))
    return None


def _event_pairs(n, stream):
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for a, b in ev:  # create the events on the device before timing
        a.record(stream)
        b.record(stream)
    return ev


def _tolerance_stats(got: torch.Tensor, ref: torch.Tensor, rtol: float, atol: float):
    got, ref = got.float(), ref.float()
    both_nan = torch.isnan(got) & torch.isnan(ref)
    d = (got - ref).abs().masked_fill(both_nan, 0.0)
    ok = bool(((d <= atol + rtol * ref.abs().masked_fill(both_nan, 0.0)) | both_nan).all())
    scale = float(ref.abs().masked_fill(both_nan, 0.0).max()) or 1.0
    return ok, float(d.max()) if d.numel() else 0.0, float(d.max()) / scale if d.numel() else 0.0


# ---------------------------------------------------------------------------
# decode inputs
# ---------------------------------------------------------------------------
def decode_layout(wl: dict, seed: int, Hkv: int = None):
    """Seeded lengths, block table (over a pool of `nblk` blocks) and
    q / k / v on the CPU. Each sequence takes its blocks from a seeded random
    permutation of the pool, in turn."""
    g = torch.Generator().manual_seed(seed)
    B, G, D, bs = wl["B"], wl["G"], wl["D"], wl["bs"]
    Hkv = Hkv or wl["Hkv"]
    lens = torch.randint(wl["lmin"], wl["lmax"] + 1, (B,), generator=g)
    max_blocks = int(math.ceil(int(lens.max()) / bs))
    nblk = wl["pool"] or int(sum(math.ceil(int(x) / bs) for x in lens)) + B
    nblk = max(nblk, B * max_blocks)
    perm = torch.randperm(nblk, generator=g)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    cursor = 0
    for b in range(B):
        n = int(math.ceil(int(lens[b]) / bs))
        bt[b, :n] = perm[cursor:cursor + n].to(torch.int32)
        cursor += n
    q = torch.randn([B, Hkv, G, 1, D], generator=g).to(torch.bfloat16)
    k = (torch.randn([B, Hkv, 1, 1, D], generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn([B, Hkv, 1, 1, D], generator=g) * 0.5).to(torch.bfloat16)
    seq = (lens - 1).to(torch.int32).reshape(B, 1)
    return dict(q=q, k=k, v=v, seq=seq, bt=bt, lens=lens, nblk=nblk)


def decode_pool(nblk, Hkv, bs, D, fp8, device, seed):
    """The KV pool, drawn on `device` (N(0,1) * 0.5 for bf16; N(0,1)
    quantised per (block, head) with scale = amax / 448 for fp8)."""
    gd = torch.Generator(device=device).manual_seed(seed)
    shape = [nblk, Hkv, 1, bs, D]
    if fp8:
        kc, ks = _fp8_pool(shape, gd, device)
        vc, vs = _fp8_pool(shape, gd, device)
        return kc, vc, ks, vs
    kc = torch.randn(shape, generator=gd, device=device, dtype=torch.bfloat16) * 0.5
    vc = torch.randn(shape, generator=gd, device=device, dtype=torch.bfloat16) * 0.5
    return kc, vc, None, None


def _fp8_pool(shape, gd, device):
    x = torch.randn(shape, generator=gd, device=device, dtype=torch.float32)
    amax = x.abs().amax(dim=(2, 3, 4)).clamp_min(1e-6)
    sc = (amax / 448.0).contiguous()
    q = (x / sc[:, :, None, None, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    del x
    return q, sc


def build_decode(wl: dict, device, seed: int = 0, pool_seed: int = None):
    """Replicated / single-GPU decode inputs: layout from `seed`, pool from
    seed + 1 (or pool_seed)."""
    lay = decode_layout(wl, seed)
    kc, vc, ks, vs = decode_pool(lay["nblk"], wl["Hkv"], wl["bs"], wl["D"], wl["fp8"], device,
                                 seed + 1 if pool_seed is None else pool_seed)
    return _decode_dict(wl, lay, kc, vc, ks, vs)


def _decode_dict(wl, lay, kc, vc, ks, vs):
    return dict(q=lay["q"], k=lay["k"], v=lay["v"], seq=lay["seq"], bt=lay["bt"], kcache=kc, vcache=vc,
                k_scale=ks, v_scale=vs, lens=lay["lens"], scale=1.0 / math.sqrt(wl["D"]), bs=wl["bs"],
                B=lay["q"].shape[0], Hkv=lay["q"].shape[1], G=wl["G"], D=wl["D"], fp8=wl["fp8"])


def build_decode_sharded(wl: dict, mode: str, rank: int, ws: int, device):
    """This rank's decode inputs under `mode` (see WORKLOADS)."""
    if mode == "replicas":
        # weak scaling: every rank runs the one-GPU workload itself (the same
        # lengths and block table, so the same bytes), over its own KV data
        return build_decode(wl, device, seed=0, pool_seed=1 + rank)
    if mode == "heads":
        # same sequences and block table on every rank; rank r holds KV heads
        # [r * Hkv / N, (r + 1) * Hkv / N) of the pool (and their query heads)
        from torch_rbln_b200 import sharding

        sharding.kv_head_range(wl["Hkv"], rank, ws)
        return build_decode(dict(wl, Hkv=wl["Hkv"] // ws), device, seed=0, pool_seed=1 + rank)
    if mode == "batch":
        # rank r holds its share of the sequences (equal counts, near-equal
        # tokens), its own pool of just their blocks and its own block table
        from torch_rbln_b200 import sharding

        lay = decode_layout(wl, seed=0)
        idx = sharding.batch_partition(lay["lens"], ws)[rank]
        blocks, table = sharding.shard_batch(lay["seq"], lay["bt"], wl["bs"], idx)
        sub = dict(q=lay["q"][idx].contiguous(), k=lay["k"][idx].contiguous(), v=lay["v"][idx].contiguous(),
                   seq=lay["seq"][idx].contiguous(), bt=table, lens=lay["lens"][idx], nblk=int(blocks.numel()))
        kc, vc, ks, vs = decode_pool(sub["nblk"], wl["Hkv"], wl["bs"], wl["D"], wl["fp8"], device, 1 + rank)
        d = _decode_dict(wl, sub, kc, vc, ks, vs)
        d["global_index"] = idx
        return d
    raise ValueError(mode)


def decode_bytes(d: dict) -> int:
    """Algorithmic HBM bytes of one decode step: every attended K/V element
    read once, q read, output written, new k/v read and written to the
    cache, block-table entries and (fp8) scales read."""
    lens = d["lens"].to(torch.int64)
    Hkv, G, D, bs = d["Hkv"], d["G"], d["D"], d["bs"]
    el = 1 if d["fp8"] else 2
    kv = int(lens.sum()) * Hkv * D * el * 2
    blocks = int(((lens + bs - 1) // bs).sum())
    scales = blocks * Hkv * 4 * 2 if d["fp8"] else 0
    qo = d["B"] * Hkv * G * D * 2 * 2
    new = d["B"] * Hkv * D * (2 * 2 + el * 2)
    return kv + scales + qo + new + blocks * 4


def decode_config(wl_name, ws, mode, global_batch, pool_bytes, step_bytes):
    """The `config` object of a decode line (rank 0's sizes); the reference
    arm prints the same."""
    wl = WORKLOADS[wl_name]
    par = {"single": "single GPU",
           "replicas": (f"replicas x{ws}: every rank the one-GPU batch of {wl['B']} sequences (same lengths "
                        f"and block table) over its own KV data, no collective"),
           "heads": (f"kv-head-sharded x{ws}: head outputs stored into every rank's buffer by the decode "
                     f"kernels (NVLink peer stores) + epoch exchange in the merge kernel"),
           "batch": f"batch-sharded x{ws}: each rank its share of the {wl['B']} sequences, own pool and table"}[mode]
    return {"workload": wl["desc"], "global_batch": global_batch, "parallelism": par,
            "l2": f"inputs larger than L2 (KV pool {pool_bytes / 1e9:.2f} GB per GPU)",
            "bytes_per_step_per_gpu": step_bytes}


def _global_batch(wl, mode, ws, local_B):
    return {"replicas": local_B * ws, "heads": local_B, "batch": wl["B"], "single": local_B}[mode]


# ---------------------------------------------------------------------------
# decode measurement (our arm)
# ---------------------------------------------------------------------------
def decode_record(args, ctx: Ctx, wl_name: str, n_parity: int = 8, cpu_leg: bool = True) -> dict:
    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi, sharding

    wl = WORKLOADS[wl_name]
    ws, rank, dev, stream = ctx.ws, ctx.rank, ctx.dev, ctx.stream
    if ws == 1:
        mode = "single"
        d = build_decode_sharded(wl, "batch", 0, 1, dev) if wl["shard"] == "batch" else build_decode(wl, dev, seed=0)
    else:
        mode = wl["shard"]
        d = build_decode_sharded(wl, mode, rank, ws, dev)
    q, k, v = d["q"].to(dev), d["k"].to(dev), d["v"].to(dev)
    seq, bt = d["seq"].to(dev), d["bt"].to(dev)
    kc, vc, ks, vs = d["kcache"], d["vcache"], d["k_scale"], d["v_scale"]
    scale_t = torch.tensor(d["scale"])
    nbytes = decode_bytes(d)
    total_bytes = int(ctx.reduce([nbytes], "sum")[0])
    global_batch = _global_batch(wl, mode, ws, d["B"])
    pool_bytes = kc.numel() * kc.element_size() * 2
    ops = torch.ops.rbln_custom_ops
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    peer, head0, e2e_ws = None, 0, {}
    if mode == "heads":
        peer = sharding.PeerHeadOutput((q.shape[0], q.shape[1] * ws) + tuple(q.shape[2:]), q.dtype, rank, ws)
        head0 = rank * q.shape[1]

    def op_call(qq, kk, vv, ss, bb):
        if d["fp8"]:
            return ops.paged_causal_attn_decode_kvfp8(qq, kk, vv, kc, vc, ks, vs, ss, scale_t, bb, d["bs"])
        if peer is not None:
            return sharding.head_sharded_paged_decode_p2p(qq, kk, vv, kc, vc, ss, d["scale"], bb, d["bs"], peer,
                                                          workspace=e2e_ws, q_is_local=True)
        return ops.paged_causal_attn_decode(qq, kk, vv, kc, vc, ss, scale_t, bb, d["bs"])

    # C-ABI parameter block (with the kernel timing hook for the roofline loop)
    p, keep = cabi.paged_params(q, k, v, kc, vc, seq, bt, d["bs"], d["scale"], k_scale=ks, v_scale=vs,
                                out=peer.outputs[0] if peer is not None else None)
    cabi.attach_workspace(p, dev, keep)
    p.error_flags = (peer.error_word if peer is not None else err).data_ptr()
    L = cabi.lib()
    pref, sh = ctypes.byref(p), ctypes.c_void_p(stream.cuda_stream)
    last_out = [keep["out"]]

    def cabi_step(ev0=None, ev1=None):
        p.prof_events[0] = ev0.cuda_event if ev0 is not None else None
        p.prof_events[1] = ev1.cuda_event if ev1 is not None else None
        if peer is not None:
            out, po = peer.next(head0)
            p.out = out.data_ptr()
            last_out[0] = out
            rc = L.rbln_paged_causal_attn_decode_peers(pref, ctypes.byref(po), sh)
        else:
            rc = L.rbln_paged_causal_attn_decode(pref, sh)
        if rc != 0:
            raise RuntimeError(f"rbln_paged_causal_attn_decode failed: {rc}")

    for _ in range(args.warmup):
        cabi_step()
        op_call(q, k, v, seq, bt)
    torch.cuda.synchronize()

    # ---- value: K steps back to back, events around the loop only
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx.barrier()
    torch.cuda.synchronize()
    with ClockSampler(ctx.local) as clk:
        t0.record(stream)
        for _ in range(args.steps):
            cabi_step()
        t1.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
    ms_step = t0.elapsed_time(t1) / args.steps

    # ---- head-sharded: the same local decode without the exchange (outputs in
    # local memory only), timed the same way, to state what the exchange costs
    local_ms = None
    if peer is not None:
        pl, keepl = cabi.paged_params(q, k, v, kc, vc, seq, bt, d["bs"], d["scale"])
        cabi.attach_workspace(pl, dev, keepl)
        pl.error_flags = err.data_ptr()
        plref = ctypes.byref(pl)
        for _ in range(args.warmup):
            L.rbln_paged_causal_attn_decode(plref, sh)
        torch.cuda.synchronize()
        ctx.barrier()
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for _ in range(args.steps):
            if L.rbln_paged_causal_attn_decode(plref, sh) != 0:
                raise RuntimeError("rbln_paged_causal_attn_decode failed")
        l1.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
        local_ms = l0.elapsed_time(l1) / args.steps
        del keepl

    # ---- roofline: the main kernel alone, events the C-ABI records around it
    kev = _event_pairs(args.steps, stream)
    ctx.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        cabi_step(*kev[i])
    torch.cuda.synchronize()
    ctx.barrier()
    kmean = statistics.mean(a.elapsed_time(b) for a, b in kev)

    # ---- e2e: public torch op, host buffers, H2D + D2H inside the timed region
    # The step's inputs (q, k, v, seq, block table) are packed into one pinned
    # staging buffer and cross PCIe as one copy per step, as a serving loop
    # would send them; the op then reads views of the device copy.
    srcs = [d[x].cpu().contiguous() for x in ("q", "k", "v", "seq", "bt")]
    offs, total = [], 0
    for t in srcs:
        offs.append(total)
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    hstage = torch.empty(total, dtype=torch.uint8).pin_memory()
    for t, o in zip(srcs, offs):
        hstage[o:o + t.numel() * t.element_size()].copy_(t.view(-1).view(torch.uint8))
    dstage = torch.empty(total, dtype=torch.uint8, device=dev)
    views = [dstage[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for t, o in zip(srcs, offs)]
    out_heads = q.shape[1] * (ws if peer is not None else 1)
    hout = torch.empty((q.shape[0], out_heads) + tuple(q.shape[2:]), dtype=q.dtype).pin_memory()
    h2d = total
    d2h = hout.numel() * hout.element_size()

    def e2e_step():
        dstage.copy_(hstage, non_blocking=True)
        o = op_call(*views)
        hout.copy_(o, non_blocking=True)

    for _ in range(max(2, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    # ---- one more C-ABI call, whose output the parity check reads
    cabi_step()
    torch.cuda.synchronize()
    ctx.barrier()
    if peer is not None:
        peer.check()  # raises ShardedDecodeError if any exchange timed out
    dev_err = int((peer.error_word if peer is not None else err).item())
    parity = decode_parity(ctx, d, last_out[0], head0, n_parity, peer is not None)
    parity["device_error_bits"] = int(ctx.reduce([dev_err], "max")[0])
    parity["ok"] = parity["ok"] and parity["device_error_bits"] == 0

    ms_step, e2e_ms, kmean = ctx.reduce([ms_step, e2e_ms, kmean], "max")
    hbm_peak, _, peak_src = load_peaks()
    achieved = nbytes / (kmean * 1e-3) / 1e9
    rec = {
        "metric": "paged decode HBM GB/s",
        "value": round(total_bytes / (ms_step * 1e-3) / 1e9, 1),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if mode in ("heads", "batch") else "weak",
        "vs_baseline": None,
        "dtype": "fp8e4m3-kv/bf16" if d["fp8"] else "bf16",
        "data": "synthetic (seeded N(0,1)*0.5 KV pool, seeded lengths and block-table permutation)",
        "config": decode_config(wl_name, ws, mode, global_batch, pool_bytes, nbytes),
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": ("torch_rbln_b200.sharding.head_sharded_paged_decode_p2p" if peer is not None else
                        "torch.ops.rbln_custom_ops.paged_causal_attn_decode" + ("_kvfp8" if d["fp8"] else ""))},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": _traffic_from_profiles(wl_name),
                     "kernel": "paged_decode_balanced_kernel (equal token chunks over the batch, mma.sync)",
                     "kernel_ms": round(kmean, 4),
                     "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs), of measured" if peak_src == "measured"
                                     else "fallback 6.65 TB/s")},
        # decode + merge per step (the exchange runs inside the merge kernel)
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
        "parity": parity,
    }
    if local_ms is not None:
        local_ms = ctx.reduce([local_ms], "max")[0]
        rec["exchange"] = {"local_decode_ms_per_step": round(local_ms, 4),
                           "exchange_us_per_step": round((ms_step - local_ms) * 1e3, 2),
                           "note": "the same rank's decode with outputs in local memory only, timed the same way; "
                                   "the difference is what the peer stores and the epoch exchange cost per call"}
    if rank == 0 and cpu_leg and ws == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_decode_baseline(d, budget_s=args.cpu_budget)
    ctx.barrier()  # every rank is past its last call before any buffer is unmapped
    if peer is not None:
        peer.close()
    ctx.barrier()
    del d, kc, vc, ks, vs, keep
    torch.cuda.empty_cache()
    return rec


def decode_parity(ctx: Ctx, d, out, head0, n, heads_sharded):
    """The last call's output against the fp32 oracle on a seeded subset of
    this rank's sequences (each rank its own; results combined over ranks).
    With the heads sharded, every rank's full output must also equal every
    other rank's, bit for bit."""
    from oracle import paged_attention as opa
    from torch_rbln_b200 import sharding

    B = d["B"]
    n = min(n, B)
    idx = torch.randperm(B, generator=torch.Generator().manual_seed(7 + ctx.rank))[:n].sort().values
    blocks, table = sharding.shard_batch(d["seq"], d["bt"], d["bs"], idx)
    dv = d["kcache"].device
    kc = d["kcache"][blocks.to(dv)].cpu()
    vc = d["vcache"][blocks.to(dv)].cpu()
    ks = d["k_scale"][blocks.to(dv)].cpu() if d["fp8"] else None
    vs = d["v_scale"][blocks.to(dv)].cpu() if d["fp8"] else None
    ref = opa.paged_decode(d["q"][idx], d["k"][idx], d["v"][idx], kc, vc, d["seq"][idx], d["scale"], table, d["bs"],
                           k_scale=ks, v_scale=vs, mode="fp32")
    got = out[idx.to(out.device), head0:head0 + d["Hkv"]].cpu()
    ok, max_abs, max_rel = _tolerance_stats(got, ref, RTOL, ATOL)
    agree = True
    if heads_sharded and ctx.pg:
        import torch.distributed as dist

        buf = torch.empty((ctx.ws,) + tuple(out.shape), dtype=out.dtype, device=out.device)
        dist.all_gather_into_tensor(buf, out.contiguous())
        agree = all(torch.equal(buf[r], out) for r in range(ctx.ws))
    okf, agreef = ctx.reduce([float(ok), float(agree)], "min")
    max_abs, max_rel = ctx.reduce([max_abs, max_rel], "max")
    n_total = int(ctx.reduce([n], "sum")[0])
    res = {"ok": bool(okf) and bool(agreef), "max_abs": round(max_abs, 6), "max_rel": round(max_rel, 6),
           "n_checked": n_total, "checked": f"{n_total} sequences (seeded subset, every rank), all their heads",
           "tolerance": f"rtol {RTOL}, atol {ATOL} (the reference's, test_custom_kernel.py:654-655)",
           "oracle": "oracle.paged_attention.paged_decode, fp32"}
    if heads_sharded:
        res["ranks_agree"] = bool(agreef)
    return res


# ---------------------------------------------------------------------------
# CPU baseline / reference arm (decode)
# ---------------------------------------------------------------------------
def cpu_sample(d: dict, n_seq: int):
    """First n_seq sequences, gathered into the reference's contiguous
    per-sequence layout [n, Hkv, 1, max_seq, D] (gather not timed; fp8
    dequantised to bf16 first)."""
    from oracle import paged_attention as opa

    n = n_seq
    lens = d["lens"][:n]
    bs = d["bs"]
    span = int(math.ceil(int(lens.max()) / bs)) * bs
    bt = d["bt"][:n, : span // bs]
    kcs, vcs = [], []
    for b in range(n):
        blocks = bt[b].long()
        kb = d["kcache"][blocks.to(d["kcache"].device)].cpu()
        vb = d["vcache"][blocks.to(d["vcache"].device)].cpu()
        if d["fp8"]:
            ksb = d["k_scale"][blocks.to(d["kcache"].device)].cpu()
            vsb = d["v_scale"][blocks.to(d["kcache"].device)].cpu()
            kb = (kb.float() * ksb[:, :, None, None, None]).to(torch.bfloat16)
            vb = (vb.float() * vsb[:, :, None, None, None]).to(torch.bfloat16)
        # [nb, Hkv, 1, bs, D] -> [Hkv, 1, nb*bs, D]
        kcs.append(kb.permute(1, 2, 0, 3, 4).reshape(d["Hkv"], 1, span, d["D"]))
        vcs.append(vb.permute(1, 2, 0, 3, 4).reshape(d["Hkv"], 1, span, d["D"]))
    kc = torch.stack(kcs)
    vc = torch.stack(vcs)
    sub = dict(d)
    sub["lens"] = lens
    sub["B"] = n
    return (d["q"][:n].clone(), d["k"][:n].clone(), d["v"][:n].clone(), kc, vc, d["seq"][:n].clone(),
            torch.tensor(d["scale"]), opa, decode_bytes(sub))


def _cpu_decode_sample_size(d, budget_s, mem_cap=1.5e9):
    """Sequences that fit the time budget (from one timed sequence) and a cap
    on the gathered caches' memory."""
    q, k, v, kc, vc, seq, sc, opa, nb = cpu_sample(d, 1)
    t = time.perf_counter()
    opa.mock_decode_contiguous(q, k, v, kc.clone(), vc.clone(), seq, sc)
    one = max(time.perf_counter() - t, 1e-4)
    per_seq_mem = 2 * kc.numel() * kc.element_size() * 2  # caches and their per-step copies
    return int(max(1, min(d["B"], budget_s / one, mem_cap / per_seq_mem)))


def cpu_decode_times(d, n, reps, warmup=1):
    """Wall-clock times of the reference's CPU decode on the first n
    sequences (the caches are re-copied outside the timed region)."""
    q, k, v, kc, vc, seq, sc, opa, nb = cpu_sample(d, n)
    for _ in range(warmup):
        opa.mock_decode_contiguous(q, k, v, kc.clone(), vc.clone(), seq, sc)
    times = []
    for _ in range(reps):
        kk, vv = kc.clone(), vc.clone()
        t = time.perf_counter()
        opa.mock_decode_contiguous(q, k, v, kk, vv, seq, sc)
        times.append(time.perf_counter() - t)
    return times, nb


def _cpu_stats_note(times):
    return (f"median of {len(times)} runs ({statistics.median(times) * 1e3:.1f} ms; min {min(times) * 1e3:.1f}, "
            f"max {max(times) * 1e3:.1f}: a shared host, so the spread is reported)")


def cpu_decode_baseline(d, budget_s=20.0, reps=5):
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    n = _cpu_decode_sample_size(d, budget_s / (reps + 1))
    times, nb = cpu_decode_times(d, n, reps)
    med = statistics.median(times)
    return {"value": round(nb / med / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} of {d['B']} sequences of the same workload, reference CPU algorithm "
                      f"(oracle.paged_attention.mock_decode_contiguous, bf16 over the gathered per-sequence "
                      f"layout), {_cpu_stats_note(times)}",
            "ms_per_sample": round(med * 1e3, 2), "bytes_per_sample": nb}


def reference_decode_inputs(wl: dict, mode: str, ws: int, kv_cap_bytes: float = 1.5e9):
    """Rank 0's share of a decode workload on the CPU, as the reference arm
    needs it: the full layout's sizes (for the config) and the inputs of
    its first sequences only, as many as fit kv_cap_bytes of KV (the CPU
    sample never reads more), with a pool of just their blocks."""
    from torch_rbln_b200 import sharding

    Hkv = wl["Hkv"] // ws if mode == "heads" else wl["Hkv"]
    lay = decode_layout(wl, seed=0, Hkv=Hkv)
    seq, bt, lens = lay["seq"], lay["bt"], lay["lens"]
    if wl["shard"] == "batch":
        idx = sharding.batch_partition(lens, ws)[0]
        blocks, bt = sharding.shard_batch(seq, bt, wl["bs"], idx)
        lay = dict(lay, q=lay["q"][idx], k=lay["k"][idx], v=lay["v"][idx], seq=seq[idx], bt=bt, lens=lens[idx],
                   nblk=int(blocks.numel()))
    el = 1 if wl["fp8"] else 2
    full = dict(lens=lay["lens"], Hkv=Hkv, G=wl["G"], D=wl["D"], bs=wl["bs"], fp8=wl["fp8"], B=lay["q"].shape[0])
    pool_bytes = lay["nblk"] * Hkv * wl["bs"] * wl["D"] * el * 2
    per_token = Hkv * wl["D"] * el * 2
    n = int(max(1, min(full["B"], (torch.cumsum(lay["lens"], 0) * per_token <= kv_cap_bytes).sum())))
    first = torch.arange(n)
    blocks, table = sharding.shard_batch(lay["seq"], lay["bt"], wl["bs"], first)
    sub = dict(q=lay["q"][:n].contiguous(), k=lay["k"][:n].contiguous(), v=lay["v"][:n].contiguous(),
               seq=lay["seq"][:n].contiguous(), bt=table, lens=lay["lens"][:n], nblk=int(blocks.numel()))
    kc, vc, ks, vs = decode_pool(sub["nblk"], Hkv, wl["bs"], wl["D"], wl["fp8"], torch.device("cpu"), 1)
    return _decode_dict(wl, sub, kc, vc, ks, vs), full, pool_bytes


def reference_decode_line(args, ctx: Ctx, wl_name: str, per_step_budget=None) -> dict:
    """--impl reference for a decode workload: the reference's CPU algorithm
    on rank 0's data, each step a bounded sample of sequences."""
    wl = WORKLOADS[wl_name]
    ws = ctx.ws
    mode = wl["shard"] if ws > 1 else "single"
    d, full, pool_bytes = reference_decode_inputs(wl, mode, ws)
    global_batch = _global_batch(wl, mode, ws, full["B"])
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    budget = per_step_budget or max(0.5, 120.0 / max(1, args.steps + args.warmup))
    n = _cpu_decode_sample_size(d, budget)
    times, nb = cpu_decode_times(d, n, args.steps, warmup=args.warmup)
    med = statistics.median(times)
    val = nb / med / 1e9
    sample = (f"{n} of {full['B']} sequences per step, reference CPU algorithm (oracle restatement of "
              f"test_custom_kernel.py paged_causal_attn_decode on the per-sequence layout), wall clock, "
              f"{_cpu_stats_note(times)}")
    return {"impl": "reference", "metric": "paged decode HBM GB/s", "value": round(val, 3), "unit": "GB/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3),
            "higher_is_better": True, "scaling": "strong" if mode in ("heads", "batch") else "weak",
            "vs_baseline": None, "dtype": "fp8e4m3-kv/bf16" if d["fp8"] else "bf16",
            "data": "synthetic (seeded N(0,1)*0.5 KV pool, seeded lengths and block-table permutation)",
            "config": decode_config(wl_name, ws, mode, global_batch, pool_bytes, decode_bytes(full)),
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# compute-bound workloads: chunked prefill and SDPA
# ---------------------------------------------------------------------------
def build_prefill(wl, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, Hkv, G, D, bs, S = wl["B"], wl["Hkv"], wl["G"], wl["D"], wl["bs"], wl["S"]
    ctx = torch.randint(wl["cmin"], wl["cmax"] + 1, (B,), generator=g)
    nb = [int(math.ceil((int(c) + S) / bs)) for c in ctx]
    max_blocks = max(nb)
    pool = sum(nb) + B
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    cur = 0
    for b in range(B):
        bt[b, :nb[b]] = perm[cur:cur + nb[b]].to(torch.int32)
        cur += nb[b]
    q = torch.randn([B, Hkv, G, S, D], generator=g).to(torch.bfloat16)
    k = torch.randn([B, Hkv, 1, S, D], generator=g).to(torch.bfloat16)
    v = torch.randn([B, Hkv, 1, S, D], generator=g).to(torch.bfloat16)
    gd = torch.Generator(device=device).manual_seed(seed + 1)
    shape = [pool, Hkv, 1, bs, D]
    kc = torch.randn(shape, generator=gd, device=device, dtype=torch.bfloat16)
    vc = torch.randn(shape, generator=gd, device=device, dtype=torch.bfloat16)
    Hq = Hkv * G
    flops = sum(4 * D * Hq * (S * int(c) + S * (S + 1) // 2) for c in ctx)
    d = dict(q=q, k=k, v=v, kcache=kc, vcache=vc, seq=ctx.to(torch.int32).reshape(B, 1), bt=bt, bs=bs,
             ctx=ctx, flops=flops, scale=1.0 / math.sqrt(D), B=B, Hkv=Hkv, G=G, D=D, S=S)
    if wl.get("keep_mask"):
        span = max_blocks * bs
        t = torch.arange(span).reshape(1, 1, span)
        qi = torch.arange(S).reshape(1, S, 1) + ctx.reshape(B, 1, 1)
        d["mask"] = (t <= qi).to(torch.bfloat16).reshape(B, 1, 1, S, span)
    return d


def build_sdpa(wl, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hkv, L, D = wl["B"], wl["Hq"], wl["Hkv"], wl["L"], wl["D"]
    q = torch.randn([B, Hq, L, D], generator=g).to(wl["dtype"])
    k = torch.randn([B, Hkv, L, D], generator=g).to(wl["dtype"])
    v = torch.randn([B, Hkv, L, D], generator=g).to(wl["dtype"])
    flops = 4 * D * Hq * B * (L * (L + 1) // 2)
    d = dict(q=q, k=k, v=v, flops=flops, scale=1.0 / math.sqrt(D))
    if wl["kind"] == "sdpa_bwd":
        # algorithmic backward FLOPs: five L x S x D products (dV, dP, dQ, dK and the
        # recomputed S) against the forward's two, i.e. 2.5x the forward count
        d["flops"] = flops * 5 // 2
        d["dout"] = torch.randn([B, Hq, L, D], generator=g).to(wl["dtype"])
    return d


L2_FLUSH_NOTE = "L2 flushed between iterations (256 MB write, outside the timed events)"


def compute_config(wl: dict, d: dict, ws: int) -> dict:
    """The `config` of a compute workload's record, the same in both arms."""
    return {"workload": wl["desc"], "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
            "l2": L2_FLUSH_NOTE, "flops_per_step": d["flops"]}


def kv_write_config(wl: dict, d: dict, ws: int) -> dict:
    """The `config` of the KV-write record, the same in both arms."""
    return {"workload": wl["desc"], "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
            "l2": L2_FLUSH_NOTE, "bytes_per_step": d["bytes"]}


def _timed_kernel_loop(args, stream, step, kernel_step, flush, kernel_events=False):
    """Per-iteration CUDA events on the launch stream around the whole op
    (`step`) and, in separate iterations, around the main kernel alone
    (`kernel_step`; with kernel_events it takes the event pair and has the
    C-ABI record it right around the kernel), each preceded by an L2 flush
    outside the timed window. The two kinds of iteration alternate, so that
    both see the same clocks: timed one loop after the other, the second
    loop of a tensor-bound op ran under the power cap and read 5 % slower
    than the first for the very same launches."""
    ev_op, ev_k = _event_pairs(args.steps, stream), _event_pairs(args.steps, stream)
    for i in range(args.steps):
        flush.zero_()
        ev_op[i][0].record(stream)
        step()
        ev_op[i][1].record(stream)
        flush.zero_()
        if kernel_events:
            kernel_step(*ev_k[i])
        else:
            ev_k[i][0].record(stream)
            kernel_step()
            ev_k[i][1].record(stream)
    torch.cuda.synchronize()
    return (statistics.mean(a.elapsed_time(b) for a, b in ev_op),
            statistics.mean(a.elapsed_time(b) for a, b in ev_k))


def compute_record(args, ctx: Ctx, wl_name: str, cpu_leg: bool = True) -> dict:
    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi

    ws, rank, dev, stream = ctx.ws, ctx.rank, ctx.dev, ctx.stream
    wl = COMPUTE[wl_name]
    sh = ctypes.c_void_p(stream.cuda_stream)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2
    L = cabi.lib()
    result = {}
    if wl["kind"] == "prefill":
        d = build_prefill(wl, dev, seed=1000 * rank)
        q, k, v, seq, bt = (d[x].to(dev) for x in ("q", "k", "v", "seq", "bt"))
        kc, vc = d["kcache"], d["vcache"]
        masked = "mask" in d
        mask = d["mask"].to(dev) if masked else None
        entry = L.rbln_paged_attn_prefill if masked else L.rbln_paged_causal_attn_prefill
        p, keep = cabi.paged_params(q, k, v, kc, vc, seq, bt, d["bs"], d["scale"], causal=1, mask=mask)
        cabi.attach_workspace(p, dev, keep, prefill=True)
        pref = ctypes.byref(p)
        scale_t = torch.tensor(d["scale"])

        def step():
            p.prof_events[0] = p.prof_events[1] = None
            rc = entry(pref, sh)
            if rc != 0:
                raise RuntimeError(f"paged prefill failed: {rc}")

        def kernel_step(ev0, ev1):  # the whole call; events recorded around the attention kernel
            p.prof_events[0], p.prof_events[1] = ev0.cuda_event, ev1.cuda_event
            rc = entry(pref, sh)
            if rc != 0:
                raise RuntimeError(f"paged prefill failed: {rc}")

        if masked:
            def op_call(qq, kk, vv, ss, bb, mm):
                return torch.ops.rbln_custom_ops.paged_attn_prefill(qq, kk, vv, mm, kc, vc, ss, scale_t, bb, d["bs"])
        else:
            def op_call(qq, kk, vv, ss, bb):
                return torch.ops.rbln_custom_ops.paged_causal_attn_prefill(qq, kk, vv, kc, vc, ss, scale_t, bb,
                                                                           d["bs"], False)

        host_inputs = [d["q"], d["k"], d["v"], d["seq"], d["bt"]] + ([d["mask"]] if masked else [])
        out_shape, out_dtype = q.shape, q.dtype
        metric = "paged chunked prefill TFLOP/s"
        # append, schedule pre-pass, attention (+ the mask pre-pass's bits and lists)
        launches = 5 if masked else 3
        kernel = ("attn_fwd_tc3_kernel<128, bf16" + (", masked" if masked else "") +
                  "> (tcgen05/TMEM/TMA, 128-key tiles, P in TMEM, two query tiles per CTA)")
        dtype = "bf16"
        kernel_events = True
        result["parity"] = lambda: prefill_parity(d, keep["out"])
    elif wl["kind"] == "sdpa_bwd":
        kernel_events = False
        d = build_sdpa(wl, seed=0)
        q, k, v, dout = (d[x].to(dev) for x in ("q", "k", "v", "dout"))
        fwd = torch.ops.aten._scaled_dot_product_fused_attention_overrideable(q, k, v, None, 0.0, True, False,
                                                                              scale=d["scale"])
        out, lse = fwd[0], fwd[1]
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        bp = cabi.sdpa_bwd_params(q, k, v, out, dout, lse, dq, dk, dv, causal=True, scale=d["scale"])
        wsz = ctypes.c_size_t(0)
        L.rbln_sdpa_bwd_workspace_size(ctypes.byref(bp), ctypes.byref(wsz))
        wsb = torch.empty(wsz.value, dtype=torch.uint8, device=dev)
        bp.workspace, bp.workspace_bytes = wsb.data_ptr(), wsz.value
        bpref = ctypes.byref(bp)

        def step():
            rc = L.rbln_sdpa_bwd(bpref, sh)
            if rc != 0:
                raise RuntimeError(f"rbln_sdpa_bwd failed: {rc}")

        kernel_step = step
        e0t = torch.empty(0, device=dev)

        def op_call(qq, kk, vv, oo, gg, ll):
            return torch.ops.aten._scaled_dot_product_fused_attention_overrideable_backward(
                gg, qq, kk, vv, e0t, [True, True, True, False], oo, ll, fwd[2], fwd[3], fwd[4], fwd[5], 0.0, True,
                fwd[6], fwd[7], scale=d["scale"])[:3]

        host_inputs = [d["q"], d["k"], d["v"], out.cpu(), d["dout"], lse.cpu()]
        out_shape, out_dtype = None, None
        metric = "SDPA backward TFLOP/s"
        launches = 3  # row pre-pass, dK/dV kernel, dQ kernel
        kernel = ("sdpa_bwd_kv_kernel<128, bf16> + sdpa_bwd_q_kernel<128, bf16> + row pre-pass "
                  "(tcgen05/TMEM/TMA; whole backward timed)")
        dtype = "bf16"
    else:
        kernel_events = False
        d = build_sdpa(wl, seed=0)
        q, k, v = (d[x].to(dev) for x in ("q", "k", "v"))
        out = torch.empty_like(q)
        lse = torch.empty(q.shape[:3], dtype=torch.float32, device=dev)
        sp = cabi.sdpa_params(q, k, v, out, lse, causal=True, scale=d["scale"])
        spref = ctypes.byref(sp)

        def step():
            rc = L.rbln_sdpa_fwd(spref, sh)
            if rc != 0:
                raise RuntimeError(f"rbln_sdpa_fwd failed: {rc}")

        kernel_step = step  # one kernel per call

        import torch.nn.functional as F

        def op_call(qq, kk, vv):
            return F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, scale=d["scale"], enable_gqa=True)

        host_inputs = [d["q"], d["k"], d["v"]]
        out_shape, out_dtype = q.shape, q.dtype
        metric = "SDPA TFLOP/s"
        launches = 1
        kernel = ("sdpa_f32_kernel<64> (exact-fp32 SIMT; tensor cores have no fp32 mode)"
                  if wl["dtype"] == torch.float32
                  else "attn_fwd_tc3_kernel<128, bf16> (tcgen05/TMEM/TMA, 128-key tiles, P in TMEM, two query tiles per CTA)")
        dtype = "f32" if wl["dtype"] == torch.float32 else "bf16"
        result["parity"] = lambda: sdpa_parity(d, out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.barrier()
    with ClockSampler(ctx.local) as clk:
        op_ms, k_ms = _timed_kernel_loop(args, stream, step, kernel_step, flush, kernel_events)
    ctx.barrier()

    # e2e through the public torch API with host buffers
    pinned = [t.cpu().pin_memory() for t in host_inputs]
    if out_shape is None:  # backward: the three gradients come back
        houts = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, k, v)]
    else:
        houts = [torch.empty(out_shape, dtype=out_dtype).pin_memory()]
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    d2h = sum(t.numel() * t.element_size() for t in houts)

    def e2e_step():
        o = op_call(*[t.to(dev, non_blocking=True) for t in pinned])
        for h, t in zip(houts, o if isinstance(o, (tuple, list)) else [o]):
            h.copy_(t, non_blocking=True)

    for _ in range(max(2, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    parity = None
    if "parity" in result:
        step()  # the output the check reads
        torch.cuda.synchronize()
        parity = result["parity"]()
    op_ms, e2e_ms, k_ms = ctx.reduce([op_ms, e2e_ms, k_ms], "max")

    _, tf_peak, peak_src = load_peaks()
    flops = d["flops"]
    achieved = flops / (k_ms * 1e-3) / 1e12
    rec = {
        "metric": metric, "value": round(ws * flops / (op_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(op_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded N(0,1) inputs" + (", seeded cached lengths and block-table permutation)"
                                                     if wl["kind"] == "prefill" else ")"),
        "config": compute_config(wl, d, ws),
        "e2e": {"value": round(ws * flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": {"prefill": ("torch.ops.rbln_custom_ops.paged_attn_prefill" if wl.get("keep_mask") else
                                    "torch.ops.rbln_custom_ops.paged_causal_attn_prefill"),
                        "sdpa_bwd": "torch.ops.aten._scaled_dot_product_fused_attention_overrideable_backward"}.get(
                            wl["kind"], "torch.nn.functional.scaled_dot_product_attention")},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_peak, 4), "traffic": _traffic_from_profiles(wl_name),
                     "kernel": kernel, "kernel_ms": round(k_ms, 4),
                     "peak_source": ("measured (MEASURED_PEAKS.json bf16_tflops, burst), of measured"
                                     if peak_src == "measured" else "fallback 1.59 PFLOP/s")},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }
    if dtype == "f32":
        # the exact-fp32 kernel runs on the FMA pipes, not the tensor cores:
        # its own ceiling is the nominal fp32 FMA rate (148 SMs x 128 lanes
        # x 2 FLOP at the 1965 MHz maximum clock; no measured figure exists)
        simt_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        rec["roofline"]["fp32_simt"] = {"peak": round(simt_peak, 1), "unit": "TFLOP/s",
                                        "frac": round(achieved / simt_peak, 4),
                                        "peak_source": "nominal fp32 FMA rate (148 x 128 x 2 x 1.965 GHz)"}
    if parity is not None:
        rec["parity"] = parity
    if rank == 0 and cpu_leg and ws == 1 and not args.no_cpu_baseline:
        rec["cpu_baseline"] = cpu_baseline_compute(wl, d, args.cpu_budget)
    del d
    torch.cuda.empty_cache()
    return rec


def prefill_parity(d, out):
    """The chunked prefill of the sequence with the median cached context
    against the fp32 oracle (its blocks gathered, caches hold the appended
    rows, which the oracle writes again)."""
    from oracle import paged_attention as opa

    b = int(torch.argsort(d["ctx"])[len(d["ctx"]) // 2])
    nb = int(math.ceil((int(d["ctx"][b]) + d["S"]) / d["bs"]))
    blocks = d["bt"][b, :nb].long()
    dv = d["kcache"].device
    kc, vc = d["kcache"][blocks.to(dv)].cpu(), d["vcache"][blocks.to(dv)].cpu()
    table = torch.arange(nb, dtype=torch.int32).reshape(1, nb)
    mask = d["mask"][b:b + 1] if "mask" in d else None  # a keep-mask run checks against the same mask
    ref = opa.paged_prefill(d["q"][b:b + 1], d["k"][b:b + 1], d["v"][b:b + 1], kc, vc, d["seq"][b:b + 1],
                            d["scale"], table, d["bs"], mask=mask, causal=True, mode="fp32")
    ok, max_abs, max_rel = _tolerance_stats(out[b:b + 1].cpu(), ref, RTOL, ATOL)
    return {"ok": ok, "max_abs": round(max_abs, 6), "max_rel": round(max_rel, 6), "n_checked": 1,
            "checked": f"sequence {b} (median cached context {int(d['ctx'][b])}), all 32 heads x 512 rows",
            "tolerance": f"rtol {RTOL}, atol {ATOL}", "oracle": "oracle.paged_attention.paged_prefill, fp32"}


def sdpa_parity(d, out):
    """fp32 SDPA against the reference's CPU path (repeat_kv + CPU SDPA):
    ||a - b||_inf / ||b||_inf <= 1e-5."""
    from oracle import sdpa as osd

    ref = osd.sdpa_reference(d["q"], d["k"], d["v"], None, 0.0, True, d["scale"]).float()
    got = out.cpu().float()
    rel = float((got - ref).abs().max() / ref.abs().max())
    return {"ok": rel <= 1e-5 if d["q"].dtype == torch.float32 else rel <= 3e-2,
            "max_abs": round(float((got - ref).abs().max()), 8), "max_rel": rel, "n_checked": 1,
            "checked": "the whole output", "tolerance": "||a-b||_inf / ||b||_inf <= 1e-5 (fp32)",
            "oracle": "oracle.sdpa.sdpa_reference (the reference's _sdpa_cpu_fallback path)"}


def _cpu_prefill_sample(d, b):
    """Sequence b gathered into the reference layout, plus its keep-mask."""
    bs, S, D = d["bs"], d["S"], d["D"]
    ctx = int(d["ctx"][b])
    nblk = int(math.ceil((ctx + S) / bs))
    blocks = d["bt"][b, :nblk].long()
    kb = d["kcache"][blocks.to(d["kcache"].device)].cpu()
    vb = d["vcache"][blocks.to(d["vcache"].device)].cpu()
    part = nblk * bs
    kc = kb.permute(1, 2, 0, 3, 4).reshape(1, d["Hkv"], 1, part, D).contiguous()
    vc = vb.permute(1, 2, 0, 3, 4).reshape(1, d["Hkv"], 1, part, D).contiguous()
    t = torch.arange(part).reshape(1, part)
    qi = torch.arange(S).reshape(S, 1) + ctx
    mask = (t <= qi).to(torch.bfloat16).reshape(1, 1, 1, S, part)
    flops = 4 * D * d["Hkv"] * d["G"] * (S * ctx + S * (S + 1) // 2)
    return d["q"][b:b + 1], d["k"][b:b + 1], d["v"][b:b + 1], kc, vc, ctx, mask, flops


def _cpu_compute_times(wl, d, reps, budget_s):
    from oracle import paged_attention as opa
    from oracle import sdpa as osd

    torch.set_num_threads(os.cpu_count() or 1)
    if wl["kind"] == "prefill":
        # the sequence with the median context stands for the workload
        b = int(torch.argsort(d["ctx"])[len(d["ctx"]) // 2])
        q, k, v, kc, vc, ctx, mask, flops = _cpu_prefill_sample(d, b)
        sc = torch.tensor(d["scale"])
        fn = lambda: opa.mock_prefill_contiguous(q, k, v, kc.clone(), vc.clone(), ctx, sc, mask)
        sample = (f"1 of {d['B']} sequences (median cached context {ctx}, 512 new tokens), reference CPU "
                  f"algorithm (oracle.paged_attention.mock_prefill_contiguous, bf16, per-sequence layout)")
    elif wl["kind"] == "sdpa_bwd":
        # one batch entry, one KV head and its 4 query heads: 1/(B * Hkv) of the workload
        G = wl["Hq"] // wl["Hkv"]
        q, k, v, go = d["q"][:1, :G], d["k"][:1, :1], d["v"][:1, :1], d["dout"][:1, :G]
        flops = d["flops"] // (wl["B"] * wl["Hkv"])
        fn = lambda: osd.sdpa_backward_reference(go, q, k, v, None, True, d["scale"])
        sample = (f"1 of {wl['B']} batch entries x 1 of {wl['Hkv']} KV heads ({G} query heads), reference CPU "
                  f"backward (oracle.sdpa.sdpa_backward_reference: attention weights + 4 products, bf16)")
    else:
        q, k, v = d["q"], d["k"], d["v"]
        flops = d["flops"]
        fn = lambda: osd.sdpa_reference(q, k, v, None, 0.0, True, d["scale"])
        sample = "the full workload, reference CPU path (oracle.sdpa.sdpa_reference: repeat_kv + torch CPU SDPA)"
    fn()
    times = []
    t_end = time.perf_counter() + budget_s
    for _ in range(reps):
        t = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t)
        if time.perf_counter() > t_end:
            break
    return times, flops, sample


def cpu_baseline_compute(wl, d, budget_s):
    times, flops, sample = _cpu_compute_times(wl, d, 5, budget_s)
    med = statistics.median(times)
    return {"value": round(flops / med / 1e12, 5), "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": sample + ", " + _cpu_stats_note(times), "ms_per_sample": round(med * 1e3, 2)}


def reference_compute_line(args, ctx: Ctx, wl_name: str, budget_s=120.0) -> dict:
    wl = COMPUTE[wl_name]
    d = build_prefill(wl, torch.device("cpu"), seed=0) if wl["kind"] == "prefill" else build_sdpa(wl, seed=0)
    for _ in range(min(args.warmup, 1)):
        _cpu_compute_times(wl, d, 1, 1e9)
    times, flops, sample = _cpu_compute_times(wl, d, args.steps, budget_s)
    med = statistics.median(times)
    val = flops / med / 1e12
    metric = {"prefill": "paged chunked prefill TFLOP/s", "sdpa_bwd": "SDPA backward TFLOP/s"}.get(wl["kind"],
                                                                                                 "SDPA TFLOP/s")
    dtype = "f32" if wl["kind"] != "prefill" and wl["dtype"] == torch.float32 else "bf16"
    return {"impl": "reference", "metric": metric, "value": round(val, 5), "unit": "TFLOP/s", "n_gpus": ctx.ws,
            "steps": len(times), "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic (seeded)",
            "config": compute_config(wl, d, ctx.ws),
            "cpu_baseline": {"value": round(val, 5), "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": sample + ", " + _cpu_stats_note(times)},
            "e2e": {"value": round(val, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# standalone KV-cache write (HBM-bound)
# ---------------------------------------------------------------------------
def build_kv_write(wl, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, Hkv, D, bs, S = wl["B"], wl["Hkv"], wl["D"], wl["bs"], wl["S"]
    starts = torch.randint(0, wl["cmax"] + 1, (B,), generator=g).to(torch.int32)
    mb = (wl["cmax"] + S) // bs + 2
    nblk = B * mb
    bt = torch.randperm(nblk, generator=g).reshape(B, mb).to(torch.int32)
    k = torch.randn([B, Hkv, 1, S, D], generator=g).to(torch.bfloat16)
    v = torch.randn([B, Hkv, 1, S, D], generator=g).to(torch.bfloat16)
    held = (starts % bs).to(torch.int64)
    # new rows read (bf16) + written (fp8), K and V; held rows of the first
    # block read and re-written; the touched blocks' two scales
    touched = sum(((int(s0) + S - 1) // bs - int(s0) // bs + 1) for s0 in starts)
    nbytes = 2 * Hkv * (B * S * D * 3 + int(held.sum()) * D * 2) + 2 * Hkv * touched * 8
    return dict(k=k, v=v, seq=starts, bt=bt, nblk=nblk, bytes=nbytes, B=B, Hkv=Hkv, D=D, bs=bs, S=S)


def _cpu_kv_write(d, budget_s):
    """oracle.paged_attention.kv_write on one sequence (all KV heads) per run."""
    from oracle import paged_attention as opa

    torch.set_num_threads(os.cpu_count() or 1)
    per_seq = d["bytes"] / d["B"]
    kc = torch.zeros([d["nblk"], d["Hkv"], 1, d["bs"], d["D"]], dtype=torch.float8_e4m3fn)
    vc = kc.clone()
    ks, vs = torch.ones(d["nblk"], d["Hkv"]), torch.ones(d["nblk"], d["Hkv"])
    times = []
    t_end = time.perf_counter() + budget_s
    b = 0
    while True:
        t = time.perf_counter()
        opa.kv_write(d["k"][b:b + 1], d["v"][b:b + 1], kc, vc, d["seq"][b:b + 1], d["bt"][b:b + 1], d["bs"], ks, vs)
        times.append(time.perf_counter() - t)
        b = (b + 1) % d["B"]
        if time.perf_counter() > t_end or len(times) >= d["B"]:
            break
    med = statistics.median(times)
    return per_seq / med / 1e9, med, times


def kv_write_parity(d, kc, vc, ks, vs, step, n=4, seed=7):
    """One more C-ABI write over the whole batch, outside the timed region,
    checked on a seeded subset of the sequences: their touched blocks (caches
    and scales) are copied out before and after the call, and the oracle
    applies the same write to the copy taken before. Caches and scales must
    match bit for bit."""
    from oracle import paged_attention as opa

    B, bs, S = d["B"], d["bs"], d["S"]
    n = min(n, B)
    idx = torch.randperm(B, generator=torch.Generator().manual_seed(seed))[:n].sort().values
    blocks, tabs = [], []
    for b in idx.tolist():
        s0 = int(d["seq"][b])
        first, last = s0 // bs, (s0 + S - 1) // bs
        tab = torch.zeros(d["bt"].shape[1], dtype=torch.int64)
        tab[first:last + 1] = torch.arange(len(blocks), len(blocks) + last - first + 1)
        blocks += d["bt"][b, first:last + 1].long().tolist()
        tabs.append(tab)
    sel = torch.tensor(blocks, dtype=torch.int64, device=kc.device)
    torch.cuda.synchronize()
    before = [t[sel].cpu() for t in (kc, vc, ks, vs)]
    step()
    torch.cuda.synchronize()
    after = [t[sel].cpu() for t in (kc, vc, ks, vs)]
    kc0, vc0, ks0, vs0 = before
    opa.kv_write(d["k"][idx], d["v"][idx], kc0, vc0, d["seq"][idx], torch.stack(tabs), bs, ks0, vs0)
    same = [torch.equal(a.view(torch.uint8), b.view(torch.uint8)) for a, b in zip((kc0, vc0), after[:2])]
    same += [torch.equal(a, b) for a, b in zip((ks0, vs0), after[2:])]
    return {"ok": all(same), "n_checked": n, "blocks_checked": len(blocks),
            "checked": f"sequences {idx.tolist()}: every touched block's K and V cache rows and scales",
            "tolerance": "bit-exact", "oracle": "oracle.paged_attention.kv_write"}


def kv_write_record(args, ctx: Ctx, wl_name: str, cpu_leg: bool = True) -> dict:
    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi

    ws, rank, dev, stream = ctx.ws, ctx.rank, ctx.dev, ctx.stream
    wl = KVWRITE[wl_name]
    d = build_kv_write(wl, seed=1000 * rank)
    k, v, seq, bt = (d[x].to(dev) for x in ("k", "v", "seq", "bt"))
    shape = [d["nblk"], d["Hkv"], 1, d["bs"], d["D"]]
    kc = torch.zeros(shape, dtype=torch.float8_e4m3fn, device=dev)
    vc = torch.zeros_like(kc)
    ks = torch.ones(d["nblk"], d["Hkv"], device=dev)
    vs = torch.ones_like(ks)
    qshape = torch.empty([d["B"], d["Hkv"], 1, d["S"], d["D"]], dtype=torch.bfloat16, device=dev)
    p, keep = cabi.paged_params(qshape, k, v, kc, vc, seq, bt, d["bs"], 1.0, k_scale=ks, v_scale=vs)
    L = cabi.lib()
    sh = ctypes.c_void_p(stream.cuda_stream)
    pref = ctypes.byref(p)

    def step():
        rc = L.rbln_paged_kv_write(pref, sh)
        if rc != 0:
            raise RuntimeError(f"rbln_paged_kv_write failed: {rc}")

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.barrier()
    with ClockSampler(ctx.local) as clk:
        op_ms, _ = _timed_kernel_loop(args, stream, step, step, flush)
    # e2e: the torch op with k / v / seq / block_table from pinned host memory, the scales read back
    pinned = [d[x].pin_memory() for x in ("k", "v", "seq", "bt")]
    hks = torch.empty(ks.shape, dtype=ks.dtype).pin_memory()
    hvs = torch.empty(vs.shape, dtype=vs.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    d2h = hks.numel() * 4 * 2

    def e2e_step():
        kk, vv, ss, bb = (t.to(dev, non_blocking=True) for t in pinned)
        torch.ops.rbln_attn.paged_kv_write(kk, vv, kc, vc, ss, bb, d["bs"], ks, vs)
        hks.copy_(ks, non_blocking=True)
        hvs.copy_(vs, non_blocking=True)

    for _ in range(max(2, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    parity = kv_write_parity(d, kc, vc, ks, vs, step, seed=7 + rank)
    failed = ctx.reduce([0.0 if parity["ok"] else 1.0], "max")[0]
    parity["ok"] = parity["ok"] and failed == 0
    op_ms, e2e_ms = ctx.reduce([op_ms, e2e_ms], "max")
    hbm_peak, _, peak_src = load_peaks()
    gbs = d["bytes"] / (op_ms * 1e-3) / 1e9
    rec = {
        "metric": "paged KV write GB/s", "value": round(ws * gbs, 1), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(op_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded N(0,1) rows, seeded starts and block-table permutation)",
        "config": kv_write_config(wl, d, ws),
        "e2e": {"value": round(ws * d["bytes"] / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": "torch.ops.rbln_attn.paged_kv_write"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(gbs / hbm_peak, 4), "traffic": _traffic_from_profiles(wl_name),
                     "kernel": "paged_kv_write_staged_kernel<bf16>", "kernel_ms": round(op_ms, 4),
                     "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs), of measured" if peak_src == "measured"
                                     else "fallback 6.65 TB/s")},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "parity": parity,
    }
    if rank == 0 and cpu_leg and ws == 1 and not args.no_cpu_baseline:
        val, med, times = _cpu_kv_write(build_kv_write(wl), min(args.cpu_budget, 10.0))
        rec["cpu_baseline"] = {"value": round(val, 4), "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
                               "sample": f"oracle.paged_attention.kv_write, 1 sequence (all KV heads) per run, "
                                         f"{_cpu_stats_note(times)}"}
    del kc, vc
    torch.cuda.empty_cache()
    return rec


def reference_kv_write_line(args, ctx: Ctx, wl_name: str, budget_s=10.0) -> dict:
    wl = KVWRITE[wl_name]
    d = build_kv_write(wl)
    val, med, times = _cpu_kv_write(d, budget_s)
    sample = f"oracle.paged_attention.kv_write, 1 sequence (all KV heads) per run, {_cpu_stats_note(times)}"
    return {"impl": "reference", "metric": "paged KV write GB/s", "value": round(val, 4),
            "unit": "GB/s", "n_gpus": ctx.ws, "steps": len(times), "warmup": args.warmup,
            "ms_per_step": round(med * 1e3 * d["B"], 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded)",
            "config": kv_write_config(wl, d, ctx.ws),
            "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": os.cpu_count() or 1,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ---------------------------------------------------------------------------
# entry points
# ---------------------------------------------------------------------------
def ours_record(args, ctx, wl_name, cpu_leg=True):
    if wl_name in KVWRITE:
        return kv_write_record(args, ctx, wl_name, cpu_leg)
    if wl_name in COMPUTE:
        return compute_record(args, ctx, wl_name, cpu_leg)
    return decode_record(args, ctx, wl_name, n_parity=4 if wl_name == "decode_long" else 8, cpu_leg=cpu_leg)


def reference_record(args, ctx, wl_name, per_step_budget=None):
    if wl_name in KVWRITE:
        return reference_kv_write_line(args, ctx, wl_name)
    if wl_name in COMPUTE:
        return reference_compute_line(args, ctx, wl_name, budget_s=30.0 if per_step_budget else 120.0)
    return reference_decode_line(args, ctx, wl_name, per_step_budget)


def _strip(rec):
    """A workload record inside the headline line (no repeated run keys)."""
    return {k: v for k, v in rec.items() if k not in ("n_gpus", "steps", "warmup", "vs_baseline")}


def run_suite_ours(args):
    ctx = Ctx()
    line = ours_record(args, ctx, SUITE_HEADLINE)
    line["workloads"] = {}
    for name, wl_name, multi in SUITE:
        if ctx.ws > 1 and not multi:
            continue  # a one-GPU configuration: measured at N = 1
        line["workloads"][name] = _strip(ours_record(args, ctx, wl_name))
    if ctx.ws > 1:
        line["workloads_note"] = ("at N > 1 only the sharded configurations run (long-context decode sharded by "
                                  "KV head, fp8 decode split by sequence); the others are one-GPU configurations")
    line["gpu_launches"] = line["gpu_launches"] + sum(r.get("gpu_launches", 0) for r in line["workloads"].values())
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


def run_suite_reference(args):
    ctx = Ctx(with_gpu=False)
    if ctx.rank != 0:
        return  # rank 0 alone times the CPU path
    line = reference_record(args, ctx, SUITE_HEADLINE)
    line["workloads"] = {}
    for name, wl_name, multi in SUITE:
        if ctx.ws > 1 and not multi:
            continue
        small = argparse.Namespace(**vars(args))
        small.steps, small.warmup = 3, 1
        line["workloads"][name] = _strip(reference_record(small, ctx, wl_name, per_step_budget=5.0))
    print(json.dumps(line), flush=True)


def peer_emulation_record(args, wl_name: str, ranks: int) -> dict:
    """One GPU: rank 0's share of a head-sharded decode at `ranks` ranks,
    timed through the plain entry point and through the peers entry point
    with n = 1, 2 and `ranks` emulated ranks whose output buffers and flag
    arrays all live in this GPU's memory, the other ranks' announcements
    pre-set. The difference is the peer path's own cost (the stores into n
    buffers, the merge kernel's arrival chain, the system-scope releases)
    without NVLink."""
    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi

    wl = WORKLOADS[wl_name]
    if wl["shard"] != "heads" or ranks < 2 or wl["Hkv"] % ranks:
        raise SystemExit(f"--emulate-ranks needs a head-sharded workload whose KV heads divide by {ranks}")
    ctx = Ctx()
    dev, stream = ctx.dev, ctx.stream
    d = build_decode_sharded(wl, "heads", 0, ranks, dev)
    q, k, v, seq, bt = (d[x].to(dev) for x in ("q", "k", "v", "seq", "bt"))
    L = cabi.lib()
    sh = ctypes.c_void_p(stream.cuda_stream)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    B, Hkv, G, _, D = q.shape

    def time_us(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps * 1e3

    p, keep = cabi.paged_params(q, k, v, d["kcache"], d["vcache"], seq, bt, d["bs"], d["scale"])
    cabi.attach_workspace(p, dev, keep)
    p.error_flags = err.data_ptr()

    def plain():
        if L.rbln_paged_causal_attn_decode(ctypes.byref(p), sh) != 0:
            raise RuntimeError("rbln_paged_causal_attn_decode failed")

    rec = {"metric": "head-sharded decode per call, peer path emulated on one GPU", "unit": "us",
           "workload": wl["desc"], "emulated_ranks": ranks, "steps": args.steps, "warmup": args.warmup,
           "plain_op_us": round(time_us(plain), 2), "peers_op_us": {}}
    with torch.cuda.stream(stream):
        for n in sorted({1, 2, ranks}):
            outs = [torch.zeros([B, n * Hkv, G, 1, D], dtype=q.dtype, device=dev) for _ in range(n)]
            flags = [torch.zeros(n, dtype=torch.int32, device=dev) for _ in range(n)]
            flags[0][1:] = 0x40000000  # every other rank has announced every epoch used here
            out_ptrs = torch.tensor([o.data_ptr() for o in outs], dtype=torch.int64, device=dev)
            flag_ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=dev)
            pp, kp = cabi.paged_params(q, k, v, d["kcache"], d["vcache"], seq, bt, d["bs"], d["scale"], out=outs[0])
            cabi.attach_workspace(pp, dev, kp)
            pp.error_flags = err.data_ptr()
            po = cabi.PeerOut()
            po.out, po.flags = out_ptrs.data_ptr(), flag_ptrs.data_ptr()
            po.n, po.rank, po.head0, po.wait_limit_us = n, 0, 0, 100000
            epoch = [0]

            def peers():
                epoch[0] += 1
                po.epoch = epoch[0]
                if L.rbln_paged_causal_attn_decode_peers(ctypes.byref(pp), ctypes.byref(po), sh) != 0:
                    raise RuntimeError("rbln_paged_causal_attn_decode_peers failed")

            rec["peers_op_us"][str(n)] = round(time_us(peers), 2)
    torch.cuda.synchronize()
    rec["device_error_bits"] = int(err.item())
    ctx.close()
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="suite",
                    choices=["suite"] + sorted(WORKLOADS) + sorted(COMPUTE) + sorted(KVWRITE))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--emulate-ranks", type=int, default=0,
                    help="one GPU: time rank 0's share of a head-sharded decode at this many ranks through the "
                         "plain and the peers entry points, every rank's buffers local (the peer path's own cost)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.emulate_ranks:
        print(json.dumps(peer_emulation_record(args, args.workload, args.emulate_ranks)), flush=True)
        return
    if args.workload == "suite":
        (run_suite_reference if args.impl == "reference" else run_suite_ours)(args)
        return
    if args.impl == "reference":
        ctx = Ctx(with_gpu=False)
        if ctx.rank == 0:
            print(json.dumps(reference_record(args, ctx, args.workload)), flush=True)
        return
    ctx = Ctx()
    rec = ours_record(args, ctx, args.workload)
    if ctx.rank == 0:
        print(json.dumps(rec), flush=True)
    ctx.close()


if __name__ == "__main__":
    main()
