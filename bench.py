#!/usr/bin/env python
"""Benchmark of the B200 attention hot path (paged decode by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|decode_fp8|decode_long|prefill|sdpa|sdpa_bf16]

Default workload (N = 1): paged-attention decode, bf16, batch 64, 32 query /
8 KV heads, head_dim 128, block_size 16, context length per sequence
uniform in [128, 4096], block table = seeded random permutation of a
20,000-block KV pool, K/V ~ N(0,1)*0.5, one new token per sequence.
Metric: algorithmic HBM bytes per step / time (GB/s).

A step is one call of rbln_custom_ops.paged_causal_attn_decode over the
batch (append + attention). `value` times K steps with inputs resident in
HBM (the KV pool, 1.3 GB, is far larger than the 126 MB L2, so no flush is
needed); `e2e` times the same op through the public torch op with the
step's inputs (q, k, v, seq, block_table) copied from pinned host memory
and the output copied back inside the timed region. `roofline` is the main
kernel alone, timed with CUDA events recorded on its launch stream around
that kernel (C-ABI measurement hook).

Under torchrun (N > 1) every rank runs its own batch of the same workload
(sequences are independent; no collective on the data path) and the JSON
line reports the whole-job aggregate over max-over-ranks time.

--impl reference times the reference's CPU algorithm for the same workload
on this host's cores (the oracle's restatement of the reference CPU op,
oracle/paged_attention.py, on a bounded sample of sequences).
"""

from __future__ import annotations

import argparse
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


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
WORKLOADS = {
    "decode": dict(desc="paged decode bf16 B=64 Hq=32 Hkv=8 D=128 bs=16 L~U[128,4096] pool=20000",
                   B=64, Hkv=8, G=4, D=128, bs=16, lmin=128, lmax=4096, pool=20000, fp8=False),
    "decode_fp8": dict(desc="paged decode fp8-e4m3 KV B=256 Hq=32 Hkv=8 D=128 bs=16 L~U[512,8192]",
                       B=256, Hkv=8, G=4, D=128, bs=16, lmin=512, lmax=8192, pool=None, fp8=True),
    # profiling case for ncu --set full: inputs still larger than L2, ~0.35 GB on the device
    "decode_small": dict(desc="paged decode bf16 B=16 Hq=32 Hkv=8 D=128 bs=16 L~U[128,4096] pool=5000",
                         B=16, Hkv=8, G=4, D=128, bs=16, lmin=128, lmax=4096, pool=5000, fp8=False),
    # long context, KV heads sharded over the ranks; each rank's kernels store its heads'
    # outputs into every rank's output buffer over NVLink (no separate all-gather)
    # profiling case for the fp8 path (~0.6 GB of fp8 KV on the device)
    "decode_fp8_small": dict(desc="paged decode fp8-e4m3 KV B=64 Hq=32 Hkv=8 D=128 bs=16 L~U[512,8192]",
                             B=64, Hkv=8, G=4, D=128, bs=16, lmin=512, lmax=8192, pool=None, fp8=True),
    "decode_long": dict(desc="paged decode bf16 B=32 Hq=64 Hkv=8 D=128 bs=16 L=32768 pool=65536",
                        B=32, Hkv=8, G=8, D=128, bs=16, lmin=32768, lmax=32768, pool=65536, fp8=False,
                        shard="heads"),
}


def build_decode(wl: dict, device, seed: int = 0, pool_seed: int = None):
    """Seeded synthetic decode inputs. Lengths / block table on the CPU
    generator; the KV pool is drawn on the device (seed + 1, or pool_seed)."""
    g = torch.Generator().manual_seed(seed)
    B, Hkv, G, D, bs = wl["B"], wl["Hkv"], wl["G"], wl["D"], wl["bs"]
    lens = torch.randint(wl["lmin"], wl["lmax"] + 1, (B,), generator=g)
    max_blocks = int(math.ceil(int(lens.max()) / bs))
    nblk = wl["pool"] or int(sum(math.ceil(int(x) / bs) for x in lens)) + B
    nblk = max(nblk, B * max_blocks)
    perm = torch.randperm(nblk, generator=g)
    # each sequence takes its blocks from the permutation in turn
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
    gd = torch.Generator(device=device).manual_seed(seed + 1 if pool_seed is None else pool_seed)
    shape = [nblk, Hkv, 1, bs, D]
    if wl["fp8"]:
        kc, ks = _fp8_pool(shape, gd, device)
        vc, vs = _fp8_pool(shape, gd, device)
    else:
        kc = (torch.randn(shape, generator=gd, device=device, dtype=torch.bfloat16) * 0.5)
        vc = (torch.randn(shape, generator=gd, device=device, dtype=torch.bfloat16) * 0.5)
        ks = vs = None
    return dict(q=q, k=k, v=v, seq=seq, bt=bt, kcache=kc, vcache=vc, k_scale=ks, v_scale=vs, lens=lens,
                scale=1.0 / math.sqrt(D), bs=bs, B=B, Hkv=Hkv, G=G, D=D, fp8=wl["fp8"])


def _fp8_pool(shape, gd, device):
    x = torch.randn(shape, generator=gd, device=device, dtype=torch.float32)
    amax = x.abs().amax(dim=(2, 3, 4)).clamp_min(1e-6)
    sc = (amax / 448.0).contiguous()
    q = (x / sc[:, :, None, None, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    del x
    return q, sc


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


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
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


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, wl_name):
    import torch.distributed as dist

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi

    wl = WORKLOADS[wl_name]
    head_shard = wl.get("shard") == "heads" and ws > 1
    if head_shard:
        # every rank sees the same sequences and block table; it holds only its
        # slice of the KV heads (and their query heads)
        from torch_rbln_b200 import sharding

        sharding.kv_head_range(wl["Hkv"], rank, ws)
        wl = dict(wl, Hkv=wl["Hkv"] // ws)
        d = build_decode(wl, dev, seed=0, pool_seed=1 + rank)
    else:
        d = build_decode(wl, dev, seed=1000 * rank)
    q, k, v = d["q"].to(dev), d["k"].to(dev), d["v"].to(dev)
    seq, bt = d["seq"].to(dev), d["bt"].to(dev)
    kc, vc = d["kcache"], d["vcache"]
    ks, vs = d["k_scale"], d["v_scale"]
    scale_t = torch.tensor(d["scale"])
    nbytes = decode_bytes(d)
    ops = torch.ops.rbln_custom_ops

    peer = None
    if head_shard:
        # every rank's full output buffers, written by all ranks' kernels over NVLink
        peer = sharding.PeerHeadOutput((q.shape[0], q.shape[1] * ws) + tuple(q.shape[2:]), q.dtype, rank, ws)
        head0 = rank * q.shape[1]
        e2e_ws = {}

    def op_call(qq, kk, vv, ss, bb):
        if d["fp8"]:
            return ops.paged_causal_attn_decode_kvfp8(qq, kk, vv, kc, vc, ks, vs, ss, scale_t, bb, d["bs"])
        if head_shard:
            return sharding.head_sharded_paged_decode_p2p(qq, kk, vv, kc, vc, ss, d["scale"], bb, d["bs"], peer,
                                                          workspace=e2e_ws, q_is_local=True)
        return ops.paged_causal_attn_decode(qq, kk, vv, kc, vc, ss, scale_t, bb, d["bs"])

    # C-ABI parameter block with the timing hook around the main kernel
    p, keep = cabi.paged_params(q, k, v, kc, vc, seq, bt, d["bs"], d["scale"], k_scale=ks, v_scale=vs,
                                out=peer.outputs[0] if head_shard else None)
    cabi.attach_workspace(p, dev, keep)
    L = cabi.lib()
    stream = torch.cuda.current_stream(dev)
    entry = L.rbln_paged_causal_attn_decode
    import ctypes

    pref = ctypes.byref(p)
    sh = ctypes.c_void_p(stream.cuda_stream)
    ws_bytes = p.workspace_bytes

    def cabi_step(ev0=None, ev1=None):
        p.prof_events[0] = ev0.cuda_event if ev0 is not None else None
        p.prof_events[1] = ev1.cuda_event if ev1 is not None else None
        if head_shard:
            # decode of the local heads, outputs stored into every rank's buffer, epoch exchange
            out, po = peer.next(head0)
            p.out = out.data_ptr()
            rc = L.rbln_paged_causal_attn_decode_peers(pref, ctypes.byref(po), sh)
        else:
            rc = entry(pref, sh)
        if rc != 0:
            raise RuntimeError(f"rbln_paged_causal_attn_decode failed: {rc}")

    for _ in range(args.warmup):
        cabi_step()
        op_call(q, k, v, seq, bt)
    torch.cuda.synchronize()

    # ---- value: device-resident inputs, K steps, events around the whole op
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in kev:  # create the events on the device before timing
        e0.record(stream)
        e1.record(stream)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            cabi_step(*kev[i])
        t1.record(stream)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
    ms_total = t0.elapsed_time(t1)
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    ms_step = ms_total / args.steps

    # ---- e2e: public torch op, host buffers, H2D + D2H inside the timed region
    pin = lambda t: t.cpu().pin_memory()
    hq, hk, hv, hs, hb = pin(d["q"]), pin(d["k"]), pin(d["v"]), pin(d["seq"]), pin(d["bt"])
    out_heads = q.shape[1] * (ws if head_shard else 1)
    hout = torch.empty((q.shape[0], out_heads) + tuple(q.shape[2:]), dtype=q.dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hs, hb))
    d2h = hout.numel() * hout.element_size()
    for _ in range(max(2, args.warmup)):
        o = op_call(hq.to(dev, non_blocking=True), hk.to(dev, non_blocking=True), hv.to(dev, non_blocking=True),
                    hs.to(dev, non_blocking=True), hb.to(dev, non_blocking=True))
        hout.copy_(o, non_blocking=True)
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        o = op_call(hq.to(dev, non_blocking=True), hk.to(dev, non_blocking=True), hv.to(dev, non_blocking=True),
                    hs.to(dev, non_blocking=True), hb.to(dev, non_blocking=True))
        hout.copy_(o, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    # max over ranks
    if ws > 1:
        tt = torch.tensor([ms_step, e2e_ms, statistics.mean(kern_ms)], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_step, e2e_ms, kmean = tt.tolist()
    else:
        kmean = statistics.mean(kern_ms)

    hbm_peak, tf_peak, peak_src = load_peaks()
    achieved = nbytes / (kmean * 1e-3) / 1e9
    value = ws * nbytes / (ms_step * 1e-3) / 1e9
    launches_per_step = 1 + (1 if ws_bytes > 0 else 0)
    line = {
        "metric": "paged decode HBM GB/s",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong" if head_shard else "weak",
        "vs_baseline": None,
        "dtype": "fp8e4m3-kv/bf16" if d["fp8"] else "bf16",
        "data": "synthetic (seeded N(0,1)*0.5 KV pool, seeded lengths and block-table permutation)",
        "config": {"workload": WORKLOADS[wl_name]["desc"], "global_batch": d["B"] if head_shard else d["B"] * ws,
                   "parallelism": (f"kv-head-sharded x{ws}, head outputs stored into every rank's buffer by the decode kernels (NVLink P2P) + epoch barrier" if head_shard
                                   else f"batch-sharded x{ws}"),
                   "l2": "inputs larger than L2 (KV pool " + f"{kc.numel() * kc.element_size() * 2 / 1e9:.2f} GB)",
                   "bytes_per_step_per_gpu": nbytes},
        "e2e": {"value": round(ws * nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "torch.ops.rbln_custom_ops.paged_causal_attn_decode" + ("_kvfp8" if d["fp8"] else "")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": None,
                     "kernel": "paged_decode_balanced_kernel (equal token chunks over the batch, mma.sync)", "kernel_ms": round(kmean, 4),
                     "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                     else "fallback 6.65 TB/s"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    traffic = _traffic_from_profiles(wl_name)
    if traffic is not None:
        line["roofline"]["traffic"] = traffic
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl_name, d, budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()  # every rank is past its last call before any buffer is unmapped
    if peer is not None:
        peer.close()
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


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


# ---------------------------------------------------------------------------
# CPU baseline / reference arm
# ---------------------------------------------------------------------------
def cpu_sample(d: dict, n_seq: int, device_pool: bool = True):
    """First n_seq sequences, gathered into the reference's contiguous
    per-sequence layout [n, Hkv, 1, max_seq, D] (gather not timed)."""
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


def cpu_baseline(wl_name, d, budget_s=20.0, steps=None):
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    # size the sample: time one sequence, then take as many as fit the budget
    q, k, v, kc, vc, seq, sc, opa, nb = cpu_sample(d, 1)
    t = time.perf_counter()
    opa.mock_decode_contiguous(q, k, v, kc.clone(), vc.clone(), seq, sc)
    one = max(time.perf_counter() - t, 1e-4)
    n = int(max(1, min(d["B"], budget_s / 4 / one)))
    q, k, v, kc, vc, seq, sc, opa, nb = cpu_sample(d, n)
    times = []
    reps = steps if steps is not None else 3
    opa.mock_decode_contiguous(q, k, v, kc.clone(), vc.clone(), seq, sc)  # warm-up
    for _ in range(reps):
        kk, vv = kc.clone(), vc.clone()
        t = time.perf_counter()
        opa.mock_decode_contiguous(q, k, v, kk, vv, seq, sc)
        times.append(time.perf_counter() - t)
    med = statistics.median(times)
    return {"value": round(nb / med / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} of {d['B']} sequences of the same workload, reference CPU algorithm "
                      f"(oracle.paged_attention.mock_decode_contiguous, bf16 over the gathered per-sequence "
                      f"layout), median of {reps} runs, {med * 1e3:.1f} ms per sample",
            "ms_per_sample": round(med * 1e3, 2), "bytes_per_sample": nb}


def run_reference(args, wl_name):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    wl = WORKLOADS[wl_name]
    dev = torch.device("cpu")
    d = build_decode(wl, dev, seed=0)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    q, k, v, kc, vc, seq, sc, opa, nb = cpu_sample(d, 1)
    t = time.perf_counter()
    opa.mock_decode_contiguous(q, k, v, kc.clone(), vc.clone(), seq, sc)
    one = max(time.perf_counter() - t, 1e-4)
    per_step_budget = max(0.5, 120.0 / max(1, args.steps + args.warmup))
    n = int(max(1, min(d["B"], per_step_budget / one)))
    q, k, v, kc, vc, seq, sc, opa, nb = cpu_sample(d, n)
    for _ in range(args.warmup):
        opa.mock_decode_contiguous(q, k, v, kc.clone(), vc.clone(), seq, sc)
    times = []
    for _ in range(args.steps):
        kk, vv = kc.clone(), vc.clone()
        t = time.perf_counter()
        opa.mock_decode_contiguous(q, k, v, kk, vv, seq, sc)
        times.append(time.perf_counter() - t)
    ms = statistics.mean(times) * 1e3
    val = nb / (ms * 1e-3) / 1e9
    sample = (f"{n} of {d['B']} sequences per step, reference CPU algorithm (oracle restatement of "
              f"test_custom_kernel.py paged_causal_attn_decode on the per-sequence layout), wall clock")
    line = {"impl": "reference", "metric": "paged decode HBM GB/s", "value": round(val, 3), "unit": "GB/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded)", "config": {"workload": wl["desc"], "global_batch": d["B"]},
            "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# compute-bound workloads: chunked prefill and SDPA
# ---------------------------------------------------------------------------
COMPUTE = {
    "prefill": dict(kind="prefill", B=8, Hkv=8, G=4, D=128, bs=16, S=512, cmin=0, cmax=8192,
                    desc="paged chunked prefill bf16 B=8 Hq=32 Hkv=8 D=128 S_q=512 new tokens, "
                         "cached ctx~U[0,8192], bs=16, causal"),
    # profiling case for ncu --set full (same per-CTA work, fewer sequences)
    "prefill_small": dict(kind="prefill", B=2, Hkv=8, G=4, D=128, bs=16, S=512, cmin=2048, cmax=6144,
                          desc="paged chunked prefill bf16 B=2 Hq=32 Hkv=8 D=128 S_q=512 ctx~U[2048,6144]"),
    "sdpa": dict(kind="sdpa", B=1, Hq=32, Hkv=8, L=512, D=64, dtype=torch.float32,
                 desc="SDPA causal GQA fp32 B=1 Hq=32 Hkv=8 L=S=512 D=64 (Llama-3.2-1B attention shape)"),
    "sdpa_bf16": dict(kind="sdpa", B=4, Hq=32, Hkv=8, L=4096, D=128, dtype=torch.bfloat16,
                      desc="SDPA causal GQA bf16 B=4 Hq=32 Hkv=8 L=S=4096 D=128"),
    "sdpa_bwd": dict(kind="sdpa_bwd", B=2, Hq=32, Hkv=8, L=4096, D=128, dtype=torch.bfloat16,
                     desc="SDPA backward causal GQA bf16 B=2 Hq=32 Hkv=8 L=S=4096 D=128 (dq, dk, dv)"),
    # profiling case for ncu --set full
    "sdpa_bwd_small": dict(kind="sdpa_bwd", B=1, Hq=32, Hkv=8, L=2048, D=128, dtype=torch.bfloat16,
                           desc="SDPA backward causal GQA bf16 B=1 Hq=32 Hkv=8 L=S=2048 D=128 (dq, dk, dv)"),
}


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
    return dict(q=q, k=k, v=v, kcache=kc, vcache=vc, seq=ctx.to(torch.int32).reshape(B, 1), bt=bt, bs=bs,
                ctx=ctx, flops=flops, scale=1.0 / math.sqrt(D), B=B, Hkv=Hkv, G=G, D=D, S=S)


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


def _timed_kernel_loop(args, stream, step, kernel_step, flush):
    """Per-iteration CUDA events on the launch stream around the whole op
    (`step`) and, in separate iterations, around the main kernel alone
    (`kernel_step`), each preceded by an L2 flush outside the timed window."""
    def timed(fn):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in ev)

    return timed(step), timed(kernel_step)


def run_compute_ours(args, wl_name):
    import ctypes

    import torch.distributed as dist

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi

    wl = COMPUTE[wl_name]
    stream = torch.cuda.current_stream(dev)
    sh = ctypes.c_void_p(stream.cuda_stream)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2
    L = cabi.lib()
    if wl["kind"] == "prefill":
        d = build_prefill(wl, dev, seed=1000 * rank)
        q, k, v, seq, bt = (d[x].to(dev) for x in ("q", "k", "v", "seq", "bt"))
        kc, vc = d["kcache"], d["vcache"]
        p, keep = cabi.paged_params(q, k, v, kc, vc, seq, bt, d["bs"], d["scale"], causal=1)
        # the same call without new rows to append launches the attention kernel alone
        pk, keepk = cabi.paged_params(q, None, None, kc, vc, seq, bt, d["bs"], d["scale"], causal=1)
        cabi.attach_workspace(p, dev, keep, prefill=True)
        cabi.attach_workspace(pk, dev, keepk, prefill=True)
        pref, pkref = ctypes.byref(p), ctypes.byref(pk)
        scale_t = torch.tensor(d["scale"])

        def step():
            rc = L.rbln_paged_causal_attn_prefill(pref, sh)
            if rc != 0:
                raise RuntimeError(f"rbln_paged_causal_attn_prefill failed: {rc}")

        def kernel_step():
            rc = L.rbln_paged_causal_attn_prefill(pkref, sh)
            if rc != 0:
                raise RuntimeError(f"rbln_paged_causal_attn_prefill failed: {rc}")

        def op_call(qq, kk, vv, ss, bb):
            return torch.ops.rbln_custom_ops.paged_causal_attn_prefill(qq, kk, vv, kc, vc, ss, scale_t, bb, d["bs"],
                                                                       False)

        host_inputs = [d["q"], d["k"], d["v"], d["seq"], d["bt"]]
        out_shape, out_dtype = q.shape, q.dtype
        metric = "paged chunked prefill TFLOP/s"
        launches = 3  # schedule pre-pass, append, attention
        kernel = "attn_fwd_tc3_kernel<128, bf16> (tcgen05/TMEM/TMA, 128-key tiles, P in TMEM, two query tiles per CTA)"
        dtype = "bf16"
        l2 = "L2 flushed between iterations (256 MB write, outside the timed events)"
    elif wl["kind"] == "sdpa_bwd":
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
        l2 = "L2 flushed between iterations (256 MB write, outside the timed events)"
    else:
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
        l2 = "L2 flushed between iterations (256 MB write, outside the timed events)"

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        op_ms, k_ms = _timed_kernel_loop(args, stream, step, kernel_step, flush)
    if ws > 1:
        dist.barrier()

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
    if ws > 1:
        tt = torch.tensor([op_ms, e2e_ms, k_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        op_ms, e2e_ms, k_ms = tt.tolist()

    hbm_peak, tf_peak, peak_src = load_peaks()
    flops = d["flops"]
    achieved = flops / (k_ms * 1e-3) / 1e12
    line = {
        "metric": metric, "value": round(ws * flops / (op_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(op_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded N(0,1) inputs" + (", seeded cached lengths and block-table permutation)"
                                                     if wl["kind"] == "prefill" else ")"),
        "config": {"workload": wl["desc"], "parallelism": f"replicas x{ws}", "l2": l2, "flops_per_step": flops},
        "e2e": {"value": round(ws * flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "api": {"prefill": "torch.ops.rbln_custom_ops.paged_causal_attn_prefill",
                        "sdpa_bwd": "torch.ops.aten._scaled_dot_product_fused_attention_overrideable_backward"}.get(
                            wl["kind"], "torch.nn.functional.scaled_dot_product_attention")},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tf_peak, 4), "traffic": _traffic_from_profiles(wl_name),
                     "kernel": kernel, "kernel_ms": round(k_ms, 4),
                     "peak_source": ("measured (MEASURED_PEAKS.json bf16_tflops, burst)" if peak_src == "measured"
                                     else "fallback 1.59 PFLOP/s")},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_compute(wl, d, args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    return statistics.median(times), flops, sample, len(times)


def cpu_baseline_compute(wl, d, budget_s):
    med, flops, sample, n = _cpu_compute_times(wl, d, 5, budget_s)
    return {"value": round(flops / med / 1e12, 5), "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": sample + f", median of {n} runs, {med * 1e3:.1f} ms", "ms_per_sample": round(med * 1e3, 2)}


def run_reference_compute(args, wl_name):
    ws, rank, local = dist_env()
    if rank != 0:
        return
    wl = COMPUTE[wl_name]
    d = build_prefill(wl, torch.device("cpu"), seed=0) if wl["kind"] == "prefill" else build_sdpa(wl, seed=0)
    for _ in range(args.warmup):
        _cpu_compute_times(wl, d, 1, 1e9)
    med, flops, sample, n = _cpu_compute_times(wl, d, args.steps, 120.0)
    val = flops / med / 1e12
    unit = "TFLOP/s"
    metric = {"prefill": "paged chunked prefill TFLOP/s", "sdpa_bwd": "SDPA backward TFLOP/s"}.get(wl["kind"],
                                                                                                 "SDPA TFLOP/s")
    line = {"impl": "reference", "metric": metric, "value": round(val, 5), "unit": unit, "n_gpus": ws, "steps": n,
            "warmup": args.warmup, "ms_per_step": round(med * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if wl["kind"] != "prefill" and wl["dtype"] == torch.float32 else "bf16",
            "data": "synthetic (seeded)", "config": {"workload": wl["desc"]},
            "cpu_baseline": {"value": round(val, 5), "unit": unit, "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(val, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# standalone KV-cache write (HBM-bound)
# ---------------------------------------------------------------------------
KVWRITE = {
    "kv_write_fp8": dict(B=64, Hkv=8, D=128, bs=16, S=512, cmax=4096,
                         desc="paged KV write bf16 -> fp8-e4m3 cache, per-(block, head) scale recompute: B=64 "
                              "sequences x 512 new rows, Hkv=8, D=128, bs=16, start ~U[0,4096]"),
    # profiling case for ncu --set full
    "kv_write_fp8_small": dict(B=16, Hkv=8, D=128, bs=16, S=512, cmax=4096,
                               desc="paged KV write bf16 -> fp8-e4m3 cache: B=16 sequences x 512 new rows, Hkv=8, "
                                    "D=128, bs=16"),
}


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
    """oracle.paged_attention.kv_write on one sequence (all KV heads)."""
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
    return per_seq / med / 1e9, med, len(times)


def run_kv_write(args, wl_name):
    import ctypes

    ws, rank, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return
        wl = KVWRITE[wl_name]
        d = build_kv_write(wl)
        val, med, n = _cpu_kv_write(d, max(10.0, args.cpu_budget))
        sample = f"oracle.paged_attention.kv_write, 1 sequence (all KV heads) per run, median of {n} runs"
        print(json.dumps({"impl": "reference", "metric": "paged KV write GB/s", "value": round(val, 4),
                          "unit": "GB/s", "n_gpus": ws, "steps": n, "warmup": args.warmup,
                          "ms_per_step": round(med * 1e3 * d["B"], 3), "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "u8", "data": "synthetic (seeded)",
                          "config": {"workload": wl["desc"]},
                          "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": os.cpu_count() or 1,
                                           "kind": "port", "sample": sample},
                          "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch_rbln_b200  # noqa: F401
    from torch_rbln_b200 import cabi

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
    stream = torch.cuda.current_stream(dev)
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
    with ClockSampler(local) as clk:
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
    hbm_peak, _, peak_src = load_peaks()
    gbs = d["bytes"] / (op_ms * 1e-3) / 1e9
    line = {
        "metric": "paged KV write GB/s", "value": round(ws * gbs, 1), "unit": "GB/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(op_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic (seeded N(0,1) rows, seeded starts and block-table permutation)",
        "config": {"workload": wl["desc"], "parallelism": f"replicas x{ws}",
                   "l2": "L2 flushed between iterations (256 MB write, outside the timed events)",
                   "bytes_per_step": d["bytes"]},
        "e2e": {"value": round(ws * d["bytes"] / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": "torch.ops.rbln_attn.paged_kv_write"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(gbs / hbm_peak, 4), "traffic": None,
                     "kernel": "paged_kv_write_kernel<bf16, fp8>", "kernel_ms": round(op_ms, 4),
                     "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                                     else "fallback 6.65 TB/s")},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        val, med, n = _cpu_kv_write(build_kv_write(wl), args.cpu_budget)
        line["cpu_baseline"] = {"value": round(val, 4), "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"oracle.paged_attention.kv_write, 1 sequence (all KV heads) per run, "
                                          f"median of {n} runs, {med * 1e3:.1f} ms"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=sorted(WORKLOADS) + sorted(COMPUTE) + sorted(KVWRITE))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in KVWRITE:
        run_kv_write(args, args.workload)
    elif args.workload in COMPUTE:
        (run_reference_compute if args.impl == "reference" else run_compute_ours)(args, args.workload)
    elif args.impl == "reference":
        run_reference(args, args.workload)
    else:
        run_ours(args, args.workload)


if __name__ == "__main__":
    main()
