#!/usr/bin/env python
"""ALUT lookup throughput on B200: the Qwen3-VL-30B-A3B-shaped decode step.

Workload (one "step"): 48 MoE layers, each with 128 experts x 2 modalities of
K=1024 x L=64 fp32 centroid keys and 1024 x 2048 bf16 value rows (random init, seeded);
16 decode tokens (text), top-8 softmax routing over Gaussian logits, a seeded 40% of the
routed (token, expert) slots looked up (the rest are "computed"). Per layer: project the
tokens onto the layer's PCA basis, scan every routed table for the best centroid
(normalised keys, hit = max >= 0: the tablemoe decode rule), gather the winning value
rows and accumulate them, renormalised over the surviving slots, into the layer output.
The layers run one after the other, as in a real decode step.

value: lookups/s with inputs resident in HBM, the 48 layers replayed as one CUDA graph.
e2e:   the same through the public LookupStepGraph API with the step's inputs copied
       host->device and the outputs device->host inside the graph (pinned buffers).
--impl reference: the CPU oracle (a restatement of the reference's torch path) on the
       host cores, over a bounded sample of the same workload.

N>1: one process per GPU, each a replica with its own tables and token batch (the decode
lookup does not shard: "replicas only"); value is the sum over ranks of lookups divided
by the max over ranks of the device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "tablemoe-sc26_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

CFG = dict(layers=48, experts=128, k=1024, l=64, h=2048, tokens=16, top_k=8, lookup_frac=0.4)
METRIC = "ALUT lookups/s (token-expert pairs)"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
KERNELS_PER_LAYER = 3  # project+plan, centroid scan, gather/combine
CPU_LAYERS = 4
PROFILE_STEPS = 20  # replays of the event-instrumented step graph for the scan-kernel timing
# DRAM bytes (read + write) per layer of k_project_mma + k_search_decode, from one ncu
# capture of this workload's layer shape (profiles/decode_kernels_full_qwen3vl_c2.md).
NCU_TRAFFIC_PER_LAYER = 1_698_048 + 12_360_448


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def layer_inputs(layer: int, rank: int):
    """Seeded synthetic inputs of one layer (host tensors)."""
    g = torch.Generator().manual_seed(1000 * rank + layer)
    q, s, e, h = CFG["tokens"], CFG["top_k"], CFG["experts"], CFG["h"]
    x = torch.randn(q, h, generator=g).to(torch.bfloat16)
    logits = torch.randn(q, e, generator=g)
    w, sel = torch.topk(torch.softmax(logits, dim=-1), s, dim=-1)
    reuse = torch.rand(q, s, generator=g) < CFG["lookup_frac"]
    return dict(x=x, sel=sel.long(), is_vision=torch.zeros(q, dtype=torch.bool), reuse=reuse,
                weights=w.float(), compute=~reuse)


def build_layer(layer: int, device, rank: int):
    """One layer's tables on the device: normalised keys (also passed as the raw keys: the
    decode rule scores normalised keys only), bf16 values, orthonormal fp32 PCA basis."""
    from table_moe.cache_engine import HybridStorageManager
    from table_moe.cache_engine.manager import normalize_rows

    e, k, l, h = CFG["experts"], CFG["k"], CFG["l"], CFG["h"]
    g = torch.Generator(device=device).manual_seed(7919 * (rank + 1) + layer)
    keys = normalize_rows(torch.randn(e, 2, k, l, generator=g, device=device), 1e-6)
    values = torch.randn(e, 2, k, h, generator=g, device=device, dtype=torch.bfloat16).mul_(0.05)
    pca = {}
    for m in ("vision", "text"):
        qm, _ = torch.linalg.qr(torch.randn(h, l, generator=g, device=device))
        pca[m] = {"proj": qm.contiguous(), "bias": torch.zeros(l, device=device)}
    return HybridStorageManager.from_tables(layer, keys, values, pca, keys=keys)


def algorithmic_bytes(inp):
    """Bytes one layer's lookup must move at minimum: the keys of every routed table once,
    the winning value rows, x, the output read+write and the basis of the modality used.
    Returns (projection + scan bytes, whole-path bytes, lookups)."""
    k, l, h = CFG["k"], CFG["l"], CFG["h"]
    r = inp["reuse"]
    tables = len(set(inp["sel"][r].tolist()))  # all tokens are text: one modality
    scan = tables * k * l * 4 + h * l * 4 + inp["x"].numel() * 2  # keys + basis + tokens
    lookups = int(r.sum())
    rest = lookups * h * 2 + 2 * inp["x"].numel() * 2  # value rows + output read/write
    return scan, scan + rest, lookups


class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(self.NAMES, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"])}, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def sum_over_ranks(v, world, device):
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())


def max_over_ranks(v, world, device):
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- secondary workloads: prefill layer (config 3) and the sharded large table (config 5) ----
# Reported under "workloads" in the same JSON line; the headline value stays the decode step.

C3 = dict(tokens=4096, vision_tokens=1024, experts=128, k=1024, l=64, h=2048, top_k=8, lookup_frac=0.4, zipf=1.1)
C5 = dict(tokens=32768, k=65536, l=128, h=4096)
L2_FLUSH_BYTES = 256 << 20  # written between timed steps (L2 is 126 MB)


def orthonormal_basis(h, l, g, device):
    qm, _ = torch.linalg.qr(torch.randn(h, l, generator=g, device=device))
    return qm.contiguous()


def timed_steps(fn, steps, warmup, device, flush, events=None):
    """Device time of `steps` calls of fn, each timed alone with CUDA events and preceded
    (outside the timed span) by an L2 flush. With events=(start, stop) set as the library's
    profile events, also returns the mean time between them (the scan kernel)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    scan = []
    for a, b in pairs:
        flush.fill_(1)
        a.record()
        fn()
        b.record()
        if events is not None:
            torch.cuda.synchronize()
            scan.append(events[0].elapsed_time(events[1]))
    torch.cuda.synchronize()
    total = sum(a.elapsed_time(b) for a, b in pairs)
    return total, (sum(scan) / len(scan) if scan else None)


def with_scan_events(lib):
    """CUDA events registered as the library's profile events (they bracket the scan)."""
    import ctypes

    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev[0].record()
    ev[1].record()
    torch.cuda.synchronize()
    lib.alut_set_profile_events(ctypes.c_void_p(ev[0].cuda_event), ctypes.c_void_p(ev[1].cuda_event))
    return ev


def c3_workload(args, device, flush, peaks):
    """One Qwen3-VL prefill layer: 4096 tokens (first 1024 image tokens ~ N(0.5, 1)), Zipf(1.1)
    top-8 routing over 128 experts, 40% of the routed slots looked up; search (raw keys,
    dot, the reference's default prefill strategy) + weighted combine of the hits."""
    from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine, _alut

    c = C3
    g = torch.Generator(device=device).manual_seed(3003)
    raw = torch.randn(c["experts"], 2, c["k"], c["l"], generator=g, device=device)
    values = torch.randn(c["experts"], 2, c["k"], c["h"], generator=g, device=device, dtype=torch.bfloat16).mul_(0.05)
    pca = {m: {"proj": orthonormal_basis(c["h"], c["l"], g, device), "bias": torch.zeros(c["l"], device=device)}
           for m in ("vision", "text")}
    mgr = HybridStorageManager.from_tables(0, raw, values, pca)
    q = c["tokens"]
    x = torch.randn(q, c["h"], generator=g, device=device)
    x[:c["vision_tokens"]] += 0.5
    x = x.to(torch.bfloat16)
    vis = torch.arange(q, device=device) < c["vision_tokens"]
    prior = torch.arange(1, c["experts"] + 1, dtype=torch.float32, device=device) ** (-c["zipf"])
    gumbel = -torch.log(-torch.log(torch.rand(q, c["experts"], generator=g, device=device)))
    w, sel = torch.topk(torch.softmax(prior.log() + gumbel, -1), c["top_k"], dim=-1)
    reuse = torch.rand(q, c["top_k"], generator=g, device=device) < c["lookup_frac"]
    comp = ~reuse
    eng = VectorSearchEngine(mgr)
    out = torch.empty(q, c["h"], dtype=torch.bfloat16, device=device)

    def step():
        out.zero_()
        eng.lookup_combine(x, sel, vis, reuse, w, compute_mask=comp, out=out, variant="prefill_dot")

    lib = _alut.load()
    total_ms, _ = timed_steps(step, args.wl_steps, args.warmup, device, flush)
    ev = with_scan_events(lib)
    _, scan_ms = timed_steps(step, 10, 1, device, flush, events=ev)
    lib.alut_set_profile_events(None, None)
    pairs = int(reuse.sum())
    tables = len(set((sel[reuse] * 2 + (~vis).long()[:, None].expand_as(sel)[reuse]).tolist()))
    flops = pairs * c["k"] * c["l"] * 2
    key_bytes = tables * c["k"] * c["l"] * 2  # bf16 operand form of every routed table, once
    achieved = flops / (scan_ms / 1e3) / 1e12
    return {
        "config": "BASELINE config 3: qwen3-vl prefill layer, 4096 tokens, 128 experts, Zipf(1.1) top-8, "
                  "K=1024, L=64, 40% looked up (prefill_dot)",
        "value": round(pairs * args.wl_steps / (total_ms / 1e3), 1), "unit": "lookups/s",
        "ms_per_step": round(total_ms / args.wl_steps, 4), "lookups_per_step": pairs, "steps": args.wl_steps,
        "l2": "flushed between steps (256 MB write outside the timed span)",
        "roofline": {"kernel": "k_search_tc (tcgen05 centroid scan)", "bound": "tensor",
                     "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / peaks["bf16_tflops"], 4), "flops_per_launch": flops,
                     "launch_us": round(scan_ms * 1e3, 2),
                     "key_bytes_per_launch": key_bytes,
                     "hbm_frac": round(key_bytes / (scan_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)},
    }


def c5_workload(args, rank, world, device, flush, peaks):
    """The large single table (K=65536, L=128 fp32 keys, 65536 x 4096 bf16 rows) sharded by
    centroid range over the ranks; 32768 tokens (hidden 4096, bf16) looked up per step:
    local tensor-core scan, NCCL all-gather of packed candidates, merge, owner gather and
    reduce-scatter of the rows. Strong scaling: the same tokens and table at every N."""
    from table_moe.cache_engine.sharded import ShardedCentroidTable, shard_range

    c = C5
    k0, k1 = shard_range(c["k"], world, rank)
    g = torch.Generator(device=device).manual_seed(5005)  # identical on every rank
    keys = torch.randn(1, 2, c["k"], c["l"], generator=g, device=device)[:, :, k0:k1].contiguous()
    pca = {m: {"proj": orthonormal_basis(c["h"], c["l"], g, device), "bias": torch.zeros(c["l"], device=device)}
           for m in ("vision", "text")}
    x = torch.randn(c["tokens"], c["h"], generator=g, device=device).to(torch.bfloat16)
    vis = torch.zeros(c["tokens"], dtype=torch.bool, device=device)
    gv = torch.Generator(device=device).manual_seed(6006 + rank)
    values = torch.randn(1, 2, k1 - k0, c["h"], generator=gv, device=device, dtype=torch.bfloat16).mul_(0.05)
    table = ShardedCentroidTable(keys, values, pca, c["k"])

    def step():
        table.lookup(x, vis)

    barrier(world)
    total_ms, _ = timed_steps(step, args.wl_steps, args.warmup, device, flush)
    total_ms = max_over_ranks(total_ms, world, device)
    flops = c["tokens"] * c["k"] * c["l"] * 2
    achieved = flops / (total_ms / args.wl_steps / 1e3) / 1e12
    return {
        "config": "BASELINE config 5: one table K=65536, L=128 fp32, 65536x4096 bf16 rows, 32768 tokens "
                  "(hidden 4096), centroid-range shards over the ranks",
        "value": round(c["tokens"] * args.wl_steps / (total_ms / 1e3), 1), "unit": "lookups/s",
        "ms_per_step": round(total_ms / args.wl_steps, 4), "steps": args.wl_steps, "scaling": "strong",
        "shards": world, "l2": "flushed between steps (256 MB write outside the timed span)",
        "whole_step_tensor": {"achieved": round(achieved, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                              "frac": round(achieved / peaks["bf16_tflops"], 4),
                              "flops": "tokens x K x L x 2 (scan only) over the whole step time"},
    }


# ---- CPU arms: the oracle (test infrastructure) timed as the baseline -----------------

def cpu_sample(managers, inputs):
    """Host copies of the sampled layers' tables and inputs for the oracle."""
    from oracle import oracle as orc

    sample = []
    for m, inp in zip(managers, inputs):
        keys = m.keys_buffer.float().cpu().numpy()
        vals = m.values_buffer.cpu().view(torch.int16).numpy().view(np.uint16)
        proj = np.stack([m.pca["vision"]["proj"].cpu().numpy(), m.pca["text"]["proj"].cpu().numpy()])
        bias = np.stack([m.pca["vision"]["bias"].cpu().numpy(), m.pca["text"]["bias"].cpu().numpy()])
        d = {k: v.numpy() for k, v in inp.items() if k != "x"}
        d["x"] = inp["x"].float().numpy()
        sample.append((keys, vals, proj, bias, d))
    return orc, sample


def cpu_step(orc, sample):
    """One oracle pass over the sampled layers: project, search (normalised keys, >= 0),
    combine (renormalised to one). Returns the lookups processed."""
    n = 0
    for keys, vals, proj, bias, inp in sample:
        q = orc.project(inp["x"], inp["is_vision"], proj, bias)
        hit, idx, _, _ = orc.search(q, keys, inp["sel"], inp["is_vision"], inp["reuse"], 0.0, 0.0, cmp_ge=True,
                                    with_gap=False)
        orc.combine(vals, inp["sel"], inp["is_vision"], hit, idx, inp["weights"], compute=inp["compute"], renorm=1)
        n += int(inp["reuse"].sum())
    return n


def time_cpu(orc, sample, *, seconds=None, steps=None, warmup=1):
    cores = len(os.sched_getaffinity(0))
    orc.set_threads(cores)
    for _ in range(warmup):
        cpu_step(orc, sample)
    t0 = time.perf_counter()
    n = done = 0
    while True:
        n += cpu_step(orc, sample)
        done += 1
        dt = time.perf_counter() - t0
        if (seconds is not None and dt >= seconds) or (steps is not None and done >= steps):
            break
    return n / dt, cores, done, dt


def config_dict(world):
    return {"workload": "qwen3-vl-30b-a3b decode step (BASELINE config 2)", "layers": CFG["layers"],
            "experts": CFG["experts"], "centroids": CFG["k"], "pca_rank": CFG["l"], "hidden": CFG["h"],
            "tokens_per_gpu": CFG["tokens"], "top_k": CFG["top_k"], "lookup_frac": CFG["lookup_frac"],
            "key_dtype": "float32", "value_dtype": "bfloat16", "search": "normalised keys, hit = max >= 0",
            "l2": "inputs larger than L2 (about 0.57 GB of keys and rows touched per step, 55 GB of tables)",
            "parallelism": f"replicas x{world}"}


def run_reference(args, rank, world, device):
    """CPU oracle arm: rank 0 only, all host threads, bounded sample per step."""
    if rank != 0:
        return
    managers = [build_layer(li, device, rank) for li in range(CPU_LAYERS)]
    inputs = [layer_inputs(li, rank) for li in range(CPU_LAYERS)]
    torch.cuda.synchronize()
    orc, sample = cpu_sample(managers, inputs)
    v, cores, steps, dt = time_cpu(orc, sample, steps=args.steps, warmup=args.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 1), "unit": "lookups/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random tables and routing)", "config": config_dict(world),
            "cpu_baseline": {"value": round(v, 1), "unit": "lookups/s", "cores": cores, "kind": "port",
                             "sample": f"each step = layers 0-{CPU_LAYERS - 1} of the decode step through the CPU "
                                       "oracle (C restatement of the reference torch path)"},
            "e2e": {"value": round(v, 1), "unit": "lookups/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["alut", "reference"], default="alut")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--wl-steps", type=int, default=20, help="timed steps of each secondary workload")
    ap.add_argument("--no-workloads", action="store_true", help="skip the config 3 / config 5 measurements")
    ap.add_argument("--only", choices=["c3", "c5"], default=None,
                    help="run only that secondary workload and print its JSON (profiling captures)")
    ap.add_argument("--layers", type=int, default=CFG["layers"],
                    help="fewer layers for profiling captures only (the benchmark is 48)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    CFG["layers"] = args.layers
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world, device)
        elif args.only:
            peaks, _ = measured_peaks()
            flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
            res = (c3_workload(args, device, flush, peaks) if args.only == "c3"
                   else c5_workload(args, rank, world, device, flush, peaks))
            if rank == 0:
                print(json.dumps({"workload": args.only, **res}), flush=True)
        else:
            run_alut(args, rank, world, local, device)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def run_alut(args, rank, world, local, device):
    from table_moe.cache_engine import VectorSearchEngine
    from table_moe.cache_engine.step_graph import LookupStepGraph

    managers = [build_layer(li, device, rank) for li in range(CFG["layers"])]
    engines = [VectorSearchEngine(m) for m in managers]
    inputs = [layer_inputs(li, rank) for li in range(CFG["layers"])]
    torch.cuda.synchronize()
    per_layer = [algorithmic_bytes(inp) for inp in inputs]
    scan_bytes = [p[0] for p in per_layer]
    path_bytes = sum(p[1] for p in per_layer)
    lookups_per_step = sum(p[2] for p in per_layer)

    # Device-resident step (timed), and a twin graph whose scan launches are bracketed by
    # event nodes (replayed after the timed region to time the scan kernels; event nodes
    # break the programmatic overlap between kernels, so they stay out of the timed graph).
    step = LookupStepGraph(engines, CFG["tokens"], CFG["top_k"], variant="decode", renorm="to_one")
    prof = LookupStepGraph(engines, CFG["tokens"], CFG["top_k"], variant="decode", renorm="to_one")
    for g in (step, prof):
        for b, inp in zip(g.layers, inputs):
            for name, t in inp.items():
                getattr(b, name).copy_(t)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in engines]
    for a, b in ev:  # the CUDA events must exist before capture
        a.record()
        b.record()
    torch.cuda.synchronize()
    step.capture()
    prof.capture(profile_events=ev)
    for _ in range(args.warmup):
        step.replay()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            step.replay()
        stop.record()
        torch.cuda.synchronize()
        barrier(world)
    dev_ms = max_over_ranks(start.elapsed_time(stop), world, device)
    ms_per_step = dev_ms / args.steps
    total_lookups = sum_over_ranks(lookups_per_step, world, device) * args.steps
    value = total_lookups / (dev_ms / 1e3)
    scan_ms = []
    for _ in range(PROFILE_STEPS):
        prof.replay()
        torch.cuda.synchronize()
        scan_ms += prof.scan_times_ms()

    # End to end through the public API: H2D inputs + lookups + D2H outputs per step.
    e2e = LookupStepGraph(engines, CFG["tokens"], CFG["top_k"], variant="decode", renorm="to_one")
    for hb, inp in zip(e2e.host_layers, inputs):
        for name, t in inp.items():
            getattr(hb, name).copy_(t)
    e2e.capture(with_copies=True)
    for _ in range(args.warmup):
        e2e.replay()
    torch.cuda.synchronize()
    barrier(world)
    s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(args.steps):
        e2e.replay()
    t2.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(s2.elapsed_time(t2), world, device)

    peaks, peak_src = measured_peaks()
    roofline = None
    if scan_ms:
        avg_ms = sum(scan_ms) / len(scan_ms)
        bpl = sum(scan_bytes) / len(scan_bytes)
        achieved = bpl / (avg_ms / 1e3) / 1e9
        roofline = {"kernel": "k_project + k_search_decode (projection + centroid scan)", "bound": "hbm", "achieved": round(achieved, 1),
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                    "traffic": NCU_TRAFFIC_PER_LAYER, "peak_source": peak_src, "bytes_per_launch": int(bpl),
                    "launch_us": round(avg_ms * 1e3, 2), "launches_timed": len(scan_ms),
                    "timed_span": "projection + centroid scan (the scan is launched as a programmatic "
                                  "dependent of the projection and streams keys while it runs)"}
    path_gbs = path_bytes / (ms_per_step / 1e3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        orc, sample = cpu_sample(managers[:CPU_LAYERS], inputs[:CPU_LAYERS])
        v, cores, n, secs = time_cpu(orc, sample, seconds=args.cpu_seconds)
        cpu = {"value": round(v, 1), "unit": "lookups/s", "cores": cores, "kind": "port",
               "sample": f"CPU oracle (C restatement of the reference torch path) over layers 0-{CPU_LAYERS - 1} "
                         f"of the step, {n} passes in {secs:.1f} s"}
    workloads = None
    if not args.no_workloads:
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        workloads = {}
        if world == 1:
            workloads["c3_prefill_layer"] = c3_workload(args, device, flush, peaks)
        workloads["c5_sharded_table"] = c5_workload(args, rank, world, device, flush, peaks)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "lookups/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random tables and routing)", "config": config_dict(world),
            "lookups_per_step": total_lookups // args.steps,
            "e2e": {"value": round(total_lookups / (e2e_ms / 1e3), 1), "unit": "lookups/s",
                    "h2d_bytes_per_step": e2e.h2d_bytes, "d2h_bytes_per_step": e2e.d2h_bytes,
                    "ms_per_step": round(e2e_ms / args.steps, 5)},
            "gpu_launches": KERNELS_PER_LAYER * CFG["layers"] * args.steps,
            "roofline": roofline,
            "path_roofline": {"bytes_per_step": path_bytes, "achieved_gbs": round(path_gbs, 1),
                              "frac": round(path_gbs / peaks["hbm_gbs"], 4), "peak_source": peak_src},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "workloads": workloads,
        }
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
