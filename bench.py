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
workloads: the other BASELINE configs, each timed with L2 flushed between steps and each
       with a roofline: config 1 (single table), config 3 (prefill layer), config 4
       (DeepSeek-VL2 prefill + decode) and config 5 (the sharded large table, at every N).
parity: before the JSON line is printed, the checker leg compares a sample of what was
       timed (layers of the replayed decode graph, tokens of each workload) with the CPU
       oracle (test infrastructure) and reports the mismatches.

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
CSRC = ROOT / "tablemoe-sc26_b200" / "csrc"
TRAFFIC_FILE = ROOT / "profiles" / "decode_layer_dram_traffic_qwen3vl_c2.txt"


def source_digest():
    """sha256 over the kernel sources and the header: names the build a capture was made of."""
    import hashlib

    h = hashlib.sha256()
    for f in sorted(CSRC.glob("*.cu*")) + [ROOT / "include" / "alut.h"]:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    return h.hexdigest()


def ncu_traffic():
    """DRAM bytes (read + write) of one decode layer's three kernels from the committed ncu
    summary, when it was captured from these exact sources; else None."""
    if not TRAFFIC_FILE.exists():
        return None, "no capture committed"
    kv = {}
    for line in TRAFFIC_FILE.read_text().splitlines():
        if ":" in line:
            k, v = line.split(":", 1)
            kv[k.strip()] = v.strip()
    if kv.get("source_sha256") != source_digest():
        return None, "committed capture is of other kernel sources"
    return int(kv["dram_bytes_per_layer"]), "ncu capture of this build (" + TRAFFIC_FILE.name + ")"


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


# ---- secondary workloads: the other BASELINE configs --------------------------------------
# Reported under "workloads" in the same JSON line; the headline value stays the decode step.

C1 = dict(tokens=256, k=256, l=64, h=2048)
C3 = dict(tokens=4096, vision_tokens=1024, experts=128, k=1024, l=64, h=2048, top_k=8, lookup_frac=0.4, zipf=1.1)
C4 = dict(layers=30, experts=72, top_k=6, k=2048, l=96, h=2560, prefill_tokens=2048, decode_steps=64,
          decode_batch=8, lookup_frac=0.4)
C5 = dict(tokens=32768, k=65536, l=128, h=4096)
L2_FLUSH_BYTES = 256 << 20  # written between timed steps (L2 is 126 MB)
SAMPLE_TOKENS = 512         # tokens of a large batch the checker leg compares with the oracle


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


def hbm_roofline(kernel, nbytes, seconds, peaks, **extra):
    gbs = nbytes / seconds / 1e9
    return {"kernel": kernel, "bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(gbs / peaks["hbm_gbs"], 4), "bytes_per_launch": int(nbytes),
            "launch_us": round(seconds * 1e6, 3), **extra}


def tensor_roofline(kernel, flops, seconds, peaks, **extra):
    tf = flops / seconds / 1e12
    return {"kernel": kernel, "bound": "tensor", "achieved": round(tf, 2), "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_tflops"], 4), "flops_per_launch": int(flops),
            "launch_us": round(seconds * 1e6, 3), **extra}


# ---- checker leg (test infrastructure: the CPU oracle checks a sample of what was timed) ----

class Checker:
    """Counts slots and elements of the timed outputs that break the parity rules of
    oracle/parity_rules.py (indices exact except near ties, rows exact, combine within 1e-2)."""

    def __init__(self):
        self.results = {}

    def _add(self, name, checked, bad, exempt=0):
        r = self.results.setdefault(name, {"checked": 0, "mismatches": 0, "exempt": 0})
        r["checked"] += int(checked)
        r["mismatches"] += int(bad)
        r["exempt"] += int(exempt)

    def lookup(self, name, *, x, vis, proj, bias, keys, sel, reuse, weights, compute, values_bits, hit, idx, out,
               renorm, cmp_ge, thr, normalize=False, accumulate_base=None):
        """Oracle project + search + combine of one batch (numpy inputs) against the GPU's
        hit / idx / out for the same batch."""
        import oracle.oracle as orc
        import oracle.parity_rules as rules

        q = orc.project(x, vis, proj, bias, normalize=normalize)
        rh, ri, _, _ = orc.search(q, keys, sel, vis, reuse, thr, thr, cmp_ge=cmp_ge, with_gap=False)
        bad, exempt = rules.search_mismatches(hit, idx, rh, ri, q, keys, sel, vis, (thr, thr), "float32")
        self._add(name, sel.size, len(bad), exempt)
        ref = orc.combine(values_bits, sel, vis, hit, idx, weights, compute=compute, renorm=renorm,
                          out=accumulate_base)
        n, _ = rules.combined_mismatches(out, ref)
        self._add(name, 0, n)

    def rows(self, name, got, ref):
        """got / ref: bit patterns of the rows (uint16)."""
        bad = int(np.count_nonzero(np.any(got != ref, axis=1)))
        self._add(name, got.shape[0], bad)

    def search_only(self, name, *, q, keys, sel, vis, hit, idx, thr, cmp_ge):
        import oracle.oracle as orc
        import oracle.parity_rules as rules

        rh, ri, _, _ = orc.search(q, keys, sel, vis, None, thr, thr, cmp_ge=cmp_ge, with_gap=False)
        bad, exempt = rules.search_mismatches(hit, idx, rh, ri, q, keys, sel, vis, (thr, thr), "float32")
        self._add(name, sel.size, len(bad), exempt)

    def summary(self):
        tot = {"checked": 0, "mismatches": 0, "exempt": 0}
        for r in self.results.values():
            for k in tot:
                tot[k] += r[k]
        return {**tot, "per_workload": self.results,
                "rule": "indices exact except near ties (1e-5 rel), rows bit-exact, combine within 1e-2 rel"}


def bits16(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def basis_np(mgr):
    proj = np.stack([mgr.pca["vision"]["proj"].cpu().numpy(), mgr.pca["text"]["proj"].cpu().numpy()])
    bias = np.stack([mgr.pca["vision"]["bias"].cpu().numpy(), mgr.pca["text"]["bias"].cpu().numpy()])
    return proj, bias


def check_engine_lookup(checker, name, mgr, x, sel, vis, reuse, w, comp, hit, idx, out, *, variant, renorm,
                        rows=None, keys=None):
    """Checker of one lookup_combine batch (device tensors), optionally on a row subset."""
    rows = slice(None) if rows is None else rows
    cmp_ge, thr, keyset = {"decode": (True, 0.0, "norm"), "prefill_dot": (False, 0.0, "raw"),
                           "decode_dot": (False, 0.0, "raw")}[variant]
    if keys is None:
        keys = (mgr.keys_buffer if keyset == "norm" else mgr.raw_keys_buffer).float().cpu().numpy()
    proj, bias = basis_np(mgr)
    rn = {"none": 0, "to_one": 1, "to_rowsum": 2}[renorm]
    checker.lookup(name, x=x[rows].float().cpu().numpy(), vis=vis[rows].cpu().numpy(), proj=proj, bias=bias,
                   keys=keys, sel=sel[rows].cpu().numpy(), reuse=reuse[rows].cpu().numpy(),
                   weights=w[rows].float().cpu().numpy(), compute=None if comp is None else comp[rows].cpu().numpy(),
                   values_bits=bits16(mgr.values_buffer), hit=hit[rows].cpu().numpy(), idx=idx[rows].cpu().numpy(),
                   out=out[rows].float().cpu().numpy(), renorm=rn, cmp_ge=cmp_ge, thr=thr)
    return keys


def c1_workload(args, device, flush, peaks, checker):
    """One table (K=256, L=64 fp32, 256 x 2048 bf16 rows), 256 tokens of hidden 2048, every
    token looked up (dot rule), rows scaled by U(0,1) weights and accumulated into the
    output (no renormalisation). The call is replayed as a one-layer CUDA graph."""
    from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine
    from table_moe.cache_engine.step_graph import LookupStepGraph

    c = C1
    g = torch.Generator(device=device).manual_seed(1001)
    x = torch.randn(c["tokens"], c["h"], generator=g, device=device).to(torch.bfloat16)
    proj = orthonormal_basis(c["h"], c["l"], g, device)
    keys = torch.randn(1, 2, c["k"], c["l"], generator=g, device=device)
    values = torch.randn(1, 2, c["k"], c["h"], generator=g, device=device, dtype=torch.bfloat16).mul_(0.05)
    w = torch.rand(c["tokens"], 1, generator=g, device=device)
    pca = {m: {"proj": proj, "bias": torch.zeros(c["l"], device=device)} for m in ("vision", "text")}
    mgr = HybridStorageManager.from_tables(0, keys, values, pca, keys=keys)
    gr = LookupStepGraph([VectorSearchEngine(mgr)], c["tokens"], 1, variant="prefill_dot", renorm="none",
                         keep_hits=True)
    b = gr.layers[0]
    b.x.copy_(x)
    b.sel.zero_()
    b.is_vision.zero_()
    b.reuse.fill_(True)
    b.weights.copy_(w)
    b.compute.zero_()
    gr.capture()
    total_ms, _ = timed_steps(gr.replay, args.wl_steps, args.warmup, device, flush)
    b.out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    hit, idx, out = gr.hits[0], gr.idx[0], b.out
    check_engine_lookup(checker, "c1", mgr, b.x, b.sel, b.is_vision, b.reuse, b.weights, None, hit, idx, out,
                        variant="prefill_dot", renorm="none")
    hits = int(hit.sum())
    nbytes = x.numel() * 2 + c["h"] * c["l"] * 4 + c["k"] * c["l"] * 4 + hits * c["h"] * 2 + 2 * out.numel() * 2
    t = total_ms / args.wl_steps / 1e3
    return {
        "config": "BASELINE config 1: one table K=256, L=64 fp32, 256x2048 bf16 rows, 256 tokens (hidden 2048), "
                  "dot rule, U(0,1) weights, rows accumulated into the output",
        "value": round(c["tokens"] / t, 1), "unit": "lookups/s", "ms_per_step": round(t * 1e3, 4),
        "steps": args.wl_steps, "l2": "flushed between steps (256 MB write outside the timed span)",
        "roofline": hbm_roofline("one alut_lookup_combine call (plan, projection, scan, combine; graph replay)",
                                 nbytes, t, peaks,
                                 bytes_note="x + text basis + table keys + hit rows + output read/write"),
    }


def c3_workload(args, device, flush, peaks, checker):
    """One Qwen3-VL prefill layer: 4096 tokens (first 1024 image tokens ~ N(0.5, 1)), Zipf(1.1)
    top-8 routing over 128 experts, 40% of the routed slots looked up; search (raw keys,
    dot, the reference's default prefill strategy) + weighted combine of the hits, replayed
    as a one-layer CUDA graph."""
    from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine
    from table_moe.cache_engine.step_graph import LookupStepGraph

    c = C3
    g = torch.Generator(device=device).manual_seed(3003)
    raw = torch.randn(c["experts"], 2, c["k"], c["l"], generator=g, device=device)
    values = torch.randn(c["experts"], 2, c["k"], c["h"], generator=g, device=device, dtype=torch.bfloat16).mul_(0.05)
    pca = {m: {"proj": orthonormal_basis(c["h"], c["l"], g, device), "bias": torch.zeros(c["l"], device=device)}
           for m in ("vision", "text")}
    mgr = HybridStorageManager.from_tables(0, raw, values, pca, keys=raw)
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
    graphs = []
    for prof in (False, True):  # the timed graph, and a twin whose scan is bracketed by events
        gr = LookupStepGraph([eng], q, c["top_k"], variant="prefill_dot", renorm="to_one", keep_hits=True)
        b = gr.layers[0]
        for name, t in (("x", x), ("sel", sel), ("is_vision", vis), ("reuse", reuse), ("weights", w),
                        ("compute", comp)):
            getattr(b, name).copy_(t)
        ev = None
        if prof:
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))]
            for e in ev[0]:
                e.record()
            torch.cuda.synchronize()
        gr.capture(profile_events=ev)
        graphs.append(gr)
    total_ms, _ = timed_steps(graphs[0].replay, args.wl_steps, args.warmup, device, flush)
    scan = []
    for _ in range(10):
        flush.fill_(1)
        graphs[1].replay()
        torch.cuda.synchronize()
        scan += graphs[1].scan_times_ms()
    scan_ms = sum(scan) / len(scan)
    gr = graphs[0]
    b = gr.layers[0]
    b.out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    rows = torch.randperm(q, generator=torch.Generator().manual_seed(3))[:SAMPLE_TOKENS].sort().values
    check_engine_lookup(checker, "c3", mgr, b.x, b.sel, b.is_vision, b.reuse, b.weights, b.compute, gr.hits[0],
                        gr.idx[0], b.out, variant="prefill_dot", renorm="to_one", rows=rows.to(device))
    pairs = int(reuse.sum())
    tables = len(set((sel[reuse] * 2 + (~vis).long()[:, None].expand_as(sel)[reuse]).tolist()))
    flops = pairs * c["k"] * c["l"] * 2
    key_bytes = tables * c["k"] * c["l"] * 2  # bf16 operand form of every routed table, once
    return {
        "config": "BASELINE config 3: qwen3-vl prefill layer, 4096 tokens, 128 experts, Zipf(1.1) top-8, "
                  "K=1024, L=64, 40% looked up (prefill_dot)",
        "value": round(pairs * args.wl_steps / (total_ms / 1e3), 1), "unit": "lookups/s",
        "ms_per_step": round(total_ms / args.wl_steps, 4), "lookups_per_step": pairs, "steps": args.wl_steps,
        "l2": "flushed between steps (256 MB write outside the timed span)",
        "roofline": tensor_roofline("k_search_tc (tcgen05 centroid scan; event nodes around it in a twin graph)",
                                    flops, scan_ms / 1e3, peaks,
                                    key_bytes_per_launch=key_bytes,
                                    hbm_frac=round(key_bytes / (scan_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)),
    }


def c4_build(device):
    """30 DeepSeek-VL2-shaped layers (72 routed experts, K=2048, L=96 fp32 keys, 2560-wide
    bf16 rows) and the routing of a 2048-token prefill and of a batch of 8 decode tokens."""
    from table_moe.cache_engine import HybridStorageManager

    c = C4
    mgrs, pre, dec = [], [], []
    for li in range(c["layers"]):
        g = torch.Generator(device=device).manual_seed(40000 + li)
        raw = torch.randn(c["experts"], 2, c["k"], c["l"], generator=g, device=device)
        values = torch.randn(c["experts"], 2, c["k"], c["h"], generator=g, device=device,
                             dtype=torch.bfloat16).mul_(0.05)
        pca = {m: {"proj": orthonormal_basis(c["h"], c["l"], g, device), "bias": torch.zeros(c["l"], device=device)}
               for m in ("vision", "text")}
        mgrs.append(HybridStorageManager.from_tables(li, raw, values, pca, keys=raw, enable_online=False))
        for n, dst in ((c["prefill_tokens"], pre), (c["decode_batch"], dec)):
            x = torch.randn(n, c["h"], generator=g, device=device).to(torch.bfloat16)
            w, sel = torch.topk(torch.softmax(torch.randn(n, c["experts"], generator=g, device=device), -1),
                                c["top_k"], dim=-1)
            reuse = torch.rand(n, c["top_k"], generator=g, device=device) < c["lookup_frac"]
            dst.append(dict(x=x, sel=sel, is_vision=torch.zeros(n, dtype=torch.bool, device=device), reuse=reuse,
                            weights=w.float(), compute=~reuse))
    return mgrs, pre, dec


def layer_bytes(inp, k, l, h, with_out=True):
    """Algorithmic bytes of one lookup batch: distinct routed tables' keys, the basis of the
    modalities present, x, the looked-up rows and the output read + write."""
    r = inp["reuse"]
    m = (~inp["is_vision"]).long()[:, None].expand_as(inp["sel"])
    tables = int(torch.unique((inp["sel"] * 2 + m)[r]).numel())
    mods = int(inp["is_vision"].any()) + int((~inp["is_vision"]).any())
    n = int(r.sum())
    return tables * k * l * 4 + mods * h * l * 4 + inp["x"].numel() * 2 + n * h * 2 + \
        (2 * inp["x"].numel() * 2 if with_out else 0), n


def c4_workload(args, device, flush, peaks, checker):
    """DeepSeek-VL2: a 2048-token prefill through 30 layers, then 64 decode steps of batch 8
    through the same 30 layers (dot rule, renormalised to the row sum of the routing
    weights, deepseek_layers.py:707-729). One step = the prefill + the 64 decode steps."""
    from table_moe.cache_engine import VectorSearchEngine
    from table_moe.cache_engine.step_graph import LookupStepGraph

    c = C4
    mgrs, pre, dec = c4_build(device)
    engines = [VectorSearchEngine(m) for m in mgrs]
    graphs = {}
    for name, q, inputs, variant in (("prefill", c["prefill_tokens"], pre, "prefill_dot"),
                                     ("decode", c["decode_batch"], dec, "decode_dot")):
        gr = LookupStepGraph(engines, q, c["top_k"], variant=variant, renorm="to_rowsum", keep_hits=True)
        for b, inp in zip(gr.layers, inputs):
            for k2, t in inp.items():
                getattr(b, k2).copy_(t)
        gr.capture()
        graphs[name] = gr

    def prefill():
        graphs["prefill"].replay()

    def decode():
        for _ in range(c["decode_steps"]):
            graphs["decode"].replay()

    def step():
        prefill()
        decode()

    total_ms, _ = timed_steps(step, args.wl_steps, args.warmup, device, flush)
    pre_ms, _ = timed_steps(prefill, args.wl_steps, 2, device, flush)
    dec_ms, _ = timed_steps(decode, args.wl_steps, 2, device, flush)
    # Checker: one fresh replay of each graph, layers 0 and 29 (prefill on a token sample).
    for gr in graphs.values():
        for b in gr.layers:
            b.out.zero_()
        gr.replay()
    torch.cuda.synchronize()
    rows = torch.randperm(c["prefill_tokens"], generator=torch.Generator().manual_seed(4))[:SAMPLE_TOKENS]
    rows = rows.sort().values.to(device)
    for li in (0, c["layers"] - 1):
        for name, inputs, rr in (("prefill", pre, rows), ("decode", dec, None)):
            gr, inp = graphs[name], inputs[li]
            check_engine_lookup(checker, f"c4_{name}", mgrs[li], inp["x"], inp["sel"], inp["is_vision"],
                                inp["reuse"], inp["weights"], inp["compute"], gr.hits[li], gr.idx[li],
                                gr.layers[li].out, variant="prefill_dot" if name == "prefill" else "decode_dot",
                                renorm="to_rowsum", rows=rr)
    pre_lookups = sum(int(i["reuse"].sum()) for i in pre)
    dec_lookups = sum(int(i["reuse"].sum()) for i in dec) * c["decode_steps"]
    dec_bytes = sum(layer_bytes(i, c["k"], c["l"], c["h"])[0] for i in dec) * c["decode_steps"]
    pre_flops = pre_lookups * c["k"] * c["l"] * 2
    t_step, t_pre, t_dec = (v / args.wl_steps / 1e3 for v in (total_ms, pre_ms, dec_ms))
    return {
        "config": "BASELINE config 4: deepseek-vl2, 30 layers x 72 routed experts top-6, K=2048, L=96 fp32, "
                  "2560-wide bf16 rows; 2048-token prefill then 64 decode steps at batch 8; 40% looked up; "
                  "dot rule, renormalised to the routing row sum",
        "value": round((pre_lookups + dec_lookups) / t_step, 1), "unit": "lookups/s",
        "ms_per_step": round(t_step * 1e3, 4), "lookups_per_step": pre_lookups + dec_lookups,
        "steps": args.wl_steps, "l2": "flushed between steps (256 MB write outside the timed span); a decode "
        "step touches about 0.4 GB of tables",
        "prefill": {"ms": round(t_pre * 1e3, 4), "lookups": pre_lookups, "value": round(pre_lookups / t_pre, 1),
                    "whole_prefill_tensor": tensor_roofline("30-layer prefill (projection, plan, tcgen05 scan, "
                                                            "combine) over its whole time", pre_flops, t_pre, peaks)},
        "decode": {"ms_per_decode_step": round(t_dec * 1e3 / c["decode_steps"], 4), "lookups": dec_lookups,
                   "value": round(dec_lookups / t_dec, 1),
                   "roofline": hbm_roofline("30-layer decode step (project -> scan -> combine per layer, PDL)",
                                            dec_bytes / c["decode_steps"], t_dec / c["decode_steps"], peaks)},
    }


def c5_workload(args, rank, world, device, flush, peaks, checker):
    """The large single table (K=65536, L=128 fp32 keys, 65536 x 4096 bf16 rows): value rows
    sharded by centroid range over the ranks, the 32 MiB key table replicated; 32768 tokens
    (hidden 4096, bf16) looked up per step: each rank projects and scans (tensor cores) its own
    Q/W tokens over the whole table, the packed winners are all-gathered (8 bytes a token) and
    merged, and each rank reads its tokens' rows from the owners (peer loads); the step is one
    CUDA graph (NCCL calls included). Strong scaling: the same tokens and table at every N."""
    from table_moe.cache_engine.sharded import ShardedCentroidTable, shard_range

    c = C5
    k0, k1 = shard_range(c["k"], world, rank)
    g = torch.Generator(device=device).manual_seed(5005)  # identical on every rank
    keys_full = torch.randn(1, 2, c["k"], c["l"], generator=g, device=device)
    proj = [orthonormal_basis(c["h"], c["l"], g, device) for _ in range(2)]
    pca = {m: {"proj": proj[i], "bias": torch.zeros(c["l"], device=device)} for i, m in enumerate(("vision", "text"))}
    x = torch.randn(c["tokens"], c["h"], generator=g, device=device).to(torch.bfloat16)
    vis = torch.zeros(c["tokens"], dtype=torch.bool, device=device)
    gv = torch.Generator(device=device).manual_seed(6006 + rank)
    values = torch.randn(1, 2, k1 - k0, c["h"], generator=gv, device=device, dtype=torch.bfloat16).mul_(0.05)
    table = ShardedCentroidTable(keys_full, values, pca, c["k"], replicate_keys=True)
    graph, (hit, idx, rows) = table.capture(x, vis)  # the whole lookup, NCCL calls included

    barrier(world)
    total_ms, _ = timed_steps(graph.replay, args.wl_steps, args.warmup, device, flush)
    total_ms = max_over_ranks(total_ms, world, device)
    # Checker: the winners of a token sample against the oracle over the full table, and the
    # rows of this rank's sampled tokens against the owning shard's (regenerated) values.
    graph.replay()
    torch.cuda.synchronize()
    n = c["tokens"] // world
    lo = rank * n
    sample = torch.randperm(c["tokens"], generator=torch.Generator().manual_seed(5))[:256].sort().values
    if rank == 0:
        import oracle.oracle as orc

        xs = x[sample].float().cpu().numpy()
        pr = np.stack([p.cpu().numpy() for p in proj])
        q = orc.project(xs, np.zeros(len(sample), bool), pr, np.zeros((2, c["l"]), np.float32))
        checker.search_only("c5", q=q, keys=keys_full.cpu().numpy(), sel=np.zeros((len(sample), 1), np.int64),
                            vis=np.zeros(len(sample), bool), hit=hit[sample].cpu().numpy()[:, None],
                            idx=idx[sample].cpu().numpy()[:, None], thr=0.0, cmp_ge=False)
    mine = sample[(sample >= lo) & (sample < lo + n)]
    ref = torch.zeros(len(mine), c["h"], dtype=torch.bfloat16, device=device)
    gi = idx[mine.to(device)]
    for r in range(world):
        r0, r1 = shard_range(c["k"], world, r)
        own = hit[mine.to(device)] & (gi >= r0) & (gi < r1)
        if own.any():
            gr = torch.Generator(device=device).manual_seed(6006 + r)
            vr = values if r == rank else torch.randn(1, 2, r1 - r0, c["h"], generator=gr, device=device,
                                                      dtype=torch.bfloat16).mul_(0.05)
            ref[own] = vr[0, 1, gi[own] - r0]
            del vr
    checker.rows("c5", bits16(rows[(mine - lo).to(device)]), bits16(ref))
    del graph
    table.close()
    flops = c["tokens"] * c["k"] * c["l"] * 2
    t = total_ms / args.wl_steps / 1e3
    achieved = flops / t / 1e12
    return {
        "config": "BASELINE config 5: one table K=65536, L=128 fp32 (replicated), 65536x4096 bf16 rows (sharded), 32768 tokens "
                  "(hidden 4096), value rows sharded by centroid range over the ranks",
        "value": round(c["tokens"] / t, 1), "unit": "lookups/s",
        "ms_per_step": round(t * 1e3, 4), "steps": args.wl_steps, "scaling": "strong",
        "shards": world, "l2": "flushed between steps (256 MB write outside the timed span)",
        "whole_step_tensor": {"achieved": round(achieved, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                              "frac_per_gpu": round(achieved / world / peaks["bf16_tflops"], 4),
                              "flops": "tokens x K x L x 2 (scan only) over the whole step time, all GPUs"},
    }


# ---- crossover sweep of the scan and projection choices -------------------------------------

CROSSOVER_CASES = [  # name, tokens, top_k, experts, K, L, H, looked-up fraction, Zipf exponent
    ("c1_single_table", 256, 1, 1, 256, 64, 2048, 1.0, None),
    ("q64", 64, 8, 128, 1024, 64, 2048, 0.4, None),
    ("q128", 128, 8, 128, 1024, 64, 2048, 0.4, None),
    ("q256", 256, 8, 128, 1024, 64, 2048, 0.4, None),
    ("q512", 512, 8, 128, 1024, 64, 2048, 0.4, None),
    ("q1024_zipf", 1024, 8, 128, 1024, 64, 2048, 0.4, 1.1),
    ("c3_prefill", 4096, 8, 128, 1024, 64, 2048, 0.4, 1.1),
    ("c4_prefill_layer", 2048, 6, 72, 2048, 96, 2560, 0.4, None),
    ("one_table_4k", 4096, 1, 1, 4096, 128, 1024, 1.0, None),
]


def crossover(args, device, flush):
    """Median device time of one lookup (graph replay, L2 flushed) per batch shape, with the
    scan the library picks for it. Builds of the library with other thresholds
    (-DALUT_TC_MIN_PAIRS, -DALUT_TC_MIN_SLOTS_PER_TABLE, -DALUT_PT_MIN_TOKENS), selected
    with TABLEMOE_ALUT_LIB, give the other side of each choice."""
    from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine, _alut
    from table_moe.cache_engine.step_graph import LookupStepGraph

    reread = torch.ones(64 << 20, dtype=torch.float32, device=device)
    lib = _alut.load()
    out = {}
    for name, q, s, e, k, l, h, frac, zipf in CROSSOVER_CASES:
        g = torch.Generator(device=device).manual_seed(1)
        raw = torch.randn(e, 2, k, l, generator=g, device=device)
        values = torch.randn(e, 2, k, h, generator=g, device=device, dtype=torch.bfloat16).mul_(0.05)
        pca = {m: {"proj": orthonormal_basis(h, l, g, device), "bias": torch.zeros(l, device=device)}
               for m in ("vision", "text")}
        mgr = HybridStorageManager.from_tables(0, raw, values, pca, keys=raw, enable_online=False)
        logits = torch.randn(q, e, generator=g, device=device)
        if zipf:
            prior = torch.arange(1, e + 1, dtype=torch.float32, device=device) ** (-zipf)
            logits = prior.log() - torch.log(-torch.log(torch.rand(q, e, generator=g, device=device)))
        w, sel = torch.topk(torch.softmax(logits, -1), s, dim=-1)
        reuse = torch.rand(q, s, generator=g, device=device) < frac
        gr = LookupStepGraph([VectorSearchEngine(mgr)], q, s, variant="prefill_dot", renorm="to_one")
        b = gr.layers[0]
        for n2, t in (("x", torch.randn(q, h, generator=g, device=device)), ("sel", sel), ("reuse", reuse),
                      ("weights", w), ("compute", ~reuse)):
            getattr(b, n2).copy_(t)
        gr.capture()
        for _ in range(5):
            gr.replay()
        ts = []
        for _ in range(30):
            flush.fill_(1)
            reread.sum()  # leaves L2 clean: the flush's dirty lines are written back here
            a, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            gr.replay()
            c.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(c) * 1e3)
        kind = lib.alut_scan_kind(mgr.alut_tables(), q, s)
        out[name] = {"us": round(sorted(ts)[len(ts) // 2], 1),
                     "scan": {0: "decode", 1: "cuda-core", 2: "tensor-core"}.get(kind, kind)}
        del gr, mgr, raw, values
        torch.cuda.empty_cache()
    return out


# ---- CPU arms: the oracle (test infrastructure) timed as the baseline -----------------

def cpu_sample(managers, inputs):
    """Host copies of the sampled layers' tables and inputs for the oracle."""
    from oracle import oracle as orc

    sample = []
    for m, inp in zip(managers, inputs):
        keys = m.keys_buffer.float().cpu().numpy()
        vals = bits16(m.values_buffer)
        proj, bias = basis_np(m)
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
    ap.add_argument("--wl-steps", type=int, default=10, help="timed steps of each secondary workload")
    ap.add_argument("--no-workloads", action="store_true", help="skip the config 1/3/4/5 measurements")
    ap.add_argument("--only", choices=["c1", "c3", "c4", "c5", "crossover"], default=None,
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
            checker = Checker()
            if args.only == "crossover":
                print(json.dumps({"workload": "crossover", "cases": crossover(args, device, flush)}), flush=True)
                return
            fn = {"c1": c1_workload, "c3": c3_workload, "c4": c4_workload}.get(args.only)
            res = fn(args, device, flush, peaks, checker) if fn else \
                c5_workload(args, rank, world, device, flush, peaks, checker)
            if rank == 0:
                print(json.dumps({"workload": args.only, **res, "parity": checker.summary()}), flush=True)
        else:
            run_alut(args, rank, world, local, device)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


def run_alut(args, rank, world, local, device):
    import gc

    from table_moe.cache_engine import VectorSearchEngine
    from table_moe.cache_engine.step_graph import LookupStepGraph

    checker = Checker()
    managers = [build_layer(li, device, rank) for li in range(CFG["layers"])]
    engines = [VectorSearchEngine(m) for m in managers]
    inputs = [layer_inputs(li, rank) for li in range(CFG["layers"])]
    torch.cuda.synchronize()
    per_layer = [algorithmic_bytes(inp) for inp in inputs]
    path_bytes = sum(p[1] for p in per_layer)
    lookups_per_step = sum(p[2] for p in per_layer)

    # Device-resident step: the 48 per-layer lookups captured as one CUDA graph (hits and
    # indices are kept in device buffers for the checker: 16 x 8 entries per layer).
    step = LookupStepGraph(engines, CFG["tokens"], CFG["top_k"], variant="decode", renorm="to_one", keep_hits=True)
    for b, inp in zip(step.layers, inputs):
        for name, t in inp.items():
            getattr(b, name).copy_(t)
    torch.cuda.synchronize()
    step.capture()
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
    e2e_io = (e2e.h2d_bytes, e2e.d2h_bytes)

    # Checker leg: one fresh replay of the timed graph, three layers against the oracle.
    for b in step.layers:
        b.out.zero_()
    step.replay()
    torch.cuda.synchronize()
    for li in (0, CFG["layers"] // 2, CFG["layers"] - 1):
        if li >= CFG["layers"]:
            continue
        inp = {k: v.to(device) for k, v in inputs[li].items()}
        check_engine_lookup(checker, "c2", managers[li], inp["x"], inp["sel"], inp["is_vision"], inp["reuse"],
                            inp["weights"], inp["compute"], step.hits[li], step.idx[li], step.layers[li].out,
                            variant="decode", renorm="to_one")

    peaks, peak_src = measured_peaks()
    # Roofline of the unit the step is made of: one layer's lookup chain (k_project_mma ->
    # k_search_decode -> k_combine, chained by programmatic dependent launch), its duration
    # the timed step divided by the layers, its bytes the layer's algorithmic bytes.
    layer_s = ms_per_step / CFG["layers"] / 1e3
    traffic, traffic_src = ncu_traffic()
    roofline = hbm_roofline("per-layer alut_lookup_combine chain: k_project_mma -> k_search_decode -> k_combine "
                            "(programmatic dependent launch)", path_bytes / CFG["layers"], layer_s, peaks,
                            traffic=traffic, traffic_source=traffic_src, peak_source=peak_src,
                            timing="timed 48-layer step / 48 (CUDA events over the timed region)",
                            bytes_note="routed tables' keys + text basis + x + looked-up rows + output read/write")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        orc, sample = cpu_sample(managers[:CPU_LAYERS], inputs[:CPU_LAYERS])
        v, cores, n, secs = time_cpu(orc, sample, seconds=args.cpu_seconds)
        cpu = {"value": round(v, 1), "unit": "lookups/s", "cores": cores, "kind": "port",
               "sample": f"CPU oracle (C restatement of the reference torch path) over layers 0-{CPU_LAYERS - 1} "
                         f"of the step, {n} passes in {secs:.1f} s"}
    # Free the decode tables before the other workloads (config 4 alone holds 49 GB).
    del step, e2e, engines, managers
    gc.collect()
    torch.cuda.empty_cache()
    workloads = None
    if not args.no_workloads:
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        workloads = {}
        if world == 1:
            workloads["c1_single_table"] = c1_workload(args, device, flush, peaks, checker)
            workloads["c3_prefill_layer"] = c3_workload(args, device, flush, peaks, checker)
            gc.collect()
            torch.cuda.empty_cache()
            workloads["c4_deepseek_prefill_decode"] = c4_workload(args, device, flush, peaks, checker)
            gc.collect()
            torch.cuda.empty_cache()
        workloads["c5_sharded_table"] = c5_workload(args, rank, world, device, flush, peaks, checker)
    parity = checker.summary()
    if world > 1:
        for k in ("checked", "mismatches", "exempt"):
            parity[k] = sum_over_ranks(parity[k], world, device)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "lookups/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random tables and routing)", "config": config_dict(world),
            "lookups_per_step": total_lookups // args.steps,
            "e2e": {"value": round(total_lookups / (e2e_ms / 1e3), 1), "unit": "lookups/s",
                    "h2d_bytes_per_step": e2e_io[0], "d2h_bytes_per_step": e2e_io[1],
                    "ms_per_step": round(e2e_ms / args.steps, 5)},
            "gpu_launches": KERNELS_PER_LAYER * CFG["layers"] * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clocks.summary(),
            "workloads": workloads,
        }
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
