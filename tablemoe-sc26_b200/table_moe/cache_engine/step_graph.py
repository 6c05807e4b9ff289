"""Fused lookups of several MoE layers replayed as one CUDA graph.

A decode step runs the same sequence of ALUT lookups on every token batch: per layer,
search the routed (token, expert) slots that were not recomputed, gather the winning
value rows and accumulate them, renormalised, into the layer output. ``LookupStepGraph``
captures that sequence once over static device buffers and replays it, so the per-layer
host work (argument marshalling, kernel launches) is paid once at capture instead of on
every step.

All per-layer inputs live in one device arena with a pinned host twin, and all layer
outputs in a second pair, so that a graph captured with ``with_copies=True`` moves a
whole step's inputs host->device and outputs device->host with one copy each.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _alut


@dataclass
class LayerBuffers:
    x: torch.Tensor          # [Q, H] hidden states
    sel: torch.Tensor        # [Q, S] int64 routed experts
    is_vision: torch.Tensor  # [Q] bool
    reuse: torch.Tensor      # [Q, S] bool, slots to look up
    weights: torch.Tensor    # [Q, S] fp32 routing weights
    compute: torch.Tensor    # [Q, S] bool, slots computed by the experts
    out: torch.Tensor        # [Q, H] layer output (accumulated into when accumulate=True)


def _nbytes(shape, dtype):
    n = 1
    for d in shape:
        n *= d
    return n * torch.empty((), dtype=dtype).element_size()


def _view(arena: torch.Tensor, off: int, shape, dtype):
    return arena[off:off + _nbytes(shape, dtype)].view(dtype).view(*shape)


class LookupStepGraph:
    # Copy plan of a captured step with copies: layers at which a new host->device input copy
    # starts (besides 0), and the layer stride of the device->host output copies.
    INPUT_CUTS = (2, 8)
    OUTPUT_EVERY = 4

    def __init__(self, engines, q, s, *, x_dtype=torch.bfloat16, variant="decode", renorm="to_one",
                 accumulate=True, keep_hits=False):
        """``keep_hits``: every layer's lookup also writes its hits and centroid indices into
        device tensors (``self.hits[i]``, ``self.idx[i]``, [q, s]) that stay out of the
        host copies, so that a replay can be checked slot by slot."""
        if not engines:
            raise ValueError("need at least one engine")
        self.engines = list(engines)
        self.device = self.engines[0].device
        self.q, self.s = q, s
        self.variant, self.renorm, self.accumulate = variant, renorm, accumulate
        in_fields = [("x", None, x_dtype), ("sel", (q, s), torch.int64), ("is_vision", (q,), torch.bool),
                     ("reuse", (q, s), torch.bool), ("weights", (q, s), torch.float32),
                     ("compute", (q, s), torch.bool)]
        # Byte layout of the two arenas: per layer, each field at a 256-byte boundary.
        plan, off_in, off_out = [], 0, 0
        self._in_ranges, self._out_ranges = [], []  # per-layer [start, stop) of each arena
        for eng in self.engines:
            h = eng.manager.values_buffer.shape[-1]
            fields = {}
            in0, out0 = off_in, off_out
            for name, shape, dt in in_fields:
                shape = shape or (q, h)
                fields[name] = ("in", off_in, shape, dt)
                off_in = (off_in + _nbytes(shape, dt) + 255) // 256 * 256
            vdt = eng.manager.values_buffer.dtype
            fields["out"] = ("out", off_out, (q, h), vdt)
            off_out = (off_out + _nbytes((q, h), vdt) + 255) // 256 * 256
            plan.append(fields)
            self._in_ranges.append((in0, off_in))
            self._out_ranges.append((out0, off_out))
        self.in_dev = torch.zeros(off_in, dtype=torch.uint8, device=self.device)
        self.out_dev = torch.zeros(off_out, dtype=torch.uint8, device=self.device)
        self.in_host = torch.zeros(off_in, dtype=torch.uint8, pin_memory=True)
        self.out_host = torch.zeros(off_out, dtype=torch.uint8, pin_memory=True)

        def views(in_arena, out_arena):
            return [LayerBuffers(**{n: _view(in_arena if a == "in" else out_arena, o, sh, dt)
                                    for n, (a, o, sh, dt) in f.items()}) for f in plan]

        self.layers = views(self.in_dev, self.out_dev)
        self.host_layers = views(self.in_host, self.out_host)
        self.hits = [torch.zeros(q, s, dtype=torch.bool, device=self.device) for _ in self.engines] \
            if keep_hits else None
        self.idx = [torch.zeros(q, s, dtype=torch.int64, device=self.device) for _ in self.engines] \
            if keep_hits else None
        self.graph = None
        self.with_copies = False
        self._events = None

    @property
    def h2d_bytes(self):
        return self.in_dev.numel()

    @property
    def d2h_bytes(self):
        return self.out_dev.numel()

    def _step(self, profile_events, lib):
        for i, (eng, b) in enumerate(zip(self.engines, self.layers)):
            if profile_events is not None:
                st, sp = profile_events[i]
                _alut.check(lib.alut_set_profile_events(st.cuda_event, sp.cuda_event), "profile events")
            out = eng.lookup_combine(b.x, b.sel, b.is_vision, b.reuse, b.weights, compute_mask=b.compute,
                                     out=b.out if self.accumulate else None, variant=self.variant,
                                     renorm=self.renorm,
                                     hit_out=None if self.hits is None else self.hits[i],
                                     idx_out=None if self.idx is None else self.idx[i])
            if not self.accumulate:
                b.out.copy_(out)

    def _step_with_copies(self, lib):
        """Inputs in three copies of growing size (layers 0-1 alone, so that the first lookup
        starts early; layers 2-7 while those run; the rest while layers 2-7 run, each copy
        landing before its first layer is reached), outputs every four layers and the last
        layer's alone (so that little is left to copy after the last lookup), all on a second
        stream. The lookups wait only at the three input boundaries, so programmatic launch
        still chains the other layers."""
        main = torch.cuda.current_stream(self.device)
        copy = torch.cuda.Stream(self.device)
        copy.wait_stream(main)
        n = len(self.engines)
        in_cuts = sorted({0, n} | {min(c, n) for c in self.INPUT_CUTS})
        out_cuts = sorted(set(range(0, n, self.OUTPUT_EVERY)) | {max(0, n - 1), n})
        landed = {}
        with torch.cuda.stream(copy):
            for lo, hi in zip(in_cuts, in_cuts[1:]):
                a, b = self._in_ranges[lo][0], self._in_ranges[hi - 1][1]
                self.in_dev[a:b].copy_(self.in_host[a:b], non_blocking=True)
                landed[lo] = torch.cuda.Event()
                landed[lo].record(copy)
        for i, (eng, b) in enumerate(zip(self.engines, self.layers)):
            if i in landed:
                main.wait_event(landed[i])
            out = eng.lookup_combine(b.x, b.sel, b.is_vision, b.reuse, b.weights, compute_mask=b.compute,
                                     out=b.out if self.accumulate else None, variant=self.variant,
                                     renorm=self.renorm,
                                     hit_out=None if self.hits is None else self.hits[i],
                                     idx_out=None if self.idx is None else self.idx[i])
            if not self.accumulate:
                b.out.copy_(out)
            if i + 1 in out_cuts:
                lo = out_cuts[out_cuts.index(i + 1) - 1]
                done = torch.cuda.Event()
                done.record(main)
                copy.wait_event(done)
                with torch.cuda.stream(copy):
                    a, b2 = self._out_ranges[lo][0], self._out_ranges[i][1]
                    self.out_host[a:b2].copy_(self.out_dev[a:b2], non_blocking=True)
        main.wait_stream(copy)

    def run_eager(self):
        """Issue the per-layer fused lookups on the current stream (no graph)."""
        self._step(None, _alut.load())

    def capture(self, *, with_copies=False, profile_events=None, warmup=2):
        """Capture one step. ``with_copies`` adds the host->device copy of the layers' inputs
        and the device->host copy of their outputs, on a second stream, overlapping the
        lookups (see ``_step_with_copies``).
        ``profile_events`` (one (start, stop) pair of timing events per layer, already
        recorded once so that they exist) brackets each layer's centroid-scan kernel."""
        if profile_events is not None and len(profile_events) != len(self.engines):
            raise ValueError("one (start, stop) event pair per layer")
        lib = _alut.load()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):  # sizes workspaces and sets kernel attributes
                self._step(None, lib)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(self.graph):
                if with_copies:
                    self._step_with_copies(lib)
                else:
                    self._step(profile_events, lib)
        finally:
            lib.alut_set_profile_events(None, None)
        self.with_copies = with_copies
        self._events = profile_events
        return self

    def replay(self):
        if self.graph is None:
            raise RuntimeError("capture() first")
        self.graph.replay()

    def check_errors(self):
        """Raise if any layer's kernels left device error bits (synchronises)."""
        for i, eng in enumerate(self.engines):
            eng.check_device_errors(f"layer {i}")

    def scan_times_ms(self):
        """Per-layer centroid-scan durations of the last replay (needs profile events)."""
        if not self._events:
            return []
        return [st.elapsed_time(sp) for st, sp in self._events]
