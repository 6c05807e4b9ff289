"""One very large centroid table split by centroid range over the ranks of a process group.

Rank r of W holds centroids [K*r/W, K*(r+1)/W) of the key table and the matching value
rows. A lookup of Q tokens then runs in three steps:

1. every rank projects its slice of Q/W tokens and the projected queries are exchanged
   (``all_gather_into_tensor``, Q x L fp32), then every rank scans its centroid slice for
   all Q tokens (``alut_search_packed``), producing one packed candidate per token:
   ``(order-preserving score bits << 32) | (0xFFFFFFFF - global index)``, so that the
   largest packed value is the best score with the lowest index;
2. the W candidate vectors are exchanged (``all_gather_into_tensor``, 8 bytes per token per
   rank) and merged by max (``alut_merge_packed``), which also applies the hit rule - every
   rank now holds the winners;
3. each rank reads the rows of its own Q/W tokens straight from the owning rank's HBM
   (``alut_gather_rows_sharded`` over CUDA IPC peer mappings, NVLink loads, no multicast):
   every remote row crosses NVLink once. Groups that cannot map peer memory (gloo, or
   IPC unavailable) use the collective form instead: each rank gathers the rows it owns
   (zeros elsewhere) and a reduce-scatter (sum) hands out the token slices - a row has
   one non-zero contribution, so the sum is an exact copy.

Failure detection (``timeout_s``): every collective of a lookup is waited on with that
limit and a timed-out wait raises ``ShardTimeoutError`` (a ``TimeoutError``); a rank that
leaves calls ``leave()`` between lookups, which the other ranks see in the process group's
store before their next launch (``PeerLeftError``). Either error marks the table failed.
``capture()`` records one whole lookup (NCCL calls included) as a CUDA graph, so that the
per-call host work - argument marshalling, launches, collective calls - is paid once.

Replicated keys (``replicate_keys=True``): the key table is small next to the value rows
(C5: 32 MiB of fp32 keys against 512 MiB of bf16 rows), so every rank may hold all of it
and only the value rows are split by centroid range. A lookup then needs no query or
candidate exchange before the scan: rank r projects and scans its own Q/W tokens over the
whole table, the packed winners (8 bytes per token) are all-gathered and merged so that
every rank holds the global (hit, idx), and step 3 is unchanged. The scan's work divides by
W with no fixed part over all Q tokens (strong scaling).

The reference is single-GPU; this is the centroid-range sharding the benchmark's large-
table configuration asks for. The device work goes through the C ABI; the three device
steps are attributes of the object so that the exchange logic can be exercised on CPU
process groups (gloo) with stand-ins.
"""
from __future__ import annotations

import ctypes
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from . import _alut

_LEFT_KEY = "alut_sharded_table/left"


class PeerLeftError(RuntimeError):
    """A rank of the table's group left (``leave()``) before this lookup."""


class ShardTimeoutError(TimeoutError):
    """A collective of the sharded lookup did not complete within ``timeout_s``."""


def shard_range(k_total: int, world: int, rank: int):
    """Centroid rows [start, stop) held by `rank`."""
    return k_total * rank // world, k_total * (rank + 1) // world


class ShardedCentroidTable:
    def __init__(self, keys, values, pca, k_total, *, group=None, keyset=_alut.KEYS_RAW,
                 normalize=False, cmp_ge=False, thr_vision=0.0, thr_text=0.0, eps=1e-6, timeout_s=None,
                 store=None, replicate_keys=False):
        """keys: [1, 2, Kr, L] this rank's slice (rows shard_range(k_total, W, r)), or with
        replicate_keys the whole [1, 2, k_total, L] table on every rank;
        values: [1, 2, Kr, H] this rank's slice; pca: {"vision": {proj, bias}, "text": {...}}.
        timeout_s: limit of every collective wait (None: the process group's own timeout);
        store: the store ``leave()`` announces through (default: the default group's)."""
        self.group = group
        self.timeout = None if timeout_s is None else timedelta(seconds=float(timeout_s))
        self._store = store
        if self._store is None and dist.is_initialized() and timeout_s is not None:
            self._store = dist.distributed_c10d._get_default_store()
        self._left_seen = 0
        self.failed = None
        self._bufs = {}
        self._capturing = False
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.k_total = int(k_total)
        self.k0, self.k1 = shard_range(self.k_total, self.world, self.rank)
        self.replicate_keys = bool(replicate_keys)
        want = self.k_total if self.replicate_keys else self.k1 - self.k0
        if keys.shape[2] != want:
            raise ValueError(f"rank {self.rank} holds {keys.shape[2]} key rows, expected {want}")
        if values.shape[2] != self.k1 - self.k0:
            raise ValueError(f"rank {self.rank} holds {values.shape[2]} value rows, expected {self.k1 - self.k0}")
        self.key_base = 0 if self.replicate_keys else self.k0  # global index of this rank's first key row
        self.keys, self.values, self.pca = keys, values, pca
        self.device = keys.device
        self.params = dict(keyset=keyset, normalize=normalize, cmp_ge=cmp_ge, thr_vision=thr_vision,
                           thr_text=thr_text, eps=eps)
        self._tables = None
        self._vtables = None
        self._ws = None
        self._peers = None  # (device pointers, shard starts, modality strides, opened mappings)
        # Device steps (replaceable for CPU tests of the exchange).
        self.local_search = self._local_search
        self.merge = self._merge
        self.gather_owned = self._gather_owned

    # ---- device steps -----------------------------------------------------------------------
    def _tables_struct(self):
        if self._tables is None:
            pv, pt = self.pca["vision"], self.pca["text"]
            k = self.keys if self.params["keyset"] == _alut.KEYS_NORMALISED else None
            r = self.keys if self.params["keyset"] == _alut.KEYS_RAW else None
            vals = None if self.replicate_keys else self.values  # replicated keys: K rows != value rows
            self._tables = _alut.make_tables(k, r, vals, pv["proj"], pv["bias"], pt["proj"], pt["bias"])
            self._split = _alut.prepare_basis(self._tables, self.device)
            if self._split is not None:
                self._tables.proj_split = self._split.data_ptr()
            # bf16 operand form of this rank's keys for the tensor-core scan (fp32 keys,
            # L % 16 == 0, L <= 128; other shapes keep the CUDA-core scans).
            self._keys_split = None
            if self.device.type == "cuda":
                lib = _alut.load()
                n = int(lib.alut_keys_split_bytes(self._tables))
                if n:
                    self._keys_split = torch.empty(n, dtype=torch.uint8, device=self.device)
                    _alut.check(lib.alut_prepare_keys(self._tables, int(self.params["keyset"]),
                                                      self._keys_split.data_ptr(), n, _alut.stream_ptr(self.device)),
                                "alut_prepare_keys")
                    if self.params["keyset"] == _alut.KEYS_RAW:
                        self._tables.raw_keys_split = self._keys_split.data_ptr()
                    else:
                        self._tables.keys_split = self._keys_split.data_ptr()
        return self._tables

    def _value_tables(self):
        """Tables whose values are this rank's slice (with replicated keys: the matching key
        rows, so that the struct's K is the slice's)."""
        if not self.replicate_keys:
            return self._tables_struct()
        if self._vtables is None:
            pv, pt = self.pca["vision"], self.pca["text"]
            ks = self.keys[:, :, self.k0:self.k1]
            k = ks if self.params["keyset"] == _alut.KEYS_NORMALISED else None
            r = ks if self.params["keyset"] == _alut.KEYS_RAW else None
            self._vtables = _alut.make_tables(k, r, self.values, pv["proj"], pv["bias"], pt["proj"], pt["bias"])
        return self._vtables

    def _params_struct(self):
        p = self.params
        return _alut.make_params(p["keyset"], p["normalize"], p["cmp_ge"], p["thr_vision"], p["thr_text"], p["eps"])

    def _buf(self, q, name, shape, dtype, zero=False):
        """Per-batch-size buffers, made once (also what a captured lookup replays on)."""
        key = (q, name)
        t = self._bufs.get(key)
        if t is None or t.shape != torch.Size(shape) or t.dtype != dtype:
            t = (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=self.device)
            self._bufs[key] = t
        return t

    def _workspace(self, q):
        lib = _alut.load()
        need = int(lib.alut_workspace_size(self._tables_struct(), q, 1))
        if self._ws is None or self._ws.numel() < need:
            if self._capturing:
                raise RuntimeError("sharded lookup: workspace must be sized before capture (run lookup once)")
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def _local_search(self, x, is_vision):
        """Packed best candidate of every token over this rank's slice -> int64 [Q]."""
        lib = _alut.load()
        q = x.shape[0]
        t = self._tables_struct()
        ws = self._workspace(q)
        sel = self._buf(q, "sel", (q, 1), torch.int64, zero=True)
        vis = is_vision.reshape(-1)
        packed = self._buf(q, "packed", (q,), torch.int64)
        b = _alut.make_batch(x, sel, vis, None)  # x, sel, vis stay referenced until the call returns
        rc = lib.alut_search_packed(t, ctypes.byref(b), self._params_struct(), None, self.key_base, packed.data_ptr(),
                                    ws.data_ptr(), ws.numel(), _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_search_packed")
        return packed

    def _merge(self, packed_all, is_vision):
        """[W, Q] packed candidates -> (hit [Q] bool, idx [Q] int64 global)."""
        lib = _alut.load()
        w, q = packed_all.shape
        vis = is_vision.reshape(-1)
        hit = self._buf(q, "hit", (q,), torch.bool)
        idx = self._buf(q, "idx", (q,), torch.int64)
        rc = lib.alut_merge_packed(w, q, 1, packed_all.data_ptr(), vis.data_ptr(), self._params_struct(),
                                   hit.data_ptr(), idx.data_ptr(), _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_merge_packed")
        return hit, idx

    def _gather_owned(self, hit, idx, is_vision):
        """[Q, H] rows of the winners this rank owns; other rows are zero."""
        lib = _alut.load()
        q = idx.shape[0]
        owned = hit & (idx >= self.k0) & (idx < self.k1)
        cids = torch.where(owned, idx - self.k0, torch.full_like(idx, -1)).contiguous()
        eids = torch.zeros(q, dtype=torch.int64, device=self.device)
        mids = torch.where(is_vision.reshape(-1).bool(), 0, 1).to(torch.int64).contiguous()
        out = torch.empty(q, self.values.shape[-1], dtype=self.values.dtype, device=self.device)
        rc = lib.alut_gather_rows(self._value_tables(), q, eids.data_ptr(), mids.data_ptr(), cids.data_ptr(), None,
                                  out.data_ptr(), out.stride(0), _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_gather_rows")
        return out

    def _nccl(self):
        return self.world > 1 and self.device.type == "cuda" and dist.get_backend(self.group) == "nccl"

    # ---- collectives with failure detection ---------------------------------------------
    def _precheck(self):
        """Before a lookup's first launch: fail fast if a peer left (store) or a previous
        lookup failed."""
        if self.failed:
            raise PeerLeftError(f"sharded table is unusable: {self.failed}")
        if self._store is not None and self.world > 1 and not self._capturing:
            left = int(self._store.add(_LEFT_KEY, 0))
            if left > self._left_seen:
                self.failed = f"{left} rank(s) left the group"
                raise PeerLeftError(self.failed)

    def _all_gather(self, out, inp):
        if self._capturing or self.timeout is None:
            dist.all_gather_into_tensor(out, inp, group=self.group)
            return
        t0 = time.monotonic()
        work = dist.all_gather_into_tensor(out, inp, group=self.group, async_op=True)
        try:
            work.wait(timeout=self.timeout)
        except RuntimeError as exc:
            waited = time.monotonic() - t0
            if waited >= 0.9 * self.timeout.total_seconds():
                self.failed = f"collective timed out after {waited:.2f} s: {exc}"
                raise ShardTimeoutError(self.failed) from exc
            self.failed = f"collective failed after {waited:.2f} s (a peer is gone): {exc}"
            raise PeerLeftError(self.failed) from exc

    def leave(self):
        """Announce, between lookups, that this rank stops taking part (the other ranks'
        next lookup raises PeerLeftError instead of waiting for it)."""
        if self._store is not None:
            self._store.add(_LEFT_KEY, 1)
        self.failed = "this rank left the group"

    def _project_split(self, x, is_vision):
        """This rank projects its Q/W tokens; the ranks all-gather the queries -> [Q, L] fp32."""
        lib = _alut.load()
        q = x.shape[0]
        lo, hi = q * self.rank // self.world, q * (self.rank + 1) // self.world
        t = self._tables_struct()
        ws = self._workspace(q)
        xs = x[lo:hi]
        vs = is_vision.reshape(-1)[lo:hi]
        sel = self._buf(q, "sel_mine", (hi - lo, 1), torch.int64, zero=True)
        mine = self._buf(q, "q_mine", (hi - lo, t.l), torch.float32)
        b = _alut.make_batch(xs, sel, vs, None)  # xs, sel, vs stay referenced until the call returns
        _alut.check(lib.alut_project(t, ctypes.byref(b), int(self.params["normalize"]), self.params["eps"],
                                     mine.data_ptr(), t.l, ws.data_ptr(), ws.numel(),
                                     _alut.stream_ptr(self.device)), "alut_project")
        q_all = self._buf(q, "q_all", (q, t.l), torch.float32)
        self._all_gather(q_all, mine)
        return q_all

    def _local_search_q(self, q_all, is_vision):
        """Packed best candidates of this slice for precomputed queries (normalisation, if
        any, was applied by the projection)."""
        lib = _alut.load()
        q = q_all.shape[0]
        t = self._tables_struct()
        ws = self._workspace(q)
        sel = self._buf(q, "sel", (q, 1), torch.int64, zero=True)
        vis = is_vision.reshape(-1)
        packed = self._buf(q, "packed", (q,), torch.int64)
        b = _alut.make_batch(None, sel, vis, None)
        p = self.params
        prm = _alut.make_params(p["keyset"], False, p["cmp_ge"], p["thr_vision"], p["thr_text"], p["eps"])
        rc = lib.alut_search_packed(t, ctypes.byref(b), prm, q_all.data_ptr(), self.key_base, packed.data_ptr(),
                                    ws.data_ptr(), ws.numel(), _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_search_packed")
        return packed

    def _peer_setup(self):
        """Exchange CUDA IPC handles of the value slices; False if peer mapping is unavailable."""
        if self._peers is not None:
            return self._peers is not False
        lib = _alut.load()
        v = self.values
        if self.world == 1:  # the one slice is local: no handles to exchange
            if not (v.is_contiguous() and v.shape[0] == 1):
                self._peers = False
                return False
            dev = self.device
            self._peers = (torch.tensor([v.data_ptr()], dtype=torch.int64, device=dev),
                           torch.tensor([self.k0, self.k1], dtype=torch.int64, device=dev),
                           torch.tensor([v.stride(1)], dtype=torch.int64, device=dev), [], v.stride(2))
            return True
        ok = v.is_contiguous() and v.shape[0] == 1
        handle = (ctypes.c_ubyte * _alut.PEER_HANDLE_BYTES)()
        off = ctypes.c_uint64(0)
        if ok:
            ok = lib.alut_peer_export(v.data_ptr(), handle, ctypes.byref(off)) == 0
        info = (bytes(handle), int(off.value), self.k0, self.k1, int(v.stride(1)), int(v.stride(2)), bool(ok))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, info, group=self.group)
        if not all(e[6] for e in everyone) or len({e[5] for e in everyone}) != 1:
            self._peers = False
            return False
        ptrs, opened = [], []
        for r, (h, o, _k0, _k1, _sm, _sk, _ok) in enumerate(everyone):
            if r == self.rank:
                ptrs.append(v.data_ptr())
                continue
            p = ctypes.c_void_p()
            _alut.check(lib.alut_peer_open(h, o, ctypes.byref(p)), "alut_peer_open")
            opened.append((p.value, o))
            ptrs.append(p.value)
        dev = self.device
        self._peers = (torch.tensor(ptrs, dtype=torch.int64, device=dev),
                       torch.tensor([e[2] for e in everyone] + [everyone[-1][3]], dtype=torch.int64, device=dev),
                       torch.tensor([e[4] for e in everyone], dtype=torch.int64, device=dev), opened,
                       everyone[0][5])
        return True

    def close(self):
        """Unmap the peers' value slices (collective: every rank calls it before freeing its
        values, so that no peer still reads them)."""
        if self._peers and self.world > 1:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            lib = _alut.load()
            for p, o in self._peers[3]:
                lib.alut_peer_close(p, o)
        self._peers = None

    def _gather_peer(self, hit, idx, is_vision, lo, hi):
        lib = _alut.load()
        ptrs, starts, strides_m, _opened, stride_k = self._peers
        q = hit.shape[0]
        n = hi - lo
        h = self.values.shape[-1]
        out = self._buf(q, "rows", (n, h), self.values.dtype)
        vis = is_vision.reshape(-1)[lo:hi]
        rc = lib.alut_gather_rows_sharded(n, hit[lo:hi].data_ptr(), idx[lo:hi].data_ptr(), vis.data_ptr(), self.world,
                                          ptrs.data_ptr(), starts.data_ptr(), strides_m.data_ptr(), stride_k, h,
                                          _alut.dtype_code(self.values.dtype), out.data_ptr(), out.stride(0),
                                          _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_gather_rows_sharded")
        return out

    # ---- lookup ---------------------------------------------------------------------------
    def search(self, x, is_vision):
        """Global (hit, idx) of every token, identical on all ranks."""
        self._precheck()
        is_vision = is_vision.reshape(-1)
        if is_vision.dtype != torch.bool or not is_vision.is_contiguous():
            is_vision = is_vision.bool().contiguous()
        q = x.shape[0]
        if self.replicate_keys:
            # Own tokens over the whole table, then the winners of every rank's tokens.
            if q % self.world:
                raise ValueError(f"token count {q} is not a multiple of the world size {self.world}")
            lo, hi = q * self.rank // self.world, q * (self.rank + 1) // self.world
            packed = self.local_search(x[lo:hi], is_vision[lo:hi])
            if self.world > 1:
                flat = self._buf(q, "flat", (q,), packed.dtype) if packed.device == self.device else \
                    torch.empty(q, dtype=packed.dtype, device=packed.device)
                self._all_gather(flat, packed.contiguous())
                packed = flat
            return self.merge(packed.view(1, -1), is_vision)
        if self._nccl() and q % self.world == 0 and self.local_search == self._local_search:
            packed = self._local_search_q(self._project_split(x, is_vision), is_vision)
        else:
            packed = self.local_search(x, is_vision)
        if self.world == 1:
            return self.merge(packed.view(1, -1), is_vision)
        q = packed.numel()
        flat = self._buf(q, "flat", (self.world * q,), packed.dtype) if packed.device == self.device else \
            torch.empty(self.world * q, dtype=packed.dtype, device=packed.device)
        self._all_gather(flat, packed.contiguous())
        return self.merge(flat.view(self.world, -1), is_vision)

    def lookup(self, x, is_vision):
        """Search, then the value rows of this rank's token slice [Q*r/W, Q*(r+1)/W) (Q must
        be a multiple of W): (hit [Q], idx [Q], rows [Q/W, H]). The returned tensors are
        this table's buffers for batches of Q tokens: the next lookup of the same size
        overwrites them."""
        q = x.shape[0]
        if self.world > 1 and q % self.world:
            raise ValueError(f"token count {q} is not a multiple of the world size {self.world}")
        is_vision = is_vision.reshape(-1)
        if is_vision.dtype != torch.bool or not is_vision.is_contiguous():
            is_vision = is_vision.bool().contiguous()
        hit, idx = self.search(x, is_vision)
        direct = self.world == 1 and self.device.type == "cuda"
        if (direct or self._nccl()) and self.gather_owned == self._gather_owned and self._peer_setup():
            lo, hi = q * self.rank // self.world, q * (self.rank + 1) // self.world
            return hit, idx, self._gather_peer(hit, idx, is_vision, lo, hi)
        rows = self.gather_owned(hit, idx, is_vision)
        if self.world == 1:
            return hit, idx, rows
        n = q // self.world
        if dist.get_backend(self.group) == "gloo":  # CPU groups: no reduce_scatter in gloo
            rows = rows.contiguous().clone()
            dist.all_reduce(rows, op=dist.ReduceOp.SUM, group=self.group)
            return hit, idx, rows[self.rank * n:(self.rank + 1) * n]
        mine = torch.empty(n, rows.shape[1], dtype=rows.dtype, device=rows.device)
        dist.reduce_scatter_tensor(mine, rows.contiguous(), op=dist.ReduceOp.SUM, group=self.group)
        return hit, idx, mine

    def capture(self, x, is_vision):
        """Record one lookup of this (static) x / is_vision as a CUDA graph: returns
        (graph, (hit, idx, rows)); ``graph.replay()`` reruns it into the same tensors. Every
        rank of the group captures together (the NCCL calls are part of the graph)."""
        if self.device.type != "cuda":
            raise ValueError("capture needs a CUDA table")
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):  # sizes buffers and the workspace, maps the peers
            for _ in range(2):
                self.lookup(x, is_vision)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        graph = torch.cuda.CUDAGraph()
        self._capturing = True
        try:
            with torch.cuda.graph(graph):
                outs = self.lookup(x, is_vision)
        finally:
            self._capturing = False
        return graph, outs
