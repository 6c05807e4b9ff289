"""Table storage of one MoE layer for the ALUT path.

Drop-in for the reference's ``HybridStorageManager`` (``table_moe/cache_engine/manager.py``):
same constructor, attributes (``pca``, ``keys_buffer``, ``raw_keys_buffer``,
``values_buffer``, the online ring buffer) and methods. One layout change, on purpose:
``values_buffer`` lives in HBM next to the keys instead of in pinned host memory
(``manager.py:54-58``), so that the value gather is a device kernel rather than a host
fancy-index plus a PCIe copy. ``gather_values`` therefore returns a device tensor; the
caller's ``.to(device, non_blocking=True)`` (``cached_layers.py:349``) is then a no-op.
"""
from __future__ import annotations

import glob
import os

import torch

from . import _alut
from .config import CacheConfig


def _resolve_cache_dtype():
    """``CacheConfig.MODEL_DTYPE`` as a torch dtype (manager.py:9-21)."""
    dtype = getattr(CacheConfig, "MODEL_DTYPE", torch.bfloat16)
    if isinstance(dtype, torch.dtype):
        return dtype
    if isinstance(dtype, str):
        name = dtype.removeprefix("torch.").lower()
        table = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
        if name in table:
            return table[name]
    raise ValueError(f"Unsupported cache dtype: {dtype!r}")


def normalize_rows(x: torch.Tensor, eps: float) -> torch.Tensor:
    """L2-normalise the last dim in fp32 with zero rows kept at zero, then cast back
    (load-time key normalisation, manager.py:24-31). CUDA tensors go through the
    ``alut_normalize_rows`` kernel; host tensors (fixtures, host-side preparation) through
    the same arithmetic in torch."""
    if x.is_cuda:
        src = x.contiguous()
        out = torch.empty_like(src)
        rows = src.numel() // src.shape[-1] if src.numel() else 0
        if rows:
            l = src.shape[-1]
            rc = _alut.load().alut_normalize_rows(rows, l, src.data_ptr(), l, out.data_ptr(), l,
                                                  _alut.dtype_code(src.dtype), float(eps),
                                                  _alut.stream_ptr(src.device))
            _alut.check(rc, "alut_normalize_rows")
        return out
    xf = x.float()
    n = torch.linalg.vector_norm(xf, dim=-1, keepdim=True)
    out = torch.where(n <= eps, torch.zeros_like(xf), xf / n.clamp_min(eps))
    return out.to(x.dtype)


class HybridStorageManager:
    def __init__(self, layer_idx, num_experts, hidden_dim, device="cuda:0", *, load=True):
        self.layer_idx = layer_idx
        self.num_experts = num_experts
        self.hidden_dim = hidden_dim
        self.device = torch.device(device)
        self.dtype = _resolve_cache_dtype()
        shape = (num_experts, 2, CacheConfig.FIXED_K, CacheConfig.COMPRESSED_DIM)
        self.pca = self._load_pca() if load else self._zero_pca()
        self.keys_buffer = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.raw_keys_buffer = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.values_buffer = torch.zeros((num_experts, 2, CacheConfig.FIXED_K, hidden_dim),
                                         dtype=self.dtype, device=self.device)
        if load:
            self._load_cache_data()
        self._init_online()
        self._tables = None

    # ---- construction from in-memory tables (synthetic runs, tests, benchmarks) ----------
    @classmethod
    def from_tables(cls, layer_idx, raw_keys, values, pca, *, keys=None, device=None,
                    eps=None, enable_online=False):
        """Build a manager around existing tensors.

        raw_keys: [E,2,K,L]; values: [E,2,K,H]; pca: {"vision": {proj, bias}, "text": ...}.
        ``keys`` (the normalised copy) is derived from raw_keys when not given.
        """
        self = cls.__new__(cls)
        self.layer_idx = layer_idx
        self.num_experts, _, _, _ = raw_keys.shape
        self.hidden_dim = values.shape[-1]
        self.device = torch.device(device) if device is not None else raw_keys.device
        self.dtype = raw_keys.dtype
        self.pca = pca
        self.raw_keys_buffer = raw_keys
        if keys is None:
            e = float(CacheConfig.OFFLINE_COSINE_EPS if eps is None else eps)
            keys = normalize_rows(raw_keys, e)
        self.keys_buffer = keys
        self.values_buffer = values
        self._init_online(force=enable_online)
        self._tables = None
        return self

    def _init_online(self, force=None):
        enable = (CacheConfig.ONLINE_MIN_LAYER_IDX <= self.layer_idx <= CacheConfig.ONLINE_MAX_LAYER_IDX)
        self.enable_online = enable if force is None else bool(force)
        self.online_ptr = 0
        self.online_size = 0
        self.online_full = False
        self.online_topk = 0
        if self.enable_online:
            self.online_size = CacheConfig.ONLINE_CACHE_SIZE
            self.online_topk = CacheConfig.ONLINE_TOP_K
            self.online_keys = torch.zeros((self.online_size, self.hidden_dim), dtype=self.dtype, device=self.device)
            self.online_values = torch.zeros((self.online_size, self.online_topk, self.hidden_dim),
                                             dtype=self.dtype, device=self.device)
            self.online_expert_ids = torch.full((self.online_size, self.online_topk), -1,
                                                dtype=torch.long, device=self.device)
        else:
            self.online_keys = None
            self.online_values = None
            self.online_expert_ids = None

    # ---- C-ABI table descriptor ---------------------------------------------------------
    def alut_tables(self):
        """The ``alut_tables_t`` of this layer (rebuilt when a buffer is replaced)."""
        pv, pt = self.pca["vision"], self.pca["text"]
        key = (self.keys_buffer.data_ptr(), self.raw_keys_buffer.data_ptr(),
               self.values_buffer.data_ptr(), pv["proj"].data_ptr(), pt["proj"].data_ptr(),
               pv["bias"].data_ptr(), pt["bias"].data_ptr())
        if self._tables is None or self._tables[0] != key:
            t = _alut.make_tables(self.keys_buffer, self.raw_keys_buffer, self.values_buffer,
                                  pv["proj"], pv["bias"], pt["proj"], pt["bias"])
            # Static tensor-core split of an fp32 basis (used for bf16 tokens, small batches).
            self._proj_split = _alut.prepare_basis(t, self.device) if self.device.type == "cuda" else None
            if self._proj_split is not None:
                t.proj_split = self._proj_split.data_ptr()
            self._keys_split = {}
            self._tables = (key, t)
        return self._tables[1]

    def prepare_tensor_core(self, keyset):
        """The tensor-core form of one key set (``_alut.KEYS_RAW`` or ``KEYS_NORMALISED``):
        made once, on the first batch large enough to use it (it takes as much memory as
        that key set). Tables that do not qualify (not fp32, L % 16, L > 128) are left alone."""
        t = self.alut_tables()
        if keyset in self._keys_split or self.device.type != "cuda":
            return t
        lib = _alut.load()
        n = int(lib.alut_keys_split_bytes(t))
        buf = None
        if n:
            buf = torch.empty(n, dtype=torch.uint8, device=self.device)
            _alut.check(lib.alut_prepare_keys(t, int(keyset), buf.data_ptr(), n, _alut.stream_ptr(self.device)),
                        "alut_prepare_keys")
            if keyset == _alut.KEYS_RAW:
                t.raw_keys_split = buf.data_ptr()
            else:
                t.keys_split = buf.data_ptr()
        self._keys_split[keyset] = buf
        return t

    # ---- online ring buffer (manager.py:89-155) -----------------------------------------
    @torch.no_grad()
    def update_online_cache_bs1(self, hidden_state, expert_ids, expert_outputs, valid_slot_mask=None):
        if not self.enable_online:
            return
        i = self.online_ptr
        self.online_keys[i].copy_(hidden_state)
        self.online_expert_ids[i].copy_(expert_ids)
        self.online_values[i].copy_(expert_outputs)
        if valid_slot_mask is not None:
            self.online_expert_ids[i].masked_fill_(~valid_slot_mask, -1)
            self.online_values[i].masked_fill_(~valid_slot_mask.unsqueeze(-1), 0)
        self.online_ptr = (i + 1) % self.online_size
        if self.online_ptr == 0:
            self.online_full = True

    @torch.no_grad()
    def update_online_cache(self, hidden_states, expert_ids, expert_outputs, valid_slot_mask=None):
        if not self.enable_online:
            return
        n = hidden_states.shape[0]
        if n == 0:
            return
        if valid_slot_mask is not None:
            bad = ~valid_slot_mask
            expert_ids = expert_ids.masked_fill(bad, -1)
            expert_outputs = expert_outputs.masked_fill(bad.unsqueeze(-1), 0)
        if n > self.online_size:
            hidden_states = hidden_states[-self.online_size:]
            expert_ids = expert_ids[-self.online_size:]
            expert_outputs = expert_outputs[-self.online_size:]
            n = self.online_size
        start = self.online_ptr
        first = min(n, self.online_size - start)
        self.online_keys[start:start + first] = hidden_states[:first]
        self.online_expert_ids[start:start + first] = expert_ids[:first]
        self.online_values[start:start + first] = expert_outputs[:first]
        rest = n - first
        if rest > 0:
            self.online_keys[:rest] = hidden_states[first:]
            self.online_expert_ids[:rest] = expert_ids[first:]
            self.online_values[:rest] = expert_outputs[first:]
            self.online_ptr = rest
            self.online_full = True
        else:
            self.online_ptr = (start + first) % self.online_size
        if self.online_ptr == 0:
            self.online_full = True

    # ---- table files (manager.py:157-210) -----------------------------------------------
    def _zero_pca(self):
        z = {}
        for mod in ("vision", "text"):
            z[mod] = {
                "proj": torch.zeros((self.hidden_dim, CacheConfig.COMPRESSED_DIM), device=self.device, dtype=self.dtype),
                "bias": torch.zeros(CacheConfig.COMPRESSED_DIM, device=self.device, dtype=self.dtype),
            }
        return z

    def _load_pca(self):
        """``L{layer}_{mod}_pca.pt`` = {mean [H], proj [H,L]} -> {proj, bias = -mean @ proj}."""
        pca = self._zero_pca()
        root = os.path.join(CacheConfig.PCA_DIR, f"layer_{self.layer_idx}")
        for mod in ("vision", "text"):
            path = os.path.join(root, f"L{self.layer_idx}_{mod}_pca.pt")
            if not os.path.exists(path):
                continue
            data = torch.load(path, map_location=self.device)
            mean = data["mean"].to(device=self.device, dtype=self.dtype)
            proj = data["proj"].to(device=self.device, dtype=self.dtype).contiguous()
            pca[mod] = {"proj": proj, "bias": -(mean @ proj)}
        return pca

    def _load_cache_data(self):
        """``L{layer}_E{e}_{mod}_cache.pt`` = {key [k,L], value [k,H]}, rows beyond k stay 0;
        the normalised key set is made from the raw one on the device after all files."""
        root = os.path.join(CacheConfig.CACHE_DIR, f"layer_{self.layer_idx}")
        eps = float(CacheConfig.OFFLINE_COSINE_EPS)
        self._load_files(root)
        self.keys_buffer.copy_(normalize_rows(self.raw_keys_buffer, eps))

    def _load_files(self, root):
        for path in glob.glob(os.path.join(root, "*_cache.pt")):
            try:
                parts = os.path.basename(path)[:-3].split("_")
                eid = int(parts[1][1:])
                mid = CacheConfig.MODALITY_MAP.get(parts[2], -1)
                if mid == -1 or eid >= self.num_experts:
                    continue
                data = torch.load(path, map_location="cpu")
                keys = data["key"].to(dtype=self.dtype)
                k = keys.shape[0]
                self.raw_keys_buffer[eid, mid, :k] = keys.to(self.device)
                self.values_buffer[eid, mid, :k] = data["value"].to(dtype=self.dtype, device=self.device)
            except Exception as exc:  # same policy as the reference: log and skip the file
                print(f"Error loading {path}: {exc}")

    # ---- value gather (manager.py:212-228) ----------------------------------------------
    def _ids(self, t):
        t = torch.as_tensor(t)
        if t.device != self.device or t.dtype != torch.int64:
            t = t.to(device=self.device, dtype=torch.int64, non_blocking=True)
        return t.contiguous()

    @torch.no_grad()
    def gather_values(self, expert_ids, modality_ids, cluster_ids):
        """values[e, m, c] rows for each i, a bit-exact device copy -> [n, H]."""
        e, m, c = self._ids(expert_ids), self._ids(modality_ids), self._ids(cluster_ids)
        e, m, c = torch.broadcast_tensors(e, m, c)
        e, m, c = e.reshape(-1).contiguous(), m.reshape(-1).contiguous(), c.reshape(-1).contiguous()
        n = e.numel()
        out = torch.empty((n, self.hidden_dim), dtype=self.values_buffer.dtype, device=self.device)
        if n:
            rc = _alut.load().alut_gather_rows(self.alut_tables(), n, e.data_ptr(), m.data_ptr(), c.data_ptr(),
                                               None, out.data_ptr(), out.stride(0), _alut.stream_ptr(self.device))
            _alut.check(rc, "gather_values")
        return out

    @torch.no_grad()
    def gather_values_decode_bs1(self, expert_ids, modality_id, cluster_ids, slot_ids, out_buffer):
        """out_buffer[slot_ids[i]] = values[expert_ids[i], modality_id, cluster_ids[i]]."""
        e = self._ids(expert_ids).reshape(-1)
        n = e.numel()
        if n == 0:
            return
        c = self._ids(cluster_ids).reshape(-1).contiguous()
        s = self._ids(slot_ids).reshape(-1).contiguous()
        m = torch.full((n,), int(modality_id), dtype=torch.int64, device=self.device)
        if out_buffer.stride(-1) != 1 or out_buffer.dtype != self.values_buffer.dtype:
            raise ValueError("out_buffer must be [top_k, H] with the value dtype and unit inner stride")
        rc = _alut.load().alut_gather_rows(self.alut_tables(), n, e.contiguous().data_ptr(), m.data_ptr(),
                                           c.data_ptr(), s.data_ptr(), out_buffer.data_ptr(),
                                           out_buffer.stride(0), _alut.stream_ptr(self.device))
        _alut.check(rc, "gather_values_decode_bs1")
