"""ALUT search engine on the sm_100a kernels of ``libalut.so``.

Drop-in for the reference's ``VectorSearchEngine`` (``table_moe/cache_engine/search.py:388``):
same constructor and public methods, same arguments, same return values and dtypes. The
Triton kernels and the torch fallback of the reference are gone; every method runs the
CUDA path and raises when the library is missing. Semantics follow the reference's torch
path, which scans all K centroids of a table:

====================================  ==========  ===================  =============
method (reference line)               query       key table            hit rule
====================================  ==========  ===================  =============
search_prefill_offline (:808)         normalised  keys_buffer          >= 0.6 / 0.7
search_prefill_offline_dot (:699)     raw         raw_keys_buffer      > DOT_THRESHOLD
search_decode_offline (:824)          raw         keys_buffer          >= 0
search_decode_offline_dot (:715)      raw         raw_keys_buffer      > DOT_THRESHOLD
search_decode_hybrid (:839)           raw         keys_buffer          >= 0 (offline part)
====================================  ==========  ===================  =============

(thresholds from ``CacheConfig``; ties resolve to the first centroid, as ``torch.max``.)
"""
from __future__ import annotations

import torch

from . import _alut
from .config import CacheConfig

# Kept for import compatibility with callers that test it; the ALUT path has no Triton.
HAS_TRITON = False


class VectorSearchEngine:
    def __init__(self, manager):
        self.manager = manager
        self.device = torch.device(manager.device)
        self.workspace_capacity = 0
        self.workspace = {}
        self._alut_ws = None
        self._alut_ws_shape = (0, 0)
        self.search_dims_cache = None
        self._lib = _alut.load()

    # ---- helpers -----------------------------------------------------------------------
    def _get_pca_pair(self):
        pca_map = getattr(self.manager, "pca", None)
        if not isinstance(pca_map, dict) or not pca_map:
            raise ValueError("manager.pca must be a non-empty dict")
        if "vision" in pca_map and "text" in pca_map:
            return pca_map["vision"], pca_map["text"]
        shared = pca_map[next(iter(pca_map))]
        return shared, shared

    def _get_search_dims(self):
        if self.search_dims_cache is None:
            pv, pt = self._get_pca_pair()
            dim = int(pv["proj"].shape[1])
            if int(pt["proj"].shape[1]) != dim:
                raise ValueError("vision/text PCA projection dims must match")
            online = getattr(self.manager, "online_expert_ids", None)
            self.search_dims_cache = {
                "pca_vis": pv, "pca_txt": pt, "compressed_dim": dim,
                "fixed_k": int(self.manager.keys_buffer.shape[2]),
                "online_topk": None if online is None else int(online.shape[1]),
            }
        return self.search_dims_cache

    def _tensor_core_wanted(self, bs, top_k):
        """Whether the library will run the tensor-core scan for this batch shape (then the
        manager prepares the key form once)."""
        fn = getattr(self.manager, "alut_tables", None)
        if fn is None or bs * top_k == 0:
            return False
        return self._lib.alut_scan_kind(fn(), bs, top_k) == _alut.SCAN_TENSOR_CORE

    def _tables(self, with_values=False, shape=(0, 0), keyset=None):
        prep = getattr(self.manager, "prepare_tensor_core", None)
        if prep is not None and keyset is not None and self._tensor_core_wanted(*shape):
            return prep(keyset)
        fn = getattr(self.manager, "alut_tables", None)
        if fn is not None:
            return fn()
        pv, pt = self._get_pca_pair()
        values = getattr(self.manager, "values_buffer", None) if with_values else None
        if values is not None and values.device != self.device:
            raise ValueError("values_buffer must be device-resident for the ALUT gather")
        return _alut.make_tables(self.manager.keys_buffer, self.manager.raw_keys_buffer, values,
                                 pv["proj"], pv["bias"], pt["proj"], pt["bias"])

    def _scratch(self, tables, q, s):
        """Zero-initialised kernel workspace, grown like the reference's _ensure_workspace."""
        cq, cs = self._alut_ws_shape
        if self._alut_ws is None or q > cq or s > cs:
            cq = max(q, cq, 128)
            cq = (cq + 127) // 128 * 128
            cs = max(s, cs)
            nbytes = int(self._lib.alut_workspace_size(tables, cq, cs))
            if nbytes == 0:
                raise ValueError("invalid table description")
            self._alut_ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._alut_ws_shape = (cq, cs)
        return self._alut_ws

    def device_errors(self, clear=True):
        """Device error bits (ALUT_ERR_*) accumulated in this engine's workspace since the last
        clear; synchronises the current stream."""
        if self._alut_ws is None:
            return 0
        return _alut.device_errors(self._alut_ws.data_ptr(), self._alut_ws.numel(), self.device, clear)

    def check_device_errors(self, what="ALUT"):
        _alut.raise_device_errors(self.device_errors(clear=True), what)

    def _ensure_workspace(self, batch_size, top_k):
        if batch_size > self.workspace_capacity or self.workspace.get("top_k") != top_k:
            cap = max(batch_size, 128)
            cap = (cap + 127) // 128 * 128
            dev = self.device
            self.workspace = {
                "top_k": top_k,
                "on_hit": torch.zeros((cap, top_k), dtype=torch.bool, device=dev),
                "off_hit": torch.zeros((cap, top_k), dtype=torch.bool, device=dev),
                "off_idx": torch.zeros((cap, top_k), dtype=torch.long, device=dev),
                "on_idx": torch.full((cap,), -1, dtype=torch.long, device=dev),
                "on_slot": torch.zeros((cap, top_k), dtype=torch.long, device=dev),
                "reuse": torch.zeros((cap, top_k), dtype=torch.bool, device=dev),
            }
            self.workspace_capacity = cap

    def _search_into(self, hidden_states, selected_experts, is_vision_mask, reuse_mask, out_hit,
                     out_idx, *, keyset, normalize, cmp_ge, thr_vision, thr_text):
        """One alut_search call writing every (token, slot) of out_hit / out_idx."""
        bs, top_k = selected_experts.shape
        if bs == 0 or top_k == 0:
            return
        x = hidden_states if hidden_states.stride(-1) == 1 else hidden_states.contiguous()
        sel = selected_experts if selected_experts.dtype == torch.int64 else selected_experts.long()
        if sel.stride(-1) != 1:
            sel = sel.contiguous()
        vis = is_vision_mask.reshape(-1)
        if vis.dtype != torch.bool:
            vis = vis.bool()
        vis = vis.contiguous()
        reuse = reuse_mask
        if reuse is not None and (reuse.dtype != torch.bool or reuse.stride(-1) != 1):
            reuse = reuse.bool().contiguous()
        if out_hit.stride() != out_idx.stride() or out_hit.stride(-1) != 1:
            raise ValueError("out_hit / out_idx must share strides with unit inner stride")
        tables = self._tables(shape=(bs, top_k), keyset=keyset)
        ws = self._scratch(tables, bs, top_k)
        batch = _alut.make_batch(x, sel, vis, reuse)
        params = _alut.make_params(keyset, normalize, cmp_ge, thr_vision, thr_text,
                                   CacheConfig.OFFLINE_COSINE_EPS)
        rc = self._lib.alut_search(tables, batch, params, None, out_hit.data_ptr(), out_idx.data_ptr(),
                                   out_hit.stride(0), ws.data_ptr(), ws.numel(),
                                   _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_search")
        if CacheConfig.ALUT_CHECK_ERRORS:
            self.check_device_errors("alut_search")

    def _new_outputs(self, selected_experts):
        bs, top_k = selected_experts.shape
        return (torch.zeros((bs, top_k), dtype=torch.bool, device=self.device),
                torch.zeros((bs, top_k), dtype=torch.long, device=self.device))

    # ---- public API (search.py:699-1105) ------------------------------------------------
    def search_prefill_offline(self, layer_idx, hidden_states, selected_experts, is_vision_mask, reuse_mask):
        hit, idx = self._new_outputs(selected_experts)
        self._search_into(hidden_states, selected_experts, is_vision_mask, reuse_mask, hit, idx,
                          keyset=_alut.KEYS_NORMALISED, normalize=True, cmp_ge=True,
                          thr_vision=CacheConfig.OFFLINE_COSINE_THRESHOLD_VISION,
                          thr_text=CacheConfig.OFFLINE_COSINE_THRESHOLD_TEXT)
        return hit, idx

    def search_prefill_offline_dot(self, layer_idx, hidden_states, selected_experts, is_vision_mask, reuse_mask):
        hit, idx = self._new_outputs(selected_experts)
        thr = float(CacheConfig.OFFLINE_DOT_THRESHOLD)
        self._search_into(hidden_states, selected_experts, is_vision_mask, reuse_mask, hit, idx,
                          keyset=_alut.KEYS_RAW, normalize=False, cmp_ge=False, thr_vision=thr, thr_text=thr)
        return hit, idx

    def search_decode_offline(self, layer_idx, hidden_states, selected_experts, is_vision_mask, reuse_mask):
        hit, idx = self._new_outputs(selected_experts)
        self._search_into(hidden_states, selected_experts, is_vision_mask, reuse_mask, hit, idx,
                          keyset=_alut.KEYS_NORMALISED, normalize=False, cmp_ge=True, thr_vision=0.0,
                          thr_text=0.0)
        return hit, idx

    def search_decode_offline_dot(self, layer_idx, hidden_states, selected_experts, is_vision_mask, reuse_mask):
        return self.search_prefill_offline_dot(layer_idx, hidden_states, selected_experts, is_vision_mask,
                                               reuse_mask)

    def _online_valid_size(self):
        m = self.manager
        if getattr(m, "online_keys", None) is None or getattr(m, "online_expert_ids", None) is None:
            return 0
        return m.online_size if m.online_full else m.online_ptr

    def _search_online_into(self, hidden_states, target_eids, out_on_hit, out_on_idx, out_on_slot):
        """Online window lookup (search.py:778-806) in one kernel (``alut_online_search``):
        best of the recent tokens by dot product in the window dtype, valid iff > 0, then
        the first cached slot holding each target expert."""
        n = self._online_valid_size()
        if n == 0 or target_eids.shape[1] == 0:
            return False
        keys = self.manager.online_keys
        eids = self.manager.online_expert_ids
        x = hidden_states if hidden_states.stride(-1) == 1 else hidden_states.contiguous()
        if x.dtype != keys.dtype:
            x = x.to(keys.dtype)
        tgt = target_eids if target_eids.dtype == torch.int64 else target_eids.long()
        if tgt.stride(-1) != 1:
            tgt = tgt.contiguous()
        if eids.dtype != torch.int64 or not eids.is_contiguous() or keys.stride(-1) != 1:
            raise ValueError("online window: keys [N,H] with unit inner stride, expert ids int64 [N,T] contiguous")
        if out_on_hit.stride() != out_on_slot.stride() or out_on_hit.stride(-1) != 1:
            raise ValueError("online outputs: on_hit / on_slot must share strides with unit inner stride")
        bs, s = tgt.shape
        rc = self._lib.alut_online_search(bs, x.shape[-1], n, eids.shape[1], s, x.data_ptr(), _alut.dtype_code(x.dtype),
                                          x.stride(0), keys.data_ptr(), _alut.dtype_code(keys.dtype), keys.stride(0),
                                          eids.data_ptr(), tgt.data_ptr(), tgt.stride(0), out_on_hit.data_ptr(),
                                          out_on_idx.data_ptr(), out_on_slot.data_ptr(), out_on_hit.stride(0),
                                          _alut.stream_ptr(self.device))
        _alut.check(rc, "alut_online_search")
        return True

    def search_decode_hybrid(self, layer_idx, hidden_states, selected_experts, is_vision_mask, keep_k=None):
        bs, top_k = selected_experts.shape
        keep_k = CacheConfig.KEEP_K if keep_k is None else keep_k
        keep_k = max(0, min(int(keep_k), top_k))
        self._ensure_workspace(bs, top_k)
        w = self.workspace
        on_hit, off_hit, off_idx = w["on_hit"][:bs], w["off_hit"][:bs], w["off_idx"][:bs]
        on_idx, on_slot, reuse = w["on_idx"][:bs], w["on_slot"][:bs], w["reuse"][:bs]
        on_hit.zero_()
        off_hit.zero_()
        off_idx.zero_()
        on_idx.fill_(-1)
        on_slot.zero_()
        reuse.zero_()
        if top_k - keep_k <= 0:
            return on_hit, on_idx, off_hit, off_idx, on_slot
        has_online = self._search_online_into(hidden_states, selected_experts[:, keep_k:], on_hit[:, keep_k:],
                                              on_idx, on_slot[:, keep_k:])
        if has_online:
            reuse[:, keep_k:].copy_(~on_hit[:, keep_k:])
        else:
            reuse[:, keep_k:].fill_(True)
        self._search_into(hidden_states, selected_experts, is_vision_mask, reuse, off_hit, off_idx,
                          keyset=_alut.KEYS_NORMALISED, normalize=False, cmp_ge=True, thr_vision=0.0,
                          thr_text=0.0)
        return on_hit, on_idx, off_hit, off_idx, on_slot

    def search_decode_offline_bs1_into(self, hidden_state, selected_experts_row, is_vision, keep_k,
                                       out_off_hit, out_off_idx):
        top_k = int(selected_experts_row.shape[0])
        out_off_hit.zero_()
        out_off_idx.zero_()
        if top_k == 0 or keep_k >= top_k:
            return
        self._ensure_workspace(1, top_k)
        reuse = self.workspace["reuse"][:1]
        reuse.zero_()
        reuse[:, keep_k:] = True
        thr = float(CacheConfig.OFFLINE_DOT_THRESHOLD)
        self._search_into(hidden_state.view(1, -1), selected_experts_row.view(1, top_k), is_vision.view(1),
                          reuse, out_off_hit.view(1, top_k), out_off_idx.view(1, top_k),
                          keyset=_alut.KEYS_RAW, normalize=False, cmp_ge=False, thr_vision=thr, thr_text=thr)

    def search_decode_hybrid_bs1_into(self, hidden_state, selected_experts_row, is_vision, keep_k,
                                      out_on_hit, out_on_idx, out_off_hit, out_off_idx, out_on_slot):
        top_k = int(selected_experts_row.shape[0])
        out_on_hit.zero_()
        out_on_idx.fill_(-1)
        out_off_hit.zero_()
        out_off_idx.zero_()
        out_on_slot.zero_()
        if top_k - keep_k <= 0:
            return
        x = hidden_state.view(1, -1)
        sel = selected_experts_row.view(1, top_k)
        self._ensure_workspace(1, top_k)
        reuse = self.workspace["reuse"][:1]
        reuse.zero_()
        has_online = self._search_online_into(x, sel[:, keep_k:], out_on_hit[keep_k:].view(1, -1),
                                              out_on_idx.view(1), out_on_slot[keep_k:].view(1, -1))
        if has_online:
            reuse[:, keep_k:].copy_(~out_on_hit[keep_k:].view(1, -1))
        else:
            reuse[:, keep_k:].fill_(True)
        self._search_into(x, sel, is_vision.view(1), reuse, out_off_hit.view(1, top_k),
                          out_off_idx.view(1, top_k), keyset=_alut.KEYS_NORMALISED, normalize=False,
                          cmp_ge=True, thr_vision=0.0, thr_text=0.0)

    # ---- fused lookup (search + gather + weighted accumulate) --------------------------
    def lookup_combine(self, hidden_states, selected_experts, is_vision_mask, reuse_mask, routing_weights,
                       *, compute_mask=None, out=None, variant="prefill_dot", renorm="to_one",
                       return_hits=False, hit_out=None, idx_out=None, computed=None):
        """Search every reuse slot, then out[t] (+)= sum over hits of w~[t,s] * value row.

        ``variant`` picks the search semantics of one of the methods above ("prefill",
        "prefill_dot", "decode", "decode_dot"); ``renorm`` is "none", "to_one" (Qwen3-VL
        combine, cached_layers.py:463-465) or "to_rowsum" (DeepSeek-VL2,
        deepseek_layers.py:715-727). ``out`` (accumulated into when given) defaults to a
        new [bs, H] tensor of the value dtype. ``hit_out`` / ``idx_out`` ([bs, top_k] bool /
        int64, unit inner stride, shared strides) receive the hits and indices in place;
        ``return_hits`` allocates them instead. ``computed`` ([bs, top_k, H] in the value
        dtype, the wrapper's collected expert outputs) adds the computed slots' outputs with
        the same renormalised weights, making the call the layer's whole combine
        (cached_layers.py:452-465); it needs ``compute_mask``.
        """
        rules = {
            "prefill": (_alut.KEYS_NORMALISED, True, True, CacheConfig.OFFLINE_COSINE_THRESHOLD_VISION,
                        CacheConfig.OFFLINE_COSINE_THRESHOLD_TEXT),
            "prefill_dot": (_alut.KEYS_RAW, False, False, CacheConfig.OFFLINE_DOT_THRESHOLD,
                            CacheConfig.OFFLINE_DOT_THRESHOLD),
            "decode": (_alut.KEYS_NORMALISED, False, True, 0.0, 0.0),
        }
        rules["decode_dot"] = rules["prefill_dot"]
        keyset, normalize, cmp_ge, tv, tt = rules[variant]
        rn = {"none": _alut.RENORM_NONE, "to_one": _alut.RENORM_TO_ONE, "to_rowsum": _alut.RENORM_TO_ROWSUM}[renorm]
        bs, top_k = selected_experts.shape
        values = self.manager.values_buffer
        accumulate = out is not None
        if out is None:
            out = torch.empty((bs, values.shape[-1]), dtype=values.dtype, device=self.device)
        hit, idx = self._new_outputs(selected_experts) if return_hits else (None, None)
        if hit_out is not None or idx_out is not None:
            if hit_out is None or idx_out is None or hit_out.shape != selected_experts.shape or \
                    idx_out.shape != selected_experts.shape or hit_out.stride() != idx_out.stride() or \
                    hit_out.stride(-1) != 1 or hit_out.dtype != torch.bool or idx_out.dtype != torch.int64:
                raise ValueError("hit_out / idx_out: [bs, top_k] bool and int64 with shared unit-inner strides")
            hit, idx = hit_out, idx_out
        if bs and top_k:
            w = routing_weights if routing_weights.dtype == torch.float32 else routing_weights.float()
            w = w if w.stride(-1) == 1 else w.contiguous()
            comp = compute_mask
            if comp is not None and (comp.dtype != torch.bool or comp.stride(-1) != 1):
                comp = comp.bool().contiguous()
            sel = selected_experts if selected_experts.dtype == torch.int64 else selected_experts.long()
            sel = sel if sel.stride(-1) == 1 else sel.contiguous()
            vis = is_vision_mask.reshape(-1).bool().contiguous()
            x = hidden_states if hidden_states.stride(-1) == 1 else hidden_states.contiguous()
            reuse = reuse_mask
            if reuse is not None and (reuse.dtype != torch.bool or reuse.stride(-1) != 1):
                reuse = reuse.bool().contiguous()
            tables = self._tables(with_values=True, shape=(bs, top_k), keyset=keyset)
            ws = self._scratch(tables, bs, top_k)
            batch = _alut.make_batch(x, sel, vis, reuse)  # x, sel, vis, reuse stay referenced
            params = _alut.make_params(keyset, normalize, cmp_ge, tv, tt, CacheConfig.OFFLINE_COSINE_EPS)
            hs = top_k if hit is None else hit.stride(0)
            if computed is not None:
                if comp is None:
                    raise ValueError("computed expert outputs need compute_mask")
                if computed.shape != (bs, top_k, values.shape[-1]) or computed.dtype != values.dtype or \
                        computed.stride(-1) != 1:
                    raise ValueError("computed: [bs, top_k, H] in the value dtype with unit inner stride")
                rc = self._lib.alut_lookup_combine_experts(
                    tables, batch, params, w.data_ptr(), w.stride(0), comp.data_ptr(), comp.stride(0),
                    computed.data_ptr(), computed.stride(0), computed.stride(1), rn, int(accumulate), out.data_ptr(),
                    out.stride(0), _alut.dtype_code(out.dtype), _alut.ptr(hit), _alut.ptr(idx), hs, ws.data_ptr(),
                    ws.numel(), _alut.stream_ptr(self.device))
                _alut.check(rc, "alut_lookup_combine_experts")
            else:
                rc = self._lib.alut_lookup_combine(
                    tables, batch, params, w.data_ptr(), w.stride(0), _alut.ptr(comp),
                    0 if comp is None else comp.stride(0), rn, int(accumulate), out.data_ptr(), out.stride(0),
                    _alut.dtype_code(out.dtype), _alut.ptr(hit), _alut.ptr(idx), hs, ws.data_ptr(), ws.numel(),
                    _alut.stream_ptr(self.device))
                _alut.check(rc, "alut_lookup_combine")
            if CacheConfig.ALUT_CHECK_ERRORS:
                self.check_device_errors("alut_lookup_combine")
        elif not accumulate:
            out.zero_()
        return (out, hit, idx) if return_hits else out
