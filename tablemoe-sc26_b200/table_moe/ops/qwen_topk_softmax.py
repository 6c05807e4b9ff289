"""Top-k softmax routing on the ``alut_route`` kernel of ``libalut.so``.

Drop-in for the reference's ``table_moe/ops/qwen_topk_softmax.py:122-153``: same name,
arguments and results (fp32 weights [Q, k] in descending order, int64 expert ids [Q, k];
``normalize_topk`` divides the weights by their sum clamped at 1e-20). There is no torch
fallback: the logits must be CUDA tensors and the library must load.

``route_for_lookup`` is new: the same routing plus the keep mask of the layer
(``table_moe/skip/pruning.py``) in one launch sequence, producing exactly the inputs of
``VectorSearchEngine.lookup_combine`` (weights, selected experts, compute mask, reuse mask).
"""
from __future__ import annotations

import torch

from ..cache_engine import _alut

_WORKSPACES = {}


def _workspace(device, num_experts):
    """Zeroed once per (device, expert count); the kernels leave it zeroed."""
    key = (device, num_experts)
    ws = _WORKSPACES.get(key)
    if ws is None:
        n = int(_alut.load().alut_route_workspace_size(num_experts))
        if n == 0:
            raise ValueError(f"unsupported expert count {num_experts}")
        ws = torch.zeros(n, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def _check_logits(router_logits):
    if router_logits.dim() != 2:
        raise ValueError(f"qwen_topk_softmax expects 2D logits, got {tuple(router_logits.shape)}")
    if router_logits.device.type != "cuda":
        raise ValueError("router logits must be a CUDA tensor (the ALUT router has no CPU path)")
    x = router_logits if router_logits.stride(-1) == 1 else router_logits.contiguous()
    return x


def route_for_lookup(router_logits, top_k, *, normalize_topk=False, keep="fixed", keep_k=None, keep_rate=0.6,
                     attn_scores=None):
    """(weights [Q,k] f32, selected_experts [Q,k] int64, compute_mask [Q,k] bool,
    reuse_mask [Q,k] bool). ``keep``: "fixed" (the first ``keep_k`` slots computed,
    build_fixed_keep_mask / build_decode_keep_mask; None keeps all) or "importance"
    (build_prefill_keep_mask with ``keep_rate`` and optional per-token ``attn_scores``)."""
    x = _check_logits(router_logits)
    q, e = x.shape
    dev = x.device
    w = torch.empty(q, top_k, dtype=torch.float32, device=dev)
    sel = torch.empty(q, top_k, dtype=torch.int64, device=dev)
    comp = torch.empty(q, top_k, dtype=torch.bool, device=dev)
    reuse = torch.empty(q, top_k, dtype=torch.bool, device=dev)
    mode = {"fixed": 0, "importance": 1}[keep]
    attn = None
    if mode == 1 and attn_scores is not None and attn_scores.numel() == q:
        attn = attn_scores.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    ws = _workspace(dev, e)
    kk = -1 if keep_k is None else int(keep_k)
    rc = _alut.load().alut_route(q, e, int(top_k), x.data_ptr(), _alut.dtype_code(x.dtype), x.stride(0),
                                 int(bool(normalize_topk)), mode, max(kk, 0) if kk >= 0 else -1, float(keep_rate),
                                 _alut.ptr(attn), w.data_ptr(), sel.data_ptr(), comp.data_ptr(), reuse.data_ptr(),
                                 top_k, ws.data_ptr(), ws.numel(), _alut.stream_ptr(dev))
    _alut.check(rc, "alut_route")
    return w, sel, comp, reuse


def qwen_topk_softmax(router_logits: torch.Tensor, top_k: int, *, normalize_topk: bool = False):
    w, sel, _, _ = route_for_lookup(router_logits, top_k, normalize_topk=normalize_topk, keep="fixed", keep_k=None)
    return w, sel
