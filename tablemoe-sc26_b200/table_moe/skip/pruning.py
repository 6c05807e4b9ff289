"""Keep masks of the skip/lookup split, drop-in for the reference's
``table_moe/skip/pruning.py`` (same functions, arguments and results).

``build_prefill_keep_mask`` runs the ``alut_keep_mask`` kernels (fixed-point expert sums,
ranking, mask; device tensors only). ``build_fixed_keep_mask`` / ``build_decode_keep_mask``
are a slice assignment and ``renormalize_surviving_weights`` a few elementwise device ops:
on the lookup path the renormalisation runs inside the combine kernel
(``alut_combine`` / ``alut_lookup_combine``), and the fixed mask inside ``alut_route``.
"""
from __future__ import annotations

import torch

from ..cache_engine import _alut


def build_fixed_keep_mask(selected_experts: torch.Tensor, keep_k: int | None) -> torch.Tensor:
    keep = torch.zeros_like(selected_experts, dtype=torch.bool)
    if selected_experts.numel() == 0:
        return keep
    k = selected_experts.shape[1] if keep_k is None else max(0, min(int(keep_k), selected_experts.shape[1]))
    if k > 0:
        keep[:, :k] = True
    return keep


def build_decode_keep_mask(selected_experts: torch.Tensor, keep_k: int | None) -> torch.Tensor:
    return build_fixed_keep_mask(selected_experts, keep_k)


def build_prefill_keep_mask(selected_experts, routing_weights, attn_scores, num_experts, keep_rate):
    if selected_experts.numel() == 0:
        return torch.zeros_like(selected_experts, dtype=torch.bool)
    if selected_experts.device.type != "cuda":
        raise ValueError("build_prefill_keep_mask: CUDA tensors only (the ALUT path has no CPU kernels)")
    from ..ops.qwen_topk_softmax import _workspace

    dev = selected_experts.device
    sel = selected_experts.to(torch.int64).contiguous()
    w = routing_weights.to(device=dev, dtype=torch.float32).contiguous()
    q, k = sel.shape
    attn = None
    if attn_scores is not None and attn_scores.numel() == q:
        attn = attn_scores.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    comp = torch.empty(q, k, dtype=torch.bool, device=dev)
    reuse = torch.empty(q, k, dtype=torch.bool, device=dev)
    ws = _workspace(dev, int(num_experts))
    rc = _alut.load().alut_keep_mask(q, int(num_experts), k, sel.data_ptr(), w.data_ptr(), k, _alut.ptr(attn),
                                     float(keep_rate), comp.data_ptr(), reuse.data_ptr(), k, ws.data_ptr(),
                                     ws.numel(), _alut.stream_ptr(dev))
    _alut.check(rc, "alut_keep_mask")
    return comp


def renormalize_surviving_weights(routing_weights, keep_mask, target_row_sum=None):
    pruned = routing_weights * keep_mask.to(routing_weights.dtype)
    kept = pruned.sum(dim=-1, keepdim=True)
    target = torch.ones_like(kept) if target_row_sum is None else target_row_sum.to(routing_weights.dtype)
    out = torch.zeros_like(routing_weights)
    valid = kept.squeeze(-1) > 0
    if valid.any():
        out[valid] = (pruned[valid] / kept[valid]) * target[valid]
    return out
