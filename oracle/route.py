"""CPU restatement of the router prologue (TEST INFRASTRUCTURE ONLY: the parity checker of
``alut_route``; the product path never imports it).

Follows the reference project fanyalun/tablemoe-sc26:
  * ``table_moe/ops/qwen_topk_softmax.py:117-119`` (``_fallback_topk_softmax``):
    softmax in fp32, then the top_k largest in descending order; ``:150-151``: with
    normalize_topk, weights / max(sum, 1e-20);
  * ``table_moe/skip/pruning.py:4-15`` ``build_fixed_keep_mask`` and ``:51``
    ``build_decode_keep_mask``;
  * ``table_moe/skip/pruning.py:18-48`` ``build_prefill_keep_mask``.
Tie rules where the reference leaves the order open (``torch.topk``, ``torch.argsort``
on equal values): lower expert id first; the parity tests exempt such near-ties.
"""
from __future__ import annotations

import numpy as np


def topk_softmax(logits, top_k, normalize_topk=False):
    """(weights [Q,k] f32, sel [Q,k] int64, probs [Q,E] f32)."""
    x = np.asarray(logits, np.float32)
    m = x.max(axis=1, keepdims=True)
    e = np.exp(x - m, dtype=np.float32)
    p = (e / e.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    order = np.argsort(-p, axis=1, kind="stable")[:, :top_k]
    w = np.take_along_axis(p, order, axis=1)
    if normalize_topk:
        tot = np.maximum(w.sum(axis=1, keepdims=True, dtype=np.float32), np.float32(1e-20))
        w = (w / tot).astype(np.float32)
    return w.astype(np.float32), order.astype(np.int64), p


def fixed_keep_mask(sel, keep_k):
    sel = np.asarray(sel)
    keep = np.zeros(sel.shape, bool)
    if sel.size == 0:
        return keep
    k = sel.shape[1] if keep_k is None else max(0, min(int(keep_k), sel.shape[1]))
    keep[:, :k] = True
    return keep


def expert_scores(sel, weights, num_experts, attn=None):
    """Per-expert importance sums in fp64 (pruning.py:29-35; the per-slot term in fp32)."""
    sel = np.asarray(sel)
    w = np.asarray(weights, np.float32)
    if attn is not None:
        terms = (np.asarray(attn, np.float32)[:, None] * w).astype(np.float32)
    else:
        terms = (w / np.float32(max(sel.shape[0], 1))).astype(np.float32)
    sums = np.zeros(num_experts, np.float64)
    np.add.at(sums, sel.reshape(-1), terms.reshape(-1).astype(np.float64))
    return sums


def prefill_keep_mask(sel, weights, num_experts, keep_rate, attn=None):
    """(keep mask, kept expert ids in rank order, per-expert sums)."""
    sel = np.asarray(sel)
    if sel.size == 0:
        return np.zeros(sel.shape, bool), np.zeros(0, np.int64), np.zeros(num_experts)
    sums = expert_scores(sel, weights, num_experts, attn)
    active = np.unique(sel)
    order = active[np.lexsort((active, -sums[active]))]  # larger sum first, lower id on ties
    keep_n = min(max(1, int(len(active) * keep_rate)), len(active))
    kept = order[:keep_n]
    return np.isin(sel, kept), kept, sums
