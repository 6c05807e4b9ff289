"""Generate the golden fixtures of the router prologue from the reference implementation.

Run where the reference project (fanyalun/tablemoe-sc26) is checked out:

    python tests/golden/make_golden_route.py --reference /path/to/tablemoe-sc26

It calls the reference's own ``table_moe.ops.qwen_topk_softmax.qwen_topk_softmax`` (on CPU
tensors it takes its torch path: softmax in fp32 + ``torch.topk``) and the keep-mask
builders of ``table_moe/skip/pruning.py`` (``build_fixed_keep_mask``,
``build_decode_keep_mask``, ``build_prefill_keep_mask``), and writes ``route_*.npz`` beside
this file: the logits (fp32), optional attention scores, the reference's weights, expert
ids and keep mask. The tests only read the ``.npz`` files.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def case(ref, name, *, Q, E, k, seed, normalize=False, mode="fixed", keep_k=3, keep_rate=0.6, attn=False,
         zipf=None, integer=False, dtype="float32"):
    topk_softmax, pruning = ref
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(Q, E, generator=g) * 2
    if zipf:
        prior = torch.arange(1, E + 1, dtype=torch.float32) ** (-zipf)
        logits = prior.log() - torch.log(-torch.log(torch.rand(Q, E, generator=g)))
    if integer:  # many equal logits: ties inside the top-k
        logits = torch.randint(0, 4, (Q, E), generator=g).float()
    if dtype == "bfloat16":
        logits = logits.to(torch.bfloat16)
    attn_scores = torch.rand(Q, generator=g) if attn else None
    w, sel = topk_softmax(logits, k, normalize_topk=normalize)
    if mode == "fixed":
        keep = pruning.build_decode_keep_mask(sel, keep_k)
    else:
        keep = pruning.build_prefill_keep_mask(sel, w, attn_scores, E, keep_rate)
    meta = dict(name=name, Q=Q, E=E, k=k, normalize=normalize, mode=mode, keep_k=keep_k, keep_rate=keep_rate,
                dtype=dtype)
    np.savez_compressed(
        HERE / f"route_{name}.npz", meta=json.dumps(meta),
        logits=logits.float().numpy(), attn=(attn_scores.numpy() if attn else np.zeros(0, np.float32)),
        weights=w.float().numpy(), sel=sel.long().numpy(), keep=keep.numpy())
    print(name, "kept slots", int(keep.sum()), "of", keep.numel())


def known_answers(pruning):
    """The reference's own known-answer tests (skip/test_pruning.py:109-121)."""
    sel = torch.tensor([[0, 1, 2, 3], [4, 5, 6, 7]])
    keep = pruning.build_fixed_keep_mask(sel, 2)
    w = torch.tensor([[0.4, 0.3, 0.2, 0.1]], dtype=torch.float32)
    ren = pruning.renormalize_surviving_weights(w, torch.tensor([[True, True, False, False]]))
    return {"fixed_keep_sel": sel.tolist(), "fixed_keep_k": 2, "fixed_keep_mask": keep.tolist(),
            "renorm_w": w.tolist(), "renorm_keep": [[True, True, False, False]], "renorm_out": ren.tolist()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from table_moe.ops.qwen_topk_softmax import qwen_topk_softmax
    from table_moe.skip import pruning

    ref = (qwen_topk_softmax, pruning)
    case(ref, "qwen_decode_keep3", Q=16, E=128, k=8, seed=1, mode="fixed", keep_k=3)
    case(ref, "qwen_decode_keep0", Q=5, E=128, k=8, seed=2, mode="fixed", keep_k=0)
    case(ref, "qwen_prefill_importance", Q=512, E=128, k=8, seed=3, mode="importance", keep_rate=0.6, zipf=1.1)
    case(ref, "prefill_attn_scores", Q=300, E=64, k=6, seed=4, mode="importance", keep_rate=0.5, attn=True)
    case(ref, "deepseek_normalized", Q=64, E=72, k=6, seed=5, normalize=True, mode="fixed", keep_k=8)
    case(ref, "bf16_logits_keep_rate_low", Q=40, E=60, k=4, seed=6, mode="importance", keep_rate=0.01,
         dtype="bfloat16")
    case(ref, "tied_logits", Q=32, E=16, k=4, seed=7, integer=True, mode="importance", keep_rate=0.6)
    (HERE / "route_known_answer.json").write_text(json.dumps(known_answers(pruning), indent=1))


if __name__ == "__main__":
    main()
