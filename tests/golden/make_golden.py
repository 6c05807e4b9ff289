"""Generate the golden fixtures of the ALUT path from the reference implementation itself.

Run in a container where the reference project (fanyalun/tablemoe-sc26) is checked out:

    python tests/golden/make_golden.py --reference /path/to/tablemoe-sc26

It imports the reference's own ``table_moe.cache_engine.search.VectorSearchEngine`` with
``HAS_TRITON`` patched to False (the torch path, which scans all K centroids), drives it
through a synthetic manager of the shape of the reference's ``DummyManager``
(``table_moe/cache_engine/test_search.py:11-26``), runs the reference's combine
(``table_moe/models/qwen3_vl_moe/cached_layers.py:455-465`` with
``table_moe/skip/pruning.py:55-73``) and writes one ``.npz`` per case next to this file:
inputs, the reference's (hit, idx), gathered rows and combined outputs. The reference is
not needed to *use* the fixtures; the tests only read the ``.npz`` files.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from unittest import mock

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


class SyntheticManager:
    """Attribute set the reference's VectorSearchEngine reads (test_search.py:11-26)."""

    def __init__(self, keys_raw, keys_norm, pca, values):
        self.device = torch.device("cpu")
        self.raw_keys_buffer = keys_raw
        self.keys_buffer = keys_norm
        self.pca = pca
        self.values_buffer = values
        self.online_keys = None
        self.online_expert_ids = None
        self.online_size = 0
        self.online_ptr = 0
        self.online_full = False


def make_case(ref, name, *, Q, S, E, K, L, H, dtype, variant, seed, vis_frac=0.5,
              plant=0.0, reuse_p=0.4, keep_k=None, all_reuse=False, no_reuse=False,
              renorm="qwen", qdist=(0.0, 1.0), dot_thr=0.0):
    search_mod, manager_mod, pruning = ref
    g = torch.Generator().manual_seed(seed)
    tdt = {"float32": torch.float32, "bfloat16": torch.bfloat16}[dtype]
    x = (torch.randn(Q, H, generator=g) * qdist[1] + qdist[0]).to(torch.bfloat16)
    is_vision = torch.rand(Q, generator=g) < vis_frac
    proj = []
    for _ in range(2):
        qm, _r = torch.linalg.qr(torch.randn(H, L, generator=g))
        proj.append(qm.contiguous())
    bias = [torch.randn(L, generator=g) * 0.1 for _ in range(2)]
    keys_raw = torch.randn(E, 2, K, L, generator=g)
    logits = torch.randn(Q, E, generator=g)
    probs = torch.softmax(logits, dim=-1)
    w, sel = torch.topk(probs, S, dim=-1)
    w = w.float()
    if plant > 0:
        # Plant near-duplicates: some keys are the projected queries plus small noise,
        # so that the cosine thresholds (0.6 / 0.7) are reached.
        xf = x.float()
        for t in range(Q):
            m = 0 if bool(is_vision[t]) else 1
            ql = xf[t] @ proj[m] + bias[m]
            for s in range(S):
                if torch.rand(1, generator=g).item() < plant:
                    k = int(torch.randint(0, K, (1,), generator=g))
                    keys_raw[sel[t, s], m, k] = ql + torch.randn(L, generator=g) * 0.3 * ql.norm() / L ** 0.5
    keys_raw = keys_raw.to(tdt)
    keys_norm = manager_mod._normalize_last_dim(keys_raw, 1e-6)
    values = (torch.randn(E, 2, K, H, generator=g) * 0.05).to(torch.bfloat16)
    if all_reuse:
        reuse = torch.ones(Q, S, dtype=torch.bool)
    elif no_reuse:
        reuse = torch.zeros(Q, S, dtype=torch.bool)
    elif keep_k is not None:
        reuse = torch.zeros(Q, S, dtype=torch.bool)
        reuse[:, keep_k:] = True
    else:
        reuse = torch.rand(Q, S, generator=g) < reuse_p
    compute = ~reuse
    pca = {"vision": {"proj": proj[0].to(tdt), "bias": bias[0].to(tdt)},
           "text": {"proj": proj[1].to(tdt), "bias": bias[1].to(tdt)}}
    mgr = SyntheticManager(keys_raw, keys_norm, pca, values)
    eng = search_mod.VectorSearchEngine(mgr)
    xin = x.to(tdt)  # addmm needs one dtype; bf16 -> fp32 is exact
    search_mod.CacheConfig.OFFLINE_DOT_THRESHOLD = float(dot_thr)
    with mock.patch.object(search_mod, "HAS_TRITON", False):
        if variant == "prefill_cos":
            hit, idx = eng.search_prefill_offline(0, xin, sel, is_vision, reuse)
        elif variant == "prefill_dot":
            hit, idx = eng.search_prefill_offline_dot(0, xin, sel, is_vision, reuse)
        elif variant == "decode_dot":
            hit, idx = eng.search_decode_offline_dot(0, xin, sel, is_vision, reuse)
        elif variant == "decode_cos":
            hit, idx = eng.search_decode_offline(0, xin, sel, is_vision, reuse)
        elif variant == "decode_hybrid":
            on_hit, on_idx, hit, idx, on_slot = eng.search_decode_hybrid(0, xin, sel, is_vision, keep_k=keep_k)
            hit, idx = hit.clone(), idx.clone()
        else:
            raise ValueError(variant)
    search_mod.CacheConfig.OFFLINE_DOT_THRESHOLD = 0.0
    # Gather (manager.py:212-213) and combine (cached_layers.py:455-465).
    rows, cols = torch.where(hit)
    mids = torch.where(is_vision[rows], 0, 1)
    gathered = values[sel[rows, cols], mids, idx[rows, cols]]
    collected = torch.zeros(Q, S, H, dtype=torch.bfloat16)
    collected[rows, cols] = gathered
    survivor = compute | hit
    if renorm == "qwen":
        ew = pruning.renormalize_surviving_weights(w, survivor).to(torch.bfloat16)
        combined = torch.bmm(ew.unsqueeze(1), collected).squeeze(1)
    else:  # deepseek_layers.py:715-727
        ew = pruning.renormalize_surviving_weights(w, survivor, target_row_sum=w.sum(dim=-1, keepdim=True))
        combined = collected.to(ew.dtype).mul_(ew.unsqueeze(-1)).sum(dim=1).to(torch.bfloat16)
    out = {
        "x_bf16": _bits(x),
        "is_vision": is_vision.numpy().astype(np.uint8),
        "proj": torch.stack([p.to(tdt).float() for p in proj]).numpy(),
        "bias": torch.stack([b.to(tdt).float() for b in bias]).numpy(),
        "values_bf16": _bits(values),
        "sel": sel.numpy().astype(np.int64),
        "weights": w.numpy().astype(np.float32),
        "reuse": reuse.numpy().astype(np.uint8),
        "compute": compute.numpy().astype(np.uint8),
        "hit": hit.numpy().astype(np.uint8),
        "idx": idx.numpy().astype(np.int64),
        "gather_rows": rows.numpy().astype(np.int64),
        "gather_cols": cols.numpy().astype(np.int64),
        "combined_bf16": _bits(combined),
    }
    # Only the key table the variant scores against is stored.
    if variant.endswith("_dot"):
        out["keys_raw"] = keys_raw.float().numpy()
    else:
        out["keys_norm"] = keys_norm.float().numpy()
    meta = dict(name=name, Q=Q, S=S, E=E, K=K, L=L, H=H, dtype=dtype, variant=variant,
                seed=seed, renorm=renorm, keep_k=keep_k, dot_thr=dot_thr)
    np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), **out)
    print(f"{name}: hits={int(hit.sum())}/{int(reuse.sum())} searched")
    return meta


def online_case(ref, name, *, B, H, size, topk_online, S, keep_k, n_valid, full, seed, dup=False,
                 negative=False, match_p=0.5):
    """The online window lookup (search.py:778-806, ``_search_decode_online_into``): bf16
    hidden states against the window's bf16 keys, first-index argmax, valid iff > 0, then
    the first cached slot holding each target expert."""
    search_mod, _, _ = ref
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, H, generator=g).to(torch.bfloat16)
    keys = torch.randn(size, H, generator=g).to(torch.bfloat16)
    if negative:  # every score < 0: no valid token
        keys = (-x.float().mean(0, keepdim=True).sign() * keys.float().abs()).to(torch.bfloat16)
    if dup:  # duplicate window entries: the first index must win
        keys[3] = keys[1]
        keys[7 % size] = keys[2]
        x[0] = keys[1]
        x[1] = keys[2]
    eids = torch.randint(0, 10, (size, topk_online), generator=g)
    eids[torch.rand(size, topk_online, generator=g) < 0.15] = -1
    sel = torch.randint(0, 10, (B, S), generator=g)
    # Route some target experts to ids present in the best window entry, so that slots hit.
    scores = (x.float() @ keys.float().T)[:, :n_valid]
    arg = scores.argmax(1)
    for b in range(B):
        for s in range(keep_k, S):
            if torch.rand(1, generator=g).item() < match_p:
                cand = eids[arg[b]][eids[arg[b]] >= 0]
                if cand.numel():
                    sel[b, s] = cand[int(torch.randint(0, cand.numel(), (1,), generator=g))]
    mgr = SyntheticManager(torch.zeros(1, 2, 1, 1), torch.zeros(1, 2, 1, 1),
                           {m: {"proj": torch.eye(1), "bias": torch.zeros(1)} for m in ("vision", "text")},
                           torch.zeros(1, 2, 1, 1, dtype=torch.bfloat16))
    mgr.online_keys, mgr.online_expert_ids = keys, eids
    mgr.online_size, mgr.online_full, mgr.online_ptr = size, full, (0 if full else n_valid)
    eng = search_mod.VectorSearchEngine(mgr)
    on_hit = torch.zeros(B, S - keep_k, dtype=torch.bool)
    on_idx = torch.full((B,), -1, dtype=torch.long)
    on_slot = torch.zeros(B, S - keep_k, dtype=torch.long)
    has = eng._search_decode_online_into(x, sel[:, keep_k:], on_hit, on_idx, on_slot)
    out = dict(x_bf16=_bits(x), keys_bf16=_bits(keys), eids=eids.numpy(), sel=sel.numpy(),
               on_hit=on_hit.numpy().astype(np.uint8), on_idx=on_idx.numpy(), on_slot=on_slot.numpy())
    meta = dict(name=name, B=B, H=H, size=size, topk_online=topk_online, S=S, keep_k=keep_k,
                n_valid=n_valid, full=full, has_online=bool(has))
    np.savez_compressed(HERE / f"online_{name}.npz", meta=json.dumps(meta), **out)
    print(f"online_{name}: valid={int((on_idx >= 0).sum())}/{B} hits={int(on_hit.sum())}")


def known_answer(ref):
    """The reference's own known-answer tests (test_search.py:36-89) as vectors."""
    search_mod, _, _ = ref
    keys = torch.zeros((2, 2, 2, 2))
    keys[0, 0] = torch.tensor([[1.0, 0.0], [-1.0, 0.0]])
    keys[1, 0] = torch.tensor([[0.0, 0.0], [-1.0, 0.0]])
    pca = {m: {"proj": torch.eye(2), "bias": torch.zeros(2)} for m in ("vision", "text")}
    mgr = SyntheticManager(keys, torch.zeros_like(keys), pca, torch.zeros(2, 2, 2, 4, dtype=torch.bfloat16))
    eng = search_mod.VectorSearchEngine(mgr)
    hs = torch.tensor([[1.0, 0.0], [1.0, 0.0]])
    sel = torch.tensor([[0], [1]])
    vis = torch.tensor([True, True])
    reuse = torch.tensor([[True], [True]])
    res = {}
    with mock.patch.object(search_mod, "HAS_TRITON", False):
        h1, i1 = eng.search_prefill_offline_dot(0, hs, sel, vis, reuse)
        h2, i2 = eng.search_decode_offline_dot(0, hs, sel, vis, reuse)
    res["prefill_dot"] = {"hit": h1.int().tolist(), "idx": i1.tolist()}
    res["decode_dot"] = {"hit": h2.int().tolist(), "idx": i2.tolist()}
    res["inputs"] = {"raw_keys": keys.tolist(), "hidden": hs.tolist(), "sel": sel.tolist(),
                     "is_vision": vis.int().tolist(), "reuse": reuse.int().tolist()}
    (HERE / "known_answer.json").write_text(json.dumps(res, indent=1))
    print("known_answer:", res["prefill_dot"], res["decode_dot"])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference project")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from table_moe.cache_engine import manager as manager_mod
    from table_moe.cache_engine import search as search_mod
    from table_moe.skip import pruning
    ref = (search_mod, manager_mod, pruning)
    known_answer(ref)
    # C1 of the benchmark configs (the reference's CPU-runnable case) with H cut to 512
    # to keep the fixture small; full-size C1 is checked against the pinned oracle.
    make_case(ref, "c1_prefill_dot_h512", Q=256, S=1, E=1, K=256, L=64, H=512, dtype="float32",
              variant="prefill_dot", seed=0, vis_frac=0.0, all_reuse=True)
    make_case(ref, "prefill_cos_mixed", Q=64, S=4, E=4, K=300, L=64, H=128, dtype="float32",
              variant="prefill_cos", seed=1, plant=0.5, reuse_p=0.6)
    make_case(ref, "decode_dot_k200", Q=16, S=8, E=9, K=200, L=32, H=128, dtype="float32",
              variant="decode_dot", seed=2, reuse_p=0.4)
    make_case(ref, "decode_cos_text", Q=16, S=8, E=9, K=130, L=40, H=128, dtype="float32",
              variant="decode_cos", seed=3, vis_frac=0.0, reuse_p=0.5)
    make_case(ref, "decode_hybrid_keep3", Q=8, S=8, E=8, K=100, L=32, H=128, dtype="float32",
              variant="decode_hybrid", seed=4, keep_k=3)
    make_case(ref, "prefill_dot_l96_deepseek", Q=48, S=6, E=6, K=140, L=96, H=160, dtype="float32",
              variant="prefill_dot", seed=5, renorm="deepseek", reuse_p=0.5)
    make_case(ref, "prefill_dot_bf16", Q=48, S=4, E=4, K=200, L=64, H=256, dtype="bfloat16",
              variant="prefill_dot", seed=6, reuse_p=0.5)
    make_case(ref, "prefill_cos_bf16", Q=48, S=4, E=4, K=160, L=64, H=256, dtype="bfloat16",
              variant="prefill_cos", seed=7, plant=0.5, reuse_p=0.6)
    make_case(ref, "no_reuse", Q=8, S=4, E=5, K=64, L=16, H=64, dtype="float32",
              variant="prefill_dot", seed=8, no_reuse=True)
    make_case(ref, "decode_dot_thr2", Q=16, S=4, E=5, K=96, L=16, H=64, dtype="float32",
              variant="decode_dot", seed=10, reuse_p=0.6, dot_thr=9.0)
    make_case(ref, "ragged_l12_k7", Q=5, S=3, E=4, K=7, L=12, H=40, dtype="float32",
              variant="prefill_dot", seed=9, reuse_p=0.7)
    # The online window (ONLINE_CACHE_SIZE 64, ONLINE_TOP_K 6, config.py:29-30).
    online_case(ref, "full64", B=16, H=256, size=64, topk_online=6, S=8, keep_k=3, n_valid=64, full=True,
                seed=40)
    online_case(ref, "partial5_bs1", B=1, H=2048, size=64, topk_online=6, S=8, keep_k=2, n_valid=5, full=False,
                seed=41, match_p=0.8)
    online_case(ref, "ties", B=4, H=128, size=16, topk_online=6, S=6, keep_k=1, n_valid=16, full=True, seed=42,
                dup=True)
    online_case(ref, "negative", B=4, H=64, size=8, topk_online=6, S=4, keep_k=1, n_valid=8, full=True, seed=43,
                negative=True)


if __name__ == "__main__":
    main()
