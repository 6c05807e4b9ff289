"""Fixture loading and the parity rules of the ALUT path, shared by the CPU and GPU tests.

Parity rules (stated with the tolerances used):
  * indices: bit-exact, except a slot whose top-2 fp64 score gap is below 1e-5 relative
    (fp32 tables) - there the chosen centroid's exact score must lie within 1e-5 relative
    of the best. For 16-bit tables the scores are compared after rounding to the table
    dtype (the reference's bmm output dtype), so a slot may differ where the two
    candidates' exact scores are within 2 ulp of that dtype.
  * hit masks: equal, except where the best score lies within the same tolerance of the
    threshold.
  * gathered rows: bit-exact.
  * combined output: |got - ref| <= 1e-2 * |ref| + 1e-2 * max|ref| (bf16 output).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

import oracle.oracle as orc
import oracle.parity_rules as rules

GOLDEN = Path(__file__).resolve().parent / "golden"

IDX_REL_TOL = rules.IDX_REL_TOL
COMBINE_RTOL = rules.COMBINE_RTOL
ULP = rules.ULP


def golden_names():
    """Search/combine fixtures (the online-window fixtures are online_*.npz)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("online_", "route_", "manager_")))


def online_names():
    return sorted(p.stem for p in GOLDEN.glob("online_*.npz"))


def load_online(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    return meta, {k: z[k] for k in z.files if k != "meta"}


def load_golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    d = {k: z[k] for k in z.files if k != "meta"}
    d["x"] = orc.bf16_to_f32(d["x_bf16"]).reshape(d["x_bf16"].shape)
    d["combined"] = orc.bf16_to_f32(d["combined_bf16"]).reshape(d["combined_bf16"].shape)
    d["values_f32"] = orc.bf16_to_f32(d["values_bf16"]).reshape(d["values_bf16"].shape)
    return meta, d


def variant_rule(variant):
    """(normalize query, key set, cmp_ge, thresholds source) of a reference entry point.

    search.py:808 search_prefill_offline: normalised query, keys_buffer, >= (0.6, 0.7)
    search.py:699 search_prefill_offline_dot: raw query, raw_keys_buffer, > OFFLINE_DOT_THRESHOLD
    search.py:715 search_decode_offline_dot: same as prefill_dot
    search.py:824 search_decode_offline (torch path): raw query, keys_buffer, >= 0
    search.py:839 search_decode_hybrid (no online window): raw query, keys_buffer, >= 0
    """
    if variant == "prefill_cos":
        return dict(normalize=True, keyset="norm", cmp_ge=True, thr=(0.6, 0.7))
    if variant in ("prefill_dot", "decode_dot"):
        return dict(normalize=False, keyset="raw", cmp_ge=False, thr=None)
    if variant in ("decode_cos", "decode_hybrid"):
        return dict(normalize=False, keyset="norm", cmp_ge=True, thr=(0.0, 0.0))
    raise ValueError(variant)


def case_inputs(meta, d):
    """Everything the oracle needs for a golden case."""
    rule = variant_rule(meta["variant"])
    thr = rule["thr"] if rule["thr"] is not None else (meta.get("dot_thr", 0.0),) * 2
    keys = d["keys_raw"] if rule["keyset"] == "raw" else d["keys_norm"]
    return rule, thr, keys


def check_search(got_hit, got_idx, ref_hit, ref_idx, q_low, keys, sel, is_vision, thr, dtype,
                 what=""):
    """Assert the index / hit parity rules; returns the number of exempted slots."""
    bad, exempt = rules.search_mismatches(got_hit, got_idx, ref_hit, ref_idx, q_low, keys, sel, is_vision, thr,
                                          dtype)
    assert not bad, f"{what}: {len(bad)} slots break the parity rule, first: {bad[:5]}"
    return exempt


def check_combined(got, ref, what=""):
    n, err = rules.combined_mismatches(got, ref)
    scale = float(np.max(np.abs(np.asarray(ref, np.float32)))) if np.size(ref) else 0.0
    assert n == 0, f"{what}: combine max err {err} (scale {scale})"


def check_online(got_hit, got_idx, got_slot, ref_hit, ref_idx, ref_slot, scores, what=""):
    """Online-window parity: exact, except for a token whose two best bf16 scores lie within
    2 bf16 ulp of each other (fp32 accumulation order): there the chosen entry's score must
    be within that tolerance of the best, and its hits follow the chosen entry."""
    got_hit, ref_hit = np.asarray(got_hit).astype(bool), np.asarray(ref_hit).astype(bool)
    got_idx, ref_idx = np.asarray(got_idx), np.asarray(ref_idx)
    bad = []
    for b in range(len(ref_idx)):
        if got_idx[b] == ref_idx[b]:
            if not (np.array_equal(got_hit[b], ref_hit[b]) and
                    np.array_equal(np.where(ref_hit[b], got_slot[b], 0), np.where(ref_hit[b], ref_slot[b], 0))):
                bad.append((b, "hits/slots"))
            continue
        best = scores[b].max()
        chosen = scores[b, got_idx[b]] if got_idx[b] >= 0 else -np.inf
        tol = 2 * ULP["bfloat16"] * max(abs(best), 1e-30)
        if got_idx[b] < 0 or ref_idx[b] < 0 or abs(best - chosen) > tol:
            bad.append((b, "idx", int(got_idx[b]), int(ref_idx[b])))
    assert not bad, f"{what}: {bad[:5]}"


def route_names():
    return sorted(p.stem for p in GOLDEN.glob("route_*.npz"))


def load_route(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    d = {k: z[k] for k in z.files if k != "meta"}
    if d["attn"].size == 0:
        d["attn"] = None
    return meta, d


def route_oracle(meta, d, weights=None, sel=None):
    """Oracle routing + keep mask of a route fixture (weights/sel: use these instead of the
    oracle's own top-k, to check a keep mask computed from them)."""
    import oracle.route as rt

    w, s, p = rt.topk_softmax(d["logits"], meta["k"], meta["normalize"])
    if weights is not None:
        w, s = weights, sel
    sums = kept = None
    if meta["mode"] == "fixed":
        keep = rt.fixed_keep_mask(s, meta["keep_k"])
    else:
        keep, kept, sums = rt.prefill_keep_mask(s, w, meta["E"], meta["keep_rate"], d["attn"])
    return w, s, keep, p, sums, kept


def check_route(got_w, got_sel, got_keep, ref_w, ref_sel, ref_keep, probs, sums=None, kept=None, what=""):
    bad = rules.route_mismatches(got_w, got_sel, got_keep, ref_w, ref_sel, ref_keep, probs, sums, kept)
    assert not bad, f"{what}: {len(bad)} router slots break the rule, first: {bad[:5]}"
