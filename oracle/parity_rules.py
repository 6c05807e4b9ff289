"""Parity rules of the ALUT path, as counting functions (TEST INFRASTRUCTURE: used by
``tests/parity.py`` as assertions and by the checker leg of ``bench.py``, which checks a
sample of what it timed; the product path never imports it).

Rules (tolerances stated where they are applied):
  * indices: bit-exact, except a slot whose chosen centroid's exact (fp64) score lies within
    1e-5 relative of the best score (fp32 tables), or within 2 ulp of the table dtype
    (16-bit tables, whose scores the reference rounds to that dtype);
  * hit masks: equal, except where the best score lies within that tolerance of the
    threshold;
  * misses carry index 0;
  * combined output: |got - ref| <= 1e-2 * |ref| + 1e-2 * max|ref| (bf16 output).
"""
from __future__ import annotations

import numpy as np

from . import oracle as orc

IDX_REL_TOL = 1e-5
COMBINE_RTOL = 1e-2
ULP = {"float32": 2.0 ** -23, "bfloat16": 2.0 ** -8, "float16": 2.0 ** -11}


def search_mismatches(got_hit, got_idx, ref_hit, ref_idx, q_low, keys, sel, is_vision, thr, dtype):
    """(list of slots breaking the rule, number of exempted near-tie slots)."""
    got_hit = np.asarray(got_hit).astype(bool)
    ref_hit = np.asarray(ref_hit).astype(bool)
    got_idx = np.asarray(got_idx)
    ref_idx = np.asarray(ref_idx)
    is_vision = np.asarray(is_vision).astype(bool)
    ulp = ULP[dtype]
    exempt = 0
    bad = []
    for t, s in zip(*np.nonzero((got_hit != ref_hit) | (got_hit & (got_idx != ref_idx)))):
        s_ref = orc.score(q_low, keys, sel, is_vision, t, s, int(ref_idx[t, s]))
        th = thr[0] if is_vision[t] else thr[1]
        if got_hit[t, s] != ref_hit[t, s]:
            best = s_ref if ref_hit[t, s] else orc.score(q_low, keys, sel, is_vision, t, s, int(got_idx[t, s]))
            tol = max(IDX_REL_TOL, 2 * ulp) * max(abs(th), abs(best), 1e-30)
            if abs(best - th) <= tol:
                exempt += 1
                continue
            bad.append((int(t), int(s), "hit", bool(got_hit[t, s]), bool(ref_hit[t, s]), best, th))
            continue
        s_got = orc.score(q_low, keys, sel, is_vision, t, s, int(got_idx[t, s]))
        tol = (IDX_REL_TOL if dtype == "float32" else 2 * ulp) * max(abs(s_ref), abs(s_got), 1e-30)
        if abs(s_ref - s_got) <= tol:
            exempt += 1
            continue
        bad.append((int(t), int(s), "idx", int(got_idx[t, s]), int(ref_idx[t, s]), s_got, s_ref))
    nz = np.nonzero(got_idx[~got_hit] != 0)[0]
    if nz.size:
        bad.append(("miss with a nonzero index", int(nz.size)))
    return bad, exempt


def combined_mismatches(got, ref):
    """Number of elements outside the combine tolerance, and the largest error."""
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    if ref.size == 0:
        return 0, 0.0
    scale = float(np.max(np.abs(ref)))
    err = np.abs(got - ref)
    tol = COMBINE_RTOL * np.abs(ref) + COMBINE_RTOL * scale + 1e-12
    return int(np.count_nonzero(err > tol)), float(err.max())


ROUTE_W_RTOL = 1e-5
ROUTE_TIE_RTOL = 1e-6
ROUTE_SUM_RTOL = 1e-5


def route_mismatches(got_w, got_sel, got_keep, ref_w, ref_sel, ref_keep, probs, sums=None, kept=None):
    """Slots breaking the router rules:
      * weights within 1e-5 relative (+1e-7) of the reference's;
      * expert ids equal, except where the two chosen probabilities are within 1e-6
        relative (the reference's top-k leaves the order of equal values open);
      * keep mask equal, except on slots whose expert id differs by such a tie, or whose
        expert's importance sum lies within 1e-5 relative of the sum at the keep boundary
        (``sums`` per expert and ``kept`` in rank order, importance mode)."""
    got_w, ref_w = np.asarray(got_w, np.float64), np.asarray(ref_w, np.float64)
    got_sel, ref_sel = np.asarray(got_sel), np.asarray(ref_sel)
    bad = []
    werr = np.abs(got_w - ref_w) > ROUTE_W_RTOL * np.abs(ref_w) + 1e-7
    for t, s in zip(*np.nonzero(werr)):
        bad.append(("weight", int(t), int(s), float(got_w[t, s]), float(ref_w[t, s])))
    tie = np.zeros(got_sel.shape, bool)
    for t, s in zip(*np.nonzero(got_sel != ref_sel)):
        pg, pr = float(probs[t, got_sel[t, s]]), float(probs[t, ref_sel[t, s]])
        if abs(pg - pr) <= ROUTE_TIE_RTOL * max(abs(pr), 1e-30):
            tie[t, s] = True
        else:
            bad.append(("expert", int(t), int(s), int(got_sel[t, s]), int(ref_sel[t, s])))
    if got_keep is not None:
        got_keep, ref_keep = np.asarray(got_keep, bool), np.asarray(ref_keep, bool)
        bounds = []
        if sums is not None and kept is not None and len(kept):
            bounds.append(sums[kept[-1]])
            rest = np.setdiff1d(np.unique(ref_sel), kept)
            if rest.size:
                bounds.append(np.max(sums[rest]))
        for t, s in zip(*np.nonzero(got_keep != ref_keep)):
            if tie[t, s]:
                continue
            e = int(got_sel[t, s])
            if sums is not None and any(abs(sums[e] - b) <= ROUTE_SUM_RTOL * max(abs(b), 1e-30) for b in bounds):
                continue
            bad.append(("keep", int(t), int(s), bool(got_keep[t, s]), bool(ref_keep[t, s])))
    return bad
