"""The router oracle (oracle/route.py) pinned to fixtures made by the reference's own
qwen_topk_softmax and keep-mask builders (tests/golden/make_golden_route.py), and to the
reference's known-answer tests (table_moe/skip/test_pruning.py:109-121)."""
import json

import numpy as np
import pytest

import oracle.route as rt
from parity import GOLDEN, check_route, load_route, route_names, route_oracle


@pytest.mark.parametrize("name", route_names())
def test_route_oracle_matches_reference(name):
    meta, d = load_route(name)
    # Top-k softmax against the reference's.
    w, s, _, p, _, _ = route_oracle(meta, d)
    check_route(w, s, None, d["weights"], d["sel"], None, p, what=name)
    # Keep mask from the reference's own routing (equal values make the reference's top-k
    # order, and with it the expert sums, depend on its sort).
    _, _, keep, _, sums, kept = route_oracle(meta, d, weights=d["weights"], sel=d["sel"])
    check_route(d["weights"], d["sel"], keep, d["weights"], d["sel"], d["keep"], p, sums, kept, what=name)


def test_route_known_answers():
    ka = json.loads((GOLDEN / "route_known_answer.json").read_text())
    keep = rt.fixed_keep_mask(np.array(ka["fixed_keep_sel"]), ka["fixed_keep_k"])
    assert keep.tolist() == ka["fixed_keep_mask"]
    # keep_k None keeps every slot, keep_k beyond top_k is clamped.
    assert rt.fixed_keep_mask(np.zeros((2, 3), np.int64), None).all()
    assert rt.fixed_keep_mask(np.zeros((2, 3), np.int64), 9).all()


def test_prefill_keep_keeps_at_least_one_expert():
    sel = np.array([[0, 1], [2, 3]])
    w = np.array([[0.6, 0.4], [0.9, 0.1]], np.float32)
    keep, kept, sums = rt.prefill_keep_mask(sel, w, 4, 0.0)
    assert kept.tolist() == [2] and keep.sum() == 1
