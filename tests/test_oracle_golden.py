"""The CPU oracle pinned against the reference's own outputs (tests/golden, made by
tests/golden/make_golden.py from the reference's torch path) and against the
reference's known-answer tests (table_moe/cache_engine/test_search.py:36-89)."""
import json

import numpy as np
import pytest

import oracle.oracle as orc
from parity import (GOLDEN, case_inputs, check_combined, check_online, check_search, golden_names, load_golden,
                    load_online, online_names)


@pytest.mark.parametrize("name", golden_names())
def test_oracle_search_matches_reference(name):
    meta, d = load_golden(name)
    rule, thr, keys = case_inputs(meta, d)
    q = orc.project(d["x"], d["is_vision"], d["proj"], d["bias"], dtype=meta["dtype"],
                    normalize=rule["normalize"])
    hit, idx, best, gap = orc.search(q, keys, d["sel"], d["is_vision"], d["reuse"], thr[0], thr[1],
                                     rule["cmp_ge"], meta["dtype"])
    check_search(hit, idx, d["hit"], d["idx"], q, keys, d["sel"], d["is_vision"], thr,
                 meta["dtype"], what=name)
    # Exact agreement on the hit masks of every slot whose score is clear of the threshold.
    assert hit.sum() == pytest.approx(d["hit"].sum(), abs=2)


@pytest.mark.parametrize("name", golden_names())
def test_oracle_gather_and_combine_match_reference(name):
    meta, d = load_golden(name)
    rows, cols = d["gather_rows"], d["gather_cols"]
    mids = np.where(d["is_vision"][rows] != 0, 0, 1)
    g = orc.gather(d["values_bf16"], d["sel"][rows, cols], mids, d["idx"][rows, cols])
    ref_rows = d["values_f32"][d["sel"][rows, cols], mids, d["idx"][rows, cols]]
    assert np.array_equal(g.view(np.uint32), ref_rows.view(np.uint32))
    renorm = 1 if meta["renorm"] == "qwen" else 2
    out = orc.combine(d["values_bf16"], d["sel"], d["is_vision"], d["hit"], d["idx"], d["weights"],
                      compute=d["compute"], renorm=renorm)
    check_combined(orc.bf16_to_f32(orc.bf16_bits(out)).reshape(out.shape), d["combined"], what=name)


def test_oracle_known_answers():
    ka = json.loads((GOLDEN / "known_answer.json").read_text())
    inp = ka["inputs"]
    keys = np.array(inp["raw_keys"], np.float32)
    hs = np.array(inp["hidden"], np.float32)
    sel = np.array(inp["sel"], np.int64)
    vis = np.array(inp["is_vision"], np.uint8)
    reuse = np.array(inp["reuse"], np.uint8)
    eye = np.stack([np.eye(2, dtype=np.float32)] * 2)
    q = orc.project(hs, vis, eye, np.zeros((2, 2), np.float32))
    hit, idx, _, _ = orc.search(q, keys, sel, vis, reuse, 0.0, 0.0, cmp_ge=False)
    assert hit.astype(int).tolist() == ka["prefill_dot"]["hit"] == ka["decode_dot"]["hit"]
    assert idx.tolist() == ka["prefill_dot"]["idx"]
    # Same inputs: hit iff max dot > 0 (test_search.py:62-64): token 0 hits idx 0, token 1 misses.
    assert hit[0, 0] and idx[0, 0] == 0 and not hit[1, 0]


def test_oracle_tie_takes_first_index():
    keys = np.zeros((1, 2, 5, 4), np.float32)
    keys[0, 1, 1] = [1, 0, 0, 0]
    keys[0, 1, 3] = [1, 0, 0, 0]
    q = np.array([[2, 0, 0, 0]], np.float32)
    hit, idx, _, gap = orc.search(q, keys, np.zeros((1, 1), np.int64), np.zeros(1, np.uint8))
    assert hit[0, 0] and idx[0, 0] == 1 and gap[0, 0] == 0.0


def test_oracle_zero_query_normalises_to_zero():
    x = np.zeros((2, 8), np.float32)
    proj = np.random.default_rng(0).standard_normal((2, 8, 4)).astype(np.float32)
    q = orc.project(x, np.array([1, 0], np.uint8), proj, np.zeros((2, 4), np.float32), normalize=True)
    assert np.all(q == 0)


@pytest.mark.parametrize("name", online_names())
def test_oracle_online_window_matches_reference(name):
    """search.py:778-806 against the reference's own outputs (online_*.npz)."""
    meta, d = load_online(name)
    keep = meta["keep_k"]
    hit, idx, slot, scores = orc.online_search(d["x_bf16"], d["keys_bf16"], d["eids"], d["sel"][:, keep:],
                                               meta["n_valid"])
    check_online(hit, idx, slot, d["on_hit"], d["on_idx"], d["on_slot"], scores, what=name)
