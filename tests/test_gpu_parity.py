"""CUDA ALUT path against the reference's golden outputs and the pinned CPU oracle.

All calls go through the C ABI of libalut.so (via the drop-in VectorSearchEngine /
HybridStorageManager or the ctypes binding directly). Tolerances are those of
tests/parity.py: indices bit-exact except ties within 1e-5 relative, gathered rows
bit-exact, combined outputs within 1e-2 relative.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle.oracle as orc
from parity import case_inputs, check_combined, check_search, golden_names, load_golden
from table_moe.cache_engine import CacheConfig, HybridStorageManager, VectorSearchEngine, _alut
from table_moe.cache_engine.manager import normalize_rows

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TDT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _bf16_tensor(bits):
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def golden_manager(meta, d):
    tdt = TDT[meta["dtype"]]
    if "keys_raw" in d:
        raw = torch.from_numpy(d["keys_raw"]).to(tdt)
        norm = normalize_rows(raw, 1e-6)
    else:
        norm = torch.from_numpy(d["keys_norm"]).to(tdt)
        raw = norm.clone()
    pca = {m: {"proj": torch.from_numpy(d["proj"][i]).to(tdt).contiguous().to(DEV),
               "bias": torch.from_numpy(d["bias"][i]).to(tdt).contiguous().to(DEV)}
           for i, m in enumerate(("vision", "text"))}
    values = _bf16_tensor(d["values_bf16"]).to(DEV)
    return HybridStorageManager.from_tables(0, raw.to(DEV), values, pca, keys=norm.to(DEV))


def run_variant(eng, meta, x, sel, vis, reuse):
    v = meta["variant"]
    if v == "prefill_cos":
        return eng.search_prefill_offline(0, x, sel, vis, reuse)
    if v == "prefill_dot":
        return eng.search_prefill_offline_dot(0, x, sel, vis, reuse)
    if v == "decode_dot":
        return eng.search_decode_offline_dot(0, x, sel, vis, reuse)
    if v == "decode_cos":
        return eng.search_decode_offline(0, x, sel, vis, reuse)
    if v == "decode_hybrid":
        on_hit, on_idx, hit, idx, on_slot = eng.search_decode_hybrid(0, x, sel, vis, keep_k=meta["keep_k"])
        assert not on_hit.any() and bool((on_idx == -1).all())
        return hit, idx
    raise ValueError(v)


@pytest.fixture(autouse=True)
def _dot_threshold():
    old = CacheConfig.OFFLINE_DOT_THRESHOLD
    yield
    CacheConfig.OFFLINE_DOT_THRESHOLD = old


@pytest.mark.parametrize("name", golden_names())
def test_engine_matches_reference_golden(name):
    meta, d = load_golden(name)
    CacheConfig.OFFLINE_DOT_THRESHOLD = meta.get("dot_thr", 0.0)
    tdt = TDT[meta["dtype"]]
    mgr = golden_manager(meta, d)
    eng = VectorSearchEngine(mgr)
    x = _bf16_tensor(d["x_bf16"]).to(tdt).to(DEV)
    sel = torch.from_numpy(d["sel"]).to(DEV)
    vis = torch.from_numpy(d["is_vision"]).bool().to(DEV)
    reuse = torch.from_numpy(d["reuse"]).bool().to(DEV)
    hit, idx = run_variant(eng, meta, x, sel, vis, reuse)
    assert hit.dtype == torch.bool and idx.dtype == torch.int64 and hit.shape == sel.shape
    rule, thr, keys = case_inputs(meta, d)
    q = orc.project(d["x"], d["is_vision"], d["proj"], d["bias"], dtype=meta["dtype"], normalize=rule["normalize"])
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), d["hit"], d["idx"], q, keys, d["sel"], d["is_vision"],
                 thr, meta["dtype"], what=name)

    # Gather: bit-exact rows (manager.py:212-213).
    rows, cols = d["gather_rows"], d["gather_cols"]
    mids = np.where(d["is_vision"][rows] != 0, 0, 1)
    g = mgr.gather_values(torch.from_numpy(d["sel"][rows, cols]), torch.from_numpy(mids),
                          torch.from_numpy(d["idx"][rows, cols]))
    ref_rows = _bf16_tensor(d["values_bf16"])[d["sel"][rows, cols], mids, d["idx"][rows, cols]]
    assert torch.equal(g.cpu().view(torch.int16), ref_rows.view(torch.int16))

    # Fused lookup + combine against the reference's combine.
    renorm = "to_one" if meta["renorm"] == "qwen" else "to_rowsum"
    variant = {"prefill_cos": "prefill", "prefill_dot": "prefill_dot", "decode_dot": "decode_dot",
               "decode_cos": "decode", "decode_hybrid": "decode"}[meta["variant"]]
    w = torch.from_numpy(d["weights"]).to(DEV)
    comp = torch.from_numpy(d["compute"]).bool().to(DEV)
    out, fh, fi = eng.lookup_combine(x, sel, vis, reuse, w, compute_mask=comp, variant=variant, renorm=renorm,
                                     return_hits=True)
    assert torch.equal(fh, hit) and torch.equal(fi, idx)
    # Reference combine recomputed from the GPU's own hits, so that exempted ties do not
    # move rows between the two sides.
    ref = orc.combine(d["values_bf16"], d["sel"], d["is_vision"], fh.cpu().numpy(), fi.cpu().numpy(), d["weights"],
                      compute=d["compute"], renorm=1 if renorm == "to_one" else 2)
    check_combined(out.float().cpu().numpy(), ref, what=name)
    if np.array_equal(fh.cpu().numpy(), d["hit"].astype(bool)) and np.array_equal(fi.cpu().numpy(), d["idx"]):
        check_combined(out.float().cpu().numpy(), d["combined"], what=name + " vs reference")


def synth(Q, S, E, K, L, H, *, seed=0, dtype=torch.float32, vis_frac=0.5, reuse_p=0.4, zipf=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(Q, H, generator=g).to(torch.bfloat16)
    vis = torch.rand(Q, generator=g) < vis_frac
    proj = torch.stack([torch.linalg.qr(torch.randn(H, L, generator=g))[0] for _ in range(2)]).contiguous()
    bias = torch.randn(2, L, generator=g) * 0.1
    raw = torch.randn(E, 2, K, L, generator=g).to(dtype)
    logits = torch.randn(Q, E, generator=g)
    if zipf:
        prior = torch.arange(1, E + 1, dtype=torch.float32) ** (-zipf)
        logits = prior.log() - torch.log(-torch.log(torch.rand(Q, E, generator=g)))
    w, sel = torch.topk(torch.softmax(logits, -1), S, dim=-1)
    reuse = torch.rand(Q, S, generator=g) < reuse_p
    return dict(x=x, vis=vis, proj=proj.to(dtype), bias=bias.to(dtype), raw=raw, sel=sel, w=w.float(), reuse=reuse)


def synth_manager(s, values=None):
    E, _, K, L = s["raw"].shape
    H = s["proj"].shape[1]
    if values is None:
        g = torch.Generator(device=DEV).manual_seed(1)
        values = (torch.randn(E, 2, K, H, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    pca = {m: {"proj": s["proj"][i].contiguous().to(DEV), "bias": s["bias"][i].contiguous().to(DEV)}
           for i, m in enumerate(("vision", "text"))}
    return HybridStorageManager.from_tables(0, s["raw"].to(DEV), values, pca)


def oracle_dot(s, dtype="float32"):
    q = orc.project(s["x"].float().numpy(), s["vis"].numpy(), s["proj"].float().numpy(), s["bias"].float().numpy(),
                    dtype=dtype)
    keys = s["raw"].float().numpy()
    hit, idx, best, gap = orc.search(q, keys, s["sel"].numpy(), s["vis"].numpy(), s["reuse"].numpy(), 0.0, 0.0,
                                     cmp_ge=False, dtype=dtype)
    return q, keys, hit, idx


def gpu_dot(mgr, s, dtype=torch.float32):
    """dtype: the dtype the tokens are handed over in (bf16 tokens with fp32 tables take the
    tensor-core projection for small batches)."""
    eng = VectorSearchEngine(mgr)
    return eng.search_prefill_offline_dot(0, s["x"].to(dtype).to(DEV), s["sel"].to(DEV), s["vis"].to(DEV),
                                          s["reuse"].to(DEV))


@pytest.mark.parametrize("Q,vis_frac,H,L", [(16, 0.0, 2048, 64), (16, 0.5, 2048, 64), (37, 0.5, 1024, 96),
                                            (300, 0.3, 512, 128), (5, 1.0, 256, 8)])
def test_tensor_core_projection_matches_oracle(Q, vis_frac, H, L):
    """bf16 tokens + fp32 basis: q from the three-part bf16 split on tensor cores."""
    s = synth(Q=Q, S=4, E=12, K=300, L=L, H=H, seed=Q + L, vis_frac=vis_frac, reuse_p=0.6)
    mgr = synth_manager(s)
    assert mgr.alut_tables().proj_split
    hit, idx = gpu_dot(mgr, s, dtype=torch.bfloat16)
    q, keys, rh, ri = oracle_dot(s)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.0, 0.0), "float32", what=f"mma Q{Q}")
    lib = _alut.load()
    t = mgr.alut_tables()
    xb, selb, visb = s["x"].to(DEV), s["sel"].to(DEV), s["vis"].to(DEV)  # alive during the call
    b = _alut.make_batch(xb, selb, visb, None)
    ws = torch.zeros(lib.alut_workspace_size(t, Q, 4), dtype=torch.uint8, device=DEV)
    qg = torch.empty(Q, L, device=DEV)
    _alut.check(lib.alut_project(t, ctypes.byref(b), 0, 1e-6, qg.data_ptr(), L, ws.data_ptr(), ws.numel(),
                                 _alut.stream_ptr(DEV)), "alut_project")
    bound = np.abs(s["x"].float().numpy()).sum(axis=1, keepdims=True) * float(np.abs(s["proj"].numpy()).max())
    assert np.all(np.abs(qg.cpu().numpy() - q) <= 1e-6 * bound + 1e-6)


@pytest.mark.parametrize("cfg", [
    dict(name="c1", Q=256, S=1, E=1, K=256, L=64, H=2048, reuse_p=1.1, vis_frac=0.0),
    dict(name="c2_layer", Q=16, S=8, E=128, K=1024, L=64, H=2048, reuse_p=0.4, vis_frac=0.0),
    dict(name="c3_prefill", Q=4096, S=8, E=128, K=1024, L=64, H=2048, reuse_p=0.4, vis_frac=0.25, zipf=1.1),
    dict(name="c4_deepseek", Q=512, S=6, E=72, K=2048, L=96, H=2560, reuse_p=0.4),
])
def test_benchmark_shapes_match_oracle(cfg):
    cfg = dict(cfg)
    name = cfg.pop("name")
    s = synth(**cfg)
    mgr = synth_manager(s)
    hit, idx = gpu_dot(mgr, s)
    q, keys, rh, ri = oracle_dot(s)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.0, 0.0), "float32", what=name)
    # Combine with the oracle from the same hits.
    eng = VectorSearchEngine(mgr)
    out = eng.lookup_combine(s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV), s["reuse"].to(DEV),
                             s["w"].to(DEV), compute_mask=(~s["reuse"]).to(DEV), variant="prefill_dot")
    vb = mgr.values_buffer.cpu().view(torch.int16).numpy().view(np.uint16)
    ref = orc.combine(vb, s["sel"].numpy(), s["vis"].numpy(), hit.cpu().numpy(), idx.cpu().numpy(), s["w"].numpy(),
                      compute=(~s["reuse"]).numpy(), renorm=1)
    check_combined(out.float().cpu().numpy(), ref, what=name)


@pytest.mark.parametrize("Q,S,E,dtype", [(100, 2, 3, torch.bfloat16), (128, 2, 2, torch.float32),
                                          (250, 1, 1, torch.bfloat16), (40, 6, 8, torch.float32)])
def test_decode_chain_runs_of_slots_per_table(Q, S, E, dtype):
    """Batches of <= 256 slots take the decode chain at any token count: a table with more
    than 32 searched slots is scanned by one leader CTA per run of 32 of them."""
    s = synth(Q=Q, S=S, E=E, K=300, L=64, H=512, seed=Q * 7 + E, vis_frac=0.3, reuse_p=0.9)
    mgr = synth_manager(s)
    assert _alut.load().alut_scan_kind(mgr.alut_tables(), Q, S) == _alut.SCAN_DECODE
    hit, idx = gpu_dot(mgr, s, dtype=dtype)
    q, keys, rh, ri = oracle_dot(s)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.0, 0.0), "float32", what=f"decode runs Q{Q} S{S} E{E}")


def test_projection_matches_oracle():
    s = synth(Q=300, S=2, E=2, K=8, L=96, H=1000, seed=3)
    mgr = synth_manager(s)
    lib = _alut.load()
    t = mgr.alut_tables()
    x, selb, visb = s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV)  # alive during the calls
    b = _alut.make_batch(x, selb, visb, None)
    ws = torch.zeros(lib.alut_workspace_size(t, 300, 2), dtype=torch.uint8, device=DEV)
    for normalize in (False, True):
        q = torch.empty(300, 96, device=DEV)
        rc = lib.alut_project(t, ctypes.byref(b), int(normalize), 1e-6, q.data_ptr(), 96, ws.data_ptr(), ws.numel(),
                              _alut.stream_ptr(DEV))
        _alut.check(rc, "alut_project")
        ref = orc.project(s["x"].float().numpy(), s["vis"].numpy(), s["proj"].numpy(), s["bias"].numpy(),
                          normalize=normalize)
        bound = np.abs(s["x"].float().numpy()).sum(axis=1, keepdims=True) * float(np.abs(s["proj"].numpy()).max())
        tol = (1e-6 * bound if not normalize else 1e-5) + 1e-6
        assert np.all(np.abs(q.cpu().numpy() - ref) <= tol)


@pytest.mark.parametrize("Q,H,L,vis,normalize", [
    (1100, 2048, 64, "mixed", False),    # tiles holding both modalities
    (4096, 2048, 64, "first1024", True),  # C3-like: image tokens first, pure tiles
    (1300, 512, 128, "mixed", True),     # ragged last tile, L = 128
    (1777, 256, 48, "none", False),      # L = 48, text only
    (300, 512, 128, "mixed", True),      # below the tcgen05 cut: decode-shaped projection
    (12000, 256, 64, "mixed", False),    # 94 tiles: persistent CTAs, no H split
])
def test_large_batch_projection_matches_oracle(Q, H, L, vis, normalize):
    """bf16 tokens, fp32 basis, >= 1024 tokens: the tcgen05 projection (128-token tiles, basis
    in three bf16 parts); q within fp32 accuracy of the oracle."""
    g = torch.Generator().manual_seed(Q + L)
    x = torch.randn(Q, H, generator=g).to(torch.bfloat16)
    is_vis = {"mixed": torch.rand(Q, generator=g) < 0.5, "none": torch.zeros(Q, dtype=torch.bool),
              "first1024": torch.arange(Q) < 1024}[vis]
    proj = torch.stack([torch.linalg.qr(torch.randn(H, L, generator=g))[0] for _ in range(2)]).contiguous()
    bias = torch.randn(2, L, generator=g) * 0.1
    raw = torch.randn(2, 2, 16, L, generator=g)
    pca = {m: {"proj": proj[i].to(DEV), "bias": bias[i].to(DEV)} for i, m in enumerate(("vision", "text"))}
    values = torch.zeros(2, 2, 16, H, dtype=torch.bfloat16, device=DEV)
    mgr = HybridStorageManager.from_tables(0, raw.to(DEV), values, pca)
    lib = _alut.load()
    t = mgr.alut_tables()
    xb, visb, selb = x.to(DEV), is_vis.to(DEV), torch.zeros(Q, 1, dtype=torch.long, device=DEV)
    b = _alut.make_batch(xb, selb, visb, None)
    ws = torch.zeros(lib.alut_workspace_size(t, Q, 1), dtype=torch.uint8, device=DEV)
    q = torch.full((Q, L), float("nan"), device=DEV)
    _alut.check(lib.alut_project(t, ctypes.byref(b), int(normalize), 1e-6, q.data_ptr(), L, ws.data_ptr(), ws.numel(),
                                 _alut.stream_ptr(DEV)), "alut_project")
    ref = orc.project(x.float().numpy(), is_vis.numpy(), proj.numpy(), bias.numpy(), normalize=normalize)
    bound = np.abs(x.float().numpy()).sum(axis=1, keepdims=True) * float(np.abs(proj.numpy()).max())
    tol = (1e-5 if normalize else 1e-6 * bound) + 1e-6
    got = q.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.all(np.abs(got - ref) <= tol), float(np.max(np.abs(got - ref) - tol))


def test_large_batch_cosine_search_bf16_tokens():
    """search_prefill_offline (normalised queries, cosine keys) with bf16 tokens at prefill
    size: tcgen05 projection + tensor-core scan against the oracle."""
    s = synth(Q=1024, S=4, E=8, K=512, L=64, H=1024, seed=21, vis_frac=0.3, reuse_p=0.6)
    q0 = orc.project(s["x"].float().numpy(), s["vis"].numpy(), s["proj"].float().numpy(), s["bias"].float().numpy())
    for t in range(64):  # planted hits: a key along the token's own query, per routed slot
        m = 0 if bool(s["vis"][t]) else 1
        for j in range(4):
            s["raw"][int(s["sel"][t, j]), m, 100 + t] = torch.from_numpy(q0[t]) * 2
    mgr = synth_manager(s)
    eng = VectorSearchEngine(mgr)
    hit, idx = eng.search_prefill_offline(0, s["x"].to(DEV), s["sel"].to(DEV), s["vis"].to(DEV), s["reuse"].to(DEV))
    q = orc.project(s["x"].float().numpy(), s["vis"].numpy(), s["proj"].float().numpy(), s["bias"].float().numpy(),
                    normalize=True)
    keys = mgr.keys_buffer.cpu().numpy()
    rh, ri, _, _ = orc.search(q, keys, s["sel"].numpy(), s["vis"].numpy(), s["reuse"].numpy(), 0.6, 0.7, cmp_ge=True)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.6, 0.7), "float32", what="cos bf16")
    assert mgr._keys_split.get(_alut.KEYS_NORMALISED) is not None
    assert rh[:64][s["reuse"].numpy()[:64]].all()


@pytest.mark.parametrize("kdt", ["bfloat16", "float16"])
def test_16bit_tables_match_oracle(kdt):
    dt = TDT[kdt]
    s = synth(Q=200, S=4, E=6, K=333, L=64, H=512, seed=4, dtype=dt)
    s["x"] = s["x"].to(dt)
    mgr = synth_manager(s)
    hit, idx = gpu_dot(mgr, s, dtype=dt)
    q, keys, rh, ri = oracle_dot(s, dtype=kdt)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.0, 0.0), kdt, what=kdt)


@pytest.mark.parametrize("L,K", [(12, 7), (20, 129), (8, 1), (256, 300)])
def test_ragged_sizes_match_oracle(L, K):
    s = synth(Q=37, S=3, E=5, K=K, L=L, H=max(72, L + 8), seed=L + K, reuse_p=0.7)
    mgr = synth_manager(s)
    hit, idx = gpu_dot(mgr, s)
    q, keys, rh, ri = oracle_dot(s)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.0, 0.0), "float32", what=f"L{L}K{K}")


def test_ties_take_the_first_index_across_chunks():
    s = synth(Q=8, S=1, E=1, K=1000, L=16, H=32, seed=5, reuse_p=1.1)
    q = orc.project(s["x"].float().numpy(), s["vis"].numpy(), s["proj"].numpy(), s["bias"].numpy())
    raw = torch.randn(1, 2, 1000, 16) * 0.01
    for t in range(8):
        m = 0 if bool(s["vis"][t]) else 1
        for k in (900 - t, 300 + t, 131 + t):  # duplicates in three different 128-centroid chunks
            raw[0, m, k] = torch.from_numpy(q[t]) * 3
    s["raw"] = raw
    hit, idx = gpu_dot(synth_manager(s), s)
    assert hit.all()
    assert idx[:, 0].cpu().tolist() == [131 + t for t in range(8)]


def test_edge_cases_empty_no_reuse_bad_ids():
    s = synth(Q=16, S=4, E=5, K=64, L=32, H=64, seed=6, reuse_p=0.8)
    mgr = synth_manager(s)
    eng = VectorSearchEngine(mgr)
    x, sel, vis = s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV)
    hit, idx = eng.search_prefill_offline_dot(0, x[:0], sel[:0], vis[:0], s["reuse"][:0].to(DEV))
    assert hit.shape == (0, 4)
    hit, idx = eng.search_prefill_offline_dot(0, x, sel, vis, torch.zeros(16, 4, dtype=torch.bool, device=DEV))
    assert not hit.any() and not idx.any()
    bad = sel.clone()
    bad[0, 0] = 99
    bad[1, 1] = -1
    reuse = torch.ones(16, 4, dtype=torch.bool, device=DEV)
    hit, idx = eng.search_prefill_offline_dot(0, x, bad, vis, reuse)
    assert not hit[0, 0] and not hit[1, 1]
    ref_hit, ref_idx = eng.search_prefill_offline_dot(0, x, sel, vis, reuse)
    keep = torch.ones_like(hit)
    keep[0, 0] = keep[1, 1] = False
    assert torch.equal(hit[keep], ref_hit[keep]) and torch.equal(idx[keep], ref_idx[keep])


def test_repeated_calls_are_bitwise_deterministic():
    s = synth(Q=2048, S=8, E=64, K=512, L=64, H=1024, seed=7, zipf=1.1)
    mgr = synth_manager(s)
    eng = VectorSearchEngine(mgr)
    args = (s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV), s["reuse"].to(DEV), s["w"].to(DEV))
    o1, h1, i1 = eng.lookup_combine(*args, return_hits=True)
    o2, h2, i2 = eng.lookup_combine(*args, return_hits=True)
    assert torch.equal(h1, h2) and torch.equal(i1, i2)
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


def test_combine_entry_accumulates_and_renormalises():
    s = synth(Q=64, S=8, E=16, K=128, L=32, H=520, seed=8, reuse_p=0.5)  # H % 8 != 0 path too
    mgr = synth_manager(s)
    eng = VectorSearchEngine(mgr)
    x, sel, vis, reuse = s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV), s["reuse"].to(DEV)
    hit, idx = eng.search_prefill_offline_dot(0, x, sel, vis, reuse)
    lib = _alut.load()
    vb = mgr.values_buffer.cpu().view(torch.int16).numpy().view(np.uint16)
    base = torch.randn(64, 520, device=DEV).to(torch.bfloat16)
    for renorm in (0, 1, 2):
        out = base.clone()
        b = _alut.make_batch(None, sel, vis, reuse)
        comp = (~reuse).contiguous()
        w = s["w"].to(DEV)
        rc = lib.alut_combine(mgr.alut_tables(), ctypes.byref(b), hit.data_ptr(), idx.data_ptr(), 8, w.data_ptr(), 8,
                              comp.data_ptr(), 8, renorm, 1, out.data_ptr(), 520, 1, _alut.stream_ptr(DEV))
        _alut.check(rc, "alut_combine")
        ref = orc.combine(vb, s["sel"].numpy(), s["vis"].numpy(), hit.cpu().numpy(), idx.cpu().numpy(),
                          s["w"].numpy(), compute=(~s["reuse"]).numpy(), renorm=renorm, out=base.float().cpu().numpy())
        check_combined(out.float().cpu().numpy(), ref, what=f"renorm{renorm}")


def test_bs1_entry_points_match_batched_search():
    s = synth(Q=1, S=8, E=32, K=256, L=64, H=512, seed=9)
    mgr = synth_manager(s)
    eng = VectorSearchEngine(mgr)
    x, sel, vis = s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV)
    hit = torch.ones(8, dtype=torch.bool, device=DEV)
    idx = torch.full((8,), 7, dtype=torch.long, device=DEV)
    eng.search_decode_offline_bs1_into(x[0], sel[0], vis[0], 3, hit, idx)
    reuse = torch.zeros(1, 8, dtype=torch.bool, device=DEV)
    reuse[:, 3:] = True
    rh, ri = eng.search_decode_offline_dot(0, x, sel, vis, reuse)
    assert torch.equal(hit, rh[0]) and torch.equal(idx, ri[0])
    on_hit = torch.ones(8, dtype=torch.bool, device=DEV)
    on_idx = torch.zeros(1, dtype=torch.long, device=DEV)
    off_hit = torch.zeros(8, dtype=torch.bool, device=DEV)
    off_idx = torch.zeros(8, dtype=torch.long, device=DEV)
    on_slot = torch.ones(8, dtype=torch.long, device=DEV)
    eng.search_decode_hybrid_bs1_into(x[0], sel[0], vis[0], 3, on_hit, on_idx, off_hit, off_idx, on_slot)
    rh2, ri2 = eng.search_decode_offline(0, x, sel, vis, reuse)
    assert not on_hit.any() and int(on_idx) == -1
    assert torch.equal(off_hit, rh2[0]) and torch.equal(off_idx, ri2[0])
    out = torch.zeros(8, 512, dtype=torch.bfloat16, device=DEV)
    hs = torch.nonzero(off_hit).flatten()
    mgr.gather_values_decode_bs1(sel[0, hs], int(not bool(vis[0])), off_idx[hs], hs, out)
    m = 0 if bool(vis[0]) else 1
    for slot in hs.tolist():
        assert torch.equal(out[slot], mgr.values_buffer[sel[0, slot], m, off_idx[slot]])


def test_centroid_shards_merge_to_the_full_search():
    s = synth(Q=512, S=1, E=1, K=4096, L=128, H=512, seed=10, reuse_p=1.1)
    mgr = synth_manager(s)
    lib = _alut.load()
    x, sel, vis = s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV)
    full_hit, full_idx = gpu_dot(mgr, s)
    world = 4
    per = 4096 // world
    packed = torch.zeros(world, 512, dtype=torch.int64, device=DEV)
    p = _alut.make_params(_alut.KEYS_RAW, False, False, 0.0, 0.0, 1e-6)
    for r in range(world):
        shard = mgr.raw_keys_buffer[:, :, r * per:(r + 1) * per]
        pv, pt = mgr.pca["vision"], mgr.pca["text"]
        t = _alut.make_tables(None, shard, None, pv["proj"], pv["bias"], pt["proj"], pt["bias"])
        ws = torch.zeros(lib.alut_workspace_size(t, 512, 1), dtype=torch.uint8, device=DEV)
        b = _alut.make_batch(x, sel, vis, None)
        rc = lib.alut_search_packed(t, ctypes.byref(b), p, None, r * per, packed[r].data_ptr(), ws.data_ptr(),
                                    ws.numel(), _alut.stream_ptr(DEV))
        _alut.check(rc, "alut_search_packed")
    hit = torch.zeros(512, dtype=torch.bool, device=DEV)
    idx = torch.zeros(512, dtype=torch.long, device=DEV)
    rc = lib.alut_merge_packed(world, 512, 1, packed.data_ptr(), vis.data_ptr(), p, hit.data_ptr(), idx.data_ptr(),
                               _alut.stream_ptr(DEV))
    _alut.check(rc, "alut_merge_packed")
    assert torch.equal(hit, full_hit[:, 0]) and torch.equal(idx, full_idx[:, 0])


@pytest.mark.parametrize("cfg", [
    dict(name="c3_tc", Q=4096, S=8, E=128, K=1024, L=64, H=2048, reuse_p=0.4, vis_frac=0.25, zipf=1.1),
    dict(name="c5_like", Q=1024, S=1, E=1, K=8192, L=128, H=512, reuse_p=1.1),
    dict(name="ragged_k", Q=600, S=2, E=3, K=300, L=48, H=256, reuse_p=0.9),
])
def test_tensor_core_scan_matches_oracle(cfg):
    """Large batches on fp32 tables take the tcgen05 scan (bf16 split candidates + exact fp32
    rescoring); the indices must still follow the exact fp32 argmax."""
    cfg = dict(cfg)
    name = cfg.pop("name")
    s = synth(**cfg)
    mgr = synth_manager(s)
    hit, idx = gpu_dot(mgr, s)
    assert mgr._keys_split.get(_alut.KEYS_RAW) is not None, "tensor-core key form was not prepared"
    q, keys, rh, ri = oracle_dot(s)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (0.0, 0.0), "float32", what=name)


def test_tensor_core_scan_ties_and_negative_scores():
    """Duplicate keys in different 128-row chunks tie to the lowest index; rows whose every
    score is negative still return their (negative) maximum under a >= -inf rule."""
    Q, K, L = 640, 1024, 64
    s = synth(Q=Q, S=1, E=1, K=K, L=L, H=128, seed=12, reuse_p=1.1)
    q = orc.project(s["x"].float().numpy(), s["vis"].numpy(), s["proj"].numpy(), s["bias"].numpy())
    raw = -torch.rand(1, 2, K, L) * 0.01 - 0.001
    for t in range(8):
        m = 0 if bool(s["vis"][t]) else 1
        for k in (900 - t, 300 + t, 131 + t):
            raw[0, m, k] = torch.from_numpy(q[t]) * 3
    s["raw"] = raw
    mgr = synth_manager(s)
    eng = VectorSearchEngine(mgr)
    x, sel, vis, reuse = s["x"].float().to(DEV), s["sel"].to(DEV), s["vis"].to(DEV), s["reuse"].to(DEV)
    old = CacheConfig.OFFLINE_DOT_THRESHOLD
    CacheConfig.OFFLINE_DOT_THRESHOLD = -1e30
    try:
        hit, idx = eng.search_prefill_offline_dot(0, x, sel, vis, reuse)
    finally:
        CacheConfig.OFFLINE_DOT_THRESHOLD = old
    assert mgr._keys_split.get(_alut.KEYS_RAW) is not None
    assert idx[:8, 0].cpu().tolist() == [131 + t for t in range(8)]
    keys = raw.float().numpy()
    rh, ri, _, _ = orc.search(q, keys, s["sel"].numpy(), s["vis"].numpy(), s["reuse"].numpy(), -1e30, -1e30,
                              cmp_ge=False)
    assert hit.all()
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, keys, s["sel"].numpy(), s["vis"].numpy(),
                 (-1e30, -1e30), "float32", what="tc ties")
