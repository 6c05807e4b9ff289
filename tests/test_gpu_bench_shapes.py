"""The exact configurations bench.py times, checked against the CPU oracle on the GPU.

* Config 2 (Qwen3-VL decode step): tables and inputs made by bench.py's own builders
  (bf16 tokens, fp32 normalised keys, decode rule hit = max >= 0, renormalised to one,
  E=128, K=1024, L=64, 16 tokens, top-8), run through the same LookupStepGraph the bench
  replays.
* Config 5 (one K=65536, L=128 table, hidden 4096): the full-size table through the
  ShardedCentroidTable at world 1 (the bench's C5 path on one GPU), with a 512-token
  sample of the bench's own tokens.
* Error reporting: out-of-range expert ids raise IndexError when device error checks are
  on (the reference's indexing raises IndexError), on the decode, single-CTA plan and
  whole-GPU plan paths.

Tolerances are tests/parity.py's: indices bit-exact except near ties (1e-5 relative),
rows bit-exact, combined output within 1e-2 relative.
"""
import numpy as np
import pytest
import torch

import bench
import oracle.oracle as orc
from parity import check_combined, check_search
from table_moe.cache_engine import CacheConfig, VectorSearchEngine

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _oracle_layer(mgr, inp):
    """Oracle project + search (normalised keys, >= 0) + combine of one bench layer."""
    keys = mgr.keys_buffer.float().cpu().numpy()
    proj = np.stack([mgr.pca["vision"]["proj"].cpu().numpy(), mgr.pca["text"]["proj"].cpu().numpy()])
    bias = np.stack([mgr.pca["vision"]["bias"].cpu().numpy(), mgr.pca["text"]["bias"].cpu().numpy()])
    x = inp["x"].float().numpy()
    vis = inp["is_vision"].numpy()
    q = orc.project(x, vis, proj, bias)
    hit, idx, _, _ = orc.search(q, keys, inp["sel"].numpy(), vis, inp["reuse"].numpy(), 0.0, 0.0, cmp_ge=True)
    return q, keys, hit, idx


@pytest.mark.parametrize("layers", [(0, 1), (5, 47)])
def test_c2_decode_step_graph_matches_oracle(layers):
    """bench.py's decode step, replayed as a CUDA graph, layer by layer against the oracle."""
    from table_moe.cache_engine.step_graph import LookupStepGraph

    mgrs = [bench.build_layer(li, DEV, 0) for li in layers]
    inputs = [bench.layer_inputs(li, 0) for li in layers]
    engines = [VectorSearchEngine(m) for m in mgrs]
    g = LookupStepGraph(engines, bench.CFG["tokens"], bench.CFG["top_k"], variant="decode", renorm="to_one",
                        keep_hits=True)
    for b, inp in zip(g.layers, inputs):
        for name, t in inp.items():
            getattr(b, name).copy_(t)
    g.capture()
    for b in g.layers:
        b.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    for i, (mgr, inp) in enumerate(zip(mgrs, inputs)):
        q, keys, rh, ri = _oracle_layer(mgr, inp)
        hit, idx = g.hits[i].cpu().numpy(), g.idx[i].cpu().numpy()
        check_search(hit, idx, rh, ri, q, keys, inp["sel"].numpy(), inp["is_vision"].numpy(), (0.0, 0.0),
                     "float32", what=f"c2 layer {layers[i]}")
        assert hit.sum() > 0.9 * inp["reuse"].sum().item()  # decode rule: almost every searched slot hits
        vb = mgr.values_buffer.cpu().view(torch.int16).numpy().view(np.uint16)
        ref = orc.combine(vb, inp["sel"].numpy(), inp["is_vision"].numpy(), hit, idx, inp["weights"].numpy(),
                          compute=inp["compute"].numpy(), renorm=1)
        check_combined(g.layers[i].out.float().cpu().numpy(), ref, what=f"c2 layer {layers[i]} combine")


def test_c5_full_table_matches_oracle():
    """Full-size config 5 table (K=65536, L=128, hidden 4096) on one GPU: tcgen05 projection,
    tensor-core scan, merge and row gather for 512 of the bench's tokens."""
    from table_moe.cache_engine.sharded import ShardedCentroidTable

    c = bench.C5
    n = 512
    g = torch.Generator(device=DEV).manual_seed(5005)
    keys = torch.randn(1, 2, c["k"], c["l"], generator=g, device=DEV)
    proj = [bench.orthonormal_basis(c["h"], c["l"], g, DEV) for _ in range(2)]
    pca = {m: {"proj": proj[i], "bias": torch.zeros(c["l"], device=DEV)} for i, m in enumerate(("vision", "text"))}
    x = torch.randn(c["tokens"], c["h"], generator=g, device=DEV).to(torch.bfloat16)[:n].contiguous()
    vis = torch.zeros(n, dtype=torch.bool, device=DEV)
    gv = torch.Generator(device=DEV).manual_seed(6006)
    values = torch.randn(1, 2, c["k"], c["h"], generator=gv, device=DEV, dtype=torch.bfloat16).mul_(0.05)
    table = ShardedCentroidTable(keys, values, pca, c["k"])
    hit, idx, rows = table.lookup(x, vis)
    torch.cuda.synchronize()
    pr = np.stack([p.cpu().numpy() for p in proj])
    q = orc.project(x.float().cpu().numpy(), vis.cpu().numpy(), pr, np.zeros((2, c["l"]), np.float32))
    kn = keys.cpu().numpy()
    sel = np.zeros((n, 1), np.int64)
    rh, ri, _, _ = orc.search(q, kn, sel, vis.cpu().numpy(), None, 0.0, 0.0, cmp_ge=False)
    gh, gi = hit.cpu().numpy()[:, None], idx.cpu().numpy()[:, None]
    check_search(gh, gi, rh, ri, q, kn, sel, vis.cpu().numpy(), (0.0, 0.0), "float32", what="c5 full table")
    ref_rows = values[0, 1, idx]
    ref_rows[~hit] = 0
    assert torch.equal(rows.view(torch.int16), ref_rows.view(torch.int16))
    table.close()


@pytest.mark.parametrize("Q,S", [(16, 8), (64, 4), (1024, 8)])
def test_bad_expert_ids_raise_with_error_checks(Q, S):
    """decode path (Q <= 32), single-CTA plan, whole-GPU plan (> 4096 slots)."""
    from table_moe.cache_engine import HybridStorageManager

    g = torch.Generator(device=DEV).manual_seed(Q)
    E, K, L, H = 8, 256, 64, 256
    keys = torch.randn(E, 2, K, L, generator=g, device=DEV)
    values = torch.zeros(E, 2, K, H, dtype=torch.bfloat16, device=DEV)
    pca = {m: {"proj": bench.orthonormal_basis(H, L, g, DEV), "bias": torch.zeros(L, device=DEV)}
           for m in ("vision", "text")}
    mgr = HybridStorageManager.from_tables(0, keys, values, pca)
    eng = VectorSearchEngine(mgr)
    x = torch.randn(Q, H, generator=g, device=DEV).to(torch.bfloat16)
    sel = torch.randint(0, E, (Q, S), generator=g, device=DEV)
    vis = torch.zeros(Q, dtype=torch.bool, device=DEV)
    reuse = torch.ones(Q, S, dtype=torch.bool, device=DEV)
    w = torch.full((Q, S), 1.0 / S, device=DEV)
    old = CacheConfig.ALUT_CHECK_ERRORS
    CacheConfig.ALUT_CHECK_ERRORS = True
    try:
        eng.search_decode_offline(0, x, sel, vis, reuse)  # valid ids: no error
        eng.lookup_combine(x, sel, vis, reuse, w, variant="decode")
        bad = sel.clone()
        bad[Q // 2, S - 1] = E  # one past the last expert
        with pytest.raises(IndexError):
            eng.search_decode_offline(0, x, bad, vis, reuse)
        bad[Q // 2, S - 1] = -3
        with pytest.raises(IndexError):
            eng.lookup_combine(x, bad, vis, reuse, w, variant="decode")
        assert eng.device_errors() == 0  # the check cleared the bits
        eng.search_decode_offline(0, x, sel, vis, reuse)
    finally:
        CacheConfig.ALUT_CHECK_ERRORS = old
    # Without the checks the bad slot is a miss and the rest is unchanged.
    h0, i0 = eng.search_decode_offline(0, x, sel, vis, reuse)
    h1, i1 = eng.search_decode_offline(0, x, bad, vis, reuse)
    assert not h1[Q // 2, S - 1]
    keep = torch.ones_like(h0)
    keep[Q // 2, S - 1] = False
    assert torch.equal(h0[keep], h1[keep]) and torch.equal(i0[keep], i1[keep])
    assert eng.device_errors() & 1


def test_step_graph_with_overlapped_copies_matches_device_graph():
    """The end-to-end graph (per-layer host->device input copies and device->host output
    copies on a second stream, overlapping the other layers) gives the device graph's
    outputs in host memory."""
    from table_moe.cache_engine.step_graph import LookupStepGraph

    layers = (0, 1, 2)
    mgrs = [bench.build_layer(li, DEV, 0) for li in layers]
    inputs = [bench.layer_inputs(li, 0) for li in layers]
    engines = [VectorSearchEngine(m) for m in mgrs]
    dev = LookupStepGraph(engines, bench.CFG["tokens"], bench.CFG["top_k"], variant="decode", accumulate=False)
    e2e = LookupStepGraph(engines, bench.CFG["tokens"], bench.CFG["top_k"], variant="decode", accumulate=False)
    for b, hb, inp in zip(dev.layers, e2e.host_layers, inputs):
        for name, t in inp.items():
            getattr(b, name).copy_(t)
            getattr(hb, name).copy_(t)
    dev.capture()
    e2e.capture(with_copies=True)
    for _ in range(2):
        dev.replay()
        e2e.replay()
    torch.cuda.synchronize()
    for b, hb in zip(dev.layers, e2e.host_layers):
        assert torch.equal(b.out.cpu().view(torch.int16), hb.out.view(torch.int16))
