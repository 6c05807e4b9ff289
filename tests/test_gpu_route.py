"""The router prologue kernels (alut_route, alut_keep_mask) against the reference's fixtures
and the router oracle, through the drop-in modules table_moe.ops.qwen_topk_softmax and
table_moe.skip. Tolerances: oracle/parity_rules.py route_mismatches (weights 1e-5 relative,
expert ids exact except ties within 1e-6, keep masks exact except ties and expert sums
within 1e-5 of the keep boundary)."""
import numpy as np
import pytest
import torch

import oracle.oracle as orc
import oracle.route as rt
from parity import check_combined, check_route, check_search, load_route, route_names, route_oracle
from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine
from table_moe.ops import qwen_topk_softmax, route_for_lookup
from table_moe.skip import build_decode_keep_mask, build_prefill_keep_mask

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _logits(meta, d):
    x = torch.from_numpy(d["logits"])
    return (x.to(torch.bfloat16) if meta["dtype"] == "bfloat16" else x).to(DEV)


def _route(meta, d):
    attn = None if d["attn"] is None else torch.from_numpy(d["attn"]).to(DEV)
    keep = "fixed" if meta["mode"] == "fixed" else "importance"
    return route_for_lookup(_logits(meta, d), meta["k"], normalize_topk=meta["normalize"], keep=keep,
                            keep_k=meta["keep_k"], keep_rate=meta["keep_rate"], attn_scores=attn)


@pytest.mark.parametrize("name", route_names())
def test_route_matches_reference_fixture(name):
    meta, d = load_route(name)
    w, sel, comp, reuse = _route(meta, d)
    w, sel, comp, reuse = (t.cpu().numpy() for t in (w, sel, comp, reuse))
    assert np.array_equal(reuse, ~comp)
    _, _, _, p, _, _ = route_oracle(meta, d)
    # top-k softmax against the reference
    check_route(w, sel, None, d["weights"], d["sel"], None, p, what=name)
    # keep mask against the oracle applied to the kernel's own routing, and, where the
    # routing equals the reference's, against the reference's mask
    _, _, keep, _, sums, kept = route_oracle(meta, d, weights=w, sel=sel)
    check_route(w, sel, comp, w, sel, keep, p, sums, kept, what=name + " keep")
    if np.array_equal(sel, d["sel"]):
        check_route(w, sel, comp, d["weights"], d["sel"], d["keep"], p, sums, kept, what=name + " vs reference")


@pytest.mark.parametrize("name", ["route_qwen_prefill_importance", "route_prefill_attn_scores",
                                  "route_bf16_logits_keep_rate_low"])
def test_build_prefill_keep_mask_kernel_matches_reference(name):
    """alut_keep_mask on the reference's own routing gives the reference's mask."""
    meta, d = load_route(name)
    attn = None if d["attn"] is None else torch.from_numpy(d["attn"]).to(DEV)
    sel = torch.from_numpy(d["sel"]).to(DEV)
    w = torch.from_numpy(d["weights"]).to(DEV)
    got = build_prefill_keep_mask(sel, w, attn, meta["E"], meta["keep_rate"]).cpu().numpy()
    _, _, keep, p, sums, kept = route_oracle(meta, d, weights=d["weights"], sel=d["sel"])
    check_route(d["weights"], d["sel"], got, d["weights"], d["sel"], d["keep"], p, sums, kept, what=name)


def test_drop_in_functions():
    meta, d = load_route("route_deepseek_normalized")
    w, sel = qwen_topk_softmax(_logits(meta, d), meta["k"], normalize_topk=True)
    _, _, _, p, _, _ = route_oracle(meta, d)
    check_route(w.cpu().numpy(), sel.cpu().numpy(), None, d["weights"], d["sel"], None, p, what="drop-in")
    assert torch.allclose(w.sum(-1), torch.ones(w.shape[0], device=DEV), atol=1e-6)
    keep = build_decode_keep_mask(sel, 2)
    assert keep[:, :2].all() and not keep[:, 2:].any()
    with pytest.raises(ValueError):
        qwen_topk_softmax(torch.zeros(4, 8), 2)  # CPU logits: no CPU path


@pytest.mark.parametrize("Q,E,k,mode", [(4096, 128, 8, "importance"), (16, 2048, 64, "fixed"), (1, 72, 6, "fixed"),
                                        (7, 4096, 8, "importance")])
def test_route_large_and_edge_shapes_match_oracle(Q, E, k, mode):
    g = torch.Generator().manual_seed(Q + E)
    logits = torch.randn(Q, E, generator=g) * 3
    meta = dict(k=k, normalize=False, mode=mode, keep_k=3, keep_rate=0.6, E=E)
    d = dict(logits=logits.numpy(), attn=None)
    w, sel, comp, _ = route_for_lookup(logits.to(DEV), k, keep=mode, keep_k=3, keep_rate=0.6)
    w, sel, comp = w.cpu().numpy(), sel.cpu().numpy(), comp.cpu().numpy()
    rw, rs, _, p, _, _ = route_oracle(meta, d)
    check_route(w, sel, None, rw, rs, None, p, what=f"Q{Q}E{E}")
    _, _, keep, _, sums, kept = route_oracle(meta, d, weights=w, sel=sel)
    check_route(w, sel, comp, w, sel, keep, p, sums, kept, what=f"Q{Q}E{E} keep")


def test_route_is_deterministic_and_reusable():
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(2048, 128, generator=g).to(DEV)
    a = route_for_lookup(logits, 8, keep="importance", keep_rate=0.6)
    b = route_for_lookup(logits, 8, keep="importance", keep_rate=0.6)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_route_feeds_lookup_combine():
    """Router prologue -> fused lookup on its outputs, against the oracle end to end."""
    g = torch.Generator().manual_seed(9)
    Q, E, K, L, H, k = 64, 32, 256, 64, 512, 8
    logits = torch.randn(Q, E, generator=g)
    x = torch.randn(Q, H, generator=g).to(torch.bfloat16)
    raw = torch.randn(E, 2, K, L, generator=g)
    proj = torch.stack([torch.linalg.qr(torch.randn(H, L, generator=g))[0] for _ in range(2)]).contiguous()
    values = (torch.randn(E, 2, K, H, generator=g) * 0.05).to(torch.bfloat16)
    pca = {m: {"proj": proj[i].to(DEV), "bias": torch.zeros(L, device=DEV)} for i, m in enumerate(("vision", "text"))}
    mgr = HybridStorageManager.from_tables(0, raw.to(DEV), values.to(DEV), pca)
    eng = VectorSearchEngine(mgr)
    vis = torch.zeros(Q, dtype=torch.bool)
    w, sel, comp, reuse = route_for_lookup(logits.to(DEV), k, keep="fixed", keep_k=3)
    out, hit, idx = eng.lookup_combine(x.to(DEV), sel, vis.to(DEV), reuse, w, compute_mask=comp,
                                       variant="prefill_dot", return_hits=True)
    sel_n, w_n, reuse_n, comp_n = sel.cpu().numpy(), w.cpu().numpy(), reuse.cpu().numpy(), comp.cpu().numpy()
    q = orc.project(x.float().numpy(), vis.numpy(), proj.numpy(), np.zeros((2, L), np.float32))
    rh, ri, _, _ = orc.search(q, raw.numpy(), sel_n, vis.numpy(), reuse_n, 0.0, 0.0, cmp_ge=False)
    check_search(hit.cpu().numpy(), idx.cpu().numpy(), rh, ri, q, raw.numpy(), sel_n, vis.numpy(), (0.0, 0.0),
                 "float32", what="route->lookup")
    vb = values.view(torch.int16).numpy().view(np.uint16)
    ref = orc.combine(vb, sel_n, vis.numpy(), hit.cpu().numpy(), idx.cpu().numpy(), w_n, compute=comp_n, renorm=1)
    check_combined(out.float().cpu().numpy(), ref, what="route->lookup combine")
    assert rt.fixed_keep_mask(sel_n, 3).tolist() == comp_n.tolist()
