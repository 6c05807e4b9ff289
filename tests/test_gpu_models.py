"""The cached MoE layer adapter (table_moe.models.ALUTCachedMoE) on a tiny random MoE: the
router, computed experts, the lookups and the combine of computed outputs and looked-up
rows in one call, against a restatement of the reference wrapper's combine
(qwen3_vl_moe/cached_layers.py:452-465: collected rows, renormalised weights, weighted
sum) built from the oracle's search. Tolerances: tests/parity.py."""
import numpy as np
import pytest
import torch

import oracle.oracle as orc
from parity import check_combined, check_search
from table_moe.cache_engine import HybridStorageManager
from table_moe.models import ALUTCachedMoE

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
E, H, L, K, S = 16, 256, 32, 64, 4


def tiny_model(seed=0):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(E, 2, K, L, generator=g)
    proj = torch.stack([torch.linalg.qr(torch.randn(H, L, generator=g))[0] for _ in range(2)]).contiguous()
    values = (torch.randn(E, 2, K, H, generator=g) * 0.05).to(torch.bfloat16)
    gate = torch.randn(H, E, generator=g) * 0.1
    experts = (torch.randn(E, H, H, generator=g) * H ** -0.5).to(torch.bfloat16)
    pca = {m: {"proj": proj[i].to(DEV), "bias": torch.zeros(L, device=DEV)} for i, m in enumerate(("vision", "text"))}
    mgr = HybridStorageManager.from_tables(0, raw.to(DEV), values.to(DEV), pca, enable_online=False)
    return mgr, raw, proj, values, gate.to(DEV), experts.to(DEV)


def run_experts_fn(experts):
    def run(x, sel, comp, collected):
        for t, s in torch.nonzero(comp).tolist():
            collected[t, s] = x[t].to(torch.bfloat16) @ experts[sel[t, s]]
    return run


@pytest.mark.parametrize("Q,prefill,renorm", [(40, True, "to_one"), (8, False, "to_one"), (24, True, "to_rowsum")])
def test_cached_moe_adapter_matches_reference_combine(Q, prefill, renorm):
    mgr, raw, proj, values, gate, experts = tiny_model(Q)
    g = torch.Generator().manual_seed(100 + Q)
    x = torch.randn(Q, H, generator=g).to(torch.bfloat16).to(DEV)
    vis = torch.zeros(Q, dtype=torch.bool, device=DEV)
    vis[: Q // 4] = prefill  # a few image tokens in the prefill batches
    moe = ALUTCachedMoE(mgr, S, decode_keep_k=2, keep_rate=0.5, renorm=renorm)
    logits = x.float() @ gate
    out, r = moe(x, logits, vis, run_experts_fn(experts), is_prefill=prefill, return_routing=True)
    torch.cuda.synchronize()
    sel, w, comp, reuse = (r[k].cpu().numpy() for k in ("selected_experts", "weights", "compute_mask", "reuse_mask"))
    hit, idx = r["hit"].cpu().numpy(), r["idx"].cpu().numpy()
    assert np.array_equal(reuse, ~comp)
    # the lookups against the oracle (dot rule, > 0)
    vn = vis.cpu().numpy()
    q = orc.project(x.float().cpu().numpy(), vn, proj.numpy(), np.zeros((2, L), np.float32))
    rh, ri, _, _ = orc.search(q, raw.numpy(), sel, vn, reuse, 0.0, 0.0, cmp_ge=False)
    check_search(hit, idx, rh, ri, q, raw.numpy(), sel, vn, (0.0, 0.0), "float32", what="adapter lookups")
    # the reference combine: collected rows, survivors' weights renormalised, weighted sum
    xf = x.to(torch.bfloat16)
    collected = np.zeros((Q, S, H), np.float32)
    vf = values.float().numpy()
    for t in range(Q):
        for s in range(S):
            if comp[t, s]:
                collected[t, s] = (xf[t] @ experts[sel[t, s]]).float().cpu().numpy()
            elif hit[t, s]:
                collected[t, s] = vf[sel[t, s], 0 if vn[t] else 1, idx[t, s]]
    surv = comp | hit
    kept = (w * surv).sum(-1, keepdims=True)
    wt = np.where(kept > 0, w * surv / np.where(kept > 0, kept, 1), 0)
    if renorm == "to_rowsum":
        wt = wt * w.sum(-1, keepdims=True)
    ref = np.einsum("ts,tsh->th", wt, collected)
    check_combined(out.float().cpu().numpy(), ref, what=f"adapter Q{Q}")
