"""Online window lookup of the hybrid decode search (search.py:778-806) on the GPU through
alut_online_search: the reference's own outputs (tests/golden/online_*.npz), randomised
windows against the oracle, and the full search_decode_hybrid flow (online hits exclude
their slots from the offline search)."""
import numpy as np
import pytest
import torch

import oracle.oracle as orc
from parity import check_online, load_online, online_names
from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _bits_to_bf16(bits):
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def _manager(H, keys, eids, n_valid, full, E=12, K=64, L=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(E, 2, K, L, generator=g)
    values = torch.zeros(E, 2, K, H, dtype=torch.bfloat16)
    pca = {m: {"proj": torch.linalg.qr(torch.randn(H, L, generator=g))[0].contiguous().to(DEV),
               "bias": torch.zeros(L, device=DEV)} for m in ("vision", "text")}
    mgr = HybridStorageManager.from_tables(1, raw.to(DEV), values.to(DEV), pca)
    mgr._init_online(force=True)
    size = keys.shape[0]
    mgr.online_size = size
    mgr.online_keys = keys.to(DEV).contiguous()
    mgr.online_expert_ids = eids.to(DEV).contiguous()
    mgr.online_values = torch.zeros(size, eids.shape[1], H, dtype=keys.dtype, device=DEV)
    mgr.online_full = full
    mgr.online_ptr = 0 if full else n_valid
    return mgr


def _run_online(mgr, x, target):
    eng = VectorSearchEngine(mgr)
    bs, s = target.shape
    on_hit = torch.zeros(bs, s, dtype=torch.bool, device=DEV)
    on_idx = torch.full((bs,), -1, dtype=torch.long, device=DEV)
    on_slot = torch.zeros(bs, s, dtype=torch.long, device=DEV)
    has = eng._search_online_into(x.to(DEV), target.to(DEV), on_hit, on_idx, on_slot)
    torch.cuda.synchronize()
    return has, on_hit.cpu().numpy(), on_idx.cpu().numpy(), on_slot.cpu().numpy()


@pytest.mark.parametrize("name", online_names())
def test_online_window_matches_reference_golden(name):
    meta, d = load_online(name)
    keys = _bits_to_bf16(d["keys_bf16"])
    x = _bits_to_bf16(d["x_bf16"])
    mgr = _manager(meta["H"], keys, torch.from_numpy(d["eids"]), meta["n_valid"], meta["full"])
    keep = meta["keep_k"]
    has, hit, idx, slot = _run_online(mgr, x, torch.from_numpy(d["sel"][:, keep:]))
    assert has == meta["has_online"]
    _, _, _, scores = orc.online_search(d["x_bf16"], d["keys_bf16"], d["eids"], d["sel"][:, keep:], meta["n_valid"])
    check_online(hit, idx, slot, d["on_hit"], d["on_idx"], d["on_slot"], scores, what=name)


@pytest.mark.parametrize("B,H,size,n_valid,full,dtype", [
    (16, 2048, 64, 64, True, torch.bfloat16),    # Qwen3-VL decode shape, full window
    (16, 2048, 64, 37, False, torch.bfloat16),   # partial window
    (3, 2560, 64, 64, True, torch.bfloat16),     # DeepSeek-VL2 hidden size
    (1, 1024, 64, 1, False, torch.float16),      # bs=1, one entry
    (8, 520, 32, 32, True, torch.float32),       # H not a power of two, fp32 window
])
def test_online_window_matches_oracle(B, H, size, n_valid, full, dtype):
    g = torch.Generator().manual_seed(B * 7 + H)
    x = torch.randn(B, H, generator=g).to(dtype)
    keys = torch.randn(size, H, generator=g).to(dtype)
    keys[5 % size] = x[0]  # a clear best for token 0
    eids = torch.randint(0, 10, (size, 6), generator=g)
    eids[torch.rand(size, 6, generator=g) < 0.2] = -1
    target = torch.randint(0, 10, (B, 5), generator=g)
    mgr = _manager(H, keys, eids, n_valid, full, seed=3)
    has, hit, idx, slot = _run_online(mgr, x, target)
    assert has
    xb = x.float().numpy()
    kb = keys.float().numpy()
    sc = xb @ kb[:n_valid].T
    if dtype == torch.bfloat16:
        sc = orc.bf16_to_f32(orc.bf16_bits(sc.astype(np.float32))).reshape(sc.shape)
    elif dtype == torch.float16:
        sc = sc.astype(np.float16).astype(np.float32)
    arg = sc.argmax(1)
    valid = sc[np.arange(B), arg] > 0
    ref_idx = np.where(valid, arg, -1)
    match = target.numpy()[:, :, None] == eids.numpy()[arg][:, None, :]
    ref_hit = match.any(-1) & valid[:, None]
    ref_slot = np.where(ref_hit, match.argmax(-1), 0)
    check_online(hit, idx, slot, ref_hit, ref_idx, ref_slot, sc, what=f"B{B} H{H} n{n_valid}")
    if n_valid > 5:
        assert idx[0] == 5 % size


def test_decode_hybrid_online_hits_skip_offline_search():
    """search_decode_hybrid: slots after keep_k that hit the online window are not searched
    offline (reuse = ~on_hit); the others are, with the decode rule (normalised keys, >= 0)."""
    B, H, S, keep = 8, 256, 8, 3
    g = torch.Generator().manual_seed(5)
    x = torch.randn(B, H, generator=g).to(torch.bfloat16)
    keys = torch.randn(64, H, generator=g).to(torch.bfloat16)
    keys[:B] = x  # token b's best window entry is b
    eids = torch.randint(0, 12, (64, 6), generator=g)
    sel = torch.stack([torch.randperm(12, generator=g)[:S] for _ in range(B)])
    sel[:, keep] = eids[torch.arange(B), 0]  # slot keep hits the window for every token
    mgr = _manager(H, keys, eids, 64, True, E=12, K=64, L=16, seed=9)
    eng = VectorSearchEngine(mgr)
    vis = torch.zeros(B, dtype=torch.bool, device=DEV)
    on_hit, on_idx, off_hit, off_idx, on_slot = eng.search_decode_hybrid(1, x.to(DEV), sel.to(DEV), vis, keep_k=keep)
    on_hit, on_idx, off_hit = on_hit.cpu(), on_idx.cpu(), off_hit.cpu()
    assert torch.equal(on_idx, torch.arange(B))
    assert on_hit[:, keep].all() and not on_hit[:, :keep].any()
    assert not off_hit[on_hit].any()  # online hits are not searched offline
    assert not off_hit[:, :keep].any()  # keep_k slots are computed, never looked up
    # The slots searched offline follow the oracle (normalised keys, hit = max >= 0).
    q = orc.project(x.float().numpy(), vis.cpu().numpy(), np.stack([mgr.pca[m]["proj"].cpu().numpy() for m in ("vision", "text")]),
                    np.stack([mgr.pca[m]["bias"].cpu().numpy() for m in ("vision", "text")]))
    reuse = np.zeros((B, S), bool)
    reuse[:, keep:] = ~on_hit[:, keep:].numpy()
    rh, ri, _, _ = orc.search(q, mgr.keys_buffer.cpu().numpy(), sel.numpy(), vis.cpu().numpy(), reuse, 0.0, 0.0,
                              cmp_ge=True)
    assert np.array_equal(off_hit.numpy(), rh)
    assert np.array_equal(np.where(rh, off_idx.cpu().numpy(), 0), np.where(rh, ri, 0))
