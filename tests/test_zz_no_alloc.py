"""alut_lookup_combine_noalloc: the fused lookup for callers that cannot allocate device
memory (they are handed only their input and output buffers, e.g. an FFI host without the
CUDA allocator, or a serving loop that forbids cudaMalloc after start-up because it can
synchronise the device). Its scratch is a fixed array inside libalut.so, so its results
must match alut_lookup_combine with a caller-owned workspace, call after call.

Collected last on purpose (file name), so that a run stopping at the first failure has
already run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from parity import check_combined
from table_moe.cache_engine import HybridStorageManager, _alut

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _case(seed, Q=16, S=8, E=32, K=512, L=64, H=1024):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(Q, H, generator=g).to(torch.bfloat16)
    vis = torch.rand(Q, generator=g) < 0.3
    w, sel = torch.topk(torch.softmax(torch.randn(Q, E, generator=g), -1), S, dim=-1)
    reuse = torch.rand(Q, S, generator=g) < 0.5
    return dict(x=x.to(DEV), vis=vis.to(DEV), sel=sel.to(DEV), w=w.float().to(DEV), reuse=reuse.to(DEV),
                comp=(~reuse).to(DEV))


@pytest.fixture(scope="module")
def manager():
    g = torch.Generator(device=DEV).manual_seed(11)
    E, K, L, H = 32, 512, 64, 1024
    raw = torch.randn(E, 2, K, L, generator=g, device=DEV)
    values = (torch.randn(E, 2, K, H, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    pca = {}
    for m in ("vision", "text"):
        q, _ = torch.linalg.qr(torch.randn(H, L, generator=g, device=DEV))
        pca[m] = {"proj": q.contiguous(), "bias": torch.zeros(L, device=DEV)}
    return HybridStorageManager.from_tables(0, raw, values, pca)


def _run(lib, mgr, c, noalloc):
    Q, S = c["sel"].shape
    # Batches of >= 512 slots take the tensor-core scan when the key form is prepared.
    tables = mgr.prepare_tensor_core(_alut.KEYS_RAW) if Q * S >= 768 else mgr.alut_tables()
    batch = _alut.make_batch(c["x"], c["sel"], c["vis"], c["reuse"])
    params = _alut.make_params(_alut.KEYS_RAW, False, False, 0.0, 0.0, 1e-6)
    out = torch.full((Q, mgr.hidden_dim), 7.0, dtype=torch.bfloat16, device=DEV)
    hit = torch.zeros(Q, S, dtype=torch.bool, device=DEV)
    idx = torch.zeros(Q, S, dtype=torch.long, device=DEV)
    common = (tables, ctypes.byref(batch), params, c["w"].data_ptr(), S, c["comp"].data_ptr(), S,
              _alut.RENORM_TO_ONE, 0, out.data_ptr(), out.stride(0), 1, hit.data_ptr(), idx.data_ptr(), S)
    if noalloc:
        rc = lib.alut_lookup_combine_noalloc(*common, _alut.stream_ptr(DEV))
        _alut.check(rc, "alut_lookup_combine_noalloc")
    else:
        ws = torch.zeros(lib.alut_workspace_size(tables, Q, S), dtype=torch.uint8, device=DEV)
        rc = lib.alut_lookup_combine(*common, ws.data_ptr(), ws.numel(), _alut.stream_ptr(DEV))
        _alut.check(rc, "alut_lookup_combine")
    torch.cuda.synchronize()
    return out, hit, idx


@pytest.mark.parametrize("Q,S", [(16, 8), (64, 4), (512, 4)])
def test_noalloc_matches_workspace_entry_on_consecutive_calls(manager, Q, S):
    """(16, 8): decode chain; (64, 4): planned CUDA-core scan; (512, 4): 2048 slots over 64
    tables with the tensor-core key form (tensor-core scan when its layout fits)."""
    lib = _alut.load()
    for seed in (1, 2):  # two calls in a row, different batches, the shared scratch reused
        c = _case(seed, Q=Q, S=S)
        ref_out, ref_hit, ref_idx = _run(lib, manager, c, noalloc=False)
        out, hit, idx = _run(lib, manager, c, noalloc=True)
        assert torch.equal(hit, ref_hit) and torch.equal(idx, ref_idx)
        check_combined(out.float().cpu().numpy(), ref_out.float().cpu().numpy(), what=f"noalloc call {seed}")


def test_noalloc_rejects_batches_beyond_the_fixed_scratch(manager):
    lib = _alut.load()
    c = _case(3)
    tables = manager.alut_tables()
    batch = _alut.make_batch(c["x"], c["sel"], c["vis"], c["reuse"])
    batch.q = 200_000  # host-side size check: nothing is launched
    params = _alut.make_params(_alut.KEYS_RAW, False, False, 0.0, 0.0, 1e-6)
    rc = lib.alut_lookup_combine_noalloc(tables, ctypes.byref(batch), params, None, 8, None, 8, 1, 0, None, 1024, 1,
                                         None, None, 8, _alut.stream_ptr(DEV))
    assert rc == _alut.ALUT_ERANGE
    assert b"scratch" in lib.alut_last_error()
    assert np.isfinite(_alut.NOALLOC_SCRATCH_BYTES)
