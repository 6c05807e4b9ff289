"""HybridStorageManager against fixtures made by the reference's own manager
(tests/golden/make_golden_manager.py): the online ring buffer on CPU tensors (its updates
are device-agnostic slice copies), and the table loader on the GPU (keys normalised by
the alut_normalize_rows kernel)."""
import json

import numpy as np
import pytest
import torch

from parity import GOLDEN
from table_moe.cache_engine import HybridStorageManager
from table_moe.cache_engine import config as cfg


@pytest.fixture
def active_config():
    saved = cfg.get_active_cache_config()
    yield cfg
    cfg.set_active_cache_config(saved)


def _load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return json.loads(str(z["meta"])), {k: z[k] for k in z.files if k != "meta"}


def test_online_ring_buffer_matches_reference(active_config):
    meta, d = _load("manager_online")
    cfg.set_active_cache_config(dict(FIXED_K=4, COMPRESSED_DIM=4, ONLINE_CACHE_SIZE=meta["size"],
                                     ONLINE_TOP_K=meta["topk"], MODEL_DTYPE="float32"))
    m = HybridStorageManager(1, 4, meta["h"], device="cpu", load=False)
    assert m.enable_online and m.online_size == meta["size"]
    for i, st in enumerate(meta["steps"]):
        x, ids, vals = (torch.from_numpy(d[f"in{i}_{k}"]) for k in ("x", "ids", "vals"))
        mask = torch.from_numpy(d[f"in{i}_mask"]) if f"in{i}_mask" in d else None
        if st["kind"] == "bs1":
            m.update_online_cache_bs1(x[0], ids[0], vals[0], None if mask is None else mask[0])
        else:
            m.update_online_cache(x, ids, vals, mask)
        assert m.online_ptr == st["ptr"] and bool(m.online_full) == st["full"], f"step {i}"
        assert np.array_equal(m.online_keys.numpy(), d[f"st{i}_keys"]), f"keys, step {i}"
        assert np.array_equal(m.online_expert_ids.numpy(), d[f"st{i}_ids"]), f"ids, step {i}"
        assert np.array_equal(m.online_values.numpy(), d[f"st{i}_vals"]), f"values, step {i}"


def _as_tensor(a, dtype):
    t = torch.from_numpy(a)
    return t.view(torch.bfloat16) if dtype == "bfloat16" else t


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_table_loader_matches_reference(dtype, tmp_path, active_config):
    meta, d = _load(f"manager_load_{dtype}")
    lay = meta["layer"]
    root = tmp_path / f"layer_{lay}"
    root.mkdir()
    torch.save({"mean": torch.from_numpy(d["pca_text_mean"]), "proj": torch.from_numpy(d["pca_text_proj"])},
               root / f"L{lay}_text_pca.pt")
    for e, mod, _ in meta["files"]:
        torch.save({"key": torch.from_numpy(d[f"file_E{e}_{mod}_key"]),
                    "value": torch.from_numpy(d[f"file_E{e}_{mod}_value"])}, root / f"L{lay}_E{e}_{mod}_cache.pt")
    cfg.set_active_cache_config(dict(PCA_DIR=str(tmp_path), CACHE_DIR=str(tmp_path), FIXED_K=meta["K"],
                                     COMPRESSED_DIM=meta["L"], MODEL_DTYPE=dtype))
    m = HybridStorageManager(lay, meta["E"], meta["H"], device="cuda:0")
    torch.cuda.synchronize()
    dt = {"bfloat16": torch.bfloat16, "float32": torch.float32}[dtype]
    # The reference allocates values_buffer uninitialised (torch.empty, manager.py:54): only the
    # rows loaded from files are defined there; ours are zero elsewhere.
    ref_vals = _as_tensor(d["ref_values"], dtype)
    mm = {"vision": 0, "text": 1}
    for e, mod, rows in meta["files"]:
        if mod in mm and e < meta["E"]:
            assert torch.equal(m.values_buffer[e, mm[mod], :rows].cpu(), ref_vals[e, mm[mod], :rows]), (e, mod)
    exact = {"raw_keys": m.raw_keys_buffer,
             "vision_proj": m.pca["vision"]["proj"], "text_proj": m.pca["text"]["proj"],
             "vision_bias": m.pca["vision"]["bias"]}
    for name, t in exact.items():
        assert torch.equal(t.cpu(), _as_tensor(d[f"ref_{name}"], dtype)), name
    # bias = -mean @ proj: a matmul, equal to rounding of the table dtype
    bias_ref = _as_tensor(d["ref_text_bias"], dtype).float()
    tol = (2 ** -7 if dtype == "bfloat16" else 1e-5) * bias_ref.abs().max()
    assert torch.allclose(m.pca["text"]["bias"].cpu().float(), bias_ref, atol=float(tol))
    # normalised keys: fp32 arithmetic on the device, rounded to the table dtype (summation
    # order of the norm may move a value by one unit of the dtype)
    got, ref = m.keys_buffer.cpu().float(), _as_tensor(d["ref_keys"], dtype).float()
    ulp = 2 ** -8 if dtype == "bfloat16" else 2 ** -23
    assert torch.all((got - ref).abs() <= 2 * ulp * ref.abs() + 1e-30)
    assert torch.equal(got == 0, ref == 0)
    assert m.keys_buffer.dtype == dt
