"""Golden fixtures of the table loader and the online ring buffer, made by the reference's
own ``HybridStorageManager`` (``table_moe/cache_engine/manager.py``).

Run where the reference project (fanyalun/tablemoe-sc26) is checked out:

    python tests/golden/make_golden_manager.py --reference /path/to/tablemoe-sc26

* ``manager_load_<dtype>.npz``: a small table tree in the reference's on-disk format
  (``layer_{l}/L{l}_{mod}_pca.pt`` = {mean, proj}; ``layer_{l}/L{l}_E{e}_{mod}_cache.pt`` =
  {key, value}), with a missing vision PCA, tables shorter than FIXED_K, a file of an
  unknown modality and one of an out-of-range expert; the file contents and the buffers
  the reference's loader (``manager.py:157-210``) builds from them.
* ``manager_online.npz``: a sequence of ``update_online_cache`` / ``update_online_cache_bs1``
  calls (``manager.py:89-155``: wrap-around, batches larger than the window, valid-slot
  masks) and the ring state (keys, expert ids, values, pointer, full flag) after each.

The reference allocates its value table in pinned host memory; this script runs on a CPU
only machine, so ``pin_memory`` is dropped while the reference manager is constructed.
"""
from __future__ import annotations

import argparse
import json
import sys
import tempfile
from pathlib import Path
from unittest import mock

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
LAYER, E, H, K_FIXED, L = 3, 4, 24, 8, 16
FILES = [  # (expert, modality, rows)
    (0, "text", 8), (0, "vision", 5), (1, "text", 3), (2, "vision", 8), (3, "text", 1),
    (1, "audio", 4),   # unknown modality: skipped
    (7, "text", 4),    # expert id beyond num_experts: skipped
]


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy() if t.dtype != torch.float32 else \
        t.contiguous().numpy().copy()


def _unpinned_empty(real_empty):
    def empty(*a, **kw):
        kw.pop("pin_memory", None)
        return real_empty(*a, **kw)
    return empty


def write_tree(root: Path, g):
    """The table tree; returns its contents as arrays (fp32)."""
    d = root / f"layer_{LAYER}"
    d.mkdir(parents=True)
    content = {}
    mean = torch.randn(H, generator=g)
    proj = torch.linalg.qr(torch.randn(H, L, generator=g))[0]
    torch.save({"mean": mean, "proj": proj}, d / f"L{LAYER}_text_pca.pt")
    content["pca_text_mean"], content["pca_text_proj"] = mean.numpy(), proj.numpy()
    for e, mod, rows in FILES:
        key = torch.randn(rows, L, generator=g) * 2
        if rows > 2:
            key[1] = 0.0  # a zero key row: normalised to zero
        value = torch.randn(rows, H, generator=g) * 0.05
        torch.save({"id": torch.arange(rows), "key": key, "value": value}, d / f"L{LAYER}_E{e}_{mod}_cache.pt")
        content[f"file_E{e}_{mod}_key"], content[f"file_E{e}_{mod}_value"] = key.numpy(), value.numpy()
    return content


def load_case(ref_mod, cfg_mod, dtype_name):
    g = torch.Generator().manual_seed(17)
    with tempfile.TemporaryDirectory() as tmp:
        content = write_tree(Path(tmp), g)
        cfg_mod.set_active_cache_config(dict(PCA_DIR=tmp, CACHE_DIR=tmp, FIXED_K=K_FIXED, COMPRESSED_DIM=L,
                                             MODEL_DTYPE=dtype_name))
        with mock.patch.object(torch, "empty", _unpinned_empty(torch.empty)):
            m = ref_mod.HybridStorageManager(LAYER, E, H, device="cpu")
    out = dict(content)
    out["ref_keys"], out["ref_raw_keys"], out["ref_values"] = (_bits(m.keys_buffer), _bits(m.raw_keys_buffer),
                                                               _bits(m.values_buffer))
    for mod in ("vision", "text"):
        out[f"ref_{mod}_proj"], out[f"ref_{mod}_bias"] = _bits(m.pca[mod]["proj"]), _bits(m.pca[mod]["bias"])
    meta = dict(layer=LAYER, E=E, H=H, K=K_FIXED, L=L, dtype=dtype_name, files=FILES)
    np.savez_compressed(HERE / f"manager_load_{dtype_name}.npz", meta=json.dumps(meta), **out)
    print("load", dtype_name, "ok")


def online_case(ref_mod, cfg_mod):
    g = torch.Generator().manual_seed(23)
    size, topk, h = 5, 3, 6
    cfg_mod.set_active_cache_config(dict(PCA_DIR="/nonexistent", CACHE_DIR="/nonexistent", FIXED_K=4,
                                         COMPRESSED_DIM=4, ONLINE_CACHE_SIZE=size, ONLINE_TOP_K=topk,
                                         MODEL_DTYPE="float32"))
    with mock.patch.object(torch, "empty", _unpinned_empty(torch.empty)):
        m = ref_mod.HybridStorageManager(1, 4, h, device="cpu")
    ops = [("bs1", 1, True), ("batch", 3, False), ("batch", 2, True), ("bs1", 1, False), ("batch", 7, True),
           ("batch", 4, False), ("bs1", 1, True), ("batch", 0, False), ("batch", 5, False)]
    arrays, steps = {}, []
    for i, (kind, n, masked) in enumerate(ops):
        nn = max(n, 1)
        x = torch.randn(nn, h, generator=g)
        ids = torch.randint(0, 4, (nn, topk), generator=g)
        vals = torch.randn(nn, topk, h, generator=g)
        mask = torch.rand(nn, topk, generator=g) < 0.7 if masked else None
        if kind == "bs1":
            m.update_online_cache_bs1(x[0], ids[0], vals[0], None if mask is None else mask[0])
        else:
            x, ids, vals = x[:n], ids[:n], vals[:n]
            mask = None if mask is None else mask[:n]
            m.update_online_cache(x, ids, vals, mask)
        arrays[f"in{i}_x"], arrays[f"in{i}_ids"], arrays[f"in{i}_vals"] = x.numpy(), ids.numpy(), vals.numpy()
        if mask is not None:
            arrays[f"in{i}_mask"] = mask.numpy()
        arrays[f"st{i}_keys"] = m.online_keys.numpy().copy()
        arrays[f"st{i}_ids"] = m.online_expert_ids.numpy().copy()
        arrays[f"st{i}_vals"] = m.online_values.numpy().copy()
        steps.append(dict(kind=kind, n=n, masked=masked, ptr=m.online_ptr, full=bool(m.online_full)))
    meta = dict(size=size, topk=topk, h=h, steps=steps)
    np.savez_compressed(HERE / "manager_online.npz", meta=json.dumps(meta), **arrays)
    print("online ok", [s["ptr"] for s in steps])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from table_moe.cache_engine import config as cfg_mod
    from table_moe.cache_engine import manager as ref_mod

    for dt in ("bfloat16", "float32"):
        load_case(ref_mod, cfg_mod, dt)
    online_case(ref_mod, cfg_mod)


if __name__ == "__main__":
    main()
