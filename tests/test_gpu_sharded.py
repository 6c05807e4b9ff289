"""Centroid-range sharded table on the GPU: world 1 in process, and world 2 over NCCL when
the box has two GPUs. The sharded lookup must give the same (hit, idx) as the unsharded
search and bit-exact value rows for each rank's token slice."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

K, L, H, Q = 4096, 128, 512, 256


def _tables(device):
    g = torch.Generator().manual_seed(21)
    keys = torch.randn(1, 2, K, L, generator=g)
    values = (torch.randn(1, 2, K, H, generator=g) * 0.05).to(torch.bfloat16)
    proj = torch.stack([torch.linalg.qr(torch.randn(H, L, generator=g))[0] for _ in range(2)]).contiguous()
    x = torch.randn(Q, H, generator=g).to(torch.bfloat16)
    vis = torch.rand(Q, generator=g) < 0.5
    return keys, values, proj, x, vis


def _reference(device):
    from table_moe.cache_engine import HybridStorageManager, VectorSearchEngine

    keys, values, proj, x, vis = _tables(device)
    pca = {m: {"proj": proj[i].to(device), "bias": torch.zeros(L, device=device)} for i, m in enumerate(("vision", "text"))}
    mgr = HybridStorageManager.from_tables(0, keys.to(device), values.to(device), pca)
    eng = VectorSearchEngine(mgr)
    sel = torch.zeros(Q, 1, dtype=torch.long, device=device)
    reuse = torch.ones(Q, 1, dtype=torch.bool, device=device)
    hit, idx = eng.search_prefill_offline_dot(0, x.to(device), sel, vis.to(device), reuse)
    return hit[:, 0].cpu(), idx[:, 0].cpu(), values


def _sharded(device, world, rank, replicate=False):
    from table_moe.cache_engine.sharded import ShardedCentroidTable, shard_range

    keys, values, proj, x, vis = _tables(device)
    k0, k1 = shard_range(K, world, rank)
    pca = {m: {"proj": proj[i].to(device), "bias": torch.zeros(L, device=device)} for i, m in enumerate(("vision", "text"))}
    kr = keys if replicate else keys[:, :, k0:k1]
    t = ShardedCentroidTable(kr.contiguous().to(device), values[:, :, k0:k1].contiguous().to(device),
                             pca, K, replicate_keys=replicate)
    xd, vd = x.to(device), vis.to(device)
    hit, idx, rows = t.lookup(xd, vd)
    torch.cuda.synchronize(device)
    return hit.cpu(), idx.cpu(), rows.cpu()


def _check(hit, idx, rows, ref_hit, ref_idx, values, vis, lo, hi):
    assert torch.equal(hit, ref_hit) and torch.equal(idx, ref_idx)
    m = torch.where(vis, 0, 1)
    ref_rows = values[0, m, idx]
    ref_rows[~hit] = 0
    assert torch.equal(rows.view(torch.int16), ref_rows[lo:hi].view(torch.int16))


@pytest.mark.parametrize("replicate", [False, True])
def test_sharded_world1_matches_search(replicate):
    dev = torch.device("cuda:0")
    ref_hit, ref_idx, values = _reference(dev)
    hit, idx, rows = _sharded(dev, 1, 0, replicate)
    _check(hit, idx, rows, ref_hit, ref_idx, values, _tables(dev)[4], 0, Q)


def _worker(rank, world, port, out, replicate):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tablemoe-sc26_b200")]
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        out[rank] = _sharded(dev, world, rank, replicate)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("replicate", [False, True])
def test_sharded_world2_nccl_matches_search(replicate):
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, port, out, replicate), nprocs=world, start_method="spawn", join=True)
    dev = torch.device("cuda:0")
    ref_hit, ref_idx, values = _reference(dev)
    vis = _tables(dev)[4]
    for r in range(world):
        hit, idx, rows = out[r]
        _check(hit, idx, rows, ref_hit, ref_idx, values, vis, Q * r // world, Q * (r + 1) // world)


def test_sharded_world1_captured_graph_matches_eager():
    """The whole sharded lookup captured as a CUDA graph gives the eager results."""
    from table_moe.cache_engine.sharded import ShardedCentroidTable

    dev = torch.device("cuda:0")
    keys, values, proj, x, vis = _tables(dev)
    pca = {m: {"proj": proj[i].to(dev), "bias": torch.zeros(L, device=dev)} for i, m in enumerate(("vision", "text"))}
    t = ShardedCentroidTable(keys.to(dev), values.to(dev), pca, K)
    xd, vd = x.to(dev), vis.to(dev)
    h0, i0, r0 = (a.clone() for a in t.lookup(xd, vd))
    graph, (h1, i1, r1) = t.capture(xd, vd)
    h1.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(h0, h1) and torch.equal(i0, i1) and torch.equal(r0.view(torch.int16), r1.view(torch.int16))
    t.close()
