"""The centroid-range sharded table's exchange (all_gather of packed candidates, max merge,
owner gather, reduction of rows to each rank's token slice) on world_size-2 gloo process
groups on CPU.

The device steps of ShardedCentroidTable (scan of the local slice, merge, owner gather) are
replaced by numpy stand-ins with the same contracts; everything else - ranges, global
index offsets, the collectives, the masking of rows owned elsewhere - is the product code.
The CUDA kernels themselves are covered by tests/test_gpu_parity.py.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from table_moe.cache_engine.sharded import ShardedCentroidTable, shard_range


def _pack(score, idx):
    u = np.asarray(score, np.float32).view(np.uint32).astype(np.uint64)
    ordered = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return ((ordered << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(idx, np.uint64))).view(np.int64)


def _unpack(p):
    p = np.asarray(p).view(np.uint64)
    ordered = (p >> np.uint64(32)).astype(np.uint32)
    u = np.where(ordered & 0x80000000, ordered & 0x7FFFFFFF, ~ordered).astype(np.uint32)
    return u.view(np.float32), (np.uint64(0xFFFFFFFF) - (p & np.uint64(0xFFFFFFFF))).astype(np.int64)


def _problem(seed=0, Q=12, K=10, L=4, H=6):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((Q, L)).astype(np.float32)
    keys = rng.standard_normal((K, L)).astype(np.float32)
    keys[7] = keys[2]  # an exact tie across the two shards: the lower index must win
    q[3] = keys[2] * 2
    values = rng.standard_normal((K, H)).astype(np.float32)
    vis = rng.random(Q) < 0.5
    return q, keys, values, vis


def _worker(rank, world, port, out, replicate=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, keys, values, vis = _problem()
        K = keys.shape[0]
        k0, k1 = shard_range(K, world, rank)
        kk = keys if replicate else keys[k0:k1]
        shard_keys = torch.from_numpy(kk).view(1, 1, len(kk), -1).expand(1, 2, -1, -1).contiguous()
        shard_vals = torch.from_numpy(values[k0:k1]).view(1, 1, k1 - k0, -1).expand(1, 2, -1, -1).contiguous()
        t = ShardedCentroidTable(shard_keys, shard_vals, pca={}, k_total=K, thr_vision=-1e9, thr_text=0.5,
                                 replicate_keys=replicate)
        seen = []

        def local_search(x, is_vision):
            seen.append(len(x))
            s = x.numpy() @ shard_keys[0, 0].numpy().T  # [Q or Q/W, Kr]
            i = s.argmax(axis=1)
            return torch.from_numpy(_pack(s[np.arange(len(i)), i], i + t.key_base))

        def merge(packed_all, is_vision):
            best = packed_all.numpy().view(np.uint64).max(axis=0)
            score, idx = _unpack(best)
            thr = np.where(is_vision.numpy(), -1e9, 0.5).astype(np.float32)
            hit = score > thr
            return torch.from_numpy(hit), torch.from_numpy(np.where(hit, idx, 0))

        def gather_owned(hit, idx, is_vision):
            owned = hit.numpy() & (idx.numpy() >= t.k0) & (idx.numpy() < t.k1)
            rows = np.zeros((len(owned), shard_vals.shape[-1]), np.float32)
            rows[owned] = shard_vals[0, 0].numpy()[idx.numpy()[owned] - t.k0]
            return torch.from_numpy(rows)

        t.local_search, t.merge, t.gather_owned = local_search, merge, gather_owned
        hit, idx, rows = t.lookup(torch.from_numpy(q), torch.from_numpy(vis))
        out[rank] = (hit.numpy().copy(), idx.numpy().copy(), rows.numpy().copy(), seen)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("replicate", [False, True])
def test_sharded_lookup_matches_unsharded(replicate):
    """Centroid-range keys (every rank scans its key slice for all tokens) and replicated keys
    (every rank scans the whole table for its own tokens) give the same lookup."""
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out, replicate), nprocs=world, start_method="spawn",
                       join=True)
    q, keys, values, vis = _problem()
    s = q @ keys.T
    idx = s.argmax(axis=1)  # first maximal index
    best = s[np.arange(len(idx)), idx]
    hit = np.where(vis, best > -1e9, best > 0.5)
    assert idx[3] == 2  # the planted tie resolves to the lower index
    Q = q.shape[0]
    for r in range(world):
        h, i, rows, seen = out[r]
        assert seen == [Q // world if replicate else Q]  # tokens each rank scanned
        assert np.array_equal(h, hit) and np.array_equal(i, np.where(hit, idx, 0))
        lo, hi = Q * r // world, Q * (r + 1) // world
        ref = np.where(hit[:, None], values[idx], 0.0)[lo:hi]
        assert np.array_equal(rows, ref)


def test_shard_ranges_cover_the_table():
    for K in (1, 7, 65536):
        for W in (1, 2, 3, 8):
            spans = [shard_range(K, W, r) for r in range(W)]
            assert spans[0][0] == 0 and spans[-1][1] == K
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _failing_worker(rank, world, port, scenario, out, replicate=False):
    """Rank 1 stops after one lookup; rank 0's next lookup must end with an error within the
    limit instead of waiting: 'leave' announces it through the store, 'silent' just stops
    (rank 0's collective times out)."""
    import time

    from table_moe.cache_engine.sharded import PeerLeftError, ShardTimeoutError

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    store = dist.distributed_c10d._get_default_store()
    q, keys, values, vis = _problem()
    K = keys.shape[0]
    k0, k1 = shard_range(K, world, rank)
    kk = keys if replicate else keys[k0:k1]
    shard_keys = torch.from_numpy(kk).view(1, 1, len(kk), -1).expand(1, 2, -1, -1).contiguous()
    shard_vals = torch.from_numpy(values[k0:k1]).view(1, 1, k1 - k0, -1).expand(1, 2, -1, -1).contiguous()
    t = ShardedCentroidTable(shard_keys, shard_vals, pca={}, k_total=K, timeout_s=2.0, replicate_keys=replicate)
    t.local_search = lambda x, v: torch.from_numpy(_pack(np.zeros(len(x), np.float32), np.full(len(x), t.k0)))
    t.merge = lambda p, v: (torch.ones(p.shape[1], dtype=torch.bool), p[0] & 0)
    t.gather_owned = lambda h, i, v: torch.zeros(len(h), shard_vals.shape[-1])
    t.lookup(torch.from_numpy(q), torch.from_numpy(vis))  # one good step on both ranks
    if rank == 1:
        if scenario == "leave":
            t.leave()
        store.set("rank1_stopped", "1")
        store.wait(["rank0_done"], __import__("datetime").timedelta(seconds=30))
        out[rank] = "stopped"
        return
    store.wait(["rank1_stopped"])
    t0 = time.monotonic()
    try:
        t.lookup(torch.from_numpy(q), torch.from_numpy(vis))
        out[rank] = ("no error", time.monotonic() - t0)
    except PeerLeftError as exc:
        out[rank] = ("left", time.monotonic() - t0, str(exc))
    except ShardTimeoutError as exc:
        out[rank] = ("timeout", time.monotonic() - t0, str(exc))
    try:  # the table stays failed: no further collective is attempted
        t.lookup(torch.from_numpy(q), torch.from_numpy(vis))
        out["again"] = "no error"
    except PeerLeftError:
        out["again"] = "refused"
    store.set("rank0_done", "1")


@pytest.mark.timeout(120)
@pytest.mark.parametrize("scenario,expect,limit,replicate", [("leave", "left", 1.0, False),
                                                             ("silent", "timeout", 10.0, False),
                                                             ("silent", "timeout", 10.0, True)])
def test_sharded_lookup_fails_fast_when_a_rank_stops(scenario, expect, limit, replicate):
    world = 2
    out = mp.get_context("spawn").Manager().dict()
    ctx = mp.start_processes(_failing_worker, args=(world, _free_port(), scenario, out, replicate), nprocs=world,
                             start_method="spawn", join=False)
    while not ctx.join(timeout=60):
        pass
    assert out[1] == "stopped"
    kind, elapsed = out[0][0], out[0][1]
    assert kind == expect, out[0]
    assert elapsed < limit
    if scenario == "silent":
        assert elapsed >= 1.5  # it waited for the limit, not for ever
    assert out["again"] == "refused"
