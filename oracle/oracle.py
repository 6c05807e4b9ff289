"""CPU oracle of the ALUT path (numpy front end of ``alut_oracle.c``).

TEST INFRASTRUCTURE ONLY: used by ``tests/`` as the parity checker, by
``__graft_entry__.smoke()`` as the checker of the smoke run, and by ``bench.py`` as the
timed CPU baseline. The product path (the ``table_moe`` package and ``libalut.so``) never
imports or calls it.

The C functions restate the reference's torch path (fanyalun/tablemoe-sc26):
``search.py:476-498`` projection, ``search.py:566-602`` / ``:661-697`` search,
``manager.py:212`` gather and ``cached_layers.py:455-465`` + ``skip/pruning.py:55-73``
combine. See ``alut_oracle.c`` for the per-function citations. ``online_search`` (numpy)
restates the online window lookup, ``search.py:778-806``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_lib = None

ROUND = {"float32": 0, "bfloat16": 1, "float16": 2}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_f = ctypes.c_float


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the Makefile beside this file."""
    src = _HERE / "alut_oracle.c"
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(_HERE), "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        L.oracle_project.argtypes = [_i64, _i64, _i64, _p, _p, _p, _p, _i, _i, _f, _p]
        L.oracle_search.argtypes = [_i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _f, _f,
                                    _i, _i, _p, _p, _p, _p]
        L.oracle_score.argtypes = [_i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64]
        L.oracle_score.restype = ctypes.c_double
        L.oracle_gather.argtypes = [_i64, _i64, _i64, _p, _i, _p, _p, _p, _p]
        L.oracle_combine.argtypes = [_i64, _i64, _i64, _i64, _i64, _p, _i, _p, _p, _p, _p, _p,
                                     _p, _i, _i, _p]
        L.oracle_round.argtypes = [_f, _i]
        L.oracle_round.restype = _f
        L.oracle_num_threads.restype = _i
        L.oracle_set_threads.argtypes = [_i]
        _lib = L
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def round_to(a, dtype: str):
    """Round fp32 values to `dtype` precision (round to nearest even), as fp32."""
    a = _c(a, np.float32)
    if dtype == "float32":
        return a.copy()
    f = lib().oracle_round
    m = ROUND[dtype]
    return np.vectorize(lambda v: f(float(v), m), otypes=[np.float32])(a)


def project(x, is_vision, proj, bias, dtype="float32", normalize=False, eps=1e-6):
    """q_low[Q,L] (fp32 holding `dtype` values). proj: [2,H,L]; bias: [2,L]."""
    x = _c(x, np.float32)
    Q, H = x.shape
    proj = _c(proj, np.float32)
    L = proj.shape[2]
    bias = _c(bias, np.float32)
    vis = _c(is_vision, np.uint8)
    out = np.empty((Q, L), np.float32)
    lib().oracle_project(Q, H, L, _ptr(x), _ptr(vis), _ptr(proj), _ptr(bias), ROUND[dtype],
                         int(bool(normalize)), float(eps), _ptr(out))
    return out


def search(q_low, keys, sel, is_vision, reuse=None, thr_vision=0.0, thr_text=0.0, cmp_ge=True,
           dtype="float32", with_gap=True):
    """Returns (hit [Q,S] bool, idx [Q,S] int64, best [Q,S] f32, gap [Q,S] f64 or None)."""
    q_low = _c(q_low, np.float32)
    keys = _c(keys, np.float32)
    sel = _c(sel, np.int64)
    Q, S = sel.shape
    E, _, K, L = keys.shape
    vis = _c(is_vision, np.uint8)
    ru = None if reuse is None else _c(reuse, np.uint8)
    hit = np.zeros((Q, S), np.uint8)
    idx = np.zeros((Q, S), np.int64)
    best = np.empty((Q, S), np.float32)
    gap = np.empty((Q, S), np.float64) if with_gap else None
    lib().oracle_search(Q, S, E, K, L, _ptr(q_low), _ptr(keys), _ptr(sel), _ptr(vis), _ptr(ru),
                        float(thr_vision), float(thr_text), int(bool(cmp_ge)), ROUND[dtype],
                        _ptr(hit), _ptr(idx), _ptr(best), _ptr(gap))
    return hit.astype(bool), idx, best, gap


def score(q_low, keys, sel, is_vision, t, s, k):
    """fp64 score of centroid k for slot (t, s)."""
    q_low = _c(q_low, np.float32)
    keys = _c(keys, np.float32)
    sel = _c(sel, np.int64)
    vis = _c(is_vision, np.uint8)
    S = sel.shape[1]
    K, L = keys.shape[2], keys.shape[3]
    return float(lib().oracle_score(S, K, L, _ptr(q_low), _ptr(keys), _ptr(sel), _ptr(vis),
                                    int(t), int(s), int(k)))


def _values(values):
    """(array, is_bf16): bf16 tables travel as their raw uint16 bits."""
    if values.dtype == np.uint16:
        return _c(values, np.uint16), 1
    return _c(values, np.float32), 0


def gather(values, eids, mids, cids):
    v, bf = _values(values)
    E, _, K, H = v.shape
    eids, mids, cids = (_c(a, np.int64) for a in (eids, mids, cids))
    n = eids.shape[0]
    out = np.empty((n, H), np.float32)
    lib().oracle_gather(n, K, H, _ptr(v), bf, _ptr(eids), _ptr(mids), _ptr(cids), _ptr(out))
    return out


def combine(values, sel, is_vision, hit, idx, weights, compute=None, renorm=1, out=None):
    """fp32 [Q,H]; `out` (fp32) is accumulated into when given."""
    v, bf = _values(values)
    E, _, K, H = v.shape
    sel = _c(sel, np.int64)
    Q, S = sel.shape
    vis = _c(is_vision, np.uint8)
    hit = _c(hit, np.uint8)
    idx = _c(idx, np.int64)
    w = _c(weights, np.float32)
    comp = None if compute is None else _c(compute, np.uint8)
    acc = 1 if out is not None else 0
    res = _c(out, np.float32).copy() if out is not None else np.empty((Q, H), np.float32)
    lib().oracle_combine(Q, S, E, K, H, _ptr(v), bf, _ptr(sel), _ptr(vis), _ptr(hit), _ptr(idx),
                         _ptr(w), _ptr(comp), int(renorm), acc, _ptr(res))
    return res


def bf16_bits(a_f32):
    """fp32 -> bf16 bit patterns (round to nearest even) as uint16."""
    a = _c(a_f32, np.float32).view(np.uint32).astype(np.uint64)
    r = (a + 0x7FFF + ((a >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(bits):
    return (_c(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


if os.environ.get("ALUT_ORACLE_REBUILD"):
    build(force=True)


def online_search(x_bits, key_bits, eids, target, n_valid):
    """The online window lookup (search.py:778-806, ``_search_decode_online_into``).

    x_bits [B,H] and key_bits [N,H] are bf16 bit patterns (the model dtype). Scores are
    the matmul of the two in bf16 - accumulated in fp32, rounded to bf16 - over the first
    n_valid window entries; per token the first index of the maximum; a token is valid iff
    its maximum is > 0 (then on_idx = that index, else -1). For each target expert id
    target[b, s]: on_hit = valid and the id is among eids[on_idx]; on_slot = the first
    position of the id there (0 where no hit). Returns (on_hit, on_idx, on_slot, scores).
    """
    x = bf16_to_f32(np.asarray(x_bits)).reshape(np.shape(x_bits))
    k = bf16_to_f32(np.asarray(key_bits)).reshape(np.shape(key_bits))[:n_valid]
    scores = bf16_to_f32(bf16_bits((x @ k.T).astype(np.float32))).reshape(x.shape[0], -1)
    arg = scores.argmax(axis=1)  # first index of the maximum
    valid = scores[np.arange(x.shape[0]), arg] > 0
    on_idx = np.where(valid, arg, -1).astype(np.int64)
    cached = np.asarray(eids)[arg]                              # [B, T]
    match = np.asarray(target)[:, :, None] == cached[:, None, :]  # [B, S, T]
    on_hit = match.any(-1) & valid[:, None]
    on_slot = np.where(on_hit, match.argmax(-1), 0).astype(np.int64)
    return on_hit, on_idx, on_slot, scores
