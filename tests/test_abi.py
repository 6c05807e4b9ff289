"""The C-ABI library loads, exports every entry point declared in include/alut.h, and
rejects bad arguments on the host before anything reaches the GPU (no CUDA call is made
by these tests)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from table_moe.cache_engine import _alut

HEADER = Path(__file__).resolve().parents[1] / "include" / "alut.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w]+\s*\*?\s*(alut_\w+)\s*\(", text, re.M)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for name in ("alut_search", "alut_project", "alut_gather_rows", "alut_combine", "alut_lookup_combine",
                 "alut_search_packed", "alut_merge_packed", "alut_workspace_size"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    lib = _alut.load()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    assert set(_alut.SIGNATURES) >= set(declared_symbols())
    assert lib.alut_version() >= 100


def _tables(E=4, K=100, L=64, H=256, dtype=torch.float32):
    keys = torch.zeros(E, 2, K, L, dtype=dtype)
    values = torch.zeros(E, 2, K, H, dtype=torch.bfloat16)
    proj = torch.zeros(H, L, dtype=dtype)
    bias = torch.zeros(L, dtype=dtype)
    return _alut.make_tables(keys, keys, values, proj, bias, proj, bias), (keys, values, proj, bias)


def test_workspace_size_is_positive_and_monotone():
    lib = _alut.load()
    t, _ = _tables()
    a = lib.alut_workspace_size(t, 16, 8)
    b = lib.alut_workspace_size(t, 4096, 8)
    assert 0 < a <= b
    assert a % 256 == 0
    assert lib.alut_workspace_size(None, 16, 8) == 0


def test_argument_errors_are_reported_without_launch():
    lib = _alut.load()
    t, _ = _tables()
    p = _alut.make_params(_alut.KEYS_RAW, False, False, 0.0, 0.0, 1e-6)
    b = _alut.Batch()
    assert lib.alut_search(None, ctypes.byref(b), p, None, None, None, 1, None, 0, None) == _alut.ALUT_EINVAL
    assert b"tables is NULL" in lib.alut_last_error()
    t.l = 1000
    assert lib.alut_search(t, ctypes.byref(b), p, None, None, None, 1, None, 0, None) == _alut.ALUT_ERANGE
    t.l = 64
    b.q, b.s = 4, 100
    assert lib.alut_search(t, ctypes.byref(b), p, None, None, None, 1, None, 0, None) == _alut.ALUT_ERANGE
    b.q, b.s = 0, 8
    # Empty batches are a no-op.
    assert lib.alut_search(t, ctypes.byref(b), p, None, None, None, 8, None, 0, None) == _alut.ALUT_OK
    t.key_dtype = 7
    b.q = 3
    assert lib.alut_search(t, ctypes.byref(b), p, None, None, None, 8, None, 0, None) == _alut.ALUT_EDTYPE


def test_check_maps_status_to_python_errors():
    _alut.load()
    with pytest.raises(ValueError):
        _alut.check(_alut.ALUT_ESHAPE, "x")
    with pytest.raises(RuntimeError):
        _alut.check(_alut.ALUT_ECUDA, "x")
    _alut.check(_alut.ALUT_OK, "x")


def test_make_tables_rejects_mismatched_shapes():
    keys = torch.zeros(4, 2, 10, 8)
    with pytest.raises(ValueError):
        _alut.make_tables(keys, keys, torch.zeros(4, 2, 11, 16, dtype=torch.bfloat16),
                          torch.zeros(16, 8), torch.zeros(8), torch.zeros(16, 8), torch.zeros(8))
    with pytest.raises(ValueError):
        _alut.make_tables(keys, keys, None, torch.zeros(16, 8), torch.zeros(8), torch.zeros(16, 4), torch.zeros(4))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setenv("TABLEMOE_ALUT_LIB", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_alut, "_lib", None)
    with pytest.raises(ImportError):
        _alut.load()


def _integration_stub_structs():
    """Run the struct definitions of the ctypes stub documented for maintainers (the python
    block of INTEGRATION.md) without its library load or calls."""
    text = (Path(__file__).resolve().parents[1] / "INTEGRATION.md").read_text()
    block = re.search(r"```python\n(.*?)```", text, re.S).group(1)
    defs = block[:block.index("lib.alut_search")].replace('lib = ctypes.CDLL("libalut.so")', "")
    ns = {}
    exec(defs, ns)
    return ns


@pytest.mark.parametrize("stub,ours", [("alut_tables_t", "Tables"), ("alut_batch_t", "Batch"),
                                       ("alut_search_params_t", "SearchParams")])
def test_integration_stub_matches_the_binding(stub, ours):
    """The documented stub has the binding's size and field offsets (a short struct would
    make the library read past its end)."""
    a, b = _integration_stub_structs()[stub], getattr(_alut, ours)
    assert ctypes.sizeof(a) == ctypes.sizeof(b)
    assert [(n, getattr(a, n).offset) for n, _ in a._fields_] == [(n, getattr(b, n).offset) for n, _ in b._fields_]


def test_scan_kind_follows_the_measured_crossovers():
    """alut_scan_kind is a host-side rule (no GPU): decode chain up to 256 slots,
    tensor-core scan from 512 slots with >= 12 slots per routed table, else CUDA-core."""
    lib = _alut.load()
    t, _ = _tables(E=128, K=1024, L=64, H=256)
    assert lib.alut_scan_kind(t, 16, 8) == _alut.SCAN_DECODE
    assert lib.alut_scan_kind(t, 256, 1) == _alut.SCAN_DECODE        # any token count up to 256 slots
    assert lib.alut_scan_kind(t, 33, 8) == _alut.SCAN_CUDA_CORE      # 264 slots
    assert lib.alut_scan_kind(t, 64, 8) == _alut.SCAN_CUDA_CORE      # 2 slots per table
    assert lib.alut_scan_kind(t, 512, 8) == _alut.SCAN_TENSOR_CORE   # 16 per table
    assert lib.alut_scan_kind(t, 4096, 8) == _alut.SCAN_TENSOR_CORE
    t96, _ = _tables(E=72, K=2048, L=96, H=256)
    assert lib.alut_scan_kind(t96, 8, 6) == _alut.SCAN_DECODE
    assert lib.alut_scan_kind(t96, 2048, 6) == _alut.SCAN_TENSOR_CORE
    t12, _ = _tables(E=4, K=100, L=12, H=256)  # L % 16 != 0: never the tensor cores
    assert lib.alut_scan_kind(t12, 4096, 8) == _alut.SCAN_CUDA_CORE
    assert lib.alut_scan_kind(None, 1, 1) < 0
