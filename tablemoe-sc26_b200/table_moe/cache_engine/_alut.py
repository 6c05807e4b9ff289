"""ctypes binding of ``libalut.so``, the sm_100a ALUT kernels behind the C ABI of
``include/alut.h``.

There is no fallback: if the library is missing or fails to load, importing the engine
raises. The library is looked up at ``$TABLEMOE_ALUT_LIB`` or at ``lib/libalut.so`` beside
this package's parent directory (the in-tree build of ``__graft_entry__.build()``),
mirroring the prebuilt-extension lookup of the reference
(``table_moe/ops/_prebuilt.py:8-50``).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_PKG_ROOT = Path(__file__).resolve().parents[2]  # .../tablemoe-sc26_b200
DEFAULT_LIB = _PKG_ROOT / "lib" / "libalut.so"

ALUT_OK = 0
ALUT_EINVAL, ALUT_EDTYPE, ALUT_ESHAPE, ALUT_ECUDA, ALUT_EWORKSPACE, ALUT_ERANGE = -1, -2, -3, -4, -5, -6
KEYS_NORMALISED, KEYS_RAW = 0, 1
RENORM_NONE, RENORM_TO_ONE, RENORM_TO_ROWSUM = 0, 1, 2
NOALLOC_SCRATCH_BYTES = 2 << 20  # ALUT_NOALLOC_SCRATCH_BYTES
PEER_HANDLE_BYTES = 64  # ALUT_PEER_HANDLE_BYTES
SCAN_DECODE, SCAN_CUDA_CORE, SCAN_TENSOR_CORE = 0, 1, 2  # alut_scan_kind
ERR_BAD_EXPERT, ERR_COPY_TIMEOUT, ERR_MMA_TIMEOUT = 1, 4, 8  # ALUT_ERR_* device error bits

_DTYPE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


class Tables(ctypes.Structure):
    _fields_ = [
        ("num_experts", ctypes.c_int32), ("k", ctypes.c_int32), ("l", ctypes.c_int32),
        ("h", ctypes.c_int32), ("key_dtype", ctypes.c_int32), ("value_dtype", ctypes.c_int32),
        ("proj_dtype", ctypes.c_int32), ("reserved0", ctypes.c_int32),
        ("keys", ctypes.c_void_p), ("raw_keys", ctypes.c_void_p), ("values", ctypes.c_void_p),
        ("proj", ctypes.c_void_p * 2), ("bias", ctypes.c_void_p * 2),
        ("key_stride", ctypes.c_int64 * 3), ("value_stride", ctypes.c_int64 * 3),
        ("proj_stride_h", ctypes.c_int64), ("proj_split", ctypes.c_void_p),
        ("keys_split", ctypes.c_void_p), ("raw_keys_split", ctypes.c_void_p),
    ]


class Batch(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_int32), ("s", ctypes.c_int32), ("x_dtype", ctypes.c_int32),
        ("reserved0", ctypes.c_int32), ("x", ctypes.c_void_p), ("x_stride", ctypes.c_int64),
        ("sel", ctypes.c_void_p), ("sel_stride", ctypes.c_int64), ("is_vision", ctypes.c_void_p),
        ("reuse", ctypes.c_void_p), ("reuse_stride", ctypes.c_int64),
    ]


class SearchParams(ctypes.Structure):
    _fields_ = [
        ("keyset", ctypes.c_int32), ("normalize_q", ctypes.c_int32), ("cmp_ge", ctypes.c_int32),
        ("reserved0", ctypes.c_int32), ("thr_vision", ctypes.c_float), ("thr_text", ctypes.c_float),
        ("eps", ctypes.c_float), ("reserved1", ctypes.c_float),
    ]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_TP = ctypes.POINTER(Tables)
_BP = ctypes.POINTER(Batch)
_PP = ctypes.POINTER(SearchParams)

SIGNATURES = {
    "alut_workspace_size": (_SZ, [_TP, _I32, _I32]),
    "alut_scan_kind": (ctypes.c_int, [_TP, _I32, _I32]),
    "alut_basis_split_bytes": (_SZ, [_TP]),
    "alut_keys_split_bytes": (_SZ, [_TP]),
    "alut_prepare_keys": (ctypes.c_int, [_TP, _I32, _P, _SZ, _P]),
    "alut_prepare_basis": (ctypes.c_int, [_TP, _P, _SZ, _P]),
    "alut_project": (ctypes.c_int, [_TP, _BP, _I32, ctypes.c_float, _P, _I64, _P, _SZ, _P]),
    "alut_search": (ctypes.c_int, [_TP, _BP, _PP, _P, _P, _P, _I64, _P, _SZ, _P]),
    "alut_gather_rows": (ctypes.c_int, [_TP, _I32, _P, _P, _P, _P, _P, _I64, _P]),
    "alut_combine": (ctypes.c_int, [_TP, _BP, _P, _P, _I64, _P, _I64, _P, _I64, _I32, _I32, _P,
                                    _I64, _I32, _P]),
    "alut_lookup_combine": (ctypes.c_int, [_TP, _BP, _PP, _P, _I64, _P, _I64, _I32, _I32, _P, _I64,
                                           _I32, _P, _P, _I64, _P, _SZ, _P]),
    "alut_lookup_combine_experts": (ctypes.c_int, [_TP, _BP, _PP, _P, _I64, _P, _I64, _P, _I64, _I64, _I32, _I32,
                                                   _P, _I64, _I32, _P, _P, _I64, _P, _SZ, _P]),
    "alut_lookup_combine_noalloc": (ctypes.c_int, [_TP, _BP, _PP, _P, _I64, _P, _I64, _I32, _I32, _P, _I64,
                                                   _I32, _P, _P, _I64, _P]),
    "alut_search_packed": (ctypes.c_int, [_TP, _BP, _PP, _P, _I64, _P, _P, _SZ, _P]),
    "alut_merge_packed": (ctypes.c_int, [_I32, _I32, _I32, _P, _P, _PP, _P, _P, _P]),
    "alut_online_search": (ctypes.c_int, [_I32, _I32, _I32, _I32, _I32, _P, _I32, _I64, _P, _I32, _I64, _P, _P,
                                          _I64, _P, _P, _P, _I64, _P]),
    "alut_peer_export": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_uint64)]),
    "alut_peer_open": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "alut_peer_close": (ctypes.c_int, [_P, ctypes.c_uint64]),
    "alut_gather_rows_sharded": (ctypes.c_int, [_I32, _P, _P, _P, _I32, _P, _P, _P, _I64, _I32, _I32, _P, _I64,
                                                _P]),
    "alut_route_workspace_size": (_SZ, [_I32]),
    "alut_route": (ctypes.c_int, [_I32, _I32, _I32, _P, _I32, _I64, _I32, _I32, _I32, ctypes.c_double, _P, _P, _P, _P,
                                  _P, _I64, _P, _SZ, _P]),
    "alut_keep_mask": (ctypes.c_int, [_I32, _I32, _I32, _P, _P, _I64, _P, ctypes.c_double, _P, _P, _I64, _P, _SZ,
                                      _P]),
    "alut_normalize_rows": (ctypes.c_int, [_I64, _I32, _P, _I64, _P, _I64, _I32, ctypes.c_float, _P]),
    "alut_workspace_errors": (ctypes.c_int, [_P, _SZ, _I32, ctypes.POINTER(ctypes.c_uint32), _P]),
    "alut_set_profile_events": (ctypes.c_int, [_P, _P]),
    "alut_last_error": (ctypes.c_char_p, []),
    "alut_version": (ctypes.c_int, []),
}

_lib = None


def lib_path() -> Path:
    raw = os.environ.get("TABLEMOE_ALUT_LIB")
    return Path(raw).expanduser().resolve() if raw else DEFAULT_LIB


def load():
    """Load libalut.so (once). Raises ImportError if it is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not path.exists():
        raise ImportError(
            f"libalut.so not found at {path}; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "or point TABLEMOE_ALUT_LIB at it (the ALUT path has no CPU or Triton fallback)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc == ALUT_OK:
        return
    msg = load().alut_last_error().decode(errors="replace")
    if rc in (ALUT_EINVAL, ALUT_EDTYPE, ALUT_ESHAPE, ALUT_ERANGE):
        raise ValueError(f"{what}: {msg} (status {rc})")
    raise RuntimeError(f"{what}: {msg} (status {rc})")


def device_errors(workspace, nbytes, device, clear=True) -> int:
    """Error bits the kernels left in a workspace (workspace None: the no-allocation
    scratch); waits for the current stream."""
    bits = ctypes.c_uint32(0)
    check(load().alut_workspace_errors(workspace, nbytes, int(clear), ctypes.byref(bits), stream_ptr(device)),
          "alut_workspace_errors")
    return int(bits.value)


def raise_device_errors(bits: int, what: str) -> None:
    """Map device error bits to the exceptions the reference raises (IndexError for an
    expert id outside the table, as its tensor indexing does) or RuntimeError."""
    if bits & ERR_BAD_EXPERT:
        raise IndexError(f"{what}: a searched slot's expert id is outside [0, num_experts)")
    if bits:
        raise RuntimeError(f"{what}: a device wait timed out (error bits {bits:#x}); results are incomplete")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _inner_contig(t: torch.Tensor, name: str) -> None:
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have unit innermost stride")


def make_tables(keys, raw_keys, values, proj_vis, bias_vis, proj_txt, bias_txt, proj_split=None) -> Tables:
    """Describe one layer's tables. keys/raw_keys: [E,2,K,L]; values: [E,2,K,H];
    proj: [H,L]; bias: [L]. keys, raw_keys or values may be None. proj_split: the bf16
    split basis written by alut_prepare_basis (optional)."""
    ref = keys if keys is not None else raw_keys
    if ref is None:
        raise ValueError("keys and raw_keys cannot both be None")
    if raw_keys is not None and keys is not None:
        if raw_keys.shape != keys.shape or raw_keys.stride() != keys.stride() or raw_keys.dtype != keys.dtype:
            raise ValueError("keys and raw_keys must share shape, strides and dtype")
    E, M, K, L = ref.shape
    if M != 2:
        raise ValueError("key tables must be [E, 2, K, L]")
    _inner_contig(ref, "keys")
    t = Tables()
    t.num_experts, t.k, t.l = E, K, L
    t.key_dtype = dtype_code(ref.dtype)
    t.keys = ptr(keys)
    t.raw_keys = ptr(raw_keys)
    t.key_stride[:] = list(ref.stride()[:3])
    H = proj_vis.shape[0] if proj_vis is not None else (values.shape[3] if values is not None else 0)
    t.h = H
    if values is not None:
        if values.shape[:3] != (E, 2, K):
            raise ValueError(f"values shape {tuple(values.shape)} does not match keys {tuple(ref.shape)}")
        _inner_contig(values, "values")
        t.h = values.shape[3]
        t.values = ptr(values)
        t.value_dtype = dtype_code(values.dtype)
        t.value_stride[:] = list(values.stride()[:3])
    else:
        t.value_dtype = 1
    if proj_vis is not None:
        for p, b in ((proj_vis, bias_vis), (proj_txt, bias_txt)):
            if p.shape != proj_vis.shape or p.stride() != proj_vis.stride() or p.dtype != proj_vis.dtype:
                raise ValueError("vision/text projections must share shape, strides and dtype")
            if p.shape[1] != L:
                raise ValueError("vision/text PCA projection dims must match the key dim")
            if b.dtype != p.dtype or b.numel() != L or (b.dim() == 1 and b.stride(0) != 1):
                raise ValueError("bias must be a contiguous [L] tensor of the projection dtype")
            _inner_contig(p, "proj")
        t.proj[0], t.proj[1] = proj_vis.data_ptr(), proj_txt.data_ptr()
        t.bias[0], t.bias[1] = bias_vis.data_ptr(), bias_txt.data_ptr()
        t.proj_dtype = dtype_code(proj_vis.dtype)
        t.proj_stride_h = proj_vis.stride(0)
        if values is not None and values.shape[3] != proj_vis.shape[0]:
            raise ValueError(f"values hidden size {values.shape[3]} != projection rows {proj_vis.shape[0]}")
        t.h = proj_vis.shape[0]
    else:
        t.proj_dtype = t.key_dtype
    if proj_split is not None:
        t.proj_split = proj_split.data_ptr()
    return t


def prepare_basis(tables: Tables, device):
    """The tensor-core split of an fp32 basis (a static [2,3,L,H] bf16 tensor), or None when
    the tables do not qualify. Made once per table load."""
    lib = load()
    n = int(lib.alut_basis_split_bytes(tables))
    if n == 0:
        return None
    out = torch.empty(n // 2, dtype=torch.bfloat16, device=device)
    check(lib.alut_prepare_basis(tables, out.data_ptr(), n, stream_ptr(device)), "alut_prepare_basis")
    return out


def make_batch(x, sel, is_vision, reuse) -> Batch:
    """Describe one batch. The struct holds raw device pointers only: the caller keeps the
    tensors alive (and unmodified) until the work using them has been issued and run."""
    b = Batch()
    Q, S = sel.shape
    b.q, b.s = Q, S
    _inner_contig(sel, "selected_experts")
    if sel.dtype != torch.int64:
        raise ValueError("selected_experts must be int64")
    b.sel, b.sel_stride = sel.data_ptr(), sel.stride(0)
    if is_vision.dtype not in (torch.bool, torch.uint8) or not is_vision.is_contiguous():
        raise ValueError("is_vision_mask must be a contiguous bool tensor")
    b.is_vision = is_vision.data_ptr()
    if x is not None:
        _inner_contig(x, "hidden_states")
        b.x, b.x_stride, b.x_dtype = x.data_ptr(), x.stride(0), dtype_code(x.dtype)
    if reuse is not None:
        if reuse.dtype not in (torch.bool, torch.uint8):
            raise ValueError("reuse_mask must be bool")
        _inner_contig(reuse, "reuse_mask")
        b.reuse, b.reuse_stride = reuse.data_ptr(), reuse.stride(0)
    return b


def make_params(keyset, normalize, cmp_ge, thr_vision, thr_text, eps) -> SearchParams:
    p = SearchParams()
    p.keyset, p.normalize_q, p.cmp_ge = int(keyset), int(bool(normalize)), int(bool(cmp_ge))
    p.thr_vision, p.thr_text, p.eps = float(thr_vision), float(thr_text), float(eps)
    return p
