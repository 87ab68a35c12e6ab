"""ctypes binding of the C ABI in ``include/fast_infer_b200.h``.

The shared library is loaded from the package directory (built in-tree by
``fast_infer_b200.build``). There is no fallback: if the library is missing or a
symbol is absent, the first call raises ``RuntimeError`` naming the build step.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfast_infer_b200.so"

FI_OK = 0
FI_ERR_INVALID_ARG = 1
FI_ERR_UNSUPPORTED = 2
FI_ERR_ALIGNMENT = 3
FI_ERR_WORKSPACE = 4
FI_ERR_CUDA = 5

FI_DEVERR_TIMEOUT = 1
FI_DEVERR_BAD_BLOCK = 2
FI_DEVERR_CONTEXT_LEN = 4
FI_STATIC_WEIGHTS = 1

_STATUS_NAMES = {
    FI_ERR_INVALID_ARG: "FI_ERR_INVALID_ARG",
    FI_ERR_UNSUPPORTED: "FI_ERR_UNSUPPORTED",
    FI_ERR_ALIGNMENT: "FI_ERR_ALIGNMENT",
    FI_ERR_WORKSPACE: "FI_ERR_WORKSPACE",
    FI_ERR_CUDA: "FI_ERR_CUDA",
}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i64p = ctypes.POINTER(ctypes.c_int64)
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); the single source of truth for the Python side.
SIGNATURES = {
    "fi_version": (ctypes.c_int, []),
    "fi_last_error": (ctypes.c_char_p, []),
    "fi_prefill_fwd": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                      _i64p, _i64p, _i64p, _i64p, _f32, _vp, _vp]),
    "fi_prefill_fwd_varlen": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                             _i64, _i64, _i64p, _i64p, _i64p, _i64p, _f32, _vp,
                                             _vp]),
    "fi_paged_decode_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "fi_paged_decode": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                       _i64, _i64, _i64, _i64, _i64, _i64p, _i64p, _i64p,
                                       _i64p, _i64p, _f32, _i64, _vp, _sz, _vp, _vp]),
    "fi_paged_decode_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                               _i64, _i64, _i64, _i64, _i64, _i64, _i64p, _i64p,
                                               _i64p, _i64p, _i64p, _f32, _i64, _vp, _vp]),
    "fi_rope_kv_write": (ctypes.c_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64p, _vp, _vp, _i64,
                                        _i64, _vp, _i64, _vp, _i64p, _vp, _i64p, _vp, _vp, _vp,
                                        _i64, _i64, _i64, _i64p, _i64p, _i64p, _vp, _vp]),
    "fi_kv_write": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64,
                                   _i64, _i64, _i64, _i64, _i64p, _i64p, _i64p, _i64p, _i64p,
                                   _vp, _vp]),
    "fi_rms_norm": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _vp]),
    "fi_int4_gemm": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64p, _i64p,
                                    _i64p, _i64p, _vp, _vp]),
    "fi_int4_dequant": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64p, _i64p, _i64p,
                                       _vp]),
    "fi_int4_quantize": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64p, _i64p, _i64p,
                                        _vp]),
    "fi_small_gemm": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _i64p,
                                     _i64p, _i64p, _i64p, _i64, _vp, _vp]),
    "fi_small_gemm_folded": (ctypes.c_int, [_vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _i64p,
                                            _i64p, _i64p, _i64p, _i64, _vp, _vp]),
    "fi_qkv_rope_kv_write": (ctypes.c_int, [_vp, _vp, _f32, _i64, _i64, _i64, _i64, _i64, _i64p,
                                            _i64p, _vp, _vp, _i64, _i64, _vp, _vp, _i64p, _vp,
                                            _vp, _vp, _i64, _i64, _i64, _i64p, _i64p, _i64p,
                                            _i64, _vp, _vp]),
    "fi_peer_gather_bytes": (_sz, [_i64, _i64, _i64]),
    "fi_peer_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(_vp), _vp]),
    "fi_peer_open": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "fi_peer_close": (ctypes.c_int, [_vp]),
    "fi_peer_free": (ctypes.c_int, [_vp]),
    "fi_peer_gather": (ctypes.c_int, [_vp, _i64, _i64, _i64, ctypes.POINTER(_vp), _i64, _i64, _i64,
                                      _i64, _i64, _vp, _vp]),
    "fi_peer_reduce_bytes": (_sz, [_i64, _i64, _i64]),
    "fi_small_gemm_peer_reduce": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64p,
                                                 _i64p, _i64p, _i64p, ctypes.POINTER(_vp),
                                                 _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} not found next to the package; build it first with "
                    "`python -m fast_infer_b200.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)  # AttributeError = stale build
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strides(*vals) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr


def check(status: int, what: str) -> None:
    """Raise on a non-FI_OK status, with the library's own message."""
    if status == FI_OK:
        return
    msg = load().fi_last_error().decode(errors="replace")
    name = _STATUS_NAMES.get(status, str(status))
    if status in (FI_ERR_INVALID_ARG, FI_ERR_ALIGNMENT):
        raise ValueError(f"{what}: {name}: {msg}")
    raise RuntimeError(f"{what}: {name}: {msg}")
