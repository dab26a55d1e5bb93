"""ctypes binding of the in-tree C ABI library ``_lib/liboscar_b200.so``.

The signatures mirror ``include/oscar_b200.h``.  There is no fallback: if the
library is missing or fails to load, every kernel entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liboscar_b200.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U32 = ctypes.c_uint32
_F32 = ctypes.c_float



class RotateSeg(ctypes.Structure):
    """struct oscar_rotate_seg of include/oscar_b200.h."""
    _fields_ = [("x", _P), ("rows", _I64), ("x_stride", _I64), ("rot", _P), ("transpose", _I32),
                ("out", _P), ("out_stride", _I64), ("out_f32", _P), ("out_f32_stride", _I64)]


# name -> (restype, argtypes), exactly the prototypes of include/oscar_b200.h
SIGNATURES = {
    "oscar_abi_version": (ctypes.c_int, []),
    "oscar_last_error": (ctypes.c_char_p, []),
    "oscar_device_error": (ctypes.c_int, [_P]),
    "oscar_launch_count": (ctypes.c_uint64, []),
    "oscar_set_attention_path": (ctypes.c_int, [ctypes.c_int]),
    "oscar_set_rotation_path": (ctypes.c_int, [ctypes.c_int]),
    "oscar_store_int2": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _F32, _F32, _P, _P, _I64, _I32,
                                        _I64, _I64, _I64, _I64, _I64, _I64, _P, _P]),
    "oscar_staging_invalidate": (ctypes.c_int, [_P, _I64, _P, _I64, _I32, _P]),
    "oscar_write_step": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _F32, _F32, _P, _P, _I64, _I32,
                                        _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _I32,
                                        _I32, _I32, _P, _P, _P, _I64, _P]),
    "oscar_staging_write": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _P, _P, _P, _I32, _I32, _I32,
                                           _P, _P, _P, _I64, _I32, _P, _U32, _P]),
    "oscar_staging_write_noalloc": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _P, _P, _P, _I32, _I32, _I32,
                                                   _P, _P, _P, _I64, _I32, _P]),
    "oscar_slab_attention": (ctypes.c_int, [_P, _P, _P, _I32, _I64, _I32, _I32, _I32, _P, _P, _I64, _I32,
                                            _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64,
                                            _P, _P, _I32, _F32, _P, _P, _P, _I64, _P, _P, _P, _I64, _P]),
    "oscar_slab_attention_shard": (ctypes.c_int, [_P, _I32, _I64, _I32, _I32, _I32, _P, _P, _I64, _I32,
                                                  _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64,
                                                  _P, _P, _I32, _F32, _P, _P, _P, _I64, _P, _P, _P, _I64, _P]),
    "oscar_slab_attention_workspace": (ctypes.c_int64, [_P, _P, _I32, _I32, _I32, _I32, _I32]),
    "oscar_merge_slab": (ctypes.c_int, [_P, _P, _I64, _P, _I32, _P, _I64, _I32, _I32, _I64, _P, _P]),
    "oscar_rotate_rows": (ctypes.c_int, [_P, _I32, _I64, _I64, _I32, _P, _I32, _P, _I32, _I64, _P, _I64, _P]),
    "oscar_rotate_rows_batch": (ctypes.c_int, [ctypes.POINTER(RotateSeg), _I32, _I32, _I32, _I32, _P]),
    "oscar_decode_layer_step": (ctypes.c_int, [_P, _P, _P, _I32, _I64, _I64, _I64, _I64, _I32, _I32, _I32,
                                               _P, _P, _P, _F32, _F32, _P, _P, _I64, _I32,
                                               _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _I64,
                                               _P, _P, _I32, _I32, _I32, _F32, _P, _P, _P, _I64, _P, _I64,
                                               _P, _I64, _P]),
    "oscar_decode_layer_step_scratch": (ctypes.c_int64, [_I64, _I32, _I32, _I32, _I32]),
}

ABI_VERSION = 1

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    """The CUDA library was not built or cannot be loaded (no fallback exists)."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("OSCAR_B200_LIB", LIB_PATH))
        if not path.exists():
            raise NativeLibraryMissing(
                f"{path} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                "(there is no CPU fallback for the OSCAR B200 kernels)")
        try:
            handle = ctypes.CDLL(str(path))
        except OSError as exc:
            raise NativeLibraryMissing(f"cannot load {path}: {exc}") from exc
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.oscar_abi_version() != ABI_VERSION:
            raise NativeLibraryMissing(f"{path}: ABI {handle.oscar_abi_version()} != expected {ABI_VERSION}")
        _lib = handle
        return _lib


def check(status: int) -> None:
    """Map a C status to the reference's exception types: layout errors raise
    ValueError (as slab_attention.py:394-410 does), device failures RuntimeError."""
    if status == OK:
        return
    msg = lib().oscar_last_error().decode(errors="replace")
    if status in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(f"OSCAR CUDA failure: {msg}")
