"""ctypes binding of libgguf_b200.so (the C ABI in include/gguf_b200.h).

The library is loaded lazily on first use.  A missing or unloadable library raises
``NativeLibraryError``: there is no CPU fallback on this path.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libgguf_b200.so"

GQ_OK = 0
ERRORS = {-1: "GQ_ERR_TYPE", -2: "GQ_ERR_SIZE", -3: "GQ_ERR_ALIGN", -4: "GQ_ERR_NULL",
          -5: "GQ_ERR_ARG", -6: "GQ_ERR_CUDA", -7: "GQ_ERR_NOMEM"}
OUT_CODES = 1
OUT_F32 = 2

# every symbol include/gguf_b200.h declares
EXPORTS = ("gq_version", "gq_strerror", "gq_last_cuda_error", "gq_kernel_errors", "gq_query", "gq_diag_reset",
           "gq_convert", "gq_convert_batch", "gq_requantize_symmetric", "gq_session_create",
           "gq_session_destroy", "gq_convert_host", "gq_convert_host_noalloc", "gq_embedding_rows",
           "gq_quantize_rows", "gq_modalix_layout", "gq_unpack_fields", "gq_remove_superblocks",
           "gq_convert_modalix", "gq_convert_modalix_batch",
           "gq_host_alloc", "gq_host_free", "gq_host_trim")


class NativeLibraryError(RuntimeError):
    pass


class GqError(RuntimeError):
    """A negative status from the C ABI."""

    def __init__(self, status: int, what: str, lib=None):
        self.status = status
        msg = f"{what}: {ERRORS.get(status, status)}"
        if lib is not None:
            msg += f" ({lib.gq_strerror(status).decode()})"
            if status == -6:
                msg += f" [cudaError {lib.gq_last_cuda_error()}]"
        super().__init__(msg)


class Diag(ctypes.Structure):
    _fields_ = [("round_err_bits", ctypes.c_uint32), ("clip_err", ctypes.c_int32)]


class Tensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("perm_heads", ctypes.c_int32),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("src", ctypes.c_void_p), ("src_bytes", ctypes.c_size_t),
                ("codes", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("values", ctypes.c_void_p), ("diag", ctypes.c_void_p)]


class Layout(ctypes.Structure):
    _fields_ = [("n_values", ctypes.c_int64), ("n_units", ctypes.c_int64),
                ("src_bytes", ctypes.c_int64), ("codes_bytes", ctypes.c_int64),
                ("scales_count", ctypes.c_int64), ("values_bytes", ctypes.c_int64),
                ("block_values", ctypes.c_int32), ("unit_values", ctypes.c_int32)]


_lib = None
_lock = threading.Lock()


def _declare(lib):
    P, I32, I64, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    sig = {
        "gq_version": ([], ctypes.c_int),
        "gq_strerror": ([ctypes.c_int], ctypes.c_char_p),
        "gq_last_cuda_error": ([], ctypes.c_int),
        "gq_kernel_errors": ([I32, I32, ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
        "gq_host_alloc": ([SZ, ctypes.POINTER(P)], ctypes.c_int),
        "gq_host_free": ([P], ctypes.c_int),
        "gq_host_trim": ([], ctypes.c_int),
        "gq_query": ([I32, I64, I64, ctypes.POINTER(Layout)], ctypes.c_int),
        "gq_diag_reset": ([P, I32, P], ctypes.c_int),
        "gq_convert": ([ctypes.POINTER(Tensor), I32, P], ctypes.c_int),
        "gq_convert_batch": ([ctypes.POINTER(Tensor), I32, I32, P], ctypes.c_int),
        "gq_requantize_symmetric": ([P, P, I64, I32, I32, P, P, P, P], ctypes.c_int),
        "gq_session_create": ([I32, SZ, ctypes.POINTER(P)], ctypes.c_int),
        "gq_session_destroy": ([P], ctypes.c_int),
        "gq_convert_host": ([P, ctypes.POINTER(Tensor), I32, I32, P], ctypes.c_int),
        "gq_convert_host_noalloc": ([I32, ctypes.POINTER(Tensor), I32, I32, P, P], ctypes.c_int),
        "gq_embedding_rows": ([I32, P, SZ, I64, I64, ctypes.c_float, I32, P, P, P, P], ctypes.c_int),
        "gq_quantize_rows": ([P, I64, I64, P, P, P], ctypes.c_int),
        "gq_modalix_layout": ([P, P, I64, I64, I32, I64, P, P, P], ctypes.c_int),
        "gq_unpack_fields": ([I32, P, SZ, I64, P, P, P, P], ctypes.c_int),
        "gq_convert_modalix": ([ctypes.POINTER(Tensor), I64, P], ctypes.c_int),
        "gq_convert_modalix_batch": ([ctypes.POINTER(Tensor), P, I32, P], ctypes.c_int),
        "gq_remove_superblocks": ([P, P, I32, I64, I32, I32, P, P, P], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def lib():
    """The loaded library (raises NativeLibraryError when it cannot be loaded)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("LLIMA_B200_LIB", LIB_PATH))
            if not path.exists():
                raise NativeLibraryError(
                    f"{path} is missing: build it with `python -m llima_b200.build` "
                    "(the GGUF path has no CPU fallback)")
            try:
                handle = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
            except OSError as exc:
                raise NativeLibraryError(f"cannot load {path}: {exc}") from exc
            missing = [s for s in EXPORTS if not hasattr(handle, s)]
            if missing:
                raise NativeLibraryError(f"{path} lacks symbols {missing}")
            _declare(handle)
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != GQ_OK:
        raise GqError(status, what, _lib)


def query(type_id: int, rows: int, cols: int) -> Layout:
    out = Layout()
    check(lib().gq_query(type_id, rows, cols, ctypes.byref(out)), "gq_query")
    return out
