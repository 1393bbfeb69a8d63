"""ctypes binding of libb2attn.so (the C ABI in include/b2attn.h).

There is no fallback: if the shared library is missing or does not export the
expected symbols, loading raises B2AError. The attention ops in this package
never run anywhere but the sm_100a kernels.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libb2attn.so")

# Status codes (mirror of the enum in include/b2attn.h).
B2A_OK = 0
B2A_ERR_INVALID_ARG = -1
B2A_ERR_HEAD_DIM = -2
B2A_ERR_GQA = -3
B2A_ERR_ALIGNMENT = -4
B2A_ERR_TMA = -5
B2A_ERR_LAUNCH = -6
B2A_ERR_WORKSPACE = -7
B2A_ERR_DEVICE = -8
B2A_ERR_DEVICE_TIMEOUT = -9
B2A_ERR_DEVICE_BAD_LEN = -10
B2A_ERR_CUDA = -11

# Size of the fixed device scratch behind b2a_decode_noalloc
# (B2A_NOALLOC_SCRATCH_BYTES in include/b2attn.h).
B2A_NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024

_c_ll3 = ctypes.c_longlong * 3
_c_ll2 = ctypes.c_longlong * 2

# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "b2a_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "b2a_version": (ctypes.c_int, []),
    "b2a_prefill": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
    ]),
    "b2a_decode_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int] * 6),
    "b2a_decode_default_split": (ctypes.c_int, [ctypes.c_int] * 3),
    "b2a_decode": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
    ]),
    "b2a_get_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_void_p]),
    "b2a_decode_noalloc": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
    ]),
    "b2a_decode_proj": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
    ]),
    "b2a_rope_append": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
    ]),
    "b2a_qk_norm_rope_append": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
    ]),
    "b2a_prefill_gated": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.c_int,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
    ]),
    "b2a_decode_gated": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
        ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), ctypes.c_int,
        ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
    ]),
    "b2a_prefill_host_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int] * 8),
    "b2a_prefill_host": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
    ]),
    # include/b2attn_diag.h
    "b2a_diag_umma_gemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                          ctypes.c_void_p]),
    "b2a_diag_wait_timeout": (ctypes.c_int, [ctypes.c_longlong, ctypes.c_void_p]),
}


class B2AError(RuntimeError):
    """A non-zero status from the C ABI (or a missing/unloadable library)."""

    def __init__(self, code: int, what: str = ""):
        self.code = code
        text = strerror(code) if code != 0 else ""
        super().__init__(f"{what}: {text} (status {code})" if what else f"{text} (status {code})")


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libb2attn.so once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise B2AError(B2A_ERR_CUDA, f"{LIB_PATH.name} is not built (run `python -m npu_b200.build`)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)  # AttributeError here means a stale or foreign library
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def strerror(code: int) -> str:
    try:
        return load().b2a_strerror(int(code)).decode()
    except Exception:  # the library itself could not be loaded
        return f"b2attn status {code}"


def check(code: int, what: str) -> None:
    if code != B2A_OK:
        raise B2AError(code, what)


def ll3(a, b, c):
    return _c_ll3(int(a), int(b), int(c))


def ll2(a, b):
    return _c_ll2(int(a), int(b))
