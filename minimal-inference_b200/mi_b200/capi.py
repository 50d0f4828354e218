"""ctypes binding of libmi_paged.so (the C ABI in include/mi_paged.h).

The library is loaded on first use. If it is missing or fails to load, every
op raises -- there is no CPU fallback. Each wrapper here takes raw integers
(device pointers, sizes, a cudaStream_t) and raises ``MiError`` with the
library's message when a call returns non-zero.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmi_paged.so")
HEADER_PATH = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include", "mi_paged.h")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
ERR_INVALID, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = 1, 2, 3, 4
STATUS_BITS = {
    1: "OUT_OF_PAGES", 2: "BAD_PAGE", 4: "BAD_POSITION", 8: "BAD_BATCH_INDEX",
    16: "POOL_OVERFLOW", 32: "SLOT_FULL", 64: "TIMEOUT",
}


class MiError(RuntimeError):
    """A libmi_paged call failed (host-side argument or launch error)."""


_c_i32, _c_i64, _c_size, _c_p, _c_f = (ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t,
                                        ctypes.c_void_p, ctypes.c_float)

# argument types per entry point, in header order
_SIGS = {
    "mi_last_error": ([], ctypes.c_char_p),
    "mi_version": ([], ctypes.c_int),
    "mi_append_paged_kv_cache": ([
        _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
        _c_p, _c_p, _c_i32,
        _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_p, _c_p, _c_i32,
        _c_p, _c_p, _c_i32, _c_p,
        _c_p, _c_i64, _c_i64,
        _c_p, _c_i64, _c_i64, _c_i32,
        _c_i32, _c_p, _c_p], ctypes.c_int),
    "mi_paged_decode_workspace_size": ([_c_i32, _c_i32, _c_i32, _c_i32], _c_size),
    "mi_paged_decode": ([
        _c_p, _c_i64, _c_i64,
        _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_f,
        _c_p, _c_p, _c_p, _c_size, _c_p, _c_p], ctypes.c_int),
    "mi_paged_decode_append": ([
        _c_p, _c_i64, _c_i64,
        _c_p, _c_i64, _c_i64,
        _c_p, _c_i64, _c_i64,
        _c_p, _c_p, _c_i32,
        _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_f,
        _c_p, _c_p, _c_p, _c_size, _c_p, _c_p], ctypes.c_int),
    "mi_paged_decode_noalloc": ([
        _c_p, _c_i64, _c_i64,
        _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_f,
        _c_p, _c_p, _c_p, _c_p], ctypes.c_int),
    "mi_paged_prefill_workspace_size": ([_c_i32, _c_i32, _c_i32, _c_i32], _c_size),
    "mi_paged_prefill": ([
        _c_p, _c_i64, _c_i64, _c_p, _c_i32,
        _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
        _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_f,
        _c_p, _c_p, _c_p, _c_size, _c_p, _c_p], ctypes.c_int),
    "mi_page_pool_init": ([_c_p, _c_p, _c_i32, _c_p], ctypes.c_int),
    "mi_page_alloc": ([_c_p, _c_p, _c_i32, _c_p, _c_i32, _c_p, _c_p, _c_p], ctypes.c_int),
    "mi_page_release": ([_c_p, _c_p, _c_i32, _c_p, _c_i32, _c_p, _c_i32, _c_i64, _c_p, _c_p],
                        ctypes.c_int),
    "mi_slot_alloc": ([_c_p, _c_p, _c_i32, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_i32, _c_p,
                       _c_p], ctypes.c_int),
    "mi_slot_release": ([_c_p, _c_p, _c_i32, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_i32, _c_p,
                         _c_i32, _c_i64, _c_p, _c_p], ctypes.c_int),
    "mi_step_prepare": ([_c_p, _c_p, _c_i32, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_i32,
                         _c_i32, _c_i32, _c_p, _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p],
                        ctypes.c_int),
    "mi_add_rmsnorm": ([_c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_f, _c_i32, _c_p], ctypes.c_int),
    "mi_silu_mul": ([_c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p], ctypes.c_int),
    "mi_proj_small_m": ([_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i32, _c_i32, _c_i32,
                         _c_i32, _c_p, _c_p], ctypes.c_int),
    "mi_allreduce_add_rmsnorm": ([_c_p, _c_i64, _c_i64, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_p,
                                 _c_i32, _c_i32, _c_f, _c_i32, _c_p, _c_p], ctypes.c_int),
    "mi_set_peer_wait_limit_ns": ([_c_i64], ctypes.c_int),
    "mi_ipc_export": ([_c_p, _c_p, _c_p], ctypes.c_int),
    "mi_ipc_open": ([_c_p, _c_p], ctypes.c_int),
    "mi_ipc_close": ([_c_p], ctypes.c_int),
}
IPC_HANDLE_BYTES = 64

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first call; raises if it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MiError(
                f"{LIB_PATH} not found: build it with "
                "`python minimal-inference_b200/csrc/build.py` (no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _lib = handle
    return _lib


def header_symbols() -> list[str]:
    """Function names declared in include/mi_paged.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mi_[a-z0-9_]+)\s*\(", text)))


def call(name: str, *args) -> None:
    """Call entry point ``name``; raise MiError on a non-zero return."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().mi_last_error().decode(errors="replace")
        raise MiError(f"{name} failed (code {rc}): {msg}")


def status_names(word: int) -> list[str]:
    return [n for bit, n in STATUS_BITS.items() if word & bit]
