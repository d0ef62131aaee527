"""ctypes binding of libsckv.so (declared in include/sckv.h).

The library is the only compute path: importing this module raises if the
shared library is missing or incomplete, and every entry point's status code
is turned into a Python exception. Nothing here falls back to a CPU
implementation.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path
from typing import Optional

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libsckv.so"

# Status codes (include/sckv.h).
SCKV_OK = 0
SCKV_ERR_INVALID_ARG = -1
SCKV_ERR_BOUNDS = -3
SCKV_ERR_ALIGNMENT = -4
SCKV_ERR_CUDA = -5
SCKV_ERR_POOL_EXHAUSTED = -6
SCKV_ERR_TIMEOUT = -7
SCKV_ERR_UNSUPPORTED = -8
SCKV_ERR_SCRATCH_LIMIT = -9

# Size of the fixed per-GPU scratch behind sckv_decode_attn_noalloc
# (SCKV_NOALLOC_SCRATCH_BYTES in include/sckv.h).
NOALLOC_SCRATCH_BYTES = 4 << 20

# Element types.
DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_INT8 = 2
DTYPE_FP8_E4M3 = 3
DTYPE_F32 = 4


class SCKVError(RuntimeError):
    """A libsckv entry point returned a nonzero status."""

    def __init__(self, code: int, where: str):
        self.code = int(code)
        super().__init__(f"{where}: {status_string(code)} (status {code})")


class SCKVPoolExhausted(SCKVError):
    pass


class SCKVBoundsError(SCKVError):
    pass


_lib: Optional[ctypes.CDLL] = None

# (name, restype, argtypes)
_SIGNATURES = [
    ("sckv_pool_required_bytes", c_int,
     [c_int, c_int, c_int, c_int, c_int64, c_int, POINTER(c_size_t), POINTER(c_size_t), POINTER(c_size_t)]),
    ("sckv_pool_create", c_int, [c_int, c_int, c_int, c_int, c_int64, c_int, c_int, POINTER(c_void_p)]),
    ("sckv_pool_wrap", c_int,
     [c_int, c_int, c_int, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, POINTER(c_void_p)]),
    ("sckv_pool_destroy", None, [c_void_p]),
    ("sckv_pool_pointers", c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p)]),
    ("sckv_append", c_int,
     [c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int,
      c_void_p]),
    ("sckv_write_pages", c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_write_pages_quantized", c_int,
     [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("sckv_gather", c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_copy_pages", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_decode_workspace_bytes", c_size_t, [c_void_p, c_int, c_int, c_int, c_int]),
    ("sckv_decode_attn", c_int,
     [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int64, c_int, c_void_p, c_int, c_float, c_void_p, c_int,
      c_void_p, c_size_t, c_int, c_void_p]),
    ("sckv_decode_attn_append", c_int,
     [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_int, c_void_p, c_int,
      c_float, c_void_p, c_int, c_void_p, c_size_t, c_int, c_void_p]),
    ("sckv_append_rope", c_int,
     [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int,
      c_void_p, c_int, c_float, c_void_p, c_float, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int,
      c_void_p]),
    ("sckv_qkv_append", c_int,
     [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
      c_void_p, c_int, c_float, c_void_p, c_float, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
      c_int, c_void_p, c_size_t, c_void_p]),
    ("sckv_split_hi_lo", c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_qkv_workspace_bytes", c_size_t, [c_void_p, c_int, c_int, c_int]),
    ("sckv_o_proj", c_int,
     [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_size_t,
      c_void_p]),
    ("sckv_o_proj_workspace_bytes", c_size_t, [c_void_p, c_int, c_int, c_int]),
    ("sckv_prefill_attn", c_int,
     [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_float,
      c_void_p, c_int, c_void_p]),
    ("sckv_decode_attn_noalloc", c_int,
     [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int64, c_int, c_void_p, c_int, c_float, c_void_p, c_int,
      c_int, c_void_p]),
    ("sckv_alloc_reset", c_int, [c_void_p, c_void_p]),
    ("sckv_alloc_pages", c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    ("sckv_free_pages", c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_touch_pages", c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_pin_pages", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    ("sckv_release_pages", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    ("sckv_evict_lru", c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    ("sckv_evict_to_watermark", c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    ("sckv_exchange_create", c_int, [c_int, c_int, c_int, c_size_t, POINTER(c_void_p)]),
    ("sckv_exchange_buffer", c_void_p, [c_void_p]),
    ("sckv_exchange_ipc_handles", c_int, [c_void_p, c_void_p]),
    ("sckv_exchange_open_peer", c_int, [c_void_p, c_int, c_void_p]),
    ("sckv_exchange_destroy", None, [c_void_p]),
    ("sckv_decode_attn_exchange", c_int,
     [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_int,
      c_void_p, c_int, c_float, c_int, c_int64, c_int, c_uint32, c_void_p, c_size_t, c_int, c_void_p]),
    ("sckv_exchange_wait", c_int, [c_void_p, c_uint32, c_uint32, c_void_p]),
    ("sckv_exchange_status", c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    ("sckv_reserve_decode", c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p]),
    ("sckv_alloc_state", c_int, [c_void_p, POINTER(c_int64), c_void_p]),
    ("sckv_get_status", c_int, [c_void_p, POINTER(c_int32), c_void_p]),
    ("sckv_clear_status", c_int, [c_void_p, c_void_p]),
    ("sckv_selftest_wait_timeout", c_int, [c_void_p, ctypes.c_uint, c_void_p]),
    ("sckv_kv_lookup", c_int, [c_void_p, c_void_p, POINTER(c_uint32)]),
    ("sckv_kv_insert", c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_double, c_void_p, POINTER(c_uint64)]),
    ("sckv_version", ctypes.c_char_p, []),
    ("sckv_last_error", ctypes.c_char_p, []),
    ("sckv_launch_count", ctypes.c_ulonglong, []),
    ("sckv_status_string", ctypes.c_char_p, [c_int]),
]

EXPORTED_SYMBOLS = tuple(name for name, _, _ in _SIGNATURES)


def load(path: Optional[os.PathLike] = None) -> ctypes.CDLL:
    """Load libsckv.so and declare every entry point. Raises if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"libsckv.so not found at {p}; build it with `python -m synapcore_b200.build` "
            "(the CUDA extension is required: there is no CPU fallback)"
        )
    lib = ctypes.CDLL(str(p))
    for name, restype, argtypes in _SIGNATURES:
        fn = getattr(lib, name)  # AttributeError if a symbol is missing
        fn.restype = restype
        fn.argtypes = argtypes
    if path is None:
        _lib = lib
    return lib


def lib() -> ctypes.CDLL:
    return load()


def launch_count() -> int:
    """Kernels libsckv has launched in this process so far."""
    return int(lib().sckv_launch_count())


def status_string(code: int) -> str:
    try:
        return lib().sckv_status_string(int(code)).decode()
    except Exception:  # pragma: no cover - message helper only
        return "unknown status"


def check(rc: int, where: str) -> None:
    if rc == SCKV_OK:
        return
    if rc == SCKV_ERR_POOL_EXHAUSTED:
        raise SCKVPoolExhausted(rc, where)
    if rc == SCKV_ERR_BOUNDS:
        raise SCKVBoundsError(rc, where)
    if rc == SCKV_ERR_CUDA and _lib is not None:
        detail = (_lib.sckv_last_error() or b"").decode(errors="replace")
        if detail:
            where = f"{where} [{detail}]"
    raise SCKVError(rc, where)


def required_bytes(num_layers: int, num_kv_heads: int, head_dim: int, page_tokens: int, max_pages: int,
                   kv_dtype: int) -> tuple[int, int, int]:
    d = c_size_t()
    s = c_size_t()
    a = c_size_t()
    check(lib().sckv_pool_required_bytes(num_layers, num_kv_heads, head_dim, page_tokens, max_pages, kv_dtype,
                                         ctypes.byref(d), ctypes.byref(s), ctypes.byref(a)),
          "sckv_pool_required_bytes")
    return d.value, s.value, a.value
