"""ctypes binding of ``liblf_sm100.so`` (declared in ``include/loopfuse_b200.h``).

There is no fallback: if the library is missing or a call fails, a
``LoopfuseError`` carrying the C status code and message is raised.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "liblf_sm100.so")

LF_OK, LF_EINVAL, LF_ENOPAGES, LF_EOVERFLOW, LF_ETIMEOUT, LF_ECUDA = range(6)
LF_PAGE_SIZE = 16
LF_CTRL_HEAD, LF_CTRL_COUNT, LF_CTRL_STATUS, LF_CTRL_WORDS = 0, 1, 2, 8

STATUS_NAMES = {LF_OK: "LF_OK", LF_EINVAL: "LF_EINVAL", LF_ENOPAGES: "LF_ENOPAGES",
                LF_EOVERFLOW: "LF_EOVERFLOW", LF_ETIMEOUT: "LF_ETIMEOUT", LF_ECUDA: "LF_ECUDA"}


class LoopfuseError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class PoolMeta(ctypes.Structure):
    _fields_ = [("free_queue", c_void_p), ("refcount", c_void_p), ("block_table", c_void_p),
                ("seq_len", c_void_p), ("ctrl", c_void_p), ("scratch", c_void_p),
                ("num_pages", c_int32), ("max_seqs", c_int32), ("max_pages_per_seq", c_int32),
                ("page_size", c_int32)]


LF_MAX_DEDUP_PAGES = 4096


class PrefixRegistry(ctypes.Structure):
    _fields_ = [("keys", c_void_p), ("pages", c_void_p), ("used", c_void_p), ("capacity", c_int)]


_P = c_void_p
# name -> argtypes (all functions return int unless listed in _RESTYPE)
_SIGS = {
    "lf_version": [],
    "lf_last_error": [],
    "lf_device_status": [POINTER(c_int)],
    "lf_selftest_bounded_wait": [c_uint, _P],
    "lf_prefill_fwd": [_P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                       c_int, _P],
    "lf_prefill_paged_fwd": [_P, _P, _P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int,
                             c_int, c_int, c_int, c_float, c_int, _P],
    "lf_decode_workspace_size": [c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_size_t)],
    "lf_decode_default_split": [c_int, c_int, c_int, c_int, c_int, POINTER(c_int)],
    "lf_decode_fwd": [_P, _P, _P, _P, _P, c_int, _P, _P, _P, c_size_t, c_int, c_int, c_int,
                      c_int, c_int, c_int, c_int, c_float, _P],
    "lf_decode_fwd_append": [_P, _P, _P, _P, _P, c_int, _P, _P, _P, _P, _P, c_size_t, c_int,
                             c_int, c_int, c_int, c_int, c_int, c_int, c_float, _P],
    "lf_decode_fwd_noalloc": [_P, _P, _P, _P, _P, c_int, _P, _P, c_int, c_int, c_int, c_int,
                              c_int, c_int, c_float, _P],
    "lf_decode_set_profile_events": [_P, _P],
    "lf_pool_init": [POINTER(PoolMeta), _P],
    "lf_pool_clear_status": [POINTER(PoolMeta), _P],
    "lf_pool_reserve": [POINTER(PoolMeta), _P, _P, c_int, _P, _P],
    "lf_pool_write_kv": [POINTER(PoolMeta), _P, _P, _P, c_int, c_int, _P, _P, c_int64, c_int64,
                         c_int64, _P, _P, c_int, c_int, c_int, _P],
    "lf_pool_fork": [POINTER(PoolMeta), c_int, _P, c_int, c_int, _P, _P, c_int, c_int, c_int, _P],
    "lf_pool_free": [POINTER(PoolMeta), _P, c_int, _P],
    "lf_pool_gather": [POINTER(PoolMeta), _P, c_int, _P, c_int, _P, _P],
    "lf_pool_read": [POINTER(PoolMeta), c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, c_int,
                     c_int, _P],
    "lf_pool_write_qkv": [POINTER(PoolMeta), _P, _P, _P, c_int, c_int, _P, c_int64, _P, _P, c_int,
                          _P, _P, _P, c_int, c_int, c_int, _P],
    "lf_add_rmsnorm": [_P, _P, _P, _P, c_int, c_int, c_float, _P],
    "lf_swiglu": [_P, _P, c_int, c_int, _P],
    "lf_gemm_skinny_workspace_size": [c_int, c_int, c_int, c_int, POINTER(c_size_t)],
    "lf_gemm_skinny": [_P, _P, _P, c_int, c_int, c_int, _P, c_size_t, c_int, _P],
    "lf_decode_fwd_gather": [_P, _P, _P, _P, _P, c_int, _P, c_int, c_int, c_int, _P, _P, c_size_t,
                             c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_float, _P],
    "lf_ipc_export": [_P, _P, POINTER(c_size_t)],
    "lf_ipc_import": [_P, POINTER(c_void_p)],
    "lf_ipc_close": [_P],
    "lf_registry_init": [POINTER(PrefixRegistry), _P],
    "lf_prefix_hashes": [_P, c_int, _P, _P],
    "lf_pool_register_prefix": [POINTER(PoolMeta), POINTER(PrefixRegistry), c_int, _P, c_int, _P, _P],
    "lf_pool_dedup_prefix": [POINTER(PoolMeta), POINTER(PrefixRegistry), _P, _P, _P, c_int, _P, _P],
    "lf_pool_unregister_all": [POINTER(PoolMeta), POINTER(PrefixRegistry), _P],
}
_RESTYPE = {"lf_version": c_char_p, "lf_last_error": c_char_p}

_lib = None


def exported_symbols():
    """Names this binding expects the library to export (every header entry point)."""
    return list(_SIGS)


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LoopfuseError(LF_ECUDA, f"{LIB_PATH} is missing: build it with "
                                          f"`python -m loopfuse_b200.build` (needs nvcc)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGS.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, c_int)
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != LF_OK:
        msg = lib().lf_last_error().decode(errors="replace")
        raise LoopfuseError(rc, f"{what}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
