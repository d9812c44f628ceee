"""The C-ABI library loads on a CPU host and exports every symbol the header declares.

No compute call is made here (there is no GPU); only pure host-side entry points
(version, workspace sizing, argument validation) are exercised.
"""
import ctypes
import os
import re

import pytest

from loopfuse_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "loopfuse_b200.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lf_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.exported_symbols())


def test_version_and_workspace_sizing():
    assert _lib.lib().lf_version().startswith(b"loopfuse_b200")
    n = ctypes.c_size_t(0)
    _lib.call("lf_decode_workspace_size", 256, 32, 128, 2048, 32, 128, ctypes.byref(n))
    slots = (2048 - 128 + 31) // 32 + 128 // 32
    assert n.value == 256 * 32 * slots * (128 * 4 + 8)


def test_host_side_validation_errors():
    lib = _lib.lib()
    rc = lib.lf_prefill_fwd(None, None, None, None, None, 1, 1, 1, 1, 1, 128, 1.0, 1, None)
    assert rc == _lib.LF_EINVAL
    assert b"null" in lib.lf_last_error()
    rc = lib.lf_decode_fwd(8, 8, 8, 8, 8, 0, 8, None, 8, 0, 1, 4, 3, 128, 1, 1, 1, 1.0, None)
    assert rc == _lib.LF_EINVAL          # unaligned pointers rejected before any launch
    m = _lib.PoolMeta()
    assert lib.lf_pool_init(ctypes.byref(m), None) == _lib.LF_EINVAL


def test_selftest_rejects_out_of_range_limits_before_any_launch():
    lib = _lib.lib()
    assert lib.lf_selftest_bounded_wait(0, None) == _lib.LF_EINVAL
    assert b"timeout_us" in lib.lf_last_error()
    assert lib.lf_selftest_bounded_wait(100001, None) == _lib.LF_EINVAL


def test_default_split_size_is_a_power_of_two_between_32_and_128_pages():
    from loopfuse_b200.attention import default_pages_per_split
    for n, hkv, max_pages, npre in [(1, 8, 64, 0), (64, 8, 319, 256), (256, 8, 2048, 128),
                                    (512, 8, 600, 256), (8, 2, 5000, 0)]:
        pps = default_pages_per_split(n, hkv, max_pages, npre)
        assert pps in (32, 64, 128), (n, hkv, max_pages, npre, pps)
    assert default_pages_per_split(256, 8, 2048, 128) == 128      # the 256-session decode


def test_skinny_gemm_workspace_and_argument_checks():
    """Partial-sum workspace = min(SMs, units) CTAs x 2 slots x M x 128 fp32; bad shapes are
    rejected on the host before any launch."""
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    _lib.call("lf_gemm_skinny_workspace_size", 64, 6144, 4096, 148, ctypes.byref(n))
    assert n.value == 148 * 2 * 64 * 128 * 4
    _lib.call("lf_gemm_skinny_workspace_size", 3, 136, 72, 148, ctypes.byref(n))
    assert n.value == 4 * 2 * 3 * 128 * 4          # 2 column blocks x 2 K chunks = 4 units
    p = 1 << 20                                     # aligned stand-in address, never touched
    assert lib.lf_gemm_skinny(p, p, p, 129, 64, 64, p, 1 << 30, 148, None) == _lib.LF_EINVAL
    assert b"M <= 128" in lib.lf_last_error()
    assert lib.lf_gemm_skinny(p, p, p, 8, 60, 64, p, 1 << 30, 148, None) == _lib.LF_EINVAL
    assert lib.lf_gemm_skinny(p + 2, p, p, 8, 64, 64, p, 1 << 30, 148, None) == _lib.LF_EINVAL
    assert lib.lf_gemm_skinny(p, p, p, 8, 64, 64, p, 16, 148, None) == _lib.LF_EINVAL
    assert b"workspace" in lib.lf_last_error()
    assert lib.lf_gemm_skinny(None, p, p, 8, 64, 64, p, 1 << 30, 148, None) == _lib.LF_EINVAL
