"""Failure reporting without a GPU fault.

Every pipelined kernel here waits on its barriers with a wall-clock limit; a wait that runs out
records a site code in the device error word instead of hanging.  ``lf_selftest_bounded_wait``
runs that same wait on a barrier that nothing arrives at: the expiry must be reported by
``lf_device_status`` (and cleared by reading it), and the context must stay usable.
"""
import ctypes
import time

import pytest
import torch

from loopfuse_b200 import _lib
from loopfuse_b200 import attention as att
from loopfuse_b200.workloads import decode_inputs

pytestmark = pytest.mark.gpu


def _status() -> int:
    v = ctypes.c_int(-1)
    assert _lib.lib().lf_device_status(ctypes.byref(v)) == _lib.LF_OK
    return v.value


def test_bounded_wait_expiry_is_reported_and_the_context_survives():
    _status()                                               # start from a clear error word
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    assert _lib.lib().lf_selftest_bounded_wait(2000, stream) == _lib.LF_OK   # 2 ms limit
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert _status() == 177                                 # 100 + the self-test's site
    assert _status() == 0                                   # reading cleared it
    w = decode_inputs(N=3, lengths=[40, 300, 17], prefix_tokens=0, seed=4)
    o = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens, pages_per_split=2)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    assert _status() == 0


def test_bounded_wait_rejects_out_of_range_limits():
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().lf_selftest_bounded_wait(0, stream) == _lib.LF_EINVAL
    assert _lib.lib().lf_selftest_bounded_wait(200000, stream) == _lib.LF_EINVAL
