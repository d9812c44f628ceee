"""The decode in a second CUDA context of the same device.

A binding that drives the GPU through the driver API (its own context rather than the device's
primary one) calls the same C entry points.  The library's per-context set-up -- each kernel's
shared-memory opt-in and the side stream the shared-prefix pass forks onto -- is made for that
context too, so the result is bit-identical to the decode in torch's primary context, on every
call.  All buffers of the second context are allocated in it (driver allocations, host copies).
"""
import pytest
import torch

from loopfuse_b200 import _lib
from loopfuse_b200 import attention as att
from loopfuse_b200.workloads import decode_inputs

pytestmark = pytest.mark.gpu


def _ok(res):
    from cuda.bindings import driver as drv
    err = res[0] if isinstance(res, tuple) else res
    assert err == drv.CUresult.CUDA_SUCCESS, err
    return res[1] if isinstance(res, tuple) and len(res) > 1 else None


def test_decode_in_a_second_context_matches_the_primary_context():
    from cuda.bindings import driver as drv
    lengths = [300, 1000, 17, 4096, 2500, 64, 777, 3000]
    w = decode_inputs(N=len(lengths), lengths=lengths, prefix_tokens=512, seed=5)
    N, Hq, D = w.q.shape
    P, Hkv = w.k_pages.shape[:2]
    maxp = w.block_table.shape[1]
    pps = att.default_pages_per_split(N, Hkv, maxp, w.n_prefix_pages)
    ref = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                           num_prefix_pages=w.n_prefix_pages, pages_per_split=pps).cpu()
    host = [t.cpu().contiguous() for t in (w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens)]
    ws_bytes = att.decode_workspace_bytes(N, Hq, D, maxp, pps, w.n_prefix_pages)
    out_bytes = N * Hq * D * 2

    _ok(drv.cuInit(0))
    dev = _ok(drv.cuDeviceGet(torch.cuda.current_device()))
    ctx = _ok(drv.cuCtxCreate(0, dev))              # pushed: current on this thread
    ptrs = []
    try:
        def alloc(nbytes):
            p = _ok(drv.cuMemAlloc(nbytes))
            ptrs.append(p)
            return p

        dq, dk, dv, dbt, dlen = (alloc(t.numel() * t.element_size()) for t in host)
        for d, t in zip((dq, dk, dv, dbt, dlen), host):
            _ok(drv.cuMemcpyHtoD(d, t.data_ptr(), t.numel() * t.element_size()))
        do, dws = alloc(out_bytes), alloc(ws_bytes)
        for _ in range(2):
            rc = _lib.lib().lf_decode_fwd(int(dq), int(dk), int(dv), int(dbt), int(dlen),
                                          w.n_prefix_pages, int(do), None, int(dws), ws_bytes, N,
                                          Hq, Hkv, D, P, maxp, pps, D ** -0.5, None)
            assert rc == _lib.LF_OK, _lib.lib().lf_last_error()
            _ok(drv.cuCtxSynchronize())
            out = torch.empty((N, Hq, D), dtype=torch.bfloat16)
            _ok(drv.cuMemcpyDtoH(out.data_ptr(), do, out_bytes))
            assert torch.equal(out, ref)
        status = _lib.ctypes.c_int(-1)
        assert _lib.lib().lf_device_status(_lib.ctypes.byref(status)) == _lib.LF_OK
        assert status.value == 0
    finally:
        for p in ptrs:
            drv.cuMemFree(p)
        drv.cuCtxPopCurrent()
        drv.cuCtxDestroy(ctx)
    # back in torch's context: the library still decodes there
    again = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                             num_prefix_pages=w.n_prefix_pages, pages_per_split=pps).cpu()
    assert torch.equal(again, ref)
