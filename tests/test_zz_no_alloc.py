"""The decode entry point that allocates nothing, checked against the allocating one.

``lf_decode_fwd_noalloc`` serves callers that cannot allocate device memory (a
binding with no device allocator, or a loop whose allocator has reserved nearly
all of HBM for the KV pool): its split partials live in a fixed array inside the
library instead of a caller workspace.  This file is collected last, so a run
that stops at the first failure has run every other test before it; it also
passes on its own in a fresh process (it builds its own inputs).
"""
import ctypes

import pytest
import torch

from oracle import attention as ora
from loopfuse_b200 import _lib
from loopfuse_b200 import attention as att
from loopfuse_b200.workloads import decode_inputs

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_MEAN = 2e-2, 2e-3


def _noalloc(w, out, lse, table=None):
    N, Hq, D = w.q.shape
    P, Hkv = w.k_pages.shape[:2]
    table = w.block_table if table is None else table
    return _lib.lib().lf_decode_fwd_noalloc(
        w.q.data_ptr(), w.k_pages.data_ptr(), w.v_pages.data_ptr(), table.data_ptr(),
        w.seq_lens.data_ptr(), w.n_prefix_pages, out.data_ptr(), lse.data_ptr(), N, Hq, Hkv, D, P,
        table.shape[1], D ** -0.5, torch.cuda.current_stream().cuda_stream)


def _check_oracle(w, out, lse, idx):
    """Sessions ``idx`` against the fp32 CPU oracle (the same tolerance as every decode test)."""
    ref, ref_lse = ora.decode_paged(w.q[idx].cpu(), w.k_pages.cpu(), w.v_pages.cpu(),
                                    w.block_table[idx].cpu(), [w.lengths[i] for i in idx])
    d = (out[idx].float().cpu() - ref).abs()
    assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN
    assert (lse[idx].cpu() - ref_lse).abs().max().item() < 1e-3


@pytest.mark.parametrize("prefix_tokens,hq,hkv,d", [(0, 32, 8, 128), (512, 32, 8, 128),
                                                     (0, 8, 2, 64), (256, 12, 12, 64)])
def test_noalloc_matches_workspace_entry_point_twice(prefix_tokens, hq, hkv, d):
    lengths = [1, 16, 17, 300, 2048, 5000, 9000, 700, 12000, 64, 4096, 3333]
    w = decode_inputs(N=len(lengths), Hq=hq, Hkv=hkv, D=d, lengths=lengths,
                      prefix_tokens=prefix_tokens, seed=21)
    ref, ref_lse = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                                    num_prefix_pages=w.n_prefix_pages, return_lse=True)
    for _ in range(2):
        out = torch.full_like(w.q, float("nan"))
        lse = torch.empty(ref_lse.shape, dtype=torch.float32, device="cuda")
        assert _noalloc(w, out, lse) == _lib.LF_OK, _lib.lib().lf_last_error()
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN
        assert (lse - ref_lse).abs().max().item() < 1e-3
    _check_oracle(w, out, lse, list(range(len(lengths))))


def test_noalloc_grows_the_split_until_the_partials_fit():
    """Many short sessions in a wide block table (256 sessions of ~64 tokens, 2048 page slots
    each): at the default split the partials would need 68 MB, twice the fixed array, so the
    entry point doubles the split size until they fit.  Two calls in a row, both against the
    allocating entry point and against the oracle."""
    g = torch.Generator().manual_seed(4)
    lengths = torch.randint(40, 91, (256,), generator=g).tolist()
    w = decode_inputs(N=256, lengths=lengths, prefix_tokens=0, seed=31)
    wide = torch.full((256, 2048), -1, dtype=torch.int32, device="cuda")
    wide[:, :w.block_table.shape[1]] = w.block_table
    ref, ref_lse = att.paged_decode(w.q, w.k_pages, w.v_pages, wide, w.seq_lens, return_lse=True)
    for _ in range(2):
        out = torch.full_like(w.q, float("nan"))
        lse = torch.empty(ref_lse.shape, dtype=torch.float32, device="cuda")
        assert _noalloc(w, out, lse, table=wide) == _lib.LF_OK, _lib.lib().lf_last_error()
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN
        assert (lse - ref_lse).abs().max().item() < 1e-3
    _check_oracle(w, out, lse, list(range(0, 256, 5)))


def test_noalloc_rejects_requests_beyond_the_fixed_scratch():
    w = decode_inputs(N=4, lengths=[64, 64, 64, 64], prefix_tokens=0, seed=2)
    out = torch.empty_like(w.q)
    lse = torch.empty((4, w.q.shape[1]), dtype=torch.float32, device="cuda")
    big_n = 65535                        # 65535 sessions x 32 heads exceed the array
    rc = _lib.lib().lf_decode_fwd_noalloc(
        w.q.data_ptr(), w.k_pages.data_ptr(), w.v_pages.data_ptr(), w.block_table.data_ptr(),
        w.seq_lens.data_ptr(), 0, out.data_ptr(), lse.data_ptr(), big_n, 32, 8, 128,
        w.k_pages.shape[0], w.block_table.shape[1], 1.0, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LF_EINVAL
    assert b"fixed scratch" in _lib.lib().lf_last_error()
