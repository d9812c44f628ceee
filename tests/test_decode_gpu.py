"""Paged split-KV decode (sm_100a) against the fp32 CPU oracle.

Tolerance: bf16 output vs fp32 oracle, max-abs <= 2e-2 and mean-abs <= 2e-3.
"""
import math

import pytest
import torch

from oracle import attention as ora
from loopfuse_b200 import attention as att
from loopfuse_b200.workloads import decode_bytes, decode_inputs

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_MEAN = 2e-2, 2e-3


def _check(o, ref, what=""):
    d = (o.float().cpu() - ref).abs()
    assert d.max().item() <= TOL_MAX, f"{what} max-abs {d.max().item()}"
    assert d.mean().item() <= TOL_MEAN, f"{what} mean-abs {d.mean().item()}"


def _oracle(w, idx=None):
    idx = list(range(w.num_seqs)) if idx is None else idx
    q = w.q[idx].cpu()
    return ora.decode_paged(q, w.k_pages.cpu(), w.v_pages.cpu(), w.block_table[idx].cpu(),
                            [w.lengths[i] for i in idx])


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (8, 8, 128), (16, 8, 128), (32, 4, 128),
                                      (12, 12, 64), (8, 2, 64)])
def test_decode_shapes(hq, hkv, d):
    lengths = [1, 15, 16, 17, 31, 33, 100, 257, 1000, 2049]
    w = decode_inputs(N=len(lengths), Hq=hq, Hkv=hkv, D=d, prefix_tokens=0, lengths=lengths, seed=3)
    o, lse = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                              pages_per_split=4, return_lse=True)
    ref, ref_lse = _oracle(w)
    _check(o, ref, f"hq={hq} hkv={hkv} d={d}")
    assert (lse.cpu() - ref_lse).abs().max().item() < 1e-3


@pytest.mark.parametrize("pps", [1, 2, 3, 8, 64, 200, 256])
def test_decode_split_sizes(pps):
    """Split sizes from one page (hundreds of partials per session for the combine) to a whole
    256-page session in one split (a warp then takes 64 pages: its page ids come in two batches
    of 32)."""
    lengths = [5, 160, 161, 999, 4096]
    w = decode_inputs(N=5, lengths=lengths, prefix_tokens=0, seed=4)
    o = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens, pages_per_split=pps)
    _check(o, _oracle(w)[0], f"pps={pps}")


@pytest.mark.parametrize("prefix_tokens", [16, 160, 2048])
def test_decode_shared_prefix(prefix_tokens):
    lengths = [1, 20, 160, 700, 2048, 2049, 3000, 5000, 31, 4000, 16, 2100]
    w = decode_inputs(N=len(lengths), lengths=lengths, prefix_tokens=prefix_tokens, seed=5)
    o_sh = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                            num_prefix_pages=w.n_prefix_pages, pages_per_split=8)
    o_ns = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens, pages_per_split=8)
    ref = _oracle(w)[0]
    _check(o_sh, ref, "shared prefix")
    _check(o_ns, ref, "no sharing")


@pytest.mark.parametrize("hq,hkv,d", [(12, 12, 64), (16, 4, 64), (8, 2, 64), (16, 2, 64),
                                      (16, 4, 128), (8, 8, 128)])
@pytest.mark.parametrize("prefix_tokens", [160, 2048])
def test_decode_shared_prefix_head_shapes(hq, hkv, d, prefix_tokens):
    """The shared-prefix pass for every GQA group size and both head dims: head_dim 64 runs the
    CUDA-core prefix kernel, 128 the tensor-core one; both write bf16 O / l partials that the
    combine scales back.  The workspace is filled with NaN bytes first."""
    lengths = [1, 20, 160, 700, 2048, 2049, 3000, 31, 4000, 16, 2100]
    w = decode_inputs(N=len(lengths), Hq=hq, Hkv=hkv, D=d, lengths=lengths,
                      prefix_tokens=prefix_tokens, seed=hq + hkv + d)
    max_pages = w.block_table.shape[1]
    need = att.decode_workspace_bytes(len(lengths), hq, d, max_pages, 8, w.n_prefix_pages)
    ws = torch.full((need,), 255, dtype=torch.uint8, device="cuda")
    o = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                         num_prefix_pages=w.n_prefix_pages, pages_per_split=8, workspace=ws)
    _check(o, _oracle(w)[0], f"hq={hq} hkv={hkv} d={d} prefix={prefix_tokens}")


def test_decode_reference_api_matches_reference_check():
    """decode_attention_fwd on [B,H,S,D] vs the reference's _reference_decode_attn (fp32 here)."""
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(2, 12, 1, 64, generator=g, device="cuda").bfloat16()
    k = torch.randn(2, 12, 300, 64, generator=g, device="cuda").bfloat16()
    v = torch.randn(2, 12, 300, 64, generator=g, device="cuda").bfloat16()
    o = att.decode_attention_fwd(q, k, v)
    ref = ora.reference_decode_attn(q.cpu().float(), k.cpu().float(), v.cpu().float())
    _check(o, ref)


def test_decode_full_size_every_session():
    """The 256-session, 2048-token-prefix workload at full size: every session against an fp32
    attention computed on the GPU, sampled sessions against the CPU oracle, and the
    shared-prefix path equal to the per-session path on every session."""
    from fp32_gpu_reference import decode_errors
    w = decode_inputs(seed=0)
    o_sh = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                            num_prefix_pages=w.n_prefix_pages)
    o_ns = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens)
    d = (o_sh.float() - o_ns.float()).abs()
    assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN
    mx, mean, n = decode_errors(w.q, w.k_pages, w.v_pages, w.block_table, w.lengths, o_sh)
    assert n == 256 and mx <= TOL_MAX and mean <= TOL_MEAN, (mx, mean)
    order = sorted(range(w.num_seqs), key=lambda i: w.lengths[i])
    idx = [order[0], order[1], order[len(order) // 2], order[-1]]
    ref, _ = _oracle(w, idx)
    _check(o_sh[idx], ref, "full-size sample")
    b = decode_bytes(w)
    assert b["unique"] < b["logical"]


def test_decode_rejects_bad_arguments():
    w = decode_inputs(N=2, lengths=[10, 20], prefix_tokens=0, seed=1)
    with pytest.raises(RuntimeError):
        att.paged_decode(w.q.float(), w.k_pages, w.v_pages, w.block_table, w.seq_lens)
    with pytest.raises(RuntimeError):
        att.paged_decode(w.q.cpu(), w.k_pages, w.v_pages, w.block_table, w.seq_lens)


def test_decode_sessions_entirely_inside_the_shared_prefix():
    """Every session's context lies within the shared prefix, so the table has no own pages and
    only the prefix pass runs (no split kernel)."""
    lengths = [1024, 17, 160, 1000, 1, 512]
    w = decode_inputs(N=len(lengths), lengths=lengths, prefix_tokens=1024, seed=9)
    assert w.block_table.shape[1] == w.n_prefix_pages
    o = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                         num_prefix_pages=w.n_prefix_pages)
    _check(o, _oracle(w)[0], "prefix only")


@pytest.mark.parametrize("lengths", [[100] * 64 + [3000], [40, 100] * 32 + [2100, 5000],
                                     [20, 3000, 5000, 257]])
def test_decode_sessions_shorter_than_the_prefix(lengths):
    """Sessions shorter than the shared prefix hold only the prefix pages they cover (the rest
    of their row is -1).  The prefix pass works on tiles of 64 sessions (4 query heads each): a
    tile whose sessions all end before a prefix chunk skips that chunk, and the combine must not
    read its slot -- the workspace is filled with NaN bytes first.  The last case's first
    session covers no chunk, so every item takes its pages from the tile's longest session."""
    w = decode_inputs(N=len(lengths), lengths=lengths, prefix_tokens=2048, seed=9)
    max_pages = w.block_table.shape[1]
    need = att.decode_workspace_bytes(len(lengths), w.q.shape[1], w.q.shape[2], max_pages, 8,
                                      w.n_prefix_pages)
    ws = torch.full((need,), 255, dtype=torch.uint8, device="cuda")
    o = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                         num_prefix_pages=w.n_prefix_pages, pages_per_split=8, workspace=ws)
    _check(o, _oracle(w)[0], f"lengths={lengths}")


@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (16, 4, 64)])
@pytest.mark.parametrize("prefix_tokens", [0, 1024])
def test_decode_empty_sessions(hq, hkv, d, prefix_tokens):
    """Sessions with no tokens yet (length 0, a table row of -1) beside others in one batch: their
    output rows are zeros and their LSE is -inf (attention over no keys is an empty sum), and the
    other sessions match the oracle.  The workspace is NaN-filled, so a read of a partial slot
    that nothing wrote would show."""
    lengths = [0, 1, 300, 0, 2049, 1100, 0]
    w = decode_inputs(N=len(lengths), Hq=hq, Hkv=hkv, D=d, lengths=lengths,
                      prefix_tokens=prefix_tokens, seed=12)
    max_pages, pps = w.block_table.shape[1], 8
    need = att.decode_workspace_bytes(len(lengths), hq, d, max_pages, pps, w.n_prefix_pages)
    ws = torch.full((need,), 255, dtype=torch.uint8, device="cuda")
    o, lse = att.paged_decode(w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens,
                              num_prefix_pages=w.n_prefix_pages, pages_per_split=pps, workspace=ws,
                              return_lse=True)
    empty = [i for i, L in enumerate(lengths) if L == 0]
    rest = [i for i, L in enumerate(lengths) if L > 0]
    assert torch.count_nonzero(o[empty]).item() == 0
    assert torch.isneginf(lse[empty]).all()
    ref, ref_lse = _oracle(w, rest)
    _check(o[rest], ref, f"hq={hq} hkv={hkv} d={d} prefix={prefix_tokens}")
    assert (lse[rest].cpu() - ref_lse).abs().max().item() < 1e-2


def test_decode_workspace_16_byte_aligned():
    """A workspace that is 16- but not 32-byte aligned takes the 16-byte store path of the
    shared-prefix pass (32-byte stores otherwise): the same bits as an aligned workspace."""
    lengths = [1, 300, 2049, 5000, 1024, 77, 4100]
    w = decode_inputs(N=len(lengths), lengths=lengths, prefix_tokens=2048, seed=13)
    max_pages = w.block_table.shape[1]
    need = att.decode_workspace_bytes(len(lengths), 32, 128, max_pages, 8, w.n_prefix_pages)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    buf = torch.empty(need + 32, dtype=torch.uint8, device="cuda")
    ws16 = buf[16:16 + need]
    assert ws.data_ptr() % 32 == 0 and ws16.data_ptr() % 32 == 16
    args = (w.q, w.k_pages, w.v_pages, w.block_table, w.seq_lens)
    o1 = att.paged_decode(*args, num_prefix_pages=w.n_prefix_pages, pages_per_split=8, workspace=ws)
    o2 = att.paged_decode(*args, num_prefix_pages=w.n_prefix_pages, pages_per_split=8, workspace=ws16)
    assert torch.equal(o1, o2)
    _check(o1, _oracle(w)[0], "aligned workspace")


@pytest.mark.parametrize("hq,hkv,d,prefix_tokens", [(32, 8, 128, 2048), (32, 8, 128, 0),
                                                    (16, 4, 64, 1024), (8, 8, 128, 256)])
def test_decode_fused_append_equals_separate_append(hq, hkv, d, prefix_tokens):
    """``paged_decode(k_new=, v_new=)`` stores each session's newest token (position L - 1)
    into its page inside the split pass and attends to it: pages and output are bit-identical
    to storing the token first and decoding after, and the output matches the oracle."""
    lengths = [prefix_tokens + x for x in (1, 16, 17, 300, 2049, 33, 1000)]
    w = decode_inputs(N=len(lengths), Hq=hq, Hkv=hkv, D=d, lengths=lengths,
                      prefix_tokens=prefix_tokens, seed=14)
    N = len(lengths)
    _device_status()                                  # start from a clear error word
    g = torch.Generator(device="cuda").manual_seed(15)
    k_new = torch.randn(N, hkv, d, generator=g, device="cuda").bfloat16()
    v_new = torch.randn(N, hkv, d, generator=g, device="cuda").bfloat16()
    kp_a, vp_a = w.k_pages.clone(), w.v_pages.clone()
    for n, L in enumerate(lengths):
        page = int(w.block_table[n, (L - 1) // 16])
        kp_a[page, :, (L - 1) % 16] = k_new[n]
        vp_a[page, :, (L - 1) % 16] = v_new[n]
    args = dict(num_prefix_pages=w.n_prefix_pages, pages_per_split=8)
    o_a = att.paged_decode(w.q, kp_a, vp_a, w.block_table, w.seq_lens, **args)
    kp_b, vp_b = w.k_pages.clone(), w.v_pages.clone()
    o_b = att.paged_decode(w.q, kp_b, vp_b, w.block_table, w.seq_lens, k_new=k_new, v_new=v_new,
                           **args)
    assert torch.equal(kp_a, kp_b) and torch.equal(vp_a, vp_b)
    assert torch.equal(o_a, o_b)
    ref = ora.decode_paged(w.q.cpu(), kp_a.cpu(), vp_a.cpu(), w.block_table.cpu(), lengths)[0]
    _check(o_b, ref, f"fused append hq={hq} hkv={hkv} d={d} prefix={prefix_tokens}")
    assert _device_status() == 0


def test_decode_fused_append_reports_a_token_inside_the_shared_prefix():
    """A session whose newest token would land inside the shared-prefix pages has no page of its
    own to store it in: nothing is stored and the device error word reports it (site 212)."""
    lengths = [1000, 3000]                       # the first ends inside the 2048-token prefix
    w = decode_inputs(N=2, lengths=lengths, prefix_tokens=2048, seed=16)
    kp, vp = w.k_pages.clone(), w.v_pages.clone()
    z = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device="cuda")
    _device_status()
    att.paged_decode(w.q, kp, vp, w.block_table, w.seq_lens, num_prefix_pages=w.n_prefix_pages,
                     pages_per_split=8, k_new=z, v_new=z)
    torch.cuda.synchronize()
    assert _device_status() == 212
    assert torch.equal(kp[w.block_table[0, :w.n_prefix_pages].long()],
                       w.k_pages[w.block_table[0, :w.n_prefix_pages].long()])


def _device_status():
    import ctypes
    from loopfuse_b200 import _lib
    torch.cuda.synchronize()
    v = ctypes.c_int(0)
    assert _lib.lib().lf_device_status(ctypes.byref(v)) == _lib.LF_OK
    return v.value
