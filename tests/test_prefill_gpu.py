"""tcgen05 prefill (sm_100a) against the fp32 CPU oracle.

Tolerance: bf16 output vs fp32 oracle, max-abs <= 2e-2 and mean-abs <= 2e-3;
LSE (natural log) within 1e-2.
"""
import pytest
import torch

from oracle import attention as ora
from loopfuse_b200 import attention as att
from loopfuse_b200.workloads import prefill_inputs

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_MEAN = 2e-2, 2e-3


def _run_and_check(B, Hq, Hkv, Sq, Sk, causal, seed=0, D=128):
    q, k, v = prefill_inputs(B, Hq, Hkv, Sq, D, seed=seed, Sk=Sk)
    o, lse = att.prefill_attention_fwd(q, k, v, causal=causal, return_lse=True)
    ref, ref_lse = ora.prefill(q.cpu(), k.cpu(), v.cpu(), causal=causal)
    d = (o.float().cpu() - ref).abs()
    assert d.max().item() <= TOL_MAX, d.max().item()
    assert d.mean().item() <= TOL_MEAN, d.mean().item()
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - ref_lse[fin]).abs().max().item() < 1e-2


@pytest.mark.parametrize("S", [128, 256, 512])
def test_prefill_causal_mha(S):
    _run_and_check(1, 2, 2, S, S, True)


@pytest.mark.parametrize("S", [1, 17, 129, 200, 383])
def test_prefill_ragged_lengths(S):
    _run_and_check(2, 4, 1, S, S, True, seed=S)


def test_prefill_gqa_noncausal():
    _run_and_check(1, 8, 2, 256, 384, False, seed=3)


@pytest.mark.parametrize("Sq,Sk", [(128, 384), (40, 300), (256, 257)])
def test_prefill_appended_queries(Sq, Sk):
    """Bottom-right causal: new tool-output tokens attend to a cached prefix."""
    _run_and_check(1, 4, 1, Sq, Sk, True, seed=Sq + Sk)


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,causal", [
    (2, 8, 2, 300, 300, False),        # head_dim 128 without the causal mask, ragged last tile
    (1, 16, 2, 256, 640, False),       # more keys than queries, no mask
    (3, 16, 2, 257, 257, True),        # GQA group 8, a tile with a single row
    (2, 24, 3, 130, 1000, True),       # group 8 over a long cached context
    (4, 4, 4, 1, 513, True),           # one new token per (batch, head) over 513 keys
])
def test_prefill_more_shapes(B, Hq, Hkv, Sq, Sk, causal):
    _run_and_check(B, Hq, Hkv, Sq, Sk, causal, seed=B * 1000 + Sq + Sk)


@pytest.mark.parametrize("Sq,Sk,causal", [(200, 200, True), (128, 512, True), (77, 300, False)])
def test_prefill_head_dim_64(Sq, Sk, causal):
    """GPT-2 style 64-dim heads (MHA 12 heads)."""
    _run_and_check(1, 12, 12, Sq, Sk, causal, seed=Sq, D=64)


def test_prefill_output_16_byte_aligned():
    """An output that is 16- but not 32-byte aligned takes the 16-byte store path of the
    epilogue (32-byte stores otherwise): same bits as the aligned output."""
    from loopfuse_b200 import _lib
    q, k, v = prefill_inputs(1, 4, 1, 200, 128, seed=2)
    o = att.prefill_attention_fwd(q, k, v, causal=True)
    buf = torch.full((q.numel() + 16,), float("nan"), dtype=torch.bfloat16, device="cuda")
    o2 = buf[8:8 + q.numel()].view(q.shape)
    assert o2.data_ptr() % 32 == 16
    _lib.call("lf_prefill_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), o2.data_ptr(), None,
              1, 4, 1, 200, 200, 128, 128 ** -0.5, 1, att._stream())
    torch.cuda.synchronize()
    assert torch.equal(o2, o)


def test_prefill_longer_sequence():
    _run_and_check(1, 8, 2, 1024, 1024, True, seed=11)


def test_prefill_full_size_every_unit():
    """B=8, Hq=32, Hkv=8, S=4096 (the benchmark's shape): all 64 (batch, KV head) units against
    an fp32 attention computed on the GPU, one GQA group of batch 5 against the CPU oracle,
    and determinism of the full launch."""
    from fp32_gpu_reference import prefill_errors
    q, k, v = prefill_inputs(seed=0)
    o = att.prefill_attention_fwd(q, k, v, causal=True)
    o2 = att.prefill_attention_fwd(q, k, v, causal=True)
    assert torch.equal(o, o2)
    mx, mean, units = prefill_errors(q, k, v, o, causal=True)
    assert units == 64
    assert mx <= TOL_MAX and mean <= TOL_MEAN, (mx, mean)
    b, g = 5, 3
    ref, _ = ora.prefill(q[b:b + 1, 4 * g:4 * g + 4].cpu(), k[b:b + 1, g:g + 1].cpu(),
                         v[b:b + 1, g:g + 1].cpu(), causal=True)
    d = (o[b:b + 1, 4 * g:4 * g + 4].float().cpu() - ref).abs()
    assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN


def test_prefill_reference_api_shape_and_dtype_checks():
    q, k, v = prefill_inputs(1, 2, 2, 64, 128, seed=1)
    with pytest.raises(RuntimeError):
        att.prefill_attention_fwd(q.float(), k, v)
    with pytest.raises(RuntimeError):
        att.prefill_attention_fwd(q, k[:, :, :, :64].contiguous(), v)


def test_prefill_work_distribution_in_graphs_and_concurrent_streams():
    """The work list is distributed by the hardware per launch (a CTA that finishes takes over a
    pending CTA's item), with no counters shared between launches.  So a launch replayed from a
    CUDA graph, and two launches running at the same time on two streams, must give the bits of
    a lone eager launch.  Both shapes have several times more items than SMs."""
    qa, ka, va = prefill_inputs(4, 32, 8, 2048, 128, seed=3)
    qb, kb, vb = prefill_inputs(2, 16, 4, 4096, 128, seed=4)
    ref_a = att.prefill_attention_fwd(qa, ka, va, causal=True)
    ref_b = att.prefill_attention_fwd(qb, kb, vb, causal=True)
    torch.cuda.synchronize()
    # graph replays
    out_a = torch.empty_like(qa)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            out_a.copy_(att.prefill_attention_fwd(qa, ka, va, causal=True))
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        out_a.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_a, ref_a)
    # two streams at once, several rounds
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(3):
        s1.wait_stream(torch.cuda.current_stream())
        s2.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s1):
            o1 = att.prefill_attention_fwd(qa, ka, va, causal=True)
        with torch.cuda.stream(s2):
            o2 = att.prefill_attention_fwd(qb, kb, vb, causal=True)
        torch.cuda.synchronize()
        assert torch.equal(o1, ref_a) and torch.equal(o2, ref_b)
