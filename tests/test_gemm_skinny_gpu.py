"""The decode-batch projection GEMM (``lf_gemm_skinny``) against an fp32 torch product.

Inputs are bf16; the kernel accumulates in fp32 and rounds once to bf16, so every element must
lie within one bf16 rounding (relative 2^-8) of the fp32 product plus a small absolute term for
the fp32 summation order (1e-3 of the output's RMS).  Shapes: the Llama-3-8B projections at
decode batches, ragged N and K (the last column block and K chunk partly out of range), and
SM counts that change how the stream-K runs split the column blocks.  Results must be
bit-identical from call to call (partials are summed in a fixed order).
"""
import ctypes

import pytest
import torch

from loopfuse_b200 import _lib
from loopfuse_b200 import model_ops as mo

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(k, n, generator=g, device="cuda") * 0.02).bfloat16()
    return x, w


def _check(y, x, w):
    ref = x.float() @ w.float()
    tol = ref.abs() * 2 ** -8 + 1e-3 * ref.pow(2).mean().sqrt()
    err = (y.float() - ref).abs()
    assert bool((err <= tol).all()), (err - tol).max().item()


@pytest.mark.parametrize("m", [1, 7, 64, 65, 100, 128])
@pytest.mark.parametrize("shape", [(4096, 6144), (4096, 4096), (14336, 4096)])
def test_llama_projection_shapes(m, shape):
    torch.backends.cuda.matmul.allow_tf32 = False
    k, n = shape
    x, w = _case(m, n, k, m * 7 + n)
    _check(mo.gemm_skinny(x, w), x, w)


@pytest.mark.parametrize("m,n,k", [(3, 136, 72), (17, 256, 64), (100, 1000, 520), (5, 392, 1032),
                                   (64, 8, 8), (128, 128264, 4096)])
def test_ragged_shapes(m, n, k):
    torch.backends.cuda.matmul.allow_tf32 = False
    x, w = _case(m, n, k, m + n + k)
    _check(mo.gemm_skinny(x, w), x, w)


@pytest.mark.parametrize("sms", [1, 7, 37, 148, 300])
def test_split_layouts_and_determinism(sms):
    """Grids of ``sms`` CTAs cut the column blocks at different units; results must not depend
    on the cut beyond fp32 summation order, and repeat bit for bit."""
    torch.backends.cuda.matmul.allow_tf32 = False
    m, n, k = 40, 768, 3072
    x, w = _case(m, n, k, sms)
    need = ctypes.c_size_t(0)
    _lib.call("lf_gemm_skinny_workspace_size", m, n, k, sms, ctypes.byref(need))
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        _lib.call("lf_gemm_skinny", x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k,
                  ws.data_ptr(), ws.numel(), sms, torch.cuda.current_stream().cuda_stream)
        outs.append(y)
    torch.cuda.synchronize()
    v = ctypes.c_int(-1)
    assert _lib.lib().lf_device_status(ctypes.byref(v)) == _lib.LF_OK and v.value == 0
    _check(outs[0], x, w)
    assert torch.equal(outs[0], outs[1])


def test_matches_library_gemm_closely():
    """Against cuBLAS bf16 (also fp32-accumulated): the two differ only by summation order."""
    x, w = _case(64, 6144, 4096, 1)
    a = mo.gemm_skinny(x, w)
    b = x @ w
    rel = ((a.float() - b.float()).abs() / b.float().abs().clamp_min(1e-2)).max().item()
    assert rel <= 2 ** -7, rel
