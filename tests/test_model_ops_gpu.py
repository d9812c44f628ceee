"""Fused decoder elementwise ops vs the eager torch sequences they replace.

The only admissible difference is the order of the fp32 sum of squares inside RMSNorm, which
can move a normalised value across a bf16 rounding boundary: outputs must match the torch
sequence exactly on >= 99% of elements and within one bf16 step (relative 2^-7) everywhere.
The residual sum and SwiGLU have no reduction and must match exactly.
"""
import pytest
import torch
import torch.nn.functional as F

from loopfuse_b200 import model_ops as mo

pytestmark = pytest.mark.gpu


def _torch_rmsnorm(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


@pytest.mark.parametrize("rows,dim", [(1, 4096), (37, 4096), (300, 768), (5, 8192), (3, 64)])
def test_add_rmsnorm_matches_torch(rows, dim):
    g = torch.Generator(device="cuda").manual_seed(rows + dim)
    x = torch.randn(rows, dim, generator=g, device="cuda").bfloat16()
    d = torch.randn(rows, dim, generator=g, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(dim, generator=g, device="cuda")).bfloat16()
    ref_x = x + d
    ref = _torch_rmsnorm(ref_x, w, 1e-5)
    got_x = x.clone()
    got = mo.add_rmsnorm(got_x, d, w, 1e-5)
    assert torch.equal(got_x, ref_x)
    same = (got == ref).float().mean().item()
    rel = ((got.float() - ref.float()).abs() / ref.float().abs().clamp_min(1e-3)).max().item()
    assert same >= 0.99 and rel <= 2 ** -7 + 1e-6, (same, rel)
    # norm only (no residual), and add only (no weight)
    got2 = mo.add_rmsnorm(ref_x.clone(), None, w, 1e-5)
    assert (got2 == ref).float().mean().item() >= 0.99
    y = x.clone()
    assert mo.add_rmsnorm(y, d, None, 1e-5) is None and torch.equal(y, ref_x)


@pytest.mark.parametrize("rows,ffn", [(1, 14336), (129, 14336), (64, 3072)])
def test_swiglu_matches_torch(rows, ffn):
    g = torch.Generator(device="cuda").manual_seed(rows)
    gu = (2 * torch.randn(rows, 2 * ffn, generator=g, device="cuda")).bfloat16()
    ref = F.silu(gu[:, :ffn]) * gu[:, ffn:]
    got = mo.swiglu(gu)
    diff = (got.float() - ref.float()).abs()
    # silu via expf may differ from torch's by an ulp in fp32 before the bf16 rounding
    assert (got == ref).float().mean().item() >= 0.999
    assert (diff / ref.float().abs().clamp_min(1e-3)).max().item() <= 2 ** -7 + 1e-6
