"""The CPU oracle against golden vectors produced by the reference's own code.

Fixtures come from ``tests/golden/make_golden.py`` (imports the reference):
``_reference_decode_attn`` outputs and the fp32 SDPA causal check of the
reference's prefill verifier.  These pin the oracle before it is trusted as
the reference computation of the sm_100a kernels' parity tests.
"""
import os

import numpy as np
import pytest
import torch

from oracle import attention as ora

TOL_MAX = 2e-2     # bf16 output vs fp32 reference, max-abs
TOL_MEAN = 2e-3    # mean-abs


@pytest.fixture(scope="module")
def att(golden_dir):
    z = np.load(os.path.join(golden_dir, "attention_fp16.npz"))
    return {k: torch.from_numpy(z[k]) for k in z.files}


def test_reference_decode_restatement_bitexact(att):
    out = ora.reference_decode_attn(att["dec_q"], att["dec_k"], att["dec_v"])
    assert torch.equal(out, att["dec_out"])


def test_decode_oracle_matches_reference(att):
    q, k, v = att["dec_q"], att["dec_k"], att["dec_v"]
    # contiguous cache -> one page table per batch row
    B, H, S, D = k.shape
    pages = k.view(B, H, S // 16, 16, D).permute(0, 2, 1, 3, 4).reshape(-1, H, 16, D)
    vpages = v.view(B, H, S // 16, 16, D).permute(0, 2, 1, 3, 4).reshape(-1, H, 16, D)
    table = torch.arange(S // 16, dtype=torch.int32).view(1, -1)
    o, lse = ora.decode_paged(q.view(B, H, D), pages, vpages, table, [S])
    ref = att["dec_out"].float().view(B, H, D)
    assert (o - ref).abs().max().item() < 1e-2          # the reference's own threshold
    o2 = ora.decode_paged_sdpa(q.view(B, H, D), pages, vpages, table, [S])
    assert torch.allclose(o, o2, atol=1e-5)


def test_prefill_oracle_matches_reference_sdpa(att):
    o, lse = ora.prefill(att["pre_q"], att["pre_k"], att["pre_v"], causal=True)
    assert torch.allclose(o, att["pre_out_fp32"], atol=1e-5, rtol=1e-5)
    assert (o.half() - att["pre_out"]).abs().max().item() <= 1e-3


def test_prefill_oracle_gqa_and_offset():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 8, 40, 32, generator=g)
    k = torch.randn(2, 2, 40, 32, generator=g)
    v = torch.randn(2, 2, 40, 32, generator=g)
    o, _ = ora.prefill(q, k, v, causal=True)
    assert torch.allclose(o, ora.sdpa_eager(q, k, v, causal=True), atol=1e-5)
    # bottom-right causal: queries appended after 24 cached keys
    qa = q[:, :, 24:]
    oa, _ = ora.prefill(qa, k, v, causal=True)
    assert torch.allclose(oa, o[:, :, 24:], atol=1e-5)


def test_merge_partials_equals_full():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 4, 1, 16, generator=g)
    k = torch.randn(1, 4, 50, 16, generator=g)
    v = torch.randn(1, 4, 50, 16, generator=g)
    o_full, lse_full = ora.prefill(q, k, v, causal=False)
    parts = [ora.prefill(q, k[:, :, a:b], v[:, :, a:b], causal=False) for a, b in ((0, 13), (13, 37), (37, 50))]
    o, lse = ora.merge_partials([p[0] for p in parts], [p[1] for p in parts])
    assert torch.allclose(o, o_full, atol=1e-5)
    assert torch.allclose(lse, lse_full, atol=1e-5)


def test_tolerance_constants_match_contract():
    assert TOL_MAX == 2e-2 and TOL_MEAN == 2e-3
