"""Fused QKV epilogue (split + RoPE + page scatter) vs the unfused torch path, bit for bit.

The unfused path is the eager fp32 torch "rotate half" formula (products and sums rounded
separately, then bf16) followed by ``KVPool.write_layer``; the fused kernel must give the same
q bytes and the same pool pages.
"""
import pytest
import torch

from loopfuse_b200 import _lib
from loopfuse_b200.llama import LlamaConfig, LlamaShaped
from loopfuse_b200.runtime.kv_pool import KVPool

pytestmark = pytest.mark.gpu


def _rope_ref(x, cos, sin):
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def _tables(D, rows, theta=500000.0):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    ang = torch.arange(rows, device="cuda").float()[:, None] * inv[None, :]
    return ang.cos().contiguous(), ang.sin().contiguous()


def _pools(hq, hkv, D, L=2):
    mk = lambda: KVPool(num_layers=L, num_heads=hq, num_kv_heads=hkv, head_dim=D, max_seq_len=1024,
                        max_slots=4, dtype=torch.bfloat16)
    return mk(), mk()


@pytest.mark.parametrize("hq,hkv,D,rope,pad", [(32, 8, 128, True, 0), (12, 12, 64, False, 0),
                                               (8, 2, 128, True, 64), (4, 4, 64, True, 16)])
def test_fused_matches_unfused(hq, hkv, D, rope, pad):
    g = torch.Generator(device="cuda").manual_seed(hq + D)
    pa, pb = _pools(hq, hkv, D)
    cached = [37, 0, 300]
    counts = [129, 1, 65]
    sa = [pa.alloc() for _ in cached]
    sb = [pb.alloc() for _ in cached]
    for pool, ss in ((pa, sa), (pb, sb)):
        pool.reserve(ss, cached)
    T = sum(counts)
    W = (hq + 2 * hkv) * D
    base = torch.randn(T, W + pad, generator=g, device="cuda").bfloat16()
    qkv = base[:, :W]                                           # strided rows when pad > 0
    cos, sin = _tables(D, 1024)
    layer = 1
    # unfused
    start_a = pa.reserve(sa, counts)
    pos = torch.cat([torch.arange(c0, c0 + n, device="cuda") for c0, n in zip(cached, counts)])
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    nq, nk = hq * D, hkv * D
    q_ref = qkv[:, :nq].reshape(T, hq, D)
    k_ref = qkv[:, nq:nq + nk].reshape(T, hkv, D)
    if rope:
        q_ref, k_ref = _rope_ref(q_ref, c, s), _rope_ref(k_ref, c, s)
    v_ref = qkv[:, nq + nk:].reshape(T, hkv, D).contiguous()
    pa.write_layer(sa, start_a, layer, k_ref.contiguous(), v_ref, counts)
    # fused
    start_b = pb.reserve(sb, counts)
    q = torch.empty(T, hq, D, dtype=torch.bfloat16, device="cuda")
    pb.write_qkv(sb, start_b, layer, qkv, q, counts, rope=(cos, sin) if rope else None)
    assert pb.status() == 0
    assert torch.equal(q, q_ref.contiguous())
    assert torch.equal(pa.keys, pb.keys) and torch.equal(pa.values, pb.values)


def test_position_past_table_sets_status():
    _, pool = _pools(4, 2, 64)
    st = pool.alloc()
    start = pool.reserve([st], [40])
    qkv = torch.zeros(40, 8 * 64, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(40, 4, 64, dtype=torch.bfloat16, device="cuda")
    cos, sin = _tables(64, 32)                                  # positions 32..39 missing
    pool.write_qkv([st], start, 0, qkv, q, [40], rope=(cos, sin))
    assert pool.status() == _lib.LF_EINVAL
    pool._call("lf_pool_clear_status", pool._meta_ref(), pool._stream())
    assert pool.status() == 0


def test_llama_forward_fused_equals_unfused():
    cfg = LlamaConfig(d_model=256, layers=2, q_heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000)
    model = LlamaShaped(cfg, seed=3)
    outs = []
    for fused in (True, False):
        model.fused_qkv = fused
        pool = KVPool(num_layers=2, num_heads=4, num_kv_heads=2, head_dim=128, max_seq_len=512,
                      max_slots=3, dtype=torch.bfloat16)
        ss = [pool.alloc() for _ in range(3)]
        toks = torch.randint(0, 1000, (90,), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
        l1 = model.forward(toks, pool, ss, [50, 30, 10], return_logits=True)
        l2 = model.forward(toks[:3], pool, ss, [1, 1, 1], return_logits=True)
        outs.append((l1, l2, pool.keys.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][2], outs[1][2])
