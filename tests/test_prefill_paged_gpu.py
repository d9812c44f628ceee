"""Prefill of appended tokens over cached paged context vs the fp32 oracle.

Sessions with cached contexts of different lengths (one forked from a shared prefix) get new
tokens appended through the device pool (reserve once, write per layer), then the new tokens
attend to their whole session through the block tables.  Tolerance: bf16 output vs fp32
oracle, max-abs <= 2e-2 and mean-abs <= 2e-3.
"""
import pytest
import torch

from oracle import attention as ora
from loopfuse_b200 import attention as att
from loopfuse_b200.runtime.kv_pool import KVPool

pytestmark = pytest.mark.gpu
TOL_MAX, TOL_MEAN = 2e-2, 2e-3


def _rand(*shape, g):
    return torch.randn(*shape, generator=g, device="cuda", dtype=torch.float32).bfloat16()


@pytest.mark.parametrize("hq,hkv,D", [(32, 8, 128), (8, 8, 128), (12, 12, 64), (16, 4, 64),
                                      (12, 4, 128), (32, 4, 128), (32, 2, 64)])
def test_paged_prefill_matches_oracle(hq, hkv, D):
    g = torch.Generator(device="cuda").manual_seed(11)
    L = 2
    pool = KVPool(num_layers=L, num_heads=hq, num_kv_heads=hkv, head_dim=D, max_seq_len=2048,
                  max_slots=6, dtype=torch.bfloat16)
    base = pool.allocate_slot()
    pre = _rand(L, 300, hkv, D, g=g)
    pool.append([base], [pre], [pre + 1])
    forked = pool.fork(base, 272)[0]                          # shares 17 full pages
    other = pool.allocate_slot()
    ctx = _rand(L, 37, hkv, D, g=g)
    pool.append([other], [ctx], [ctx - 1])
    fresh = pool.allocate_slot()                              # no cached context
    states = [base, forked, other, fresh]
    new_counts = [129, 1, 300, 64]
    start = pool.reserve(states, new_counts)
    T = sum(new_counts)
    layer = 1
    newk = [_rand(T, hkv, D, g=g) for _ in range(L)]
    newv = [_rand(T, hkv, D, g=g) for _ in range(L)]
    for l in range(L):
        pool.write_layer(states, start, l, newk[l], newv[l], new_counts)
    q = _rand(T, hq, D, g=g)
    table, lens = pool.block_table(states)
    cu = torch.tensor([0] + list(torch.tensor(new_counts).cumsum(0)), dtype=torch.int32, device="cuda")
    kp, vp = pool.layer_pages(layer)
    o, lse = att.prefill_paged(q, kp, vp, table, cu, lens, max(new_counts), return_lse=True)
    into = torch.full_like(q, float("nan"))
    att.prefill_paged(q, kp, vp, table, cu, lens, max(new_counts), out=into)
    assert torch.equal(into, o)                               # the out= path writes the same bits
    off = 0
    for i, s in enumerate(states):
        n = new_counts[i]
        k, v = pool.read(s, layer)                            # [Hkv, Lk, D]
        qi = q[off:off + n].permute(1, 0, 2).unsqueeze(0)     # [1, Hq, n, D]
        ref, ref_lse = ora.prefill(qi.cpu(), k.unsqueeze(0).cpu(), v.unsqueeze(0).cpu(), causal=True)
        got = o[off:off + n].permute(1, 0, 2).unsqueeze(0).float().cpu()
        d = (got - ref).abs()
        assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN, (i, d.max().item())
        gl = lse[off:off + n].permute(1, 0).unsqueeze(0).cpu()
        assert (gl - ref_lse).abs().max().item() < 1e-2
        off += n


def test_paged_prefill_equals_dense_prefill_on_contiguous_context():
    g = torch.Generator(device="cuda").manual_seed(5)
    S, hq, hkv, D = 512, 8, 2, 128
    pool = KVPool(num_layers=1, num_heads=hq, num_kv_heads=hkv, head_dim=D, max_seq_len=S,
                  max_slots=1, dtype=torch.bfloat16)
    s = pool.allocate_slot()
    k = _rand(1, S, hkv, D, g=g)
    v = _rand(1, S, hkv, D, g=g)
    pool.append([s], [k], [v])
    q = _rand(S, hq, D, g=g)
    table, lens = pool.block_table([s])
    cu = torch.tensor([0, S], dtype=torch.int32, device="cuda")
    kp, vp = pool.layer_pages(0)
    o = att.prefill_paged(q, kp, vp, table, cu, lens, S)
    od = att.prefill_attention_fwd(q.permute(1, 0, 2).unsqueeze(0).contiguous(),
                                   k[0].permute(1, 0, 2).unsqueeze(0).contiguous(),
                                   v[0].permute(1, 0, 2).unsqueeze(0).contiguous())
    # The two modes share the tile loop but not the exp2 split between MUFU and FMA, so some
    # bf16 outputs differ by a rounding step; a paging error would be far larger.
    d = (o.permute(1, 0, 2).float() - od[0].float()).abs()
    same, worst, mean = (d == 0).float().mean().item(), d.max().item(), d.mean().item()
    assert same >= 0.9 and worst <= 5e-3 and mean <= 1e-4, (same, worst, mean)


def test_paged_prefill_sessions_without_new_tokens():
    """A batch may list sessions that append nothing (cu_seqlens repeats): they get no rows and
    the other sessions' results are unchanged."""
    g = torch.Generator(device="cuda").manual_seed(21)
    hq, hkv, D = 8, 2, 128
    pool = KVPool(num_layers=1, num_heads=hq, num_kv_heads=hkv, head_dim=D, max_seq_len=1024,
                  max_slots=4, dtype=torch.bfloat16)
    ss = [pool.allocate_slot() for _ in range(4)]
    ctx = _rand(1, 200, hkv, D, g=g)
    pool.append([ss[1]], [ctx], [ctx])                       # cached context, no new tokens
    counts = [70, 0, 33, 0]
    start = pool.reserve(ss, counts)
    T = sum(counts)
    nk = _rand(T, hkv, D, g=g)
    pool.write_layer(ss, start, 0, nk, nk, counts)
    q = _rand(T, hq, D, g=g)
    table, lens = pool.block_table(ss)
    cu = torch.tensor([0, 70, 70, 103, 103], dtype=torch.int32, device="cuda")
    kp, vp = pool.layer_pages(0)
    o = att.prefill_paged(q, kp, vp, table, cu, lens, max(counts))
    off = 0
    for s, n in zip(ss, counts):
        if n == 0:
            continue
        k, v = pool.read(s, 0)
        qi = q[off:off + n].permute(1, 0, 2).unsqueeze(0)
        ref, _ = ora.prefill(qi.cpu(), k.unsqueeze(0).cpu(), v.unsqueeze(0).cpu(), causal=True)
        d = (o[off:off + n].permute(1, 0, 2).unsqueeze(0).float().cpu() - ref).abs()
        assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN
        off += n


def test_paged_prefill_many_ragged_items_fp32():
    """Agent-shaped appends with far more work items than SMs: 96 sessions forked from a
    1024-token prefix, 1-300 new tokens each (3840 items, most CTAs take over pending ones).
    Every session and KV head against the fp32 GPU reference; a second launch must give the
    same bits (an item is computed whole by whichever CTA takes it)."""
    from fp32_gpu_reference import prefill_unit
    g = torch.Generator(device="cuda").manual_seed(21)
    gc = torch.Generator().manual_seed(21)
    N, hq, hkv, D, L = 96, 32, 8, 128, 1
    counts = [int(x) for x in torch.randint(1, 301, (N,), generator=gc)]
    pool = KVPool(num_layers=L, num_heads=hq, num_kv_heads=hkv, head_dim=D, max_seq_len=1400,
                  max_slots=N + 1, dtype=torch.bfloat16)
    root = pool.allocate_slot()
    pre = _rand(L, 1024, hkv, D, g=g)
    pool.append([root], [pre], [pre * 0.5])
    states = pool.fork(root, 1024, n=N)
    start = pool.reserve(states, counts)
    T = sum(counts)
    pool.write_layer(states, start, 0, _rand(T, hkv, D, g=g), _rand(T, hkv, D, g=g), counts)
    q = _rand(T, hq, D, g=g)
    table, lens = pool.block_table(states)
    cu = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32, device="cuda")
    kp, vp = pool.layer_pages(0)
    o = att.prefill_paged(q, kp, vp, table, cu, lens, max(counts))
    again = att.prefill_paged(q, kp, vp, table, cu, lens, max(counts))
    assert torch.equal(o, again)
    G = hq // hkv
    worst, total, cnt = 0.0, 0.0, 0
    off = 0
    for i, s in enumerate(states):
        n = counts[i]
        k, v = pool.read(s, 0)                                # [Hkv, Lk, D]
        for h in range(hkv):
            qi = q[off:off + n, h * G:(h + 1) * G].permute(1, 0, 2)        # [G, n, D]
            ref, _ = prefill_unit(qi, k[h], v[h], causal=True)
            d = (o[off:off + n, h * G:(h + 1) * G].permute(1, 0, 2).float() - ref).abs()
            worst = max(worst, d.max().item())
            total += d.sum().item()
            cnt += d.numel()
        off += n
    assert worst <= TOL_MAX and total / cnt <= TOL_MEAN, (worst, total / cnt)


def test_paged_prefill_sessions_with_no_new_tokens():
    """Sessions that append nothing this step (equal cu_seqlens_q entries; one of them has no
    context either) beside sessions that do: they own no query rows, every row of a NaN-filled
    output is written, and the other sessions match the oracle."""
    g = torch.Generator(device="cuda").manual_seed(21)
    hq, hkv, D = 32, 8, 128
    pool = KVPool(num_layers=1, num_heads=hq, num_kv_heads=hkv, head_dim=D, max_seq_len=2048,
                  max_slots=5, dtype=torch.bfloat16)
    states = [pool.allocate_slot() for _ in range(4)]
    ctx = [300, 37, 0, 500]
    for s, n in zip(states, ctx):
        if n:
            kk = _rand(1, n, hkv, D, g=g)
            pool.append([s], [kk], [kk - 0.5])
    new_counts = [0, 64, 0, 129]
    start = pool.reserve(states, new_counts)
    T = sum(new_counts)
    newk, newv = _rand(T, hkv, D, g=g), _rand(T, hkv, D, g=g)
    pool.write_layer(states, start, 0, newk, newv, new_counts)
    q = _rand(T, hq, D, g=g)
    table, lens = pool.block_table(states)
    cu = torch.tensor([0] + list(torch.tensor(new_counts).cumsum(0)), dtype=torch.int32, device="cuda")
    kp, vp = pool.layer_pages(0)
    o = torch.full_like(q, float("nan"))
    att.prefill_paged(q, kp, vp, table, cu, lens, max(new_counts), out=o)
    assert not torch.isnan(o).any()
    # an output 16- but not 32-byte aligned takes the 16-byte store path: same bits
    buf = torch.full((q.numel() + 16,), float("nan"), dtype=torch.bfloat16, device="cuda")
    o16 = buf[8:8 + q.numel()].view(q.shape)
    assert o16.data_ptr() % 32 == 16
    att.prefill_paged(q, kp, vp, table, cu, lens, max(new_counts), out=o16)
    assert torch.equal(o16, o)
    off = 0
    for i, s in enumerate(states):
        n = new_counts[i]
        if n == 0:
            continue
        k, v = pool.read(s, 0)
        qi = q[off:off + n].permute(1, 0, 2).unsqueeze(0)
        ref, _ = ora.prefill(qi.cpu(), k.unsqueeze(0).cpu(), v.unsqueeze(0).cpu(), causal=True)
        d = (o[off:off + n].permute(1, 0, 2).unsqueeze(0).float().cpu() - ref).abs()
        assert d.max().item() <= TOL_MAX and d.mean().item() <= TOL_MEAN, (i, d.max().item())
        off += n
