"""The KV-fusion loop on a small configuration: device pool metadata bit-exact against the pool
oracle after every fork, append (reserve) and free; decode output against the fp32 oracle."""
import pytest
import torch

from oracle import attention as ora
from oracle.pool_spec import PagedKVPoolSpec
from loopfuse_b200 import attention as att
from loopfuse_b200.kv_fusion_loop import FusionLoop, FusionLoopConfig

pytestmark = pytest.mark.gpu


def test_small_loop_is_bitexact_with_the_pool_oracle():
    cfg = FusionLoopConfig(sessions=6, steps=3, layers=2, prefix_tokens=64, decode_tokens=3,
                           tool_mean=20, tool_cap=50, seed=3)
    probe = FusionLoop(cfg)
    spec = PagedKVPoolSpec(probe.pool.num_pages, probe.pool.max_slots, probe.pool.max_pages_per_seq)
    del probe
    loop = FusionLoop(cfg, spec=spec)
    res = loop.run()
    assert res.checks == 2 + cfg.steps * (1 + cfg.decode_tokens) + 1
    for st in res.steps:
        assert st.bytes_read < st.bytes_read_unshared
        assert st.ms > 0


def test_decode_in_the_loop_matches_oracle():
    cfg = FusionLoopConfig(sessions=5, steps=1, layers=1, prefix_tokens=128, decode_tokens=1,
                           tool_mean=30, tool_cap=60, seed=4)
    loop = FusionLoop(cfg)
    loop.setup()
    loop.step(0)
    pool, S = loop.pool, loop.sessions
    table, lens = pool.block_table(S)
    kp, vp = pool.layer_pages(0)
    o = att.paged_decode(loop.qdec, kp, vp, table, lens, num_prefix_pages=loop.n_prefix_pages)
    ref, _ = ora.decode_paged(loop.qdec.cpu(), kp.cpu(), vp.cpu(), table.cpu(), lens.cpu())
    d = (o.float().cpu() - ref).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3
    loop.teardown()


def test_graphed_decode_iterations_equal_eager():
    """Graph replays of the decode iteration leave the pool exactly as eager iterations do."""
    res = []
    for graphs in (False, True):
        cfg = FusionLoopConfig(sessions=7, steps=2, layers=3, prefix_tokens=96, decode_tokens=5,
                               tool_mean=25, tool_cap=60, seed=11, graphs=graphs)
        loop = FusionLoop(cfg)
        loop.setup()
        for st in range(cfg.steps):
            loop.step(st)
        torch.cuda.synchronize()
        res.append((loop.pool.snapshot(), loop.pool.keys.clone(), loop.pool.values.clone(),
                    [s.current_len for s in loop.sessions]))
    (se, ke, ve, le), (sg, kg, vg, lg) = res
    assert le == lg and se == sg
    assert torch.equal(ke, kg) and torch.equal(ve, vg)
