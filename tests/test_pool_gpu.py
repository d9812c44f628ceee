"""Device paged pool vs the pool oracle: bit-exact metadata after every operation.

Also re-runs the reference's KVPool unit tests (tests/test_runtime.py of the
reference) and its golden trace against the device pool.
"""
import json
import os
import random

import pytest
import torch

from oracle.pool_spec import PagedKVPoolSpec, PoolError
from loopfuse_b200.runtime.kv_pool import KVPool, KVState

pytestmark = pytest.mark.gpu

GPT2_KV = {"num_layers": 12, "num_heads": 12, "head_dim": 64, "max_seq_len": 1024, "dtype": "fp16"}


def _same(pool, spec):
    snap = pool.snapshot()
    want = spec.snapshot()
    assert snap["status"] == 0
    assert snap["free_queue"] == want["free_queue"]
    assert snap["refcount"] == want["refcount"]
    assert snap["block_table"] == want["block_table"]
    assert snap["seq_len"] == want["seq_len"]


def test_random_operation_sequences_bitexact():
    rng = random.Random(1)
    L, H, D = 2, 2, 64
    pool = KVPool(num_layers=L, num_heads=H, head_dim=D, max_seq_len=16 * 12, max_slots=6,
                  dtype=torch.bfloat16, num_pages=40)
    spec = PagedKVPoolSpec(num_pages=40, max_seqs=6, max_pages_per_seq=12, num_layers=L,
                           num_kv_heads=H, head_dim=D, dtype=torch.bfloat16, with_data=True)
    states = {}
    gen = torch.Generator().manual_seed(0)
    for step in range(150):
        op = rng.random()
        live = list(states)
        try:
            if op < 0.2 and pool._free_slots:
                s = pool.allocate_slot()
                assert spec.open_seq() == s.slot_id
                states[s.slot_id] = s
            elif op < 0.55 and live:
                pick = rng.sample(live, rng.randint(1, len(live)))
                counts = [rng.randint(0, 37) for _ in pick]
                if any(states[p].current_len + c > pool.max_seq_len for p, c in zip(pick, counts)):
                    continue
                ks = [torch.randn(L, c, H, D, generator=gen).bfloat16() for c in counts]
                vs = [torch.randn(L, c, H, D, generator=gen).bfloat16() for c in counts]
                try:
                    spec.append(pick, ks, vs)
                except PoolError:
                    with pytest.raises(RuntimeError, match="exhausted"):
                        pool.append([states[p] for p in pick], [k.cuda() for k in ks],
                                    [v.cuda() for v in vs])
                    continue
                pool.append([states[p] for p in pick], [k.cuda() for k in ks], [v.cuda() for v in vs])
            elif op < 0.7 and live and pool._free_slots:
                src = states[rng.choice(live)]
                plen = rng.randint(0, src.current_len)
                dst_id = spec.free_seqs[0]
                try:
                    spec.open_seq()
                    spec.fork(src.slot_id, [dst_id], plen)
                except PoolError:
                    spec.free_seqs.insert(0, dst_id)
                    with pytest.raises(RuntimeError, match="exhausted"):
                        pool.fork(src, plen)
                    assert pool._free_slots[0] == dst_id
                    continue
                d = pool.fork(src, plen)[0]
                assert d.slot_id == dst_id
                states[d.slot_id] = d
            elif live:
                pick = rng.sample(live, rng.randint(1, len(live)))
                for p in pick:
                    spec.close_seq(p)
                pool.release_all([states.pop(p) for p in pick])
        finally:
            _same(pool, spec)
        for sid, st in states.items():
            if st.current_len:
                k, v = pool.read(st, layer=1)
                ks, vs = spec.session_kv(sid, 1)
                assert torch.equal(k.cpu(), ks) and torch.equal(v.cpu(), vs)


def test_reference_runtime_tests_on_device_pool():
    """The reference's TestKVPool (tests/test_runtime.py:13-97) against the device pool."""
    pool = KVPool.from_config(GPT2_KV, device="cuda", max_slots=4)
    assert (pool.num_layers, pool.num_heads, pool.head_dim, pool.max_seq_len) == (12, 12, 64, 1024)
    s0 = pool.allocate_slot()
    assert isinstance(s0, KVState) and s0.slot_id == 0 and s0.current_len == 0
    s1 = pool.allocate_slot()
    assert s0.slot_id != s1.slot_id
    pool.allocate_slot(), pool.allocate_slot()
    with pytest.raises(RuntimeError, match="exhausted"):
        pool.allocate_slot()
    pool.release(s1)
    assert pool.allocate_slot() is not None
    nl, nh, hd = 12, 12, 64
    st = s0
    k = torch.zeros(nl, nh, 8, hd, dtype=torch.float16, device="cuda")
    assert pool.write(st, k, torch.zeros_like(k)) == 8 and st.current_len == 8
    for _ in range(4):
        k = torch.zeros(nl, nh, 4, hd, dtype=torch.float16, device="cuda")
        pool.write(st, k, torch.zeros_like(k))
    assert st.current_len == 24
    k = torch.zeros(nl, nh, 1025, hd, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="overflow"):
        pool.write(st, k, torch.zeros_like(k))
    pool.release(st)
    st = pool.allocate_slot()
    k_in = torch.randn(nl, nh, 16, hd, dtype=torch.float16, device="cuda")
    v_in = torch.randn_like(k_in)
    pool.write(st, k_in, v_in)
    k_out, v_out = pool.read(st, layer=0)
    assert k_out.shape == (nh, 16, hd) and torch.equal(k_out, k_in[0]) and torch.equal(v_out, v_in[0])
    ka, va = pool.read_all_layers(st)
    assert ka.shape == (nl, nh, 16, hd) and torch.equal(ka, k_in)
    kr, _ = pool.read(st, layer=3, seq_start=4, seq_end=12)
    assert torch.equal(kr, k_in[3, :, 4:12])
    assert pool.hbm_usage_bytes() > 0
    assert {"hbm_mb", "active_slots", "free_slots", "writes"} <= set(pool.stats())
    assert st.step_id == 0
    st.advance_step()
    assert st.step_id == 1


def test_reference_trace_replay(golden_dir):
    tr = json.load(open(os.path.join(golden_dir, "kvpool_trace.json")))
    ev = {e["op"]: e for e in tr["events"]}
    pool = KVPool.from_config(tr["config"], device="cuda", max_slots=tr["max_slots"])
    st = [pool.allocate_slot() for _ in range(4)]
    assert [s.slot_id for s in st] == ev["allocate x4"]["slots"]
    with pytest.raises(RuntimeError) as ei:
        pool.allocate_slot()
    assert str(ei.value) == ev["allocate (exhausted)"]["error"]
    pool.release(st[1])
    pool.release(st[3])
    assert [pool.allocate_slot().slot_id, pool.allocate_slot().slot_id] == \
        ev["release 1,3 then allocate x2"]["slots"]
    nl, nh, hd = 12, 12, 64
    lens = []
    for n in (8, 4, 4, 4, 4):
        k = torch.zeros(nl, nh, n, hd, dtype=torch.float16, device="cuda")
        lens.append(pool.write(st[0], k, torch.zeros_like(k)))
    assert lens == ev["write 8,4,4,4,4 to slot 0"]["returned"]
    with pytest.raises(RuntimeError) as ei:
        k = torch.zeros(nl, nh, 1024, hd, dtype=torch.float16, device="cuda")
        pool.write(st[0], k, torch.zeros_like(k))
    assert str(ei.value) == ev["write max_seq_len more (overflow)"]["error"]
    s = pool.stats()
    assert (s["active_slots"], s["free_slots"], s["writes"]) == (4, 0, 5)


def test_oversubscribed_pool_reports_exhaustion_without_side_effects():
    pool = KVPool(num_layers=1, num_heads=1, head_dim=64, max_seq_len=256, max_slots=4,
                  dtype=torch.bfloat16, num_pages=5)
    a, b = pool.allocate_slot(), pool.allocate_slot()
    k = torch.randn(1, 1, 64, 64, dtype=torch.bfloat16, device="cuda")
    pool.write(a, k, k)                                # 4 pages
    before = pool.snapshot()
    with pytest.raises(RuntimeError, match="exhausted"):
        pool.write(b, torch.cat([k, k], 2), torch.cat([k, k], 2))
    after = pool.snapshot()
    assert after == before


def _raw_meta_args(pool):
    return pool._meta_ref(), torch.cuda.current_stream().cuda_stream


def test_reserve_with_a_repeated_session_is_rejected_like_the_spec():
    """The host API refuses a repeated session; the device kernel, called directly, reports
    LF_EINVAL through the sticky status and changes nothing -- the spec's answer."""
    from loopfuse_b200 import _lib
    from loopfuse_b200._lib import LoopfuseError
    pool = KVPool(num_layers=1, num_heads=2, head_dim=64, max_seq_len=128, max_slots=3,
                  dtype=torch.bfloat16, num_pages=16)
    spec = PagedKVPoolSpec(num_pages=16, max_seqs=3, max_pages_per_seq=8)
    a, b = pool.alloc(), pool.alloc()
    spec.open_seq(), spec.open_seq()
    pool.reserve([a], [20])
    spec.reserve([a.slot_id], [20])
    _same(pool, spec)
    with pytest.raises(LoopfuseError):
        pool.reserve([a, b, a], [1, 1, 1])
    ids = torch.tensor([b.slot_id, a.slot_id, b.slot_id], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([16, 16, 16], dtype=torch.int32, device="cuda")
    start = torch.empty(3, dtype=torch.int32, device="cuda")
    meta, st = _raw_meta_args(pool)
    assert _lib.lib().lf_pool_reserve(meta, ids.data_ptr(), cnt.data_ptr(), 3, start.data_ptr(),
                                      st) == _lib.LF_OK
    with pytest.raises(PoolError) as e:
        spec.reserve([b.slot_id, a.slot_id, b.slot_id], [16, 16, 16])
    assert pool.status() == e.value.code == _lib.LF_EINVAL
    _lib.call("lf_pool_clear_status", meta, st)
    _same(pool, spec)
    # zero-count rows (a fixed-size batch's padding) may repeat a session that does not grow
    assert pool.reserve([b, a, b, b], [0, 5, 0, 0]).tolist() == \
        spec.reserve([b.slot_id, a.slot_id, b.slot_id, b.slot_id], [0, 5, 0, 0])
    _same(pool, spec)


def test_write_to_a_position_without_a_page_sets_the_status_and_stores_nothing():
    """A K/V row whose position has no reserved page (a stale start position) is skipped and
    reported (LF_EINVAL in the sticky status) instead of being stored through page id -1; the
    rows that do have pages are stored."""
    from loopfuse_b200 import _lib
    L, H, D = 2, 2, 64
    pool = KVPool(num_layers=L, num_heads=H, head_dim=D, max_seq_len=64, max_slots=2,
                  dtype=torch.bfloat16, num_pages=8)
    a = pool.alloc()
    pool.reserve([a], [16])                       # one page
    keys_before = pool.keys.clone()
    kv = torch.randn(L, 20, H, D, device="cuda").bfloat16()
    ids = torch.tensor([a.slot_id], dtype=torch.int32, device="cuda")
    start = torch.tensor([0], dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, 20], dtype=torch.int32, device="cuda")      # rows 16..19 have no page
    meta, st = _raw_meta_args(pool)
    rc = _lib.lib().lf_pool_write_kv(meta, ids.data_ptr(), start.data_ptr(), cu.data_ptr(), 1, 20,
                                     kv.data_ptr(), kv.data_ptr(), kv.stride(0), kv.stride(1),
                                     kv.stride(2), pool.keys.data_ptr(), pool.values.data_ptr(), L,
                                     H, D, st)
    assert rc == _lib.LF_OK
    assert pool.status() == _lib.LF_EINVAL
    page = pool.snapshot()["block_table"][a.slot_id][0]
    for l in range(L):
        assert torch.equal(pool.keys[l, page].permute(1, 0, 2), kv[l, :16])
    other = [p for p in range(pool.num_pages) if p != page]
    assert torch.equal(pool.keys[:, other], keys_before[:, other])
    _lib.call("lf_pool_clear_status", meta, st)
    # a stale start position past the session's pages is skipped the same way
    start.fill_(40)
    cu[1] = 4
    rc = _lib.lib().lf_pool_write_kv(meta, ids.data_ptr(), start.data_ptr(), cu.data_ptr(), 1, 4,
                                     kv.data_ptr(), kv.data_ptr(), kv.stride(0), kv.stride(1),
                                     kv.stride(2), pool.keys.data_ptr(), pool.values.data_ptr(), L,
                                     H, D, st)
    assert rc == _lib.LF_OK and pool.status() == _lib.LF_EINVAL
    assert torch.equal(pool.keys[:, other], keys_before[:, other])
    _lib.call("lf_pool_clear_status", meta, st)
