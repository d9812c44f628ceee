"""The paged-pool oracle: reference slot semantics (golden trace) and page-level rules."""
import json
import os
import random

import pytest
import torch

from oracle.pool_spec import EINVAL, ENOPAGES, EOVERFLOW, PAGE, PagedKVPoolSpec, PoolError, page_hash


def test_reference_slot_trace(golden_dir):
    """Slot FIFO, exhaustion/overflow messages and write lengths of the reference KVPool."""
    tr = json.load(open(os.path.join(golden_dir, "kvpool_trace.json")))
    cfg = tr["config"]
    sp = PagedKVPoolSpec(num_pages=tr["max_slots"] * cfg["max_seq_len"] // PAGE,
                         max_seqs=tr["max_slots"], max_pages_per_seq=cfg["max_seq_len"] // PAGE)
    ev = {e["op"]: e for e in tr["events"]}
    slots = [sp.open_seq() for _ in range(4)]
    assert slots == ev["allocate x4"]["slots"]
    with pytest.raises(PoolError) as ei:
        sp.open_seq()
    assert str(ei.value) == ev["allocate (exhausted)"]["error"]
    sp.close_seq(slots[1])
    sp.close_seq(slots[3])
    assert [sp.open_seq(), sp.open_seq()] == ev["release 1,3 then allocate x2"]["slots"]
    lens = []
    for n in (8, 4, 4, 4, 4):
        sp.reserve([slots[0]], [n])
        lens.append(sp.seq_len[slots[0]])
    assert lens == ev["write 8,4,4,4,4 to slot 0"]["returned"]
    with pytest.raises(PoolError) as ei:
        sp.reserve([slots[0]], [cfg["max_seq_len"]])
    assert ei.value.code == EOVERFLOW
    assert str(ei.value) == ev["write max_seq_len more (overflow)"]["error"]
    assert sp.seq_len[slots[0]] == ev["write max_seq_len more (overflow)"]["current_len_after"]


def test_reserve_order_and_all_or_nothing():
    sp = PagedKVPoolSpec(num_pages=8, max_seqs=4, max_pages_per_seq=8)
    a, b, c = sp.open_seq(), sp.open_seq(), sp.open_seq()
    assert sp.reserve([a, b], [20, 40]) == [0, 0]
    assert sp.block_table[a][:2] == [0, 1] and sp.block_table[b][:3] == [2, 3, 4]
    assert sp.reserve([a], [12]) == [20]            # fills page 1, no new page
    assert sp.block_table[a][:3] == [0, 1, -1]
    before = sp.snapshot()
    with pytest.raises(PoolError) as ei:
        sp.reserve([c, a], [32, 40])                  # needs 2 + 3 > 3 free
    assert ei.value.code == ENOPAGES
    assert sp.snapshot() == before


def test_fork_shares_full_pages_and_copies_partial():
    sp = PagedKVPoolSpec(num_pages=16, max_seqs=4, max_pages_per_seq=8, num_layers=1,
                         num_kv_heads=1, head_dim=8, dtype=torch.float32, with_data=True)
    s = sp.open_seq()
    k = torch.arange(40 * 8, dtype=torch.float32).view(1, 40, 1, 8)
    sp.append([s], [k], [k + 0.5])
    d1, d2 = sp.open_seq(), sp.open_seq()
    sp.fork(s, [d1, d2], 37)                          # 2 full pages shared, 5 rows copied
    assert sp.block_table[d1][:2] == sp.block_table[s][:2] == sp.block_table[d2][:2]
    assert sp.refcount[sp.block_table[s][0]] == 3
    assert sp.block_table[d1][2] == 3 and sp.block_table[d2][2] == 4
    kd, vd = sp.session_kv(d2, 0)
    ks, vs = sp.session_kv(s, 0)
    assert torch.equal(kd, ks[:, :37]) and torch.equal(vd, vs[:, :37])


def test_free_first_occurrence_order():
    sp = PagedKVPoolSpec(num_pages=10, max_seqs=4, max_pages_per_seq=8)
    s = sp.open_seq()
    sp.reserve([s], [48])                             # pages 0,1,2
    d = sp.open_seq()
    sp.fork(s, [d], 32)                               # shares 0,1
    sp.reserve([d], [20])                             # 16 + 4 more tokens -> pages 3,4
    sp.free([d, s])
    # d's pages in order: 0(shared),1(shared),3,4 ; s: 0,1,2
    # zero after batch: all; first occurrences: 0,1,3,4 (from d), then 2 (from s)
    assert sp.free_queue == [5, 6, 7, 8, 9, 0, 1, 3, 4, 2]


def _check_invariants(sp):
    used = {}
    for s in range(sp.max_seqs):
        for p in sp.pages_of(s):
            used[p] = used.get(p, 0) + 1
    for p in sp.registry.values():
        used[p] = used.get(p, 0) + 1
    for p in range(sp.num_pages):
        assert sp.refcount[p] == used.get(p, 0)
    assert len(set(sp.free_queue)) == len(sp.free_queue)
    assert set(sp.free_queue) == {p for p in range(sp.num_pages) if sp.refcount[p] == 0}


def test_random_sequences_keep_invariants():
    rng = random.Random(0)
    sp = PagedKVPoolSpec(num_pages=64, max_seqs=8, max_pages_per_seq=16)
    live = []
    for _ in range(400):
        op = rng.random()
        try:
            if op < 0.25 and sp.free_seqs:
                live.append(sp.open_seq())
            elif op < 0.55 and live:
                k = rng.sample(live, rng.randint(1, len(live)))
                sp.reserve(k, [rng.randint(0, 40) for _ in k])
            elif op < 0.7 and live and sp.free_seqs:
                src = rng.choice(live)
                dst = sp.open_seq()
                live.append(dst)
                sp.fork(src, [dst], rng.randint(0, sp.seq_len[src]))
            elif live:
                k = rng.sample(live, rng.randint(1, len(live)))
                for s in k:
                    live.remove(s)
                    sp.close_seq(s)
        except PoolError:
            pass
        _check_invariants(sp)


def test_prefix_hash_dedup():
    sp = PagedKVPoolSpec(num_pages=32, max_seqs=4, max_pages_per_seq=8)
    toks = list(range(100, 150))                      # 3 full pages + 2 tokens
    a = sp.open_seq()
    sp.reserve([a], [len(toks)])
    assert sp.register(a, toks) == 3
    b = sp.open_seq()
    covered = sp.dedup(b, toks[:40] + [7] * 20)       # 2 pages match, 3rd differs
    assert covered == 32
    assert sp.block_table[b][:2] == sp.block_table[a][:2]
    assert page_hash(0, toks[:16]) == sp.hashes(toks)[0]
    assert sp.hashes(toks)[1] == page_hash(sp.hashes(toks)[0], toks[16:32])
    _check_invariants(sp)
    sp.close_seq(a)
    sp.close_seq(b)
    sp.unregister_all()
    assert sorted(sp.free_queue) == list(range(32))


def test_dedup_registry_capacity_and_order():
    """Registry limit is capacity // 2 (all or nothing); unregister frees in page order."""
    sp = PagedKVPoolSpec(num_pages=16, max_seqs=3, max_pages_per_seq=8, registry_capacity=8)
    a = sp.open_seq()
    sp.reserve([a], [80])                             # 5 pages: more than the limit of 4
    toks = list(range(80))
    before = sp.snapshot()
    with pytest.raises(PoolError) as e:
        sp.register(a, toks)
    assert e.value.code == ENOPAGES and sp.snapshot() == before and not sp.registry
    sp.close_seq(a)
    a = sp.open_seq()
    sp.reserve([a], [64])                             # pages popped after the 5 freed
    assert sp.register(a, toks) == 4
    b, c = sp.open_seq(), sp.open_seq()
    assert sp.dedup_many([b, c], [toks[:64], toks[:20] + [9] * 40]) == [64, 16]
    with pytest.raises(PoolError):
        sp.dedup_many([b], [toks])                    # not empty
    sp.close_seq(a)
    sp.close_seq(b)
    sp.close_seq(c)
    q0 = len(sp.free_queue)
    sp.unregister_all()
    tail = sp.free_queue[q0:]
    assert tail == sorted(tail) and len(tail) == 4
    _check_invariants(sp)


def test_reserve_rejects_a_repeated_session_without_side_effects():
    sp = PagedKVPoolSpec(num_pages=16, max_seqs=4, max_pages_per_seq=8)
    a, b = sp.open_seq(), sp.open_seq()
    sp.reserve([a], [20])
    before = sp.snapshot()
    for seqs, counts in (([a, b, a], [1, 2, 3]), ([b, b], [16, 16])):
        try:
            sp.reserve(seqs, counts)
            raise AssertionError("a repeated session must be rejected")
        except PoolError as e:
            assert e.code == EINVAL
        assert sp.snapshot() == before
    # the first offending entry in call order decides: an overflow before the repeat wins
    try:
        sp.reserve([b, a, a], [8 * 16 + 1, 1, 1])
    except PoolError as e:
        assert e.code == EOVERFLOW
    # zero-count entries (padding rows) may repeat, unless their session also grows
    assert sp.reserve([b, a, b, b], [0, 3, 0, 0]) == [0, 20, 0, 0]
    for seqs, counts in (([a, b, a], [0, 1, 2]), ([a, b, a], [2, 1, 0])):
        try:
            sp.reserve(seqs, counts)
            raise AssertionError("a growing session must appear once")
        except PoolError as e:
            assert e.code == EINVAL
