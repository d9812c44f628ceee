"""Device prefix-hash dedup (register / dedup / unregister) vs the pool oracle, bit for bit.

Every step is mirrored in ``PagedKVPoolSpec`` and the full device metadata (free queue from
its head, refcounts, block tables, lengths) is compared after it.  Page hashes computed on the
device must equal the oracle's ``page_hash`` chain.
"""
import ctypes
import random

import pytest
import torch

from oracle.pool_spec import MAX_DEDUP_PAGES, PAGE, PagedKVPoolSpec, PoolError
from loopfuse_b200 import _lib
from loopfuse_b200.runtime.kv_pool import KVPool, prefix_hashes

pytestmark = pytest.mark.gpu


def _as_u64(x: int) -> int:
    return x & ((1 << 64) - 1)


def _pair(num_pages=64, slots=6, max_len=512, layers=2, hkv=2, d=64):
    pool = KVPool(num_layers=layers, num_heads=hkv, num_kv_heads=hkv, head_dim=d,
                  max_seq_len=max_len, max_slots=slots, dtype=torch.bfloat16,
                  num_pages=num_pages)
    cap = 1 << max(10, (2 * num_pages - 1).bit_length())
    spec = PagedKVPoolSpec(num_pages=num_pages, max_seqs=slots,
                           max_pages_per_seq=pool.max_pages_per_seq, registry_capacity=cap)
    return pool, spec


def _same(pool, spec):
    got, want = pool.snapshot(), spec.snapshot()
    for key in ("free_queue", "refcount", "block_table", "seq_len"):
        assert got[key] == want[key], key
    assert got["status"] == 0


@pytest.mark.parametrize("n_tokens", [0, 15, 16, 100, 16 * 300 + 7, 16 * MAX_DEDUP_PAGES + 40])
def test_device_hashes_match_oracle(n_tokens):
    rng = random.Random(n_tokens)
    toks = [rng.randint(-2**31, 2**31 - 1) for _ in range(n_tokens)]
    got = prefix_hashes(torch.tensor(toks, dtype=torch.int32, device="cuda")).cpu().tolist()
    want = PagedKVPoolSpec(1, 1, 1).hashes(toks)
    assert [_as_u64(x) for x in got] == want


def test_register_dedup_unregister_bit_exact():
    pool, spec = _pair()
    rng = random.Random(3)
    toks = [rng.randint(0, 50000) for _ in range(100)]          # 6 full pages + 4 tokens
    a = pool.alloc()
    assert spec.open_seq() == a.slot_id
    start = pool.reserve([a], [100])
    spec.reserve([a.slot_id], [100])
    k = torch.randn(100, 2, 64, device="cuda").bfloat16()
    pool.write_layer([a], start, 0, k, k + 1, [100])
    assert pool.register_prefix(a, toks) == spec.register(a.slot_id, toks) == 6
    _same(pool, spec)
    assert pool.register_prefix(a, toks) == spec.register(a.slot_id, toks) == 0     # idempotent
    _same(pool, spec)
    b, c, d = pool.alloc(), pool.alloc(), pool.alloc()
    ids = [spec.open_seq() for _ in range(3)]
    assert ids == [b.slot_id, c.slot_id, d.slot_id]
    streams = [toks, toks[:40] + [7] * 30, [1] * 64]
    got = pool.dedup_prefix([b, c, d], streams)
    want = spec.dedup_many(ids, streams)
    assert got == want == [96, 32, 0]
    assert [b.current_len, c.current_len, d.current_len] == want
    _same(pool, spec)
    # the shared pages hold the registered session's K/V
    kb, _ = pool.read(b, 0)
    ka, _ = pool.read(a, 0)
    assert torch.equal(kb, ka[:, :96])
    # appends after a dedup go to fresh pages (the shared ones are full)
    pool.reserve([b, c], [20, 5])
    spec.reserve([b.slot_id, c.slot_id], [20, 5])
    _same(pool, spec)
    # a non-empty destination fails on the device and changes nothing
    e = pool.alloc()
    spec.open_seq()
    with pytest.raises(_lib.LoopfuseError):
        pool.dedup_prefix([e, b], [toks, toks])
    with pytest.raises(PoolError):
        spec.dedup_many([e.slot_id, b.slot_id], [toks, toks])
    _same(pool, spec)
    # free everything, then drop the registry: its pages come back in page order
    everyone = [a, b, c, d, e]
    pool.release_all(everyone)
    spec.free([s.slot_id for s in everyone])
    spec.free_seqs.extend(s.slot_id for s in everyone)
    _same(pool, spec)
    pool.unregister_all()
    spec.unregister_all()
    _same(pool, spec)
    assert sorted(pool.snapshot()["free_queue"]) == list(range(pool.num_pages))


def test_many_sessions_share_a_registered_prompt():
    pool, spec = _pair(num_pages=256, slots=34, max_len=1024)
    rng = random.Random(9)
    prompt = [rng.randint(0, 1000) for _ in range(512 + 9)]
    root = pool.alloc()
    spec.open_seq()
    pool.reserve([root], [len(prompt)])
    spec.reserve([root.slot_id], [len(prompt)])
    assert pool.register_prefix(root, prompt) == spec.register(root.slot_id, prompt) == 32
    sess = [pool.alloc() for _ in range(33)]
    ids = [spec.open_seq() for _ in range(33)]
    streams = [prompt[:rng.randint(0, len(prompt))] + [rng.randint(0, 1000)] * 17 for _ in ids]
    assert pool.dedup_prefix(sess, streams) == spec.dedup_many(ids, streams)
    _same(pool, spec)
    table, lens = pool.block_table(sess)
    assert lens.tolist() == [spec.seq_len[i] for i in ids]


def test_registry_full_is_all_or_nothing():
    """Through the C ABI with a 4-entry registry (limit 2 entries)."""
    pool, _ = _pair()
    keys = torch.zeros(4, dtype=torch.int64, device="cuda")
    pages = torch.empty(4, dtype=torch.int32, device="cuda")
    used = torch.zeros(1, dtype=torch.int32, device="cuda")
    reg = _lib.PrefixRegistry(keys.data_ptr(), pages.data_ptr(), used.data_ptr(), 4)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("lf_registry_init", ctypes.byref(reg), st)
    a = pool.alloc()
    pool.reserve([a], [48])
    toks = torch.arange(48, dtype=torch.int32, device="cuda")
    before = pool.snapshot()
    _lib.call("lf_pool_register_prefix", pool._meta_ref(), ctypes.byref(reg), a.slot_id,
              toks.data_ptr(), 48, None, st)
    assert pool.status() == _lib.LF_ENOPAGES
    pool._call("lf_pool_clear_status", pool._meta_ref(), st)
    after = pool.snapshot()
    assert after["refcount"] == before["refcount"] and int(used.item()) == 0
    assert int((keys != 0).sum().item()) == 0
    _lib.call("lf_pool_register_prefix", pool._meta_ref(), ctypes.byref(reg), a.slot_id,
              toks.data_ptr(), 32, None, st)
    assert pool.status() == 0 and int(used.item()) == 2


def test_bad_registry_capacity_rejected_on_host():
    pool, _ = _pair()
    t = torch.zeros(8, dtype=torch.int64, device="cuda")
    reg = _lib.PrefixRegistry(t.data_ptr(), t.data_ptr(), t.data_ptr(), 6)
    with pytest.raises(_lib.LoopfuseError):
        _lib.call("lf_registry_init", ctypes.byref(reg), 0)
