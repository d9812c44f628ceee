"""Deterministic Python specification of the paged, refcounted KV pool.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  The device pool in
``loopfuse_b200`` must reproduce every state this spec reaches, bit for bit:
free-queue contents and order, refcounts, block tables and sequence lengths,
and the K/V bytes each session sees.

What is kept from the reference (``runtime/kv_pool.py``)
--------------------------------------------------------
* Session slots are handed out first-in first-out from ``range(max_slots)``
  and returned to the back on release (``allocate_slot`` ``:103-115``,
  ``release`` ``:117-121``).
* ``write`` appends at ``current_len`` and returns the new length
  (``:123-149``); more than ``max_seq_len`` tokens raises ``RuntimeError``
  with "KV cache overflow" (``:135-139``); no free slot raises "KVPool
  exhausted" (``:105-109``).

What the reference does not have and is specified here
------------------------------------------------------
The reference pool is one dense ``[max_seq_len]`` strip per slot: no pages,
no sharing.  Pages are ``PAGE`` (16) tokens.  Free pages sit in a FIFO queue,
initially ``0, 1, ..., P-1``.

``reserve(seqs, n_new)``  (the allocation step of ``append``)
    For each session, in the order given, ``need = ceil((len + n)/16) -
    ceil(len/16)`` pages are popped from the queue head and appended to its
    block table with refcount 1; ``len += n``.  All or nothing: if the total
    need exceeds the free count (ENOPAGES) or any session would pass
    ``max_pages_per_seq`` pages (EOVERFLOW), nothing changes.  Counts must be
    non-negative and a session that grows must appear once: an entry is
    EINVAL when an earlier entry names the same session and either of the two
    counts is non-zero (zero-count entries, e.g. padding rows, may repeat).
    The first offending entry in call order decides between EINVAL and
    EOVERFLOW.
``fork(src, dsts, prefix_len)``
    Each destination (empty) gets the source's first ``prefix_len // 16`` page
    ids (shared; refcount += 1 per destination).  If ``prefix_len % 16`` is
    not zero, each destination, in order, pops one page from the queue and
    receives a copy of the first ``prefix_len % 16`` token rows of the source's
    partial page (copy-on-write at fork time, so appends never write a shared
    page).  ``len = prefix_len``.  All or nothing on ENOPAGES.
``free(seqs)``
    Every (session, page) occurrence, sessions in the order given and pages
    in block-table order, decrements the page's refcount once.  A page whose
    refcount is zero after the whole batch is pushed to the queue tail once,
    at the position of its first occurrence in that order.  Block-table rows
    are reset to -1 and lengths to 0.
``gather(seqs)``
    Block-table rows and lengths of the given sessions, in order (the batch
    block table a decode launch reads).
``dedup(seq, tokens)``  (prefix-hash KV fusion)
    Full pages are identified by a chained 64-bit hash of their token ids
    (``page_hash``).  ``register`` records, for each full page of a session,
    hash -> page (first writer wins; the registry holds one reference, so a
    registered page is not freed until ``unregister_all``).  The registry
    holds at most ``registry_capacity // 2`` entries: a ``register`` that
    would pass that adds nothing (ENOPAGES).  ``dedup`` maps the longest run
    of leading full pages of a new (empty) session whose hashes are
    registered onto those pages (refcount += 1) and returns the number of
    tokens it covered; ``dedup_many`` does that for a batch of distinct empty
    sessions (all or nothing on EINVAL).  ``unregister_all`` drops the
    registry's references; pages reaching zero re-enter the queue tail in
    ascending page-id order.  Both consider at most ``MAX_DEDUP_PAGES`` pages
    of a session.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

PAGE = 16

OK = 0
EINVAL = 1
ENOPAGES = 2
EOVERFLOW = 3

MAX_DEDUP_PAGES = 4096

_MASK64 = (1 << 64) - 1
_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x100000001B3
_MIX_A = 0xFF51AFD7ED558CCD
_MIX_B = 0xC4CEB9FE1A85EC53


def _fmix64(h: int) -> int:
    """64-bit finaliser (the MurmurHash3 ``fmix64`` avalanche step)."""
    h ^= h >> 33
    h = (h * _MIX_A) & _MASK64
    h ^= h >> 33
    h = (h * _MIX_B) & _MASK64
    h ^= h >> 33
    return h


def page_local_hash(tokens: Sequence[int]) -> int:
    """FNV-1a (64-bit) over the little-endian bytes of one page's 32-bit token ids."""
    h = _FNV_OFFSET
    for t in tokens:
        for b in int(t & 0xFFFFFFFF).to_bytes(4, "little"):
            h = ((h ^ b) * _FNV_PRIME) & _MASK64
    return h


def page_hash(prev: int, tokens: Sequence[int]) -> int:
    """Chained hash of one full page: ``fmix64(prev ^ page_local_hash(tokens))``.

    The first page of a session chains from ``prev = 0``, so a page's hash covers every token
    before it.  The per-page FNV part has no dependence on ``prev`` (the device computes it for
    all pages in parallel); only the cheap ``fmix64`` step is serial.  0 marks an empty
    registry slot, so a hash of 0 becomes 1.
    """
    h = _fmix64((prev ^ page_local_hash(tokens)) & _MASK64)
    return h if h != 0 else 1


class PoolError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class PagedKVPoolSpec:
    """Host model of the device pool (metadata plus optional K/V contents)."""

    def __init__(self, num_pages: int, max_seqs: int, max_pages_per_seq: int,
                 num_layers: int = 0, num_kv_heads: int = 0, head_dim: int = 0,
                 dtype: torch.dtype = torch.bfloat16, with_data: bool = False,
                 registry_capacity: int = 4096):
        self.num_pages = num_pages
        self.registry_capacity = registry_capacity
        self.max_seqs = max_seqs
        self.max_pages_per_seq = max_pages_per_seq
        self.free_queue: List[int] = list(range(num_pages))
        self.refcount = [0] * num_pages
        self.block_table = [[-1] * max_pages_per_seq for _ in range(max_seqs)]
        self.seq_len = [0] * max_seqs
        self.free_seqs: List[int] = list(range(max_seqs))
        self.registry: Dict[int, int] = {}
        self.with_data = with_data
        if with_data:
            shape = (num_layers, num_pages, num_kv_heads, PAGE, head_dim)
            self.k = torch.zeros(shape, dtype=dtype)
            self.v = torch.zeros(shape, dtype=dtype)

    # -- session slots (reference FIFO semantics) -------------------------
    def open_seq(self) -> int:
        if not self.free_seqs:
            raise PoolError(ENOPAGES, f"KVPool exhausted: all {self.max_seqs} slots in use. "
                                      f"Increase max_slots or wait for a trajectory to complete.")
        return self.free_seqs.pop(0)

    def close_seq(self, seq: int) -> None:
        self.free([seq])
        self.free_seqs.append(seq)

    # -- helpers ----------------------------------------------------------
    @staticmethod
    def pages_for(n_tokens: int) -> int:
        return (n_tokens + PAGE - 1) // PAGE

    def pages_of(self, seq: int) -> List[int]:
        return self.block_table[seq][: self.pages_for(self.seq_len[seq])]

    # -- reserve ----------------------------------------------------------
    def reserve(self, seqs: Sequence[int], n_new: Sequence[int]) -> List[int]:
        """Returns each session's start position; raises PoolError on failure."""
        needs = []
        grows = {}                                  # session -> an earlier entry adds tokens
        for s, n in zip(seqs, n_new):
            if n < 0 or (s in grows and (n != 0 or grows[s])):
                raise PoolError(EINVAL, "negative token count or repeated growing session")
            grows[s] = grows.get(s, False) or n != 0
            old = self.pages_for(self.seq_len[s])
            new = self.pages_for(self.seq_len[s] + n)
            if new > self.max_pages_per_seq:
                raise PoolError(EOVERFLOW, f"KV cache overflow: current_len={self.seq_len[s]} + "
                                           f"seq_new={n} > max_seq_len="
                                           f"{self.max_pages_per_seq * PAGE}")
            needs.append(new - old)
        if sum(needs) > len(self.free_queue):
            raise PoolError(ENOPAGES, f"KVPool exhausted: need {sum(needs)} pages, "
                                      f"{len(self.free_queue)} free")
        starts = []
        for s, n, need in zip(seqs, n_new, needs):
            old = self.pages_for(self.seq_len[s])
            for j in range(need):
                p = self.free_queue.pop(0)
                self.refcount[p] = 1
                self.block_table[s][old + j] = p
            starts.append(self.seq_len[s])
            self.seq_len[s] += n
        return starts

    def write(self, seqs: Sequence[int], starts: Sequence[int], k_new: List[torch.Tensor],
              v_new: List[torch.Tensor]) -> None:
        """Store ``k_new[i]`` (``[L, n_i, Hkv, D]``) at session ``seqs[i]`` from ``starts[i]``."""
        assert self.with_data
        for s, st, kn, vn in zip(seqs, starts, k_new, v_new):
            for t in range(kn.shape[1]):
                pos = st + t
                page = self.block_table[s][pos // PAGE]
                self.k[:, page, :, pos % PAGE] = kn[:, t]
                self.v[:, page, :, pos % PAGE] = vn[:, t]

    def append(self, seqs, k_new, v_new) -> List[int]:
        starts = self.reserve(seqs, [kn.shape[1] for kn in k_new])
        if self.with_data:
            self.write(seqs, starts, k_new, v_new)
        return starts

    # -- fork -------------------------------------------------------------
    def fork(self, src: int, dsts: Sequence[int], prefix_len: int) -> None:
        if prefix_len > self.seq_len[src] or prefix_len < 0:
            raise PoolError(EINVAL, "fork prefix longer than the source")
        for d in dsts:
            if self.seq_len[d] != 0:
                raise PoolError(EINVAL, "fork destination is not empty")
        full, part = divmod(prefix_len, PAGE)
        if part and len(dsts) > len(self.free_queue):
            raise PoolError(ENOPAGES, f"KVPool exhausted: need {len(dsts)} pages, "
                                      f"{len(self.free_queue)} free")
        src_pages = self.block_table[src]
        for d in dsts:
            for j in range(full):
                p = src_pages[j]
                self.block_table[d][j] = p
                self.refcount[p] += 1
            if part:
                p = self.free_queue.pop(0)
                self.refcount[p] = 1
                self.block_table[d][full] = p
                if self.with_data:
                    sp = src_pages[full]
                    self.k[:, p, :, :part] = self.k[:, sp, :, :part]
                    self.v[:, p, :, :part] = self.v[:, sp, :, :part]
            self.seq_len[d] = prefix_len

    # -- free -------------------------------------------------------------
    def free(self, seqs: Sequence[int]) -> None:
        occ = []
        for s in seqs:
            for p in self.pages_of(s):
                occ.append(p)
                self.refcount[p] -= 1
        seen = set()
        for p in occ:
            if p in seen:
                continue
            seen.add(p)
            if self.refcount[p] == 0:
                self.free_queue.append(p)
        for s in seqs:
            self.block_table[s] = [-1] * self.max_pages_per_seq
            self.seq_len[s] = 0

    # -- gather -----------------------------------------------------------
    def gather(self, seqs: Sequence[int]):
        return [list(self.block_table[s]) for s in seqs], [self.seq_len[s] for s in seqs]

    # -- prefix-hash dedup ------------------------------------------------
    def hashes(self, tokens: Sequence[int]) -> List[int]:
        out, h = [], 0
        for j in range(min(len(tokens) // PAGE, MAX_DEDUP_PAGES)):
            h = page_hash(h, tokens[j * PAGE:(j + 1) * PAGE])
            out.append(h)
        return out

    def register(self, seq: int, tokens: Sequence[int]) -> int:
        """Record hash -> page for the session's full pages; returns pages added."""
        if not 0 <= seq < self.max_seqs:
            raise PoolError(EINVAL, f"register: bad session {seq}")
        hs = self.hashes(tokens[: self.seq_len[seq]])[: self.max_pages_per_seq]
        new = [j for j, h in enumerate(hs) if h not in self.registry]
        if len(self.registry) + len(new) > self.registry_capacity // 2:
            raise PoolError(ENOPAGES, "prefix registry full")
        for j in new:
            p = self.block_table[seq][j]
            self.registry[hs[j]] = p
            self.refcount[p] += 1
        return len(new)

    def dedup(self, seq: int, tokens: Sequence[int]) -> int:
        """Share the longest registered run of leading full pages; returns tokens covered."""
        return self.dedup_many([seq], [tokens])[0]

    def dedup_many(self, seqs: Sequence[int], tokens: Sequence[Sequence[int]]) -> List[int]:
        if len(set(seqs)) != len(seqs) or any(
                not 0 <= s < self.max_seqs or self.seq_len[s] != 0 for s in seqs):
            raise PoolError(EINVAL, "dedup destination is not empty")
        out = []
        for seq, toks in zip(seqs, tokens):
            n = 0
            for j, h in enumerate(self.hashes(toks)):
                if j >= self.max_pages_per_seq or h not in self.registry:
                    break
                p = self.registry[h]
                self.block_table[seq][j] = p
                self.refcount[p] += 1
                n += 1
            self.seq_len[seq] = n * PAGE
            out.append(n * PAGE)
        return out

    def unregister_all(self) -> None:
        """Drop the registry's references (pages reaching zero return to the queue in
        ascending page-id order)."""
        freed = []
        for h, p in self.registry.items():
            self.refcount[p] -= 1
            if self.refcount[p] == 0:
                freed.append(p)
        self.free_queue.extend(sorted(freed))
        self.registry.clear()

    # -- snapshot ---------------------------------------------------------
    def snapshot(self) -> dict:
        return {
            "free_queue": list(self.free_queue),
            "refcount": list(self.refcount),
            "block_table": [list(r) for r in self.block_table],
            "seq_len": list(self.seq_len),
        }

    def session_kv(self, seq: int, layer: int):
        """Contiguous ``[Hkv, len, D]`` K and V of one session (data mode)."""
        pages = self.pages_of(seq)
        L = self.seq_len[seq]
        idx = torch.as_tensor(pages, dtype=torch.long)
        k = self.k[layer].index_select(0, idx).permute(1, 0, 2, 3).reshape(
            self.k.shape[2], -1, self.k.shape[4])[:, :L]
        v = self.v[layer].index_select(0, idx).permute(1, 0, 2, 3).reshape(
            self.v.shape[2], -1, self.v.shape[4])[:, :L]
        return k, v
