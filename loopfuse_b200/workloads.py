"""Seeded synthetic workloads for the attention hot path (bench and tests).

The reference measures on HotpotQA agent traces, which are not available
here; these generators build inputs with the shapes, sizes and value
distributions of the named workloads instead:

* ``prefill_inputs``: causal GQA prefill, Q ``[B,Hq,S,D]``, K/V ``[B,Hkv,S,D]``,
  i.i.d. N(0,1) bf16.  Default: B=8, Hq=32, Hkv=8, S=4096, D=128.
* ``decode_inputs``: paged decode over a shared prefix.  N sessions with context
  lengths uniform in [lmin, lmax]; the first ``prefix_tokens`` tokens are one
  set of pages shared by every session; each session's remaining pages are a
  slice of a random permutation of a pool sized to 1.1x the page demand; K/V
  and q i.i.d. N(0,1) bf16.  Default: N=256, Hq=32, Hkv=8, D=128,
  L ~ U[1024, 32768], 2048-token prefix, 16-token pages.

``decode_bytes`` / ``prefill_flops`` give the algorithmic work the roofline
numbers divide by.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch

PAGE = 16


@dataclass
class DecodeWorkload:
    q: torch.Tensor             # [N, Hq, D]
    k_pages: torch.Tensor       # [P, Hkv, 16, D]
    v_pages: torch.Tensor
    block_table: torch.Tensor   # [N, max_pages] int32, -1 padded
    seq_lens: torch.Tensor      # [N] int32
    n_prefix_pages: int
    lengths: List[int]
    prefix_pages: List[int]

    @property
    def num_seqs(self) -> int:
        return self.q.shape[0]


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def prefill_inputs(B: int = 8, Hq: int = 32, Hkv: int = 8, S: int = 4096, D: int = 128,
                   seed: int = 0, device="cuda", Sk: Optional[int] = None):
    g = _gen(seed, device)
    Sk = S if Sk is None else Sk
    q = torch.randn((B, Hq, S, D), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn((B, Hkv, Sk, D), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((B, Hkv, Sk, D), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    return q, k, v


def prefill_flops(B: int, Hq: int, S: int, D: int, Sk: Optional[int] = None, causal: bool = True) -> float:
    """Algorithmic FLOPs: 4*D per visible (query, key) pair; causal S(S+1)/2 pairs per head."""
    Sk = S if Sk is None else Sk
    if causal:
        off = Sk - S
        pairs = sum(min(Sk, i + 1 + off) for i in range(S)) if S <= 65536 else S * (S + 1) / 2
    else:
        pairs = S * Sk
    return 4.0 * B * Hq * D * pairs


def decode_lengths(n: int, lmin: int, lmax: int, seed: int) -> List[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lmin, lmax + 1, (n,), generator=g).tolist()


def decode_inputs(N: int = 256, Hq: int = 32, Hkv: int = 8, D: int = 128, lmin: int = 1024,
                  lmax: int = 32768, prefix_tokens: int = 2048, seed: int = 0, device="cuda",
                  lengths: Optional[List[int]] = None, pool_factor: float = 1.1,
                  table_seed: Optional[int] = None) -> DecodeWorkload:
    """``seed`` draws the lengths (unless given), the page permutation (unless ``table_seed``
    is given: then the block table is that seed's, shared by every caller using it) and the
    q / K / V values."""
    lengths = lengths if lengths is not None else decode_lengths(N, lmin, lmax, seed)
    n_pre = prefix_tokens // PAGE
    own = [max(0, math.ceil(L / PAGE) - n_pre) for L in lengths]
    P = math.ceil(pool_factor * (n_pre + sum(own)))
    gcpu = torch.Generator().manual_seed((seed if table_seed is None else table_seed) + 1)
    perm = torch.randperm(P, generator=gcpu).tolist()
    prefix = perm[:n_pre]
    max_pages = max(math.ceil(L / PAGE) for L in lengths)
    table = torch.full((N, max_pages), -1, dtype=torch.int32)
    cur = n_pre
    for i, L in enumerate(lengths):
        npg = math.ceil(L / PAGE)
        row = prefix[:min(npg, n_pre)] + perm[cur:cur + own[i]]
        cur += own[i]
        table[i, :len(row)] = torch.tensor(row, dtype=torch.int32)
    g = _gen(seed + 2, device)
    k_pages = torch.empty((P, Hkv, PAGE, D), dtype=torch.bfloat16, device=device)
    v_pages = torch.empty_like(k_pages)
    chunk = max(1, (1 << 28) // (Hkv * PAGE * D))      # <= 256M elements per fill
    for t in (k_pages, v_pages):
        for s in range(0, P, chunk):
            e = min(P, s + chunk)
            t[s:e] = torch.randn((e - s, Hkv, PAGE, D), generator=g, device=device,
                                 dtype=torch.float32).to(torch.bfloat16)
    q = torch.randn((N, Hq, D), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    return DecodeWorkload(q, k_pages, v_pages, table.to(device),
                          torch.tensor(lengths, dtype=torch.int32, device=device),
                          n_pre if prefix_tokens else 0, lengths, prefix)


def decode_bytes(w: DecodeWorkload, shared_prefix: bool = True) -> dict:
    """Algorithmic HBM bytes of one decode step.

    ``unique``: every K/V page touched, counted once (the shared prefix once),
    plus q, o, the block-table entries read and the lengths.  ``logical``: the
    prefix counted once per session that reads it (what a kernel without
    prefix sharing must move).
    """
    N, Hq, D = w.q.shape
    return decode_bytes_from_lengths(w.lengths, Hq, w.k_pages.shape[1], D, w.n_prefix_pages,
                                     w.k_pages.element_size())


def decode_bytes_from_lengths(lengths: List[int], Hq: int, Hkv: int, D: int, n_pre: int,
                              elem: int = 2) -> dict:
    """``decode_bytes`` from the session lengths alone (no device tensors needed)."""
    N = len(lengths)
    page_bytes = 2 * Hkv * PAGE * D * elem                            # K + V, all heads
    pages_own = sum(max(0, math.ceil(L / PAGE) - n_pre) for L in lengths)
    pages_pre_used = max((min(math.ceil(L / PAGE), n_pre) for L in lengths), default=0)
    pages_logical = sum(math.ceil(L / PAGE) for L in lengths)
    small = 2 * N * Hq * D * 2 + 4 * N + 4 * pages_logical
    return {"unique": (pages_pre_used + pages_own) * page_bytes + small,
            "logical": pages_logical * page_bytes + small,
            "suffix_kv": pages_own * page_bytes,
            "page_bytes": page_bytes,
            "pool_pages": math.ceil(1.1 * (n_pre + pages_own))}
