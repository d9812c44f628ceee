"""fp32 CPU restatement of the reference's attention semantics (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Every function computes in float32 on the CPU and returns float32 results.
Shapes follow the reference: prefill tensors are ``[batch, heads, seq, dim]``
(``kernels/triton/prefill_attn.py:136-143``); decode queries are one token per
session.  Grouped-query attention maps query head ``hq`` to KV head
``hq // (Hq // Hkv)``, which is what ``scaled_dot_product_attention(...,
enable_gqa=True)`` does.

Softmax scale defaults to ``head_dim ** -0.5`` (``prefill_attn.py:150``,
``decode_attn.py:344``).  The log-sum-exp returned next to an output is the
natural log of ``sum_j exp(scale * q.k_j)`` over the unmasked keys, the
convention the split-KV combine uses.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

PAGE_SIZE = 16


def _expand_kv(k: torch.Tensor, hq: int) -> torch.Tensor:
    """Repeat KV heads so head ``hq`` sees KV head ``hq // group``."""
    hkv = k.shape[-3]
    if hq == hkv:
        return k
    assert hq % hkv == 0, f"Hq={hq} not a multiple of Hkv={hkv}"
    return k.repeat_interleave(hq // hkv, dim=-3)


def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
            scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Causal (or full) attention of ``q [B,Hq,Sq,D]`` over ``k,v [B,Hkv,Sk,D]``.

    Restates ``_prefill_attn_kernel`` (``kernels/triton/prefill_attn.py:35-124``):
    scores ``q.k * scale``, mask, softmax, ``p @ v``.  The reference masks
    ``q_idx >= k_idx`` with ``Sq == Sk`` (``:97-99``); when ``Sq < Sk`` (new
    tokens appended after a cached prefix) the mask is aligned bottom-right,
    query ``i`` sitting at key position ``Sk - Sq + i``, which reduces to the
    reference's mask when ``Sq == Sk``.

    Returns ``(o, lse)``: ``o [B,Hq,Sq,D]`` fp32 and ``lse [B,Hq,Sq]`` fp32.
    Rows with no visible key (only possible when ``Sq > Sk``) get ``o = 0``
    and ``lse = -inf``.
    """
    qf, kf, vf = q.float(), k.float(), v.float()
    B, Hq, Sq, D = qf.shape
    Sk = kf.shape[2]
    if scale is None:
        scale = D ** -0.5
    kf = _expand_kv(kf, Hq)
    vf = _expand_kv(vf, Hq)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    if causal:
        qi = torch.arange(Sq).view(Sq, 1) + (Sk - Sq)
        kj = torch.arange(Sk).view(1, Sk)
        s = s.masked_fill(kj > qi, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse.unsqueeze(-1))
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.matmul(p, vf)
    return o, lse


def sdpa_eager(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               causal: bool = True) -> torch.Tensor:
    """The reference's EAGER kernel choice, run in fp32.

    ``PHASE_KERNEL_MAP[(EAGER, *)]`` names ``torch.nn.functional.
    scaled_dot_product_attention`` (``passes/phase_select.py:80-89``) and the
    reference checks its prefill kernel against it in fp32
    (``kernels/triton/prefill_attn.py:180-182``).  ``enable_gqa`` extends it to
    grouped-query heads.
    """
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                          is_causal=causal, enable_gqa=True)


def reference_decode_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Restates the reference's decode check ``_reference_decode_attn``.

    ``kernels/triton/decode_attn.py:178-184``: scores in the input dtype,
    softmax in fp32, probabilities cast back to the input dtype, then
    ``p @ v`` in the input dtype.  Kept to pin the oracle against the
    reference's own definition on its MHA fp16 shapes.
    """
    scale = q.shape[-1] ** -0.5
    attn = torch.matmul(q, k.transpose(-2, -1)) * scale
    attn = F.softmax(attn.float(), dim=-1).to(q.dtype)
    return torch.matmul(attn, v)


def gather_pages(pool: torch.Tensor, pages, length: int) -> torch.Tensor:
    """Contiguous ``[Hkv, length, D]`` view of one session's paged K or V.

    ``pool`` is ``[P, Hkv, PAGE_SIZE, D]``; ``pages`` lists the session's page
    ids in token order (its block-table row).
    """
    n = (length + PAGE_SIZE - 1) // PAGE_SIZE
    idx = torch.as_tensor(list(pages[:n]), dtype=torch.long)
    g = pool.index_select(0, idx)                     # [n, Hkv, 16, D]
    g = g.permute(1, 0, 2, 3).reshape(pool.shape[1], n * PAGE_SIZE, pool.shape[3])
    return g[:, :length]


def decode_paged(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                 block_table: torch.Tensor, seq_lens, scale: Optional[float] = None
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """One-token attention per session over paged K/V.

    ``q [N,Hq,D]``; ``k_pool, v_pool [P,Hkv,16,D]``; ``block_table [N,max_pages]``
    int32; ``seq_lens [N]``.  Restates ``_decode_attn_kernel``
    (``kernels/triton/decode_attn.py:57-130``) after gathering each session's
    pages into contiguous ``[Hkv, L, D]`` -- the reference's decode reads a
    contiguous cache (``:95-123``) and has no paging of its own.

    Returns ``(o [N,Hq,D], lse [N,Hq])`` in fp32.
    """
    N, Hq, D = q.shape
    if scale is None:
        scale = D ** -0.5
    bt = block_table.tolist()
    lens = [int(x) for x in (seq_lens.tolist() if torch.is_tensor(seq_lens) else seq_lens)]
    outs, lses = [], []
    for i in range(N):
        L = lens[i]
        kf = gather_pages(k_pool, bt[i], L).float()   # [Hkv, L, D]
        vf = gather_pages(v_pool, bt[i], L).float()
        kf = _expand_kv(kf, Hq)
        vf = _expand_kv(vf, Hq)
        qf = q[i].float().unsqueeze(1)                 # [Hq, 1, D]
        s = torch.matmul(qf, kf.transpose(-1, -2)).squeeze(1) * scale   # [Hq, L]
        lse = torch.logsumexp(s, dim=-1)
        p = torch.exp(s - lse.unsqueeze(-1))
        outs.append(torch.einsum("hl,hld->hd", p, vf))
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def decode_paged_sdpa(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      block_table: torch.Tensor, seq_lens) -> torch.Tensor:
    """Decode through the reference's EAGER path: gather, then fp32 SDPA.

    This is the CPU torch path timed as the baseline: the reference selects
    ``scaled_dot_product_attention`` for EAGER decode (``passes/
    phase_select.py:85-89``); pages are gathered through the block table first.
    """
    N, Hq, D = q.shape
    bt = block_table.tolist()
    lens = [int(x) for x in (seq_lens.tolist() if torch.is_tensor(seq_lens) else seq_lens)]
    outs = []
    for i in range(N):
        kf = gather_pages(k_pool, bt[i], lens[i]).float().unsqueeze(0)
        vf = gather_pages(v_pool, bt[i], lens[i]).float().unsqueeze(0)
        outs.append(sdpa_eager(q[i].float().view(1, Hq, 1, D), kf, vf, causal=False)[0, :, 0])
    return torch.stack(outs)


def merge_partials(o_parts, lse_parts):
    """Combine attention over disjoint key sets from ``(o_i, lse_i)`` pairs.

    ``o = sum_i exp(lse_i - lse) o_i`` with ``lse = logsumexp_i lse_i``: the
    split-KV / shared-prefix merge, restated for tests.
    """
    lse = torch.logsumexp(torch.stack(lse_parts), dim=0)
    o = sum(torch.exp(l - lse).unsqueeze(-1) * o for o, l in zip(o_parts, lse_parts))
    return o, lse


def attention_flops_causal(B: int, Hq: int, S: int, D: int) -> float:
    """Algorithmic FLOPs of causal prefill: ``4 * B * Hq * D * S(S+1)/2``."""
    return 4.0 * B * Hq * D * S * (S + 1) / 2.0


def log2e() -> float:
    return 1.0 / math.log(2.0)
