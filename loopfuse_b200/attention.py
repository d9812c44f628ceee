"""PyTorch-facing attention ops over the sm_100a C ABI.

Tensors must be CUDA, bf16 and contiguous; the ops launch on
``torch.cuda.current_stream()`` and return without synchronising.  There is no
CPU or eager fallback: a missing library, a wrong device or dtype raises.

* ``prefill_attention_fwd(q, k, v, causal)`` -- drop-in for the reference's
  ``kernels/triton/prefill_attn.py:127-168`` (``[B,H,S,D]`` layout), extended to
  grouped-query heads (``k, v`` may have fewer heads) and to ``Sq < Sk``
  (queries appended after a cached prefix, bottom-right causal mask).
* ``paged_decode(q, k_pages, v_pages, block_table, seq_lens, ...)`` -- split-KV
  decode over a paged pool, optional shared prefix.
* ``decode_attention_fwd(q, k, v)`` -- drop-in for
  ``kernels/triton/decode_attn.py:133-171`` (contiguous ``[B,H,S,D]`` cache):
  the cache is laid out as pages and handed to ``paged_decode``.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import LF_PAGE_SIZE, LoopfuseError

SM_COUNT = 148          # B200; the split heuristic uses the current device's count when it can


def _sm_count() -> int:
    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return SM_COUNT


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require(t: torch.Tensor, name: str, dtype=torch.bfloat16) -> None:
    if not t.is_cuda:
        raise LoopfuseError(_lib.LF_EINVAL, f"{name} must be a CUDA tensor (no CPU path)")
    if t.dtype != dtype:
        raise LoopfuseError(_lib.LF_EINVAL, f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise LoopfuseError(_lib.LF_EINVAL, f"{name} must be contiguous")


def prefill_attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                          scale: Optional[float] = None, return_lse: bool = False):
    """Causal GQA attention: ``q [B,Hq,Sq,D]``, ``k, v [B,Hkv,Sk,D]`` -> ``o [B,Hq,Sq,D]``, D 64 or 128."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _require(t, n)
    B, Hq, Sq, D = q.shape
    Bk, Hkv, Sk, Dk = k.shape
    if Bk != B or Dk != D or v.shape != k.shape:
        raise LoopfuseError(_lib.LF_EINVAL, f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} "
                                            f"v{tuple(v.shape)}")
    scale = D ** -0.5 if scale is None else float(scale)
    o = torch.empty_like(q)
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device) if return_lse else None
    _lib.call("lf_prefill_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
              lse.data_ptr() if lse is not None else None, B, Hq, Hkv, Sq, Sk, D, scale,
              int(bool(causal)), _stream())
    return (o, lse) if return_lse else o


def prefill_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                  block_table: torch.Tensor, cu_seqlens_q: torch.Tensor, seqlens_k: torch.Tensor,
                  max_seqlen_q: int, causal: bool = True, scale: Optional[float] = None,
                  return_lse: bool = False, out: Optional[torch.Tensor] = None):
    """Attention of newly appended tokens over each session's cached paged K/V.

    ``q [T, Hq, D]``: the new tokens of N sessions back to back, session ``n`` owning rows
    ``cu_seqlens_q[n] .. cu_seqlens_q[n+1]``; ``k_pages, v_pages [P, Hkv, 16, D]`` (one layer,
    new tokens already appended); ``block_table [N, max_pages]``; ``seqlens_k [N]`` context
    lengths including the new tokens.  Causal with the queries at the end of their session.
    Returns ``o [T, Hq, D]`` (and ``lse [T, Hq]``); ``out``, when given, is a contiguous
    ``[T, Hq, D]`` bf16 tensor that receives ``o``.
    """
    for t, n in ((q, "q"), (k_pages, "k_pages"), (v_pages, "v_pages")):
        _require(t, n)
    for t, n in ((block_table, "block_table"), (cu_seqlens_q, "cu_seqlens_q"),
                 (seqlens_k, "seqlens_k")):
        _require(t, n, torch.int32)
    T, Hq, D = q.shape
    P, Hkv, page, Dk = k_pages.shape
    N = block_table.shape[0]
    if page != LF_PAGE_SIZE or Dk != D or cu_seqlens_q.shape != (N + 1,) or seqlens_k.shape != (N,):
        raise LoopfuseError(_lib.LF_EINVAL, "prefill_paged: inconsistent shapes")
    scale = D ** -0.5 if scale is None else float(scale)
    if out is None:
        o = torch.empty_like(q)
    else:
        _require(out, "out")
        if out.shape != q.shape:
            raise LoopfuseError(_lib.LF_EINVAL, "prefill_paged: out must have q's shape")
        o = out
    lse = torch.empty((T, Hq), dtype=torch.float32, device=q.device) if return_lse else None
    _lib.call("lf_prefill_paged_fwd", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
              block_table.data_ptr(), cu_seqlens_q.data_ptr(), seqlens_k.data_ptr(), o.data_ptr(),
              lse.data_ptr() if lse is not None else None, N, T, int(max_seqlen_q), Hq, Hkv, D, P,
              block_table.shape[1], scale, int(bool(causal)), _stream())
    return (o, lse) if return_lse else o


def default_pages_per_split(num_seqs: int, num_kv_heads: int, max_pages: int,
                            num_prefix_pages: int = 0) -> int:
    """Split size for the sessions' own pages (the shared prefix is read separately): enough
    CTAs for several waves on the device's SMs, 32 to 128 pages each.  ``max_pages`` is the
    block-table width, each session's capacity; sessions are taken to be half full on average.
    The floor of 32 keeps small batches from launching many short or empty splits: the grid is
    sized for the table's capacity, and three split CTAs fit on an SM at a time.  The formula
    lives in the library (``lf_decode_default_split``), shared with the no-allocation decode."""
    out = _lib.c_int(0)
    _lib.call("lf_decode_default_split", int(num_seqs), int(num_kv_heads), int(max_pages),
              int(num_prefix_pages), _sm_count(), _lib.ctypes.byref(out))
    return int(out.value)


def decode_workspace_bytes(num_seqs: int, num_q_heads: int, head_dim: int, max_pages: int,
                           pages_per_split: int, num_prefix_pages: int = 0) -> int:
    n = _lib.c_size_t(0)
    _lib.call("lf_decode_workspace_size", num_seqs, num_q_heads, head_dim, max_pages,
              pages_per_split, num_prefix_pages, _lib.ctypes.byref(n))
    return int(n.value)


def paged_decode(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                 block_table: torch.Tensor, seq_lens: torch.Tensor, num_prefix_pages: int = 0,
                 scale: Optional[float] = None, pages_per_split: Optional[int] = None,
                 out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
                 return_lse: bool = False, k_new: Optional[torch.Tensor] = None,
                 v_new: Optional[torch.Tensor] = None):
    """One-token attention per session over paged K/V.

    ``q [N,Hq,D]``; ``k_pages, v_pages [P,Hkv,16,D]`` (one layer of the pool);
    ``block_table [N,max_pages]`` int32; ``seq_lens [N]`` int32.  With
    ``num_prefix_pages > 0`` the first that many block-table entries must be the
    same pages for all sessions; they are then read once per group of sessions.

    ``k_new, v_new [N,Hkv,D]`` (both or neither): each session's newest token, at position
    ``seq_lens[i] - 1`` in a page already reserved in ``block_table`` past the shared-prefix
    pages, is stored into ``k_pages`` / ``v_pages`` by the decode itself before it is attended
    (``lf_decode_fwd_append``): the pages end up as a separate ``KVPool.write_layer`` would leave
    them, one kernel launch fewer.
    """
    _require(q, "q")
    _require(k_pages, "k_pages")
    _require(v_pages, "v_pages")
    _require(block_table, "block_table", torch.int32)
    _require(seq_lens, "seq_lens", torch.int32)
    N, Hq, D = q.shape
    P, Hkv, page, Dk = k_pages.shape
    if page != LF_PAGE_SIZE or Dk != D or v_pages.shape != k_pages.shape:
        raise LoopfuseError(_lib.LF_EINVAL, f"pages must be [P,Hkv,{LF_PAGE_SIZE},{D}]")
    if block_table.dim() != 2 or block_table.shape[0] != N or seq_lens.shape != (N,):
        raise LoopfuseError(_lib.LF_EINVAL, "block_table must be [N,max_pages], seq_lens [N]")
    max_pages = block_table.shape[1]
    pps = pages_per_split or default_pages_per_split(N, Hkv, max_pages, num_prefix_pages)
    scale = D ** -0.5 if scale is None else float(scale)
    need = decode_workspace_bytes(N, Hq, D, max_pages, pps, num_prefix_pages)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    o = out if out is not None else torch.empty_like(q)
    lse = torch.empty((N, Hq), dtype=torch.float32, device=q.device) if return_lse else None
    if (k_new is None) != (v_new is None):
        raise LoopfuseError(_lib.LF_EINVAL, "paged_decode: give both k_new and v_new, or neither")
    if k_new is not None:
        for t, n in ((k_new, "k_new"), (v_new, "v_new")):
            _require(t, n)
            if tuple(t.shape) != (N, Hkv, D):
                raise LoopfuseError(_lib.LF_EINVAL, f"{n} must be [N,Hkv,D] = {(N, Hkv, D)}")
        _lib.call("lf_decode_fwd_append", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
                  block_table.data_ptr(), seq_lens.data_ptr(), int(num_prefix_pages),
                  k_new.data_ptr(), v_new.data_ptr(), o.data_ptr(),
                  lse.data_ptr() if lse is not None else None, workspace.data_ptr(),
                  workspace.numel() * workspace.element_size(), N, Hq, Hkv, D, P, max_pages, pps,
                  scale, _stream())
        return (o, lse) if return_lse else o
    _lib.call("lf_decode_fwd", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
              block_table.data_ptr(), seq_lens.data_ptr(), int(num_prefix_pages), o.data_ptr(),
              lse.data_ptr() if lse is not None else None, workspace.data_ptr(),
              workspace.numel() * workspace.element_size(), N, Hq, Hkv, D, P, max_pages, pps,
              scale, _stream())
    return (o, lse) if return_lse else o


def contiguous_to_pages(k: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """``[B,H,S,D]`` cache -> pages ``[B*ceil(S/16), H, 16, D]`` and block table ``[B, S/16]``."""
    B, H, S, D = k.shape
    npg = math.ceil(S / LF_PAGE_SIZE)
    pad = npg * LF_PAGE_SIZE - S
    if pad:
        k = torch.nn.functional.pad(k, (0, 0, 0, pad))
    pages = k.view(B, H, npg, LF_PAGE_SIZE, D).permute(0, 2, 1, 3, 4).reshape(B * npg, H,
                                                                              LF_PAGE_SIZE, D)
    table = torch.arange(B * npg, dtype=torch.int32, device=k.device).view(B, npg)
    return pages.contiguous(), table


def decode_attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         scale: Optional[float] = None) -> torch.Tensor:
    """Reference-compatible decode: ``q [B,H,1,D]``, ``k, v [B,Hkv,S,D]`` -> ``[B,H,1,D]``."""
    if q.dim() != 4 or q.shape[2] != 1:
        raise LoopfuseError(_lib.LF_EINVAL, f"decode expects seq_q=1, got {tuple(q.shape)}")
    B, H, _, D = q.shape
    S = k.shape[2]
    kp, table = contiguous_to_pages(k)
    vp, _ = contiguous_to_pages(v)
    lens = torch.full((B,), S, dtype=torch.int32, device=q.device)
    o = paged_decode(q.reshape(B, H, D).contiguous(), kp, vp, table, lens, scale=scale)
    return o.view(B, H, 1, D)
