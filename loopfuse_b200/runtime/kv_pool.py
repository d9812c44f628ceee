"""Paged, refcounted KV pool in device memory -- drop-in for ``runtime/kv_pool.py``.

The reference pool (``runtime/kv_pool.py:28-235``) preallocates one dense
``[max_seq_len]`` strip per slot.  This pool keeps the same public API and
error behaviour but stores K/V in 16-token pages that sessions can share:

* ``allocate_slot`` / ``release`` / ``write`` / ``read`` / ``read_all_layers``
  / ``prefetch_next_slot`` / ``stats`` / ``hbm_usage_bytes`` / ``from_config``
  behave as in the reference: slots are FIFO (``:103-121``), ``write`` appends
  at ``current_len`` and returns the new length (``:123-149``), overflow and
  exhaustion raise ``RuntimeError`` with the reference's messages
  (``:105-109``, ``:135-139``), ``read`` returns ``[H, S, D]`` (a gathered
  copy, since pages are not contiguous).
* New paged API: ``alloc``, ``append`` (batched), ``fork`` (share a prefix by
  reference), ``free``, ``block_table`` (batch table for ``paged_decode``),
  ``layer_pages``, ``snapshot``, and content-addressed sharing:
  ``register_prefix`` / ``dedup_prefix`` / ``unregister_all`` (a device hash
  registry of full pages keyed by the chained hash of their token ids).

Every metadata operation (page allocation, fork, free, block-table gather,
prefix-hash register / dedup) is a device kernel from ``liblf_sm100.so`` launched on the pool's stream; no
CPU-side page bookkeeping exists.  K/V storage is ``[L, P, Hkv, 16, D]`` per
tensor: one layer's pages are ``[P, Hkv, 16, D]``, a page of one head 4 KB
contiguous at D = 128.

The pool lives on the GPU only: ``device`` must be CUDA.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch

from .. import _lib
from .._lib import LF_PAGE_SIZE, LoopfuseError, PoolMeta

_DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}


def prefix_hashes(tokens: torch.Tensor) -> torch.Tensor:
    """Chained 64-bit hashes (as int64) of the full 16-token pages of a CUDA int32 token
    vector, computed on the device: the keys ``KVPool.register_prefix`` / ``dedup_prefix``
    use.  At most ``LF_MAX_DEDUP_PAGES`` pages."""
    if tokens.device.type != "cuda" or tokens.dtype != torch.int32:
        raise LoopfuseError(_lib.LF_EINVAL, "prefix_hashes: tokens must be a CUDA int32 tensor")
    toks = tokens.reshape(-1).contiguous()
    n = min(toks.numel() // LF_PAGE_SIZE, _lib.LF_MAX_DEDUP_PAGES)
    out = torch.empty(n, dtype=torch.int64, device=toks.device)
    _lib.call("lf_prefix_hashes", toks.data_ptr(), toks.numel(), out.data_ptr(),
              torch.cuda.current_stream(toks.device).cuda_stream)
    return out


class KVState:
    """Handle to one session (trajectory) in the pool: ``slot_id`` is its block-table row."""

    def __init__(self, slot_id: int, pool: "KVPool"):
        self.slot_id = slot_id
        self.pool = pool
        self.current_len = 0
        self.step_id = 0

    @property
    def seq_id(self) -> int:
        return self.slot_id

    def advance_step(self) -> None:
        self.step_id += 1

    def __repr__(self):
        return f"KVState(slot={self.slot_id}, len={self.current_len}, step={self.step_id})"


class KVPool:
    def __init__(self, num_layers: int, num_heads: int, head_dim: int, max_seq_len: int,
                 max_slots: int = 8, dtype: torch.dtype = torch.float16, device: str = "cuda",
                 num_kv_heads: Optional[int] = None, num_pages: Optional[int] = None):
        dev = torch.device(device)
        if dev.type != "cuda":
            raise LoopfuseError(_lib.LF_EINVAL, "loopfuse_b200.KVPool keeps its pages and metadata "
                                                "in GPU memory; device must be CUDA")
        if dtype not in (torch.bfloat16, torch.float16):
            raise LoopfuseError(_lib.LF_EINVAL, f"pool dtype must be bf16 or fp16, got {dtype}")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads or num_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.max_slots = max_slots
        self.dtype = dtype
        self.device = dev
        self.page_size = LF_PAGE_SIZE
        self.max_pages_per_seq = math.ceil(max_seq_len / LF_PAGE_SIZE)
        self.num_pages = num_pages or max_slots * self.max_pages_per_seq

        shape = (num_layers, self.num_pages, self.num_kv_heads, LF_PAGE_SIZE, head_dim)
        self.keys = torch.zeros(shape, dtype=dtype, device=dev)
        self.values = torch.zeros(shape, dtype=dtype, device=dev)

        i32 = dict(dtype=torch.int32, device=dev)
        self._free_queue = torch.empty(self.num_pages, **i32)
        self._refcount = torch.empty(self.num_pages, **i32)
        self._table = torch.empty(max_slots * self.max_pages_per_seq, **i32)
        self._seq_len = torch.empty(max_slots, **i32)
        self._ctrl = torch.zeros(_lib.LF_CTRL_WORDS, **i32)
        self._scratch = torch.empty(self.num_pages, **i32)
        self._meta = PoolMeta(self._free_queue.data_ptr(), self._refcount.data_ptr(),
                              self._table.data_ptr(), self._seq_len.data_ptr(),
                              self._ctrl.data_ptr(), self._scratch.data_ptr(), self.num_pages,
                              max_slots, self.max_pages_per_seq, LF_PAGE_SIZE)
        # Same two-stream arrangement as the reference (kv_pool.py:76-81): compute stays hot,
        # background work (speculative prefill) goes to the low-priority stream.
        self.compute_stream = torch.cuda.Stream(device=dev, priority=0)
        self.prefetch_stream = torch.cuda.Stream(device=dev, priority=-1)
        self._oversubscribed = self.num_pages < max_slots * self.max_pages_per_seq

        self._free_slots: List[int] = list(range(max_slots))
        self._active: Dict[int, KVState] = {}
        self._write_count = 0
        self._bytes_written = 0
        self._reg: Optional[_lib.PrefixRegistry] = None
        with torch.cuda.device(dev):
            self._call("lf_pool_init", self._meta_ref(), self._stream())

    # -- construction --------------------------------------------------------
    @classmethod
    def from_config(cls, kv_config: dict, device: str = "cuda", max_slots: int = 8,
                    num_pages: Optional[int] = None) -> "KVPool":
        return cls(num_layers=kv_config["num_layers"], num_heads=kv_config["num_heads"],
                   head_dim=kv_config["head_dim"], max_seq_len=kv_config["max_seq_len"],
                   dtype=_DTYPES.get(kv_config.get("dtype", "fp16"), torch.float16),
                   device=device, max_slots=max_slots,
                   num_kv_heads=kv_config.get("num_kv_heads"), num_pages=num_pages)

    # -- plumbing -------------------------------------------------------------
    def _meta_ref(self):
        return _lib.ctypes.byref(self._meta)

    def _stream(self, stream: Optional[torch.cuda.Stream] = None) -> int:
        return (stream or torch.cuda.current_stream(self.device)).cuda_stream

    def _call(self, name: str, *args) -> None:
        _lib.call(name, *args)

    def _ids(self, xs: Sequence[int]) -> torch.Tensor:
        return torch.tensor(list(xs), dtype=torch.int32).to(self.device, non_blocking=True)

    def status(self) -> int:
        """Sticky device status (one host sync)."""
        return int(self._ctrl[_lib.LF_CTRL_STATUS].item())

    def _raise_if_failed(self, what: str, detail: str = "") -> None:
        st = self.status()
        if st == _lib.LF_OK:
            return
        self._call("lf_pool_clear_status", self._meta_ref(), self._stream())
        if st == _lib.LF_ENOPAGES:
            raise RuntimeError(f"KVPool exhausted: no free pages for {what} "
                               f"({self.num_pages} pages). {detail}".strip())
        if st == _lib.LF_EOVERFLOW:
            raise RuntimeError(f"KV cache overflow in {what}. {detail}".strip())
        raise LoopfuseError(st, f"pool {what} failed on the device. {detail}".strip())

    # -- reference API ----------------------------------------------------------
    def allocate_slot(self) -> KVState:
        """Start a trajectory: FIFO slot (reference ``kv_pool.py:103-115``)."""
        if not self._free_slots:
            raise RuntimeError(f"KVPool exhausted: all {self.max_slots} slots in use. "
                               f"Increase max_slots or wait for a trajectory to complete.")
        slot = self._free_slots.pop(0)
        state = KVState(slot, self)
        self._active[slot] = state
        return state

    def release(self, state: KVState) -> None:
        """End a trajectory: its pages are dereferenced on the device, the slot recycled."""
        if state.slot_id in self._active:
            self.free(state)
            del self._active[state.slot_id]
            self._free_slots.append(state.slot_id)

    def write(self, state: KVState, new_keys: torch.Tensor, new_values: torch.Tensor,
              stream: Optional[torch.cuda.Stream] = None) -> int:
        """Append ``[L, Hkv, S_new, D]`` keys/values at ``current_len``; returns the new length."""
        seq_new = new_keys.shape[2]
        if state.current_len + seq_new > self.max_seq_len:
            raise RuntimeError(f"KV cache overflow: current_len={state.current_len} + "
                               f"seq_new={seq_new} > max_seq_len={self.max_seq_len}")
        self.append([state], [new_keys], [new_values], layout="lhsd", stream=stream)
        return state.current_len

    def read(self, state: KVState, layer: int, seq_start: int = 0,
             seq_end: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Gathered copy of one layer's keys/values, ``[Hkv, seq_range, D]``."""
        seq_end = seq_end or state.current_len
        count = max(0, seq_end - seq_start)
        k = torch.empty((self.num_kv_heads, count, self.head_dim), dtype=self.dtype, device=self.device)
        v = torch.empty_like(k)
        self._call("lf_pool_read", self._meta_ref(), state.slot_id, layer, seq_start,
                   seq_start + count, self.keys.data_ptr(), self.values.data_ptr(), k.data_ptr(),
                   v.data_ptr(), self.num_layers, self.num_kv_heads, self.head_dim, self._stream())
        return k, v

    def read_all_layers(self, state: KVState, seq_start: int = 0,
                        seq_end: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        ks, vs = zip(*(self.read(state, l, seq_start, seq_end) for l in range(self.num_layers)))
        return torch.stack(ks), torch.stack(vs)

    def prefetch_next_slot(self, state: KVState) -> None:
        """Kept for the executor's speculative-prefill hook (reference ``:189-198``).

        The dense pool zeroed the next slot here.  Pages are never zeroed: a
        session only reads positions below its length, so there is nothing to do.
        """
        return None

    def hbm_usage_bytes(self) -> int:
        meta = sum(t.numel() * 4 for t in (self._free_queue, self._refcount, self._table,
                                            self._seq_len, self._ctrl, self._scratch))
        return (self.keys.numel() + self.values.numel()) * self.keys.element_size() + meta

    def stats(self) -> dict:
        ctrl = self._ctrl.tolist()
        return {
            "hbm_mb": round(self.hbm_usage_bytes() / 1e6, 1),
            "active_slots": len(self._active),
            "free_slots": len(self._free_slots),
            "writes": self._write_count,
            "mb_written": round(self._bytes_written / 1e6, 1),
            "pages_total": self.num_pages,
            "pages_free": ctrl[_lib.LF_CTRL_COUNT],
            "status": ctrl[_lib.LF_CTRL_STATUS],
        }

    def __repr__(self):
        return (f"KVPool(layers={self.num_layers}, heads={self.num_heads}/{self.num_kv_heads}, "
                f"dim={self.head_dim}, seq={self.max_seq_len}, slots={self.max_slots}, "
                f"pages={self.num_pages})")

    # -- paged API --------------------------------------------------------------
    def alloc(self, n_tokens: int = 0) -> KVState:
        """Open a session, optionally reserving pages for ``n_tokens`` (no data written)."""
        st = self.allocate_slot()
        if n_tokens:
            self._reserve([st], [n_tokens])
        return st

    def _reserve(self, states: Sequence[KVState], counts: Sequence[int],
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        for s, n in zip(states, counts):
            if s.current_len + n > self.max_seq_len:
                raise RuntimeError(f"KV cache overflow: current_len={s.current_len} + "
                                   f"seq_new={n} > max_seq_len={self.max_seq_len}")
        grows = {}
        for s, n in zip(states, counts):
            if s.slot_id in grows and (n != 0 or grows[s.slot_id]):
                raise LoopfuseError(_lib.LF_EINVAL, "reserve: a growing session appears twice "
                                                    "in one call")
            grows[s.slot_id] = grows.get(s.slot_id, False) or n != 0
        ids = self._ids([s.slot_id for s in states])
        cnt = self._ids(counts)
        start = torch.empty(len(states), dtype=torch.int32, device=self.device)
        self._call("lf_pool_reserve", self._meta_ref(), ids.data_ptr(), cnt.data_ptr(), len(states),
                   start.data_ptr(), self._stream(stream))
        if self._oversubscribed:
            self._raise_if_failed("reserve")
        for s, n in zip(states, counts):
            s.current_len += n
        return start

    def reserve(self, states: Sequence[KVState], counts: Sequence[int],
                stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Grow sessions by ``counts`` tokens (pages from the device queue); returns the device
        tensor of their old lengths, the write offsets for ``write_layer``."""
        return self._reserve(states, counts, stream)

    def batch_index(self, states: Sequence[KVState], counts: Sequence[int]
                    ) -> Tuple[torch.Tensor, torch.Tensor, int]:
        """Device (session ids, token offsets, total) of a batch, reusable across layers."""
        cu = [0]
        for c in counts:
            cu.append(cu[-1] + int(c))
        return self._ids([s.slot_id for s in states]), self._ids(cu), cu[-1]

    def write_layer(self, states: Sequence[KVState], start: torch.Tensor, layer: int,
                    keys: torch.Tensor, values: torch.Tensor, counts: Sequence[int],
                    stream: Optional[torch.cuda.Stream] = None, index=None) -> None:
        """Store one layer's new K/V (``[T_total, Hkv, D]``, sessions back to back with
        ``counts[i]`` tokens each) at the offsets a ``reserve`` returned.  A model forward
        reserves once and then writes each layer as soon as its K/V exist."""
        ids, cu_t, total = index if index is not None else self.batch_index(states, counts)
        if total == 0:
            return
        for t in (keys, values):
            if t.device != self.device or t.dtype != self.dtype or not t.is_contiguous() or \
                    tuple(t.shape) != (total, self.num_kv_heads, self.head_dim):
                raise LoopfuseError(_lib.LF_EINVAL, "write_layer expects contiguous "
                                                    "[T_total, Hkv, D] tensors of the pool dtype")
        elem = self.keys.element_size()
        layer_off = layer * self.keys.stride(0) * elem
        self._call("lf_pool_write_kv", self._meta_ref(), ids.data_ptr(), start.data_ptr(),
                   cu_t.data_ptr(), len(states), total, keys.data_ptr(), values.data_ptr(), 0,
                   keys.stride(0), keys.stride(1), self.keys.data_ptr() + layer_off,
                   self.values.data_ptr() + layer_off, 1, self.num_kv_heads, self.head_dim,
                   self._stream(stream))
        self._bytes_written += 2 * keys.numel() * elem

    def append(self, states: Sequence[KVState], keys: Sequence[torch.Tensor],
               values: Sequence[torch.Tensor], layout: str = "lthd",
               stream: Optional[torch.cuda.Stream] = None) -> None:
        """Append new tokens to several sessions in one reserve + one scatter.

        ``layout="lthd"``: each tensor is ``[L, T_i, Hkv, D]``; ``"lhsd"``: the
        reference's ``[L, Hkv, T_i, D]``.  Tensors of one call share strides.
        """
        if len(states) == 0:
            return
        tdim = 1 if layout == "lthd" else 2
        counts = [int(k.shape[tdim]) for k in keys]
        start = self._reserve(states, counts, stream)
        total = sum(counts)
        if total == 0:
            return
        if len(keys) == 1:
            k_all, v_all = keys[0], values[0]
        else:
            k_all = torch.cat(list(keys), dim=tdim)
            v_all = torch.cat(list(values), dim=tdim)
        for t in (k_all, v_all):
            if t.device != self.device or t.dtype != self.dtype or t.stride(-1) != 1:
                raise LoopfuseError(_lib.LF_EINVAL, "new K/V must be on the pool's device, in the "
                                                    "pool dtype, with contiguous head_dim")
        if v_all.stride() != k_all.stride():
            v_all = v_all.contiguous()
            k_all = k_all.contiguous()
        sl = k_all.stride(0)
        st_tok = k_all.stride(1) if layout == "lthd" else k_all.stride(2)
        st_head = k_all.stride(2) if layout == "lthd" else k_all.stride(1)
        cu = [0]
        for c in counts:
            cu.append(cu[-1] + c)
        ids = self._ids([s.slot_id for s in states])
        cu_t = self._ids(cu)
        self._call("lf_pool_write_kv", self._meta_ref(), ids.data_ptr(), start.data_ptr(),
                   cu_t.data_ptr(), len(states), total, k_all.data_ptr(), v_all.data_ptr(), sl,
                   st_tok, st_head, self.keys.data_ptr(), self.values.data_ptr(), self.num_layers,
                   self.num_kv_heads, self.head_dim, self._stream(stream))
        self._write_count += 1
        self._bytes_written += 2 * k_all.numel() * k_all.element_size()

    def fork(self, state: KVState, prefix_len: Optional[int] = None, n: int = 1) -> List[KVState]:
        """``n`` new sessions sharing ``state``'s first ``prefix_len`` tokens (KV fusion)."""
        prefix_len = state.current_len if prefix_len is None else prefix_len
        if prefix_len > state.current_len or prefix_len < 0:
            raise LoopfuseError(_lib.LF_EINVAL, f"fork prefix {prefix_len} > length "
                                                f"{state.current_len}")
        if len(self._free_slots) < n:
            raise RuntimeError(f"KVPool exhausted: all {self.max_slots} slots in use. "
                               f"Increase max_slots or wait for a trajectory to complete.")
        dsts = [self.allocate_slot() for _ in range(n)]
        ids = self._ids([d.slot_id for d in dsts])
        self._call("lf_pool_fork", self._meta_ref(), state.slot_id, ids.data_ptr(), n, prefix_len,
                   self.keys.data_ptr(), self.values.data_ptr(), self.num_layers,
                   self.num_kv_heads, self.head_dim, self._stream())
        if self._oversubscribed and prefix_len % LF_PAGE_SIZE:
            try:
                self._raise_if_failed("fork")
            except RuntimeError:
                # nothing changed on the device: hand the slots back, first in line again
                for d in dsts:
                    del self._active[d.slot_id]
                self._free_slots[0:0] = [d.slot_id for d in dsts]
                raise
        for d in dsts:
            d.current_len = prefix_len
        return dsts

    def free(self, states: Union[KVState, Sequence[KVState]]) -> None:
        """Drop the sessions' page references (slots stay allocated; see ``release``)."""
        states = [states] if isinstance(states, KVState) else list(states)
        if not states:
            return
        ids = self._ids([s.slot_id for s in states])
        self._call("lf_pool_free", self._meta_ref(), ids.data_ptr(), len(states), self._stream())
        for s in states:
            s.current_len = 0

    def adopt(self, keep: KVState, branch: KVState) -> None:
        """``keep`` takes over ``branch``'s block-table row (a speculative branch that turned
        out right): keep's own pages are dropped on the device, the handle is re-pointed at the
        branch's row and length, and keep's old row returns to the free slots at the tail, as
        ``release`` would return it.  ``branch`` is spent: use ``keep`` from now on."""
        if keep.slot_id not in self._active or branch.slot_id not in self._active or \
                keep.slot_id == branch.slot_id:
            raise LoopfuseError(_lib.LF_EINVAL, "adopt: both sessions must be open and distinct")
        self.free(keep)
        old = keep.slot_id
        del self._active[branch.slot_id]
        del self._active[old]
        keep.slot_id, keep.current_len = branch.slot_id, branch.current_len
        branch.current_len = 0
        self._active[keep.slot_id] = keep
        self._free_slots.append(old)

    def release_all(self, states: Sequence[KVState]) -> None:
        """Batched ``release``: one device free for all, slots back in the given order."""
        states = [s for s in states if s.slot_id in self._active]
        self.free(states)
        for s in states:
            del self._active[s.slot_id]
            self._free_slots.append(s.slot_id)

    # -- device-buffer forms (no host bookkeeping, no sync: usable inside CUDA-graph capture) --
    def reserve_device(self, slot_ids: torch.Tensor, counts: torch.Tensor, start: torch.Tensor,
                       n: int) -> None:
        """``lf_pool_reserve`` on device int32 buffers of ``n`` entries.  The caller keeps the
        host ``KVState.current_len`` in step and reads ``status()`` when it next syncs."""
        self._call("lf_pool_reserve", self._meta_ref(), slot_ids.data_ptr(), counts.data_ptr(), n,
                   start.data_ptr(), self._stream())

    def gather_device(self, slot_ids: torch.Tensor, n: int, table: torch.Tensor,
                      lens: torch.Tensor) -> None:
        """Block-table rows and lengths of ``n`` slots into ``table [n, W]`` / ``lens [n]``."""
        self._call("lf_pool_gather", self._meta_ref(), slot_ids.data_ptr(), n, table.data_ptr(),
                   table.shape[1], lens.data_ptr(), self._stream())

    def pad_session(self, root: Optional[KVState] = None, prefix_len: int = 0) -> KVState:
        """A session for the padding rows of fixed-size batches: it shares ``root``'s first
        ``prefix_len`` tokens (when given) and has a free row in its last page, so a batch row
        that appends 0 tokens can write its K/V at position ``current_len`` harmlessly."""
        st = self.fork(root, prefix_len, n=1)[0] if root is not None else self.alloc()
        self.reserve([st], [1 if st.current_len % LF_PAGE_SIZE == 0 else 0])
        return st

    def write_qkv(self, states: Sequence[KVState], start: torch.Tensor, layer: int,
                  qkv: torch.Tensor, q_out: torch.Tensor, counts: Sequence[int],
                  rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                  stream: Optional[torch.cuda.Stream] = None, index=None) -> None:
        """Fused QKV epilogue of one layer: ``qkv [T_total, (Hq + 2 Hkv) * D]`` (q heads, then
        k heads, then v heads per row; rows may be strided) is split, q and k are rotated with
        ``rope = (cos, sin)`` tables ``[rows, D/2]`` fp32 indexed by each token's position in
        its session ("rotate half" form; None skips it), q goes to ``q_out [T_total, Hq, D]``
        and k, v to this layer's pages -- one kernel."""
        ids, cu_t, total = index if index is not None else self.batch_index(states, counts)
        if total == 0:
            return
        Hq, Hkv, D = q_out.shape[1], self.num_kv_heads, self.head_dim
        if qkv.dtype != self.dtype or qkv.device != self.device or qkv.dim() != 2 or \
                qkv.shape[0] != total or qkv.shape[1] != (Hq + 2 * Hkv) * D or qkv.stride(1) != 1:
            raise LoopfuseError(_lib.LF_EINVAL, "write_qkv expects qkv [T_total, (Hq+2Hkv)*D] "
                                                "rows of the pool dtype")
        if q_out.dtype != self.dtype or not q_out.is_contiguous() or \
                tuple(q_out.shape) != (total, Hq, D):
            raise LoopfuseError(_lib.LF_EINVAL, "write_qkv: q_out must be contiguous [T, Hq, D]")
        cos = sin = None
        rows = 0
        if rope is not None:
            cos, sin = rope
            for t in (cos, sin):
                if t.dtype != torch.float32 or not t.is_contiguous() or t.dim() != 2 or \
                        t.shape[1] != D // 2 or t.device != self.device:
                    raise LoopfuseError(_lib.LF_EINVAL, "write_qkv: rope tables must be "
                                                        "contiguous fp32 [rows, D/2] on the pool device")
            rows = cos.shape[0]
        elem = self.keys.element_size()
        layer_off = layer * self.keys.stride(0) * elem
        self._call("lf_pool_write_qkv", self._meta_ref(), ids.data_ptr(), start.data_ptr(),
                   cu_t.data_ptr(), ids.numel(), total, qkv.data_ptr(), qkv.stride(0),
                   cos.data_ptr() if cos is not None else None,
                   sin.data_ptr() if sin is not None else None, rows, q_out.data_ptr(),
                   self.keys.data_ptr() + layer_off, self.values.data_ptr() + layer_off, Hq, Hkv, D,
                   self._stream(stream))
        self._bytes_written += 2 * total * Hkv * D * elem

    # -- prefix-hash dedup (content-addressed KV fusion) ----------------------------------
    def _registry(self) -> "_lib.PrefixRegistry":
        if self._reg is None:
            cap = 1 << max(10, (2 * self.num_pages - 1).bit_length())
            self._reg_keys = torch.zeros(cap, dtype=torch.int64, device=self.device)
            self._reg_pages = torch.empty(cap, dtype=torch.int32, device=self.device)
            self._reg_used = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._reg = _lib.PrefixRegistry(self._reg_keys.data_ptr(), self._reg_pages.data_ptr(),
                                            self._reg_used.data_ptr(), cap)
            self._call("lf_registry_init", _lib.ctypes.byref(self._reg), self._stream())
        return self._reg

    def _tokens(self, tokens) -> torch.Tensor:
        return torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).to(self.device)

    def register_prefix(self, state: KVState, tokens) -> int:
        """Publish the session's full pages under the chained hash of their token ids (the
        first ``state.current_len`` of ``tokens`` count); returns pages added (host sync)."""
        toks = self._tokens(tokens)
        added = torch.zeros(1, dtype=torch.int32, device=self.device)
        reg = self._registry()
        self._call("lf_pool_register_prefix", self._meta_ref(), _lib.ctypes.byref(reg),
                   state.slot_id, toks.data_ptr(), toks.numel(), added.data_ptr(), self._stream())
        self._raise_if_failed("register_prefix", "prefix registry full or bad session")
        return int(added.item())

    def dedup_prefix(self, states: Sequence[KVState], tokens: Sequence) -> List[int]:
        """Map each (empty) session's longest registered run of leading full pages onto the
        registered pages; returns the tokens each one now holds (host sync)."""
        states = list(states)
        if not states:
            return []
        chunks = [self._tokens(t) for t in tokens]
        cu = torch.tensor([0] + [int(c.numel()) for c in chunks], dtype=torch.int64).cumsum(0)
        toks = torch.cat(chunks) if chunks else torch.empty(0, dtype=torch.int32, device=self.device)
        ids = self._ids([s.slot_id for s in states])
        cu_d = cu.to(torch.int32).to(self.device)
        covered = torch.zeros(len(states), dtype=torch.int32, device=self.device)
        reg = self._registry()
        self._call("lf_pool_dedup_prefix", self._meta_ref(), _lib.ctypes.byref(reg), ids.data_ptr(),
                   toks.data_ptr(), cu_d.data_ptr(), len(states), covered.data_ptr(), self._stream())
        self._raise_if_failed("dedup_prefix", "destinations must be distinct empty sessions")
        out = covered.tolist()
        for s, n in zip(states, out):
            s.current_len = n
        return out

    def unregister_all(self) -> None:
        """Drop the registry's page references and empty it."""
        if self._reg is None:
            return
        self._call("lf_pool_unregister_all", self._meta_ref(), _lib.ctypes.byref(self._reg),
                   self._stream())

    def block_table(self, states: Sequence[KVState], max_pages: Optional[int] = None
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Device ``[N, max_pages]`` int32 table and ``[N]`` lengths for ``paged_decode``."""
        max_pages = max_pages or self.max_pages_per_seq
        ids = self._ids([s.slot_id for s in states])
        table = torch.empty((len(states), max_pages), dtype=torch.int32, device=self.device)
        lens = torch.empty(len(states), dtype=torch.int32, device=self.device)
        self._call("lf_pool_gather", self._meta_ref(), ids.data_ptr(), len(states),
                   table.data_ptr(), max_pages, lens.data_ptr(), self._stream())
        return table, lens

    def layer_pages(self, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """``[P, Hkv, 16, D]`` views of one layer's K and V pages."""
        return self.keys[layer], self.values[layer]

    def snapshot(self) -> dict:
        """Host copy of the metadata (free queue from its head, refcounts, tables, lengths)."""
        ctrl = self._ctrl.tolist()
        head, count = ctrl[_lib.LF_CTRL_HEAD], ctrl[_lib.LF_CTRL_COUNT]
        fq = self._free_queue.tolist()
        P = self.num_pages
        return {
            "free_queue": [fq[(head + i) % P] for i in range(count)],
            "refcount": self._refcount.tolist(),
            "block_table": self._table.view(self.max_slots, self.max_pages_per_seq).tolist(),
            "seq_len": self._seq_len.tolist(),
            "status": ctrl[_lib.LF_CTRL_STATUS],
        }
