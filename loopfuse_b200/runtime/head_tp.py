"""Head-tensor-parallel paged decode: KV heads split over the ranks of a node, outputs gathered.

Each of the ``world`` ranks (one process per GPU) holds ``Hkv / world`` of the model's KV heads
for every session and computes the matching ``Hq / world`` query heads; every rank then needs
all heads' outputs ``[N, Hq, D]``.  Two ways to get there:

* ``decode`` (fused): ``lf_decode_fwd_gather`` -- the combine kernel that finishes a row stores
  it straight into every rank's output buffer (peer-memory stores over NVLink; the buffers are
  mapped into each process with CUDA IPC, plain peer mappings), then a one-element NCCL
  all-reduce on the same stream orders every rank's readers after every rank's stores.
* ``decode_nccl`` (baseline): local decode, then ``all_gather_into_tensor`` and a head-major
  re-layout.

Both give the same bits (each head's attention is computed the same way whichever rank runs
it).  Outputs alternate between two buffers, so a rank may run one call ahead of a slower
peer; a returned tensor stays valid until the caller's second-next ``decode``.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import _lib
from .. import attention as att
from .._lib import LF_PAGE_SIZE, LoopfuseError


class HeadParallelDecode:
    def __init__(self, num_seqs: int, num_q_heads_total: int, head_dim: int,
                 device: torch.device, group: Optional[dist.ProcessGroup] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if num_q_heads_total % self.world:
            raise LoopfuseError(_lib.LF_EINVAL, "query heads must split evenly over the ranks")
        self.N, self.Hq, self.D, self.device = num_seqs, num_q_heads_total, head_dim, device
        self.hq_local = num_q_heads_total // self.world
        self._opened: List[int] = []
        self._bufs, self._peers = [], []
        for _ in range(2):
            out = torch.empty((num_seqs, num_q_heads_total, head_dim), dtype=torch.bfloat16,
                              device=device)
            self._bufs.append(out)
            self._peers.append(self._share(out))
        self._flag = torch.zeros(1, dtype=torch.float32, device=device)
        self._calls = 0

    def _share(self, out: torch.Tensor) -> torch.Tensor:
        """Device array of every rank's pointer to its copy of ``out``'s buffer."""
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t(0)
        _lib.call("lf_ipc_export", out.data_ptr(), handle, ctypes.byref(off))
        mine = (bytes(handle.raw), int(off.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=self.group)
        ptrs = []
        for r, (h, o) in enumerate(everyone):
            if r == self.rank:
                ptrs.append(out.data_ptr())
                continue
            base = ctypes.c_void_p(0)
            _lib.call("lf_ipc_import", ctypes.create_string_buffer(h, 64), ctypes.byref(base))
            self._opened.append(int(base.value))
            ptrs.append(int(base.value) + o)
        return torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    def _check(self, q: torch.Tensor, k_pages: torch.Tensor) -> None:
        N, Hq, D = q.shape
        if (N, Hq, D) != (self.N, self.hq_local, self.D) or k_pages.shape[2] != LF_PAGE_SIZE:
            raise LoopfuseError(_lib.LF_EINVAL, f"head-parallel decode expects q [{self.N}, "
                                                f"{self.hq_local}, {self.D}] (this rank's heads)")

    def decode(self, q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
               block_table: torch.Tensor, seq_lens: torch.Tensor, num_prefix_pages: int = 0,
               pages_per_split: Optional[int] = None, workspace: Optional[torch.Tensor] = None,
               scale: Optional[float] = None) -> torch.Tensor:
        """This rank's heads in, every head out ``[N, Hq_total, D]`` (fused gather)."""
        self._check(q, k_pages)
        P, Hkv, _, D = k_pages.shape
        max_pages = block_table.shape[1]
        pps = pages_per_split or att.default_pages_per_split(self.N, Hkv, max_pages, num_prefix_pages)
        need = att.decode_workspace_bytes(self.N, self.hq_local, D, max_pages, pps, num_prefix_pages)
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=self.device)
        i = self._calls & 1
        self._calls += 1
        _lib.call("lf_decode_fwd_gather", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
                  block_table.data_ptr(), seq_lens.data_ptr(), int(num_prefix_pages),
                  self._peers[i].data_ptr(), self.world, self.rank * self.hq_local, self.Hq, None,
                  workspace.data_ptr(), workspace.numel() * workspace.element_size(), self.N,
                  self.hq_local, Hkv, D, P, max_pages, pps,
                  D ** -0.5 if scale is None else float(scale),
                  torch.cuda.current_stream(self.device).cuda_stream)
        dist.all_reduce(self._flag, group=self.group)     # every rank's stores have landed
        return self._bufs[i]

    def decode_nccl(self, q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                    block_table: torch.Tensor, seq_lens: torch.Tensor, num_prefix_pages: int = 0,
                    pages_per_split: Optional[int] = None,
                    workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Baseline: local decode, then NCCL all-gather and head-major re-layout."""
        self._check(q, k_pages)
        local = att.paged_decode(q, k_pages, v_pages, block_table, seq_lens,
                                 num_prefix_pages=num_prefix_pages, pages_per_split=pages_per_split,
                                 workspace=workspace)
        gathered = torch.empty((self.world,) + tuple(local.shape), dtype=local.dtype,
                               device=self.device)
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        return gathered.permute(1, 0, 2, 3).reshape(self.N, self.Hq, self.D)

    def close(self) -> None:
        for base in self._opened:
            _lib.call("lf_ipc_close", base)
        self._opened = []
