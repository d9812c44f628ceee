"""Session sharding across GPUs (one process per GPU, torch.distributed for the plumbing).

Sessions are independent: each one's block table, pages and decode state live on exactly one
GPU, so a decode or prefill step needs no data-path collective.  ``lpt_assign`` balances ranks
by expected work (longest-processing-time-first on context length); ``RankGroup`` wraps the
process group for the few host-side collectives a run needs (barrier, max of step times, sums
of counters), all of which stay outside the timed kernels.
"""
from __future__ import annotations

import datetime
import heapq
import os
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def lpt_assign(work: Sequence[float], world_size: int) -> List[List[int]]:
    """Indices of ``work`` per rank: largest first onto the least-loaded rank (ties: lowest rank).

    Deterministic for a given input, so every rank computes the same assignment locally.
    """
    heap = [(0.0, r) for r in range(world_size)]
    heapq.heapify(heap)
    out: List[List[int]] = [[] for _ in range(world_size)]
    for i in sorted(range(len(work)), key=lambda i: (-work[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + float(work[i]), r))
    return [sorted(x) for x in out]


class RankGroup:
    """The process group of a run: rank / world size from the launcher's environment."""

    def __init__(self, backend: Optional[str] = None, timeout_s: float = 120.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        self.device = (torch.device("cuda", self.local_rank) if self.backend == "nccl"
                       else torch.device("cpu"))
        if self.world > 1 and not dist.is_initialized():
            kw = {"device_id": self.device} if self.backend == "nccl" else {}
            if self.backend == "nccl":
                torch.cuda.set_device(self.device)
            dist.init_process_group(self.backend, timeout=datetime.timedelta(seconds=timeout_s),
                                    **kw)

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def close(self) -> None:
        if self.world > 1 and dist.is_initialized():
            dist.destroy_process_group()
