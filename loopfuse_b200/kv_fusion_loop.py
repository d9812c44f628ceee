"""KV-fusion loop: many agent sessions sharing one forked prompt prefix, step after step.

The reference's KV fusion is a compile-time pass that, on real programs, never fires
(``passes/kv_fusion.py:80-107``: it keys on ``seq_pos == 0`` writes, and the builder gives only
step 0 that position).  Here the fusion happens in the pool: the shared prefix is written once
into pages that every session references (``KVPool.fork``), decode reads those pages once per
group of sessions (``paged_decode(num_prefix_pages=...)``), and each step's new tokens go to
private pages.

Workload (all sizes configurable): ``sessions`` sessions forked from a ``prefix_tokens`` prompt;
for ``steps`` agent steps each session appends a tool output of geometric length (mean
``tool_mean``, capped at ``tool_cap``) -- written layer by layer and attended by the paged
prefill -- then decodes ``decode_tokens`` tokens, each one appended to the pool and attended
by the paged split-KV decode with the shared prefix, in every one of ``layers`` layers.
Attention shapes are Llama-3-8B's (32 layers, 32 query / 8 KV heads, head_dim 128, bf16);
the K/V/q values are synthetic (no model weights are involved).

Every decode iteration (all sessions, one token, every layer) is replayed from one CUDA graph,
captured during setup: the session set is fixed, so its shapes are.

Per step it reports the algorithmic HBM bytes the attention reads with prefix sharing
(``bytes_read``: every page a kernel must touch, the prefix once per decode call) and without
it (``bytes_read_unshared``: the prefix once per session), the K/V bytes written, and the GPU
time.  ``check`` mirrors every pool operation in the pool oracle and compares the device
metadata bit for bit after each fork, append and free (test use).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from . import attention as att
from .runtime.kv_pool import KVPool

PAGE = 16


@dataclass
class FusionLoopConfig:
    sessions: int = 64
    steps: int = 8
    layers: int = 32
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    prefix_tokens: int = 4096
    decode_tokens: int = 64
    tool_mean: float = 120.0
    tool_cap: int = 1024
    seed: int = 0
    graphs: bool = True          # decode iterations replayed from a CUDA graph captured in setup


def tool_lengths(cfg: FusionLoopConfig) -> np.ndarray:
    """[steps, sessions] tool-output lengths: geometric with mean ``tool_mean``, capped."""
    rng = np.random.default_rng(cfg.seed)
    return np.minimum(rng.geometric(1.0 / cfg.tool_mean, size=(cfg.steps, cfg.sessions)),
                      cfg.tool_cap).astype(np.int64)


@dataclass
class StepStats:
    step: int
    tool_tokens: int
    ms: float
    bytes_read: int
    bytes_read_unshared: int
    bytes_written: int
    launches: int
    prefill_ms: float = 0.0          # tool-output append + paged prefill, all layers
    decode_ms: float = 0.0           # the decode iterations
    decode_bytes_read: int = 0       # bytes_read of the decode iterations alone


@dataclass
class LoopResult:
    steps: List[StepStats] = field(default_factory=list)
    pages_total: int = 0
    checks: int = 0


class FusionLoop:
    def __init__(self, cfg: FusionLoopConfig, device=None, spec=None):
        self.cfg = cfg
        self.device = torch.device(device or "cuda")
        self.tools = tool_lengths(cfg)
        c = cfg
        self.n_prefix_pages = c.prefix_tokens // PAGE
        assert c.prefix_tokens % PAGE == 0, "prefix must be a whole number of pages"
        max_len = c.prefix_tokens + int(self.tools.sum(axis=0).max()) + c.steps * c.decode_tokens
        own = [math.ceil((int(self.tools[:, s].sum()) + c.steps * c.decode_tokens) / PAGE) + 1
               for s in range(c.sessions)]
        num_pages = self.n_prefix_pages + sum(own) + 8
        self.pool = KVPool(num_layers=c.layers, num_heads=c.q_heads, num_kv_heads=c.kv_heads,
                           head_dim=c.head_dim, max_seq_len=max_len, max_slots=c.sessions + 1,
                           dtype=torch.bfloat16, device=self.device, num_pages=num_pages)
        self.spec = spec
        g = torch.Generator(device=self.device)
        g.manual_seed(c.seed + 1)
        big = max(c.prefix_tokens, int(self.tools.sum(axis=1).max()))

        def rnd(*shape):
            return torch.randn(shape, generator=g, device=self.device,
                               dtype=torch.float32).to(torch.bfloat16)
        self.kbuf, self.vbuf = rnd(big, c.kv_heads, c.head_dim), rnd(big, c.kv_heads, c.head_dim)
        self.qbuf = rnd(big, c.q_heads, c.head_dim)
        self.qdec = rnd(c.sessions, c.q_heads, c.head_dim)
        self.page_bytes = 2 * c.kv_heads * PAGE * c.head_dim * 2       # K+V of one page, one layer
        self.checks = 0
        self._graph: Optional[dict] = None
        self._dec_idx = None
        self._ws: Optional[torch.Tensor] = None
        self._pps = 0

    # -- oracle mirror ----------------------------------------------------------------------
    def _check(self):
        if self.spec is None:
            return
        snap, want = self.pool.snapshot(), self.spec.snapshot()
        for key in ("free_queue", "refcount", "block_table", "seq_len"):
            if snap[key] != want[key]:
                raise AssertionError(f"device pool {key} differs from the oracle")
        self.checks += 1

    # -- phases -------------------------------------------------------------------------------
    def setup(self):
        c, pool = self.cfg, self.pool
        self.root = pool.alloc()
        start = pool.reserve([self.root], [c.prefix_tokens])
        idx = pool.batch_index([self.root], [c.prefix_tokens])
        for layer in range(c.layers):
            pool.write_layer([self.root], start, layer, self.kbuf[:c.prefix_tokens],
                             self.vbuf[:c.prefix_tokens], [c.prefix_tokens], index=idx)
        if self.spec is not None:
            self.spec.open_seq()
            self.spec.reserve([self.root.slot_id], [c.prefix_tokens])
            self._check()
        self.sessions = pool.fork(self.root, c.prefix_tokens, n=c.sessions)
        if self.spec is not None:
            ids = [self.spec.open_seq() for _ in range(c.sessions)]
            self.spec.fork(self.root.slot_id, ids, c.prefix_tokens)
            self._check()
        S = self.sessions
        self._dec_idx = pool.batch_index(S, [1] * len(S))
        table, lens = pool.block_table(S)
        self._pps = att.default_pages_per_split(len(S), c.kv_heads, table.shape[1], self.n_prefix_pages)
        self._ws = torch.empty(att.decode_workspace_bytes(len(S), c.q_heads, c.head_dim, table.shape[1],
                                                          self._pps, self.n_prefix_pages),
                               dtype=torch.uint8, device=self.device)
        if c.graphs:
            # One read-only decode initialises the kernels (and the library's side stream) outside
            # capture; the decode graph is then captured here, so no step times a capture.
            kp, vp = pool.layer_pages(0)
            att.paged_decode(self.qdec[:len(S)], kp, vp, table, lens,
                             num_prefix_pages=self.n_prefix_pages, pages_per_split=self._pps,
                             workspace=self._ws)
            torch.cuda.synchronize(self.device)
            self._graph = self._capture_decode(S, self._dec_idx)

    def _pages(self, n_tokens: int) -> int:
        return (n_tokens + PAGE - 1) // PAGE

    def step(self, step: int) -> StepStats:
        c, pool, S = self.cfg, self.pool, self.sessions
        T = [int(x) for x in self.tools[step]]
        total = sum(T)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        launches = 0
        bytes_read = bytes_unshared = 0
        # tool output: append (all layers) and attend over each session's whole context
        start = pool.reserve(S, T)
        idx = pool.batch_index(S, T)
        table, lens = pool.block_table(S)
        cu = torch.tensor([0] + list(np.cumsum(T)), dtype=torch.int32, device=self.device)
        for layer in range(c.layers):
            pool.write_layer(S, start, layer, self.kbuf[:total], self.vbuf[:total], T, index=idx)
            kp, vp = pool.layer_pages(layer)
            att.prefill_paged(self.qbuf[:total], kp, vp, table, cu, lens, max(T))
            launches += 2
        ev_mid = torch.cuda.Event(enable_timing=True)
        ev_mid.record()
        ctx = [s.current_len for s in S]
        pre_pages = sum(self._pages(L) for L in ctx)
        bytes_read += c.layers * pre_pages * self.page_bytes
        bytes_unshared += c.layers * pre_pages * self.page_bytes
        prefill_bytes = bytes_read
        if self.spec is not None:
            self.spec.reserve([s.slot_id for s in S], T)
            self._check()
        # decode: one token per session per iteration, every layer
        ones = [1] * len(S)
        dec_idx = self._dec_idx
        for _ in range(c.decode_tokens):
            if self._graph is not None:
                for s in S:
                    if s.current_len + 1 > pool.max_seq_len:
                        raise RuntimeError(f"KV cache overflow: current_len={s.current_len} + "
                                           f"seq_new=1 > max_seq_len={pool.max_seq_len}")
                self._graph["graph"].replay()
                for s in S:
                    s.current_len += 1
            else:
                start = pool.reserve(S, ones)
                table, lens = pool.block_table(S)
                for layer in range(c.layers):
                    pool.write_layer(S, start, layer, self.kbuf[:len(S)], self.vbuf[:len(S)], ones,
                                     index=dec_idx)
                    kp, vp = pool.layer_pages(layer)
                    att.paged_decode(self.qdec[:len(S)], kp, vp, table, lens,
                                     num_prefix_pages=self.n_prefix_pages,
                                     pages_per_split=self._pps, workspace=self._ws)
            # reserve + gather, then per layer the decode's prefix pass, split and combine (the
            # graphed iteration fuses the K/V append into the split; eager appends separately)
            launches += 2 + (3 if self._graph is not None else 4) * c.layers
            own = sum(self._pages(s.current_len) - self.n_prefix_pages for s in S)
            bytes_read += c.layers * (self.n_prefix_pages + own) * self.page_bytes
            bytes_unshared += c.layers * sum(self._pages(s.current_len) for s in S) * self.page_bytes
            if self.spec is not None:
                self.spec.reserve([s.slot_id for s in S], ones)
                self._check()
        ev1.record()
        ev1.synchronize()
        if pool.status() != 0:
            pool._raise_if_failed("fusion-loop decode")
        written = c.layers * (total + c.decode_tokens * len(S)) * 2 * c.kv_heads * c.head_dim * 2
        return StepStats(step, total, ev0.elapsed_time(ev1), bytes_read, bytes_unshared, written,
                         launches, ev0.elapsed_time(ev_mid), ev_mid.elapsed_time(ev1),
                         bytes_read - prefill_bytes)

    def _capture_decode(self, S, dec_idx) -> dict:
        """One decode iteration of every session as a CUDA graph: pool reserve and block-table
        gather on device buffers, then per layer the paged decode with the new token's K/V append
        fused in (the split pass stores each session's newest token into its page before reading
        it; the pages end up as ``write_layer`` would leave them).  Captured in setup, after a
        read-only decode has initialised the decode kernels; nothing in it allocates."""
        c, pool, n = self.cfg, self.pool, len(S)
        i32 = dict(dtype=torch.int32, device=self.device)
        g = {"start": torch.empty(n, **i32), "ones": torch.ones(n, **i32),
             "table": torch.empty((n, pool.max_pages_per_seq), **i32), "lens": torch.empty(n, **i32),
             "out": torch.empty_like(self.qdec[:n])}
        kb, vb, qd = self.kbuf[:n], self.vbuf[:n], self.qdec[:n]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            pool.reserve_device(dec_idx[0], g["ones"], g["start"], n)
            pool.gather_device(dec_idx[0], n, g["table"], g["lens"])
            for layer in range(c.layers):
                kp, vp = pool.layer_pages(layer)
                att.paged_decode(qd, kp, vp, g["table"], g["lens"],
                                 num_prefix_pages=self.n_prefix_pages, pages_per_split=self._pps,
                                 out=g["out"], workspace=self._ws,
                                 k_new=kb.view(n, c.kv_heads, c.head_dim),
                                 v_new=vb.view(n, c.kv_heads, c.head_dim))
        g["graph"] = graph
        return g

    def teardown(self):
        everyone = self.sessions + [self.root]
        self.pool.release_all(everyone)
        if self.spec is not None:
            ids = [s.slot_id for s in everyone]
            self.spec.free(ids)                   # one batched free, like release_all
            self.spec.free_seqs.extend(ids)
            self._check()

    def run(self) -> LoopResult:
        res = LoopResult(pages_total=self.pool.num_pages)
        self.setup()
        for step in range(self.cfg.steps):
            res.steps.append(self.step(step))
        self.teardown()
        res.checks = self.checks
        return res
