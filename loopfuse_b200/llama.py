"""Llama-3-8B-shaped decoder whose attention runs on the sm_100a kernels and the paged pool.

Weights are random (N(0, 0.02), bf16): the agent-loop workload measures throughput, and no
checkpoint is available.  Shapes: 32 layers, d_model 4096, 32 query / 8 KV heads of 128, SwiGLU
FFN 14336, vocab 128256, RoPE theta 500000, RMSNorm eps 1e-5.  The dense projections are plain
library GEMMs (``torch.matmul`` -> cuBLAS bf16); normalisation and the SwiGLU gate are
elementwise torch ops.  The QKV GEMM's output goes through one fused kernel
(``KVPool.write_qkv``): split, rotary embedding of q and k from a cached cos/sin table, q
written contiguous, k and v scattered into the session's pages.  Attention is the package's own: ``prefill_paged`` for a batch of
new prompt / tool-output tokens over each session's cached pages, ``paged_decode`` (with the
forked shared prefix read once per group of sessions) for one token per session.  New K/V are
appended to the pool layer by layer (``KVPool.reserve`` once per forward, ``write_qkv`` per
layer).

``forward(tokens, pool, states, counts)`` advances every listed session by ``counts[i]`` tokens
(``tokens`` holds them back to back) and returns the greedy next token of each session.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
import torch.nn.functional as F

from . import _lib
from . import attention as att
from . import model_ops as mo
from .runtime.kv_pool import KVPool, KVState


@dataclass
class LlamaConfig:
    d_model: int = 4096
    layers: int = 32
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5

    @property
    def kv_config(self) -> dict:
        return {"num_layers": self.layers, "num_heads": self.q_heads,
                "num_kv_heads": self.kv_heads, "head_dim": self.head_dim, "dtype": "bf16"}


class OpTimer:
    """CUDA-event attribution of one forward's GPU time to op classes.

    ``lap(name)`` records an event on the current stream and charges the time since the previous
    event to ``name``.  Call ``start()`` first; ``totals()`` (after a sync) returns milliseconds
    per name.  To keep host launch gaps out of the measured spans, ``start`` can hold the stream
    in a device-side spin (``hold_cycles``) while the host enqueues the whole forward."""

    def __init__(self):
        self.events: List[tuple] = []

    def start(self, hold_cycles: int = 0) -> None:
        if hold_cycles:
            torch.cuda._sleep(int(hold_cycles))
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.events = [(None, ev)]

    def lap(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.events.append((name, ev))

    def totals(self) -> dict:
        out: dict = {}
        for (_, a), (name, b) in zip(self.events, self.events[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


def _lap(timer: Optional[OpTimer], name: str) -> None:
    if timer is not None:
        timer.lap(name)


class LlamaShaped:
    def __init__(self, cfg: LlamaConfig, device="cuda", seed: int = 0, std: float = 0.02):
        self.cfg = cfg
        self.device = torch.device(device)
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        c = cfg

        def w(*shape):
            out = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
            flat = out.view(-1)
            step = 1 << 26
            for s in range(0, flat.numel(), step):
                e = min(flat.numel(), s + step)
                flat[s:e] = (torch.randn(e - s, generator=g, device=self.device) * std).to(torch.bfloat16)
            return out

        qkv = (c.q_heads + 2 * c.kv_heads) * c.head_dim
        self.embed = w(c.vocab, c.d_model)
        self.wqkv = [w(c.d_model, qkv) for _ in range(c.layers)]
        self.wo = [w(c.q_heads * c.head_dim, c.d_model) for _ in range(c.layers)]
        self.w13 = [w(c.d_model, 2 * c.ffn) for _ in range(c.layers)]
        self.w2 = [w(c.ffn, c.d_model) for _ in range(c.layers)]
        ones = torch.ones(c.d_model, dtype=torch.bfloat16, device=self.device)
        self.attn_norm = [ones.clone() for _ in range(c.layers)]
        self.ffn_norm = [ones.clone() for _ in range(c.layers)]
        self.final_norm = ones.clone()
        self.lm_head = w(c.d_model, c.vocab)
        self.inv_freq = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, device=self.device,
                                                               dtype=torch.float32) / c.head_dim))
        self._ws: Optional[torch.Tensor] = None
        self._rope_rows = 0
        self._cos = self._sin = None
        self._rope_old: list = []      # replaced tables stay alive: captured graphs point at them
        self.fused_qkv = True          # False: the unfused torch split / rotate / pool write path
        self.fused_ops = True          # False: torch RMSNorm / residual adds / SwiGLU

    def rope_tables(self, rows: int):
        """``[rows, D/2]`` fp32 cos / sin of position x inverse frequency (grown on demand)."""
        if rows > self._rope_rows:
            if self._cos is not None:
                self._rope_old.append((self._cos, self._sin))
            rows = max(rows, 2 * self._rope_rows, 4096)
            ang = torch.arange(rows, device=self.device).float()[:, None] * self.inv_freq[None, :]
            self._cos, self._sin = ang.cos().contiguous(), ang.sin().contiguous()
            self._rope_rows = rows
        return self._cos, self._sin

    def param_bytes(self) -> int:
        ts = [self.embed, self.lm_head] + self.wqkv + self.wo + self.w13 + self.w2
        return sum(t.numel() * t.element_size() for t in ts)

    def flops_per_token(self) -> int:
        """2 x parameters touched per token (attention scores excluded)."""
        c = self.cfg
        per_layer = c.d_model * (c.q_heads + 2 * c.kv_heads) * c.head_dim + \
            c.q_heads * c.head_dim * c.d_model + 3 * c.d_model * c.ffn
        return 2 * (c.layers * per_layer + c.d_model * c.vocab)

    # -- pieces -------------------------------------------------------------------------------
    def _rmsnorm(self, x: torch.Tensor, wgt: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(x.dtype) * wgt

    def _rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        half = x.shape[-1] // 2
        xf = x.float()
        x1, x2 = xf[..., :half], xf[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)

    def _norm_in(self, x: torch.Tensor, delta: Optional[torch.Tensor], w: Optional[torch.Tensor]):
        """``x += delta``; returns ``rmsnorm(x) * w`` (None when ``w`` is None)."""
        if self.fused_ops:
            return mo.add_rmsnorm(x, delta, w, self.cfg.eps)
        if delta is not None:
            x.add_(delta)
        return self._rmsnorm(x, w) if w is not None else None

    def _mlp_block(self, x: torch.Tensor, attn: torch.Tensor, l: int,
                   timer: Optional[OpTimer] = None):
        """Rest of layer ``l`` after attention: output projection, residual, FFN norm, SwiGLU
        FFN, residual, and the next layer's input norm.  Returns (x, normed input of l + 1)."""
        c = self.cfg
        o = attn @ self.wo[l]
        _lap(timer, "o_gemm")
        h = self._norm_in(x, o, self.ffn_norm[l])
        _lap(timer, "add_rmsnorm")
        gu = h @ self.w13[l]
        _lap(timer, "gate_up_gemm")
        act = mo.swiglu(gu) if self.fused_ops else F.silu(gu[:, :c.ffn]) * gu[:, c.ffn:]
        _lap(timer, "swiglu")
        nxt = self.attn_norm[l + 1] if l + 1 < c.layers else None
        d = act @ self.w2[l]
        _lap(timer, "down_gemm")
        out = self._norm_in(x, d, nxt)
        _lap(timer, "add_rmsnorm")
        return x, out

    # -- forward ------------------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, pool: KVPool, states: Sequence[KVState],
                counts: Sequence[int], n_prefix_pages: int = 0,
                return_logits: bool = False, timer: Optional[OpTimer] = None) -> torch.Tensor:
        c = self.cfg
        counts = [int(x) for x in counts]
        T = sum(counts)
        starts_host = [s.current_len for s in states]
        start = pool.reserve(states, counts)
        index = pool.batch_index(states, counts)
        table, lens = pool.block_table(states)
        if self.fused_qkv:
            rope = self.rope_tables(max(s0 + n for s0, n in zip(starts_host, counts)))
        else:
            pos = torch.cat([torch.arange(s0, s0 + n, device=self.device) for s0, n in
                             zip(starts_host, counts)]).float()
            ang = pos[:, None] * self.inv_freq[None, :]
            cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
        decode = all(n == 1 for n in counts)
        if not decode:
            cu = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32,
                              device=self.device)
        else:
            pps = att.default_pages_per_split(len(states), c.kv_heads, table.shape[1], n_prefix_pages)
            need = att.decode_workspace_bytes(len(states), c.q_heads, c.head_dim, table.shape[1],
                                              pps, n_prefix_pages)
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        if timer is not None:
            timer.lap("setup")
        x = self.embed[tokens]
        nq, nk = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
        h = self._norm_in(x, None, self.attn_norm[0])
        _lap(timer, "embed_norm")
        for l in range(c.layers):
            qkv = h @ self.wqkv[l]
            _lap(timer, "qkv_gemm")
            if self.fused_qkv:
                q = torch.empty((T, c.q_heads, c.head_dim), dtype=qkv.dtype, device=self.device)
                pool.write_qkv(states, start, l, qkv, q, counts, rope=rope, index=index)
                _lap(timer, "qkv_rope_append")
            else:
                q = self._rope(qkv[:, :nq].view(T, c.q_heads, c.head_dim), cos, sin).contiguous()
                k = self._rope(qkv[:, nq:nq + nk].view(T, c.kv_heads, c.head_dim), cos, sin)
                v = qkv[:, nq + nk:].reshape(T, c.kv_heads, c.head_dim).contiguous()
                pool.write_layer(states, start, l, k.contiguous(), v, counts, index=index)
            kp, vp = pool.layer_pages(l)
            if decode:
                a = att.paged_decode(q, kp, vp, table, lens,
                                     num_prefix_pages=n_prefix_pages, pages_per_split=pps,
                                     workspace=self._ws)
            else:
                a = att.prefill_paged(q, kp, vp, table, cu, lens, max(counts))
            _lap(timer, "attention")
            x, h = self._mlp_block(x, a.view(T, nq), l, timer)
        last = torch.tensor(counts, device=self.device).cumsum(0) - 1
        h = self._norm_in(x[last].contiguous(), None, self.final_norm)
        logits = h @ self.lm_head
        _lap(timer, "lm_head")
        out = logits.float() if return_logits else torch.argmax(logits, dim=-1)
        _lap(timer, "argmax")
        return out

    # -- AgentExecutor model contract ------------------------------------------------------------
    def prefill(self, tokens: torch.Tensor, kv_state: KVState, attention=None) -> torch.Tensor:
        nxt = self.forward(tokens.to(self.device).long(), kv_state.pool, [kv_state], [tokens.numel()])
        return torch.nn.functional.one_hot(nxt, self.cfg.vocab).float()

    def decode(self, tokens: torch.Tensor, kv_state: KVState, attention=None) -> torch.Tensor:
        nxt = self.forward(tokens.to(self.device).long(), kv_state.pool, [kv_state], [1])
        return torch.nn.functional.one_hot(nxt, self.cfg.vocab).float()


_BUCKETS = (16, 32, 64, 96, 128, 192, 256, 320, 384, 448, 512)


def _bucket(n: int) -> int:
    for b in _BUCKETS:
        if n <= b:
            return b
    return -(-n // 128) * 128


class GraphedDecode:
    """One-token decode steps replayed from CUDA graphs, one graph per batch-size bucket.

    A decode step of the model is ~700 kernel launches, so at small batches the host's launch
    rate, not the GPU, sets the step time.  Here a step is: one pinned host -> device copy of
    (tokens, slot ids, counts), one graph replay (pool reserve and block-table gather, every
    layer, final norm, LM head, argmax), and the caller's read of the result.  A batch of n
    sessions runs in the graph of the smallest bucket >= n; rows past n take 0 new tokens in
    ``pad`` (a ``KVPool.pad_session``): their pages never grow and their outputs are ignored.
    Each graph has its own memory pool; the pool's device status is copied back with the
    output (``raise_if_failed`` after the caller's sync).
    """

    def __init__(self, model: "LlamaShaped", pool: KVPool, pad: KVState, n_prefix_pages: int = 0):
        self.model, self.pool, self.pad, self.npp = model, pool, pad, n_prefix_pages
        self.graphs = {}
        self.status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)

    def _build(self, nb: int):
        m, pool, dev = self.model, self.pool, self.model.device
        c = m.cfg
        s = {"nb": nb,
             "host": torch.zeros((3, nb), dtype=torch.int32, pin_memory=True),
             "dev": torch.zeros((3, nb), dtype=torch.int32, device=dev),
             "cu": torch.arange(nb + 1, dtype=torch.int32, device=dev),
             "start": torch.zeros(nb, dtype=torch.int32, device=dev),
             "table": torch.empty((nb, pool.max_pages_per_seq), dtype=torch.int32, device=dev),
             "lens": torch.empty(nb, dtype=torch.int32, device=dev),
             "copied": torch.cuda.Event()}
        s["pps"] = att.default_pages_per_split(nb, c.kv_heads, pool.max_pages_per_seq, self.npp)
        s["ws"] = torch.empty(att.decode_workspace_bytes(nb, c.q_heads, c.head_dim,
                                                         pool.max_pages_per_seq, s["pps"], self.npp),
                              dtype=torch.uint8, device=dev)
        # rows: real sessions take 1 token; a fresh graph's warm-up runs every row as padding
        s["host"][1].fill_(self.pad.slot_id)
        s["dev"].copy_(s["host"])
        m.rope_tables(pool.max_seq_len + 1)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._body(s)                          # warm-up outside capture (allocator, cuBLAS)
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            s["out"] = self._body(s)
        s["graph"] = g
        return s

    @torch.no_grad()
    def _body(self, s) -> torch.Tensor:
        m, pool = self.model, self.pool
        c = m.cfg
        nb = s["nb"]
        toks, ids, cnt = s["dev"][0], s["dev"][1], s["dev"][2]
        pool.reserve_device(ids, cnt, s["start"], nb)
        pool.gather_device(ids, nb, s["table"], s["lens"])
        rope = (m._cos, m._sin)
        index = (ids, s["cu"], nb)
        x = m.embed[toks.long()]
        nq = c.q_heads * c.head_dim
        h = m._norm_in(x, None, m.attn_norm[0])
        for l in range(c.layers):
            qkv = h @ m.wqkv[l]
            q = torch.empty((nb, c.q_heads, c.head_dim), dtype=qkv.dtype, device=m.device)
            pool.write_qkv(None, s["start"], l, qkv, q, None, rope=rope, index=index)
            kp, vp = pool.layer_pages(l)
            a = att.paged_decode(q, kp, vp, s["table"], s["lens"], num_prefix_pages=self.npp,
                                 pages_per_split=s["pps"], workspace=s["ws"])
            x, h = m._mlp_block(x, a.view(nb, nq), l)
        return torch.argmax(m._norm_in(x, None, m.final_norm) @ m.lm_head, dim=-1)

    def prepare(self, max_batch: int) -> None:
        """Capture the graphs of every bucket up to ``max_batch`` sessions."""
        for b in _BUCKETS:
            if b not in self.graphs:
                self.graphs[b] = self._build(b)
            if b >= max_batch:
                break

    def step(self, states: Sequence[KVState], tokens: Sequence[int]) -> torch.Tensor:
        """Advance each session by its token; returns the device tensor of greedy next tokens
        (the first ``len(states)`` rows are valid)."""
        n = len(states)
        nb = _bucket(n)
        s = self.graphs.get(nb)
        if s is None:
            s = self.graphs[nb] = self._build(nb)
        for st in states:
            if st.current_len + 1 > self.pool.max_seq_len:
                raise RuntimeError(f"KV cache overflow: current_len={st.current_len} + seq_new=1 > "
                                   f"max_seq_len={self.pool.max_seq_len}")
        s["copied"].synchronize()                  # the previous copy out of this buffer is done
        host = s["host"]
        host[0, :n] = torch.as_tensor(list(tokens), dtype=torch.int32)
        host[1, :n] = torch.as_tensor([st.slot_id for st in states], dtype=torch.int32)
        host[2, :n] = 1
        host[0, n:] = 0
        host[1, n:] = self.pad.slot_id
        host[2, n:] = 0
        s["dev"].copy_(host, non_blocking=True)
        s["copied"].record()
        s["graph"].replay()
        self.status_host.copy_(self.pool._ctrl[_lib.LF_CTRL_STATUS:_lib.LF_CTRL_STATUS + 1],
                               non_blocking=True)
        for st in states:
            st.current_len += 1
        return s["out"]

    def raise_if_failed(self) -> None:
        """Call after a sync that follows ``step`` (e.g. reading its output)."""
        if int(self.status_host[0]) != _lib.LF_OK:
            self.pool._raise_if_failed("graphed decode")
