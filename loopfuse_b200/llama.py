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

from . import attention as att
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
        self.fused_qkv = True          # False: the unfused torch split / rotate / pool write path

    def rope_tables(self, rows: int):
        """``[rows, D/2]`` fp32 cos / sin of position x inverse frequency (grown on demand)."""
        if rows > self._rope_rows:
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

    # -- forward ------------------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, pool: KVPool, states: Sequence[KVState],
                counts: Sequence[int], n_prefix_pages: int = 0,
                return_logits: bool = False) -> torch.Tensor:
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
            pps = att.default_pages_per_split(len(states), c.kv_heads, table.shape[1])
            need = att.decode_workspace_bytes(len(states), c.q_heads, c.head_dim, table.shape[1],
                                              pps, n_prefix_pages)
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        x = self.embed[tokens]
        nq, nk = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
        for l in range(c.layers):
            h = self._rmsnorm(x, self.attn_norm[l])
            qkv = h @ self.wqkv[l]
            if self.fused_qkv:
                q = torch.empty((T, c.q_heads, c.head_dim), dtype=qkv.dtype, device=self.device)
                pool.write_qkv(states, start, l, qkv, q, counts, rope=rope, index=index)
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
            x = x + a.view(T, nq) @ self.wo[l]
            h = self._rmsnorm(x, self.ffn_norm[l])
            gu = h @ self.w13[l]
            x = x + (F.silu(gu[:, :c.ffn]) * gu[:, c.ffn:]) @ self.w2[l]
        last = torch.tensor(counts, device=self.device).cumsum(0) - 1
        h = self._rmsnorm(x[last], self.final_norm)
        logits = h @ self.lm_head
        return logits.float() if return_logits else torch.argmax(logits, dim=-1)

    # -- AgentExecutor model contract ------------------------------------------------------------
    def prefill(self, tokens: torch.Tensor, kv_state: KVState, attention=None) -> torch.Tensor:
        nxt = self.forward(tokens.to(self.device).long(), kv_state.pool, [kv_state], [tokens.numel()])
        return torch.nn.functional.one_hot(nxt, self.cfg.vocab).float()

    def decode(self, tokens: torch.Tensor, kv_state: KVState, attention=None) -> torch.Tensor:
        nxt = self.forward(tokens.to(self.device).long(), kv_state.pool, [kv_state], [1])
        return torch.nn.functional.one_hot(nxt, self.cfg.vocab).float()
