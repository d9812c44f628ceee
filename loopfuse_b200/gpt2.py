"""GPT-2-small decoder whose attention runs on the sm_100a kernels and the paged pool.

The reference names GPT-2 small as its CPU-runnable program (``ir/dialect.py:525-532``: 12 layers,
d_model 768, 12 heads of 64, ffn 3072, vocab 50257) and runs it through
``scaled_dot_product_attention`` (``passes/phase_select.py:80-89``).  Here the attention is the
package's own: ``prefill_paged`` (tcgen05 core, 64-dim heads, one KV head per query head) for a
chunk of new tokens over the session's cached pages, ``paged_decode`` for one token.  Each
layer's QKV output is split by the fused ``KVPool.write_qkv`` kernel: q contiguous, K/V into
the bf16 pool pages.  The dense parts (embeddings, LayerNorm, QKV / output / MLP
projections, GELU-tanh) are torch ops in ``dense_dtype`` (fp32 by default, so that the only
reduced-precision step is the bf16 attention).

``weights`` is a dict of host tensors keyed like ``{"wte", "wpe", "ln_f.w", "ln_f.b",
"<l>.ln_1.w", "<l>.attn.w" [768, 2304], "<l>.attn.b", "<l>.proj.w", "<l>.proj.b", "<l>.ln_2.w",
"<l>.fc.w" [768, 3072], "<l>.fc.b", "<l>.fc2.w", "<l>.fc2.b", ...}`` (x @ W layout); ``None``
draws N(0, 0.02) weights from ``seed``.  The position table may be longer than GPT-2's 1024
rows (``GPT2Config.positions``) so that programs longer than 1024 tokens run.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch
import torch.nn.functional as F

from . import attention as att
from ._lib import LF_PAGE_SIZE
from .runtime.kv_pool import KVPool, KVState


@dataclass
class GPT2Config:
    layers: int = 12
    d_model: int = 768
    heads: int = 12
    head_dim: int = 64
    ffn: int = 3072
    vocab: int = 50257
    positions: int = 1280
    eps: float = 1e-5

    @property
    def kv_config(self) -> dict:
        return {"num_layers": self.layers, "num_heads": self.heads, "num_kv_heads": self.heads,
                "head_dim": self.head_dim, "dtype": "bf16"}


class GPT2Model:
    def __init__(self, cfg: GPT2Config = GPT2Config(), weights: Optional[Dict[str, torch.Tensor]] = None,
                 device="cuda", dense_dtype: torch.dtype = torch.float32, seed: int = 0):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dense_dtype
        if weights is None:
            weights = self._random(seed)
        self.w = {k: v.to(self.device, self.dtype) for k, v in weights.items()}
        self._ws: Optional[torch.Tensor] = None

    def _random(self, seed: int) -> Dict[str, torch.Tensor]:
        c = self.cfg
        g = torch.Generator().manual_seed(seed)
        d, f = c.d_model, c.ffn

        def n(*shape):
            return torch.randn(*shape, generator=g) * 0.02
        w = {"wte": n(c.vocab, d), "wpe": n(c.positions, d),
             "ln_f.w": torch.ones(d), "ln_f.b": torch.zeros(d)}
        for l in range(c.layers):
            w.update({f"{l}.ln_1.w": torch.ones(d), f"{l}.ln_1.b": torch.zeros(d),
                      f"{l}.attn.w": n(d, 3 * d), f"{l}.attn.b": torch.zeros(3 * d),
                      f"{l}.proj.w": n(d, d), f"{l}.proj.b": torch.zeros(d),
                      f"{l}.ln_2.w": torch.ones(d), f"{l}.ln_2.b": torch.zeros(d),
                      f"{l}.fc.w": n(d, f), f"{l}.fc.b": torch.zeros(f),
                      f"{l}.fc2.w": n(f, d), f"{l}.fc2.b": torch.zeros(d)})
        return w

    def new_pool(self, num_pages: int, max_slots: int, max_seq_len: Optional[int] = None) -> KVPool:
        c = self.cfg
        return KVPool(num_layers=c.layers, num_heads=c.heads, num_kv_heads=c.heads,
                      head_dim=c.head_dim, max_seq_len=max_seq_len or c.positions,
                      max_slots=max_slots, dtype=torch.bfloat16, device=self.device,
                      num_pages=num_pages)

    def _ln(self, x: torch.Tensor, p: str) -> torch.Tensor:
        return F.layer_norm(x, (self.cfg.d_model,), self.w[p + ".w"], self.w[p + ".b"], self.cfg.eps)

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, pool: KVPool, states: Sequence[KVState],
                counts: Sequence[int], n_prefix_pages: int = 0,
                attn_last: Optional[List[torch.Tensor]] = None) -> torch.Tensor:
        """Advance each session by ``counts[i]`` tokens; returns [n_sessions, vocab] logits of
        each session's last new position.  ``attn_last``, if given, receives per layer the
        attention output ([n_sessions, d_model], ``dense_dtype``) at those positions."""
        c, w = self.cfg, self.w
        counts = [int(x) for x in counts]
        T = sum(counts)
        starts_host = [s.current_len for s in states]
        if max(starts_host[i] + counts[i] for i in range(len(counts))) > c.positions:
            raise ValueError(f"GPT-2 position table has {c.positions} rows")
        start = pool.reserve(states, counts)
        index = pool.batch_index(states, counts)
        table, lens = pool.block_table(states)
        pos = torch.cat([torch.arange(s0, s0 + n, device=self.device)
                         for s0, n in zip(starts_host, counts)])
        decode = all(n == 1 for n in counts)
        if decode:
            pps = att.default_pages_per_split(len(states), c.heads, table.shape[1], n_prefix_pages)
            need = att.decode_workspace_bytes(len(states), c.heads, c.head_dim, table.shape[1],
                                              pps, n_prefix_pages)
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        else:
            cu = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32,
                              device=self.device)
        last = torch.tensor(counts, device=self.device).cumsum(0) - 1
        x = w["wte"][tokens.to(self.device)] + w["wpe"][pos]
        for l in range(c.layers):
            h = self._ln(x, f"{l}.ln_1")
            qkv = (h @ w[f"{l}.attn.w"] + w[f"{l}.attn.b"]).to(torch.bfloat16)
            q = torch.empty((T, c.heads, c.head_dim), dtype=torch.bfloat16, device=self.device)
            pool.write_qkv(states, start, l, qkv, q, counts, index=index)   # no rotary in GPT-2
            kp, vp = pool.layer_pages(l)
            if decode:
                a = att.paged_decode(q, kp, vp, table, lens, num_prefix_pages=n_prefix_pages,
                                     pages_per_split=pps, workspace=self._ws)
            else:
                a = att.prefill_paged(q, kp, vp, table, cu, lens, max(counts))
            a = a.reshape(T, c.d_model).to(self.dtype)
            if attn_last is not None:
                attn_last.append(a[last])
            x = x + a @ w[f"{l}.proj.w"] + w[f"{l}.proj.b"]
            h = self._ln(x, f"{l}.ln_2")
            x = x + F.gelu(h @ w[f"{l}.fc.w"] + w[f"{l}.fc.b"], approximate="tanh") @ w[f"{l}.fc2.w"] \
                + w[f"{l}.fc2.b"]
        return self._ln(x[last], "ln_f") @ w["wte"].t()

    # -- AgentExecutor model contract ------------------------------------------------------
    def prefill(self, tokens: torch.Tensor, kv_state: KVState, attention=None) -> torch.Tensor:
        """Append ``tokens`` to the session; last-position logits ``[1, vocab]``."""
        return self.forward(tokens.to(self.device).long(), kv_state.pool, [kv_state], [tokens.numel()])

    def decode(self, tokens: torch.Tensor, kv_state: KVState, attention=None) -> torch.Tensor:
        return self.forward(tokens.to(self.device).long(), kv_state.pool, [kv_state], [1])


@dataclass
class ReactTrace:
    choices: List[int]                       # greedy argmax after every prompt / decode position
    tables: List[List[int]]                  # the session's block-table row after each step
    lengths: List[int]
    attn_last: List[torch.Tensor]            # per chunk [layers, d_model] (when recorded)


def run_react(model: GPT2Model, prefix: Sequence[int], prompts: Sequence[Sequence[int]],
              tools: Sequence[Sequence[int]], decode_tokens: int = 32,
              forced: Optional[Sequence[int]] = None, record: bool = False,
              num_pages: Optional[int] = None) -> ReactTrace:
    """Batch-1 ReAct program: ``prefix`` written once into a root session and forked (its pages
    shared), then per step: the prompt chunk, ``decode_tokens`` greedy decodes, the step's tool
    output (when there is one).  ``forced`` replaces the greedy tokens fed back (teacher
    forcing); the argmax choices are recorded either way."""
    c = model.cfg
    per_seq = -(-c.positions // LF_PAGE_SIZE)
    pool = model.new_pool(num_pages or 2 * per_seq, max_slots=2)
    n_prefix_pages = len(prefix) // LF_PAGE_SIZE
    tr = ReactTrace([], [], [], [])
    dev = model.device

    def run(st, ids, prefix_pages=0):
        rec: Optional[List[torch.Tensor]] = [] if record else None
        logits = model.forward(torch.tensor(list(ids), dtype=torch.long, device=dev), pool, [st],
                               [len(ids)], n_prefix_pages=prefix_pages, attn_last=rec)
        if record:
            tr.attn_last.append(torch.stack([r[0] for r in rec]).float().cpu())
        return logits

    root = pool.alloc()
    run(root, prefix)
    seq = pool.fork(root, len(prefix), n=1)[0]
    k = 0
    for step, prompt in enumerate(prompts):
        logits = run(seq, prompt)
        for _ in range(decode_tokens):
            tok = int(torch.argmax(logits[0]))
            tr.choices.append(tok)
            logits = run(seq, [forced[k] if forced is not None else tok], n_prefix_pages)
            k += 1
        if step < len(tools):
            run(seq, tools[step])
        tr.tables.append(pool.snapshot()["block_table"][seq.slot_id])
        tr.lengths.append(seq.current_len)
    pool.release_all([seq, root])
    return tr
