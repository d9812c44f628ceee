"""CPU GPT-2-small ReAct program through the reference's torch path (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

The reference has no GPT-2 implementation (its configs only name the shapes:
``ir/dialect.py:525-532``) and its "reference path" is ``scaled_dot_product_attention``
(``passes/phase_select.py:80-89``) with KV in its pool.  This restates that path for the
3-step ReAct program: GPT-2 small (12 layers, d_model 768, 12 heads of 64, ffn 3072, vocab
50257), random N(0, 0.02) fp32 weights, batch 1; a 512-token system prefix written once and
forked (KV fusion); per step 128 uniform-random prompt ids; tool outputs of 150 then 80 ids
appended after steps 0 and 1; 32 greedy decode tokens per step; KV in 16-token pages held by
the pool oracle.  The program is 512 + 3*128 + 150 + 80 + 3*32 = 1222 tokens, more than GPT-2's
1024 positions, so the learned position table has 1280 rows (a deliberate extension; the
weights are random, so nothing is lost).

``run()`` returns every token fed to the model in order (teacher-forcing input for another
implementation), the chunk boundaries, each chunk's per-layer attention output at its last
position, the final logits' argmax choices and the pool's block table after each step.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List

import torch
import torch.nn.functional as F

from .pool_spec import PAGE, PagedKVPoolSpec


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


def gpt2_weights(cfg: GPT2Config, seed: int = 0, std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Random fp32 weights, keyed as the GPU model expects them."""
    g = torch.Generator().manual_seed(seed)

    def n(*shape):
        return torch.randn(*shape, generator=g) * std
    d, f = cfg.d_model, cfg.ffn
    w = {"wte": n(cfg.vocab, d), "wpe": n(cfg.positions, d),
         "ln_f.w": torch.ones(d), "ln_f.b": torch.zeros(d)}
    for l in range(cfg.layers):
        w.update({f"{l}.ln_1.w": torch.ones(d), f"{l}.ln_1.b": torch.zeros(d),
                  f"{l}.attn.w": n(d, 3 * d), f"{l}.attn.b": torch.zeros(3 * d),
                  f"{l}.proj.w": n(d, d), f"{l}.proj.b": torch.zeros(d),
                  f"{l}.ln_2.w": torch.ones(d), f"{l}.ln_2.b": torch.zeros(d),
                  f"{l}.fc.w": n(d, f), f"{l}.fc.b": torch.zeros(f),
                  f"{l}.fc2.w": n(f, d), f"{l}.fc2.b": torch.zeros(d)})
    return w


@dataclass
class ProgramTrace:
    tokens: List[int] = field(default_factory=list)
    chunks: List[tuple] = field(default_factory=list)        # (kind, start, length)
    attn_last: List[torch.Tensor] = field(default_factory=list)   # per chunk [layers, d_model]
    choices: List[int] = field(default_factory=list)
    tables: List[list] = field(default_factory=list)         # block-table row after each step
    lengths: List[int] = field(default_factory=list)


class GPT2Program:
    PREFIX, PROMPT, DECODE, TOOLS = 512, 128, 32, (150, 80)

    def __init__(self, cfg: GPT2Config = GPT2Config(), seed: int = 0):
        self.cfg, self.w = cfg, gpt2_weights(cfg, seed)
        self.rng = torch.Generator().manual_seed(seed + 1)
        pages = math.ceil(cfg.positions / PAGE)
        self.pool = PagedKVPoolSpec(num_pages=2 * pages, max_seqs=2, max_pages_per_seq=pages,
                                    num_layers=cfg.layers, num_kv_heads=cfg.heads,
                                    head_dim=cfg.head_dim, dtype=torch.float32, with_data=True)

    def _ln(self, x, p):
        return F.layer_norm(x, (self.cfg.d_model,), self.w[p + ".w"], self.w[p + ".b"], self.cfg.eps)

    def _chunk(self, seq: int, ids: List[int], trace: ProgramTrace, kind: str) -> torch.Tensor:
        """Append ``ids`` to session ``seq``; returns logits of the last position."""
        c, w = self.cfg, self.w
        start = self.pool.seq_len[seq]
        T = len(ids)
        x = w["wte"][torch.tensor(ids)] + w["wpe"][start:start + T]
        ks, vs, attn_last = [], [], []
        self.pool.reserve([seq], [T])
        for l in range(c.layers):
            h = self._ln(x, f"{l}.ln_1")
            qkv = h @ w[f"{l}.attn.w"] + w[f"{l}.attn.b"]
            q, k, v = qkv.split(c.d_model, dim=-1)
            k = k.view(T, c.heads, c.head_dim)
            v = v.view(T, c.heads, c.head_dim)
            for t in range(T):                                 # this layer's new rows
                pos = start + t
                page = self.pool.block_table[seq][pos // PAGE]
                self.pool.k[l, page, :, pos % PAGE] = k[t]
                self.pool.v[l, page, :, pos % PAGE] = v[t]
            kc, vc = self.pool.session_kv(seq, l)              # [H, start+T, D]
            qh = q.view(T, c.heads, c.head_dim).permute(1, 0, 2)
            L = start + T
            mask = torch.arange(L)[None, :] <= (torch.arange(T)[:, None] + start)
            a = F.scaled_dot_product_attention(qh[None], kc[None], vc[None], attn_mask=mask[None, None])[0]
            a = a.permute(1, 0, 2).reshape(T, c.d_model)
            attn_last.append(a[-1].clone())
            x = x + a @ w[f"{l}.proj.w"] + w[f"{l}.proj.b"]
            h = self._ln(x, f"{l}.ln_2")
            x = x + F.gelu(h @ w[f"{l}.fc.w"] + w[f"{l}.fc.b"], approximate="tanh") @ w[f"{l}.fc2.w"] + w[f"{l}.fc2.b"]
        trace.tokens.extend(ids)
        trace.chunks.append((kind, start, T))
        trace.attn_last.append(torch.stack(attn_last))
        return self._ln(x[-1:], "ln_f") @ w["wte"].t()

    def _rand(self, n: int) -> List[int]:
        return torch.randint(0, self.cfg.vocab, (n,), generator=self.rng).tolist()

    def run(self) -> ProgramTrace:
        tr = ProgramTrace()
        root = self.pool.open_seq()
        self._chunk(root, self._rand(self.PREFIX), tr, "prefix")
        seq = self.pool.open_seq()
        self.pool.fork(root, [seq], self.PREFIX)              # KV fusion: the prefix is shared
        for step in range(3):
            logits = self._chunk(seq, self._rand(self.PROMPT), tr, "prompt")
            for _ in range(self.DECODE):
                tok = int(torch.argmax(logits[0]))
                tr.choices.append(tok)
                logits = self._chunk(seq, [tok], tr, "decode")
            if step < 2:
                self._chunk(seq, self._rand(self.TOOLS[step]), tr, "tool")
            tr.tables.append(list(self.pool.block_table[seq]))
            tr.lengths.append(self.pool.seq_len[seq])
        return tr
