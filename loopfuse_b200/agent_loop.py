"""Many concurrent ReAct agent sessions on one GPU: batched prefill / decode with tool waits.

This is the runtime side of the reference's agent programs (``runtime/executor.py`` runs one
program's steps sequentially; ``passes/spec_prefill.py:59-124`` inserts speculative prefills
before tool calls).  Every session runs ``steps`` ReAct steps: the observation tokens (the
user question on the first step, the previous tool's output after that) are prefilled, the
model decodes ``decode_tokens`` tokens (thought + action), then the tool runs on the host for an
exponentially distributed latency (mean ``tool_ms``) while the GPU serves other sessions.

Scheduling (one host thread per GPU, a loop of GPU batches):
  1. sessions whose tool has returned move to "prefill";
  2. if sessions wait for prefill -- and, while others are decoding, either at least
     ``min_prefill_tokens`` tokens are pending or the oldest request has waited
     ``max_prefill_wait_ms`` -- one varlen prefill batch of them (capped at
     ``max_prefill_tokens``) runs and yields each session's first decoded token;
  3. otherwise one decode iteration advances every decoding session by one token; sessions
     that finish their thought/action start their tool call;
  4. if nothing is runnable, the GPU would idle until the next tool returns: speculative
     prefill fills that window.  Every observation begins with the same template tokens
     ("Observation:"), so while a session's tool runs, those ``spec_tokens`` tokens are
     prefilled ahead of time (on the pool's low-priority stream); when the tool returns only
     the tool output itself is left to prefill.
The system prompt (``prefix_tokens``) is prefilled once (``setup``, before the loop) and forked
to every session, so the decode attention reads it once per group of sessions.  Decode
iterations replay CUDA graphs (``llama.GraphedDecode``), one per batch-size bucket, captured in
``setup``; prefill batches run eagerly.

Token ids are synthetic (seeded uniform ids; tool outputs of geometric length, mean
``tool_len_mean``, capped).  The reported metric is agent steps per second: completed ReAct
steps of all sessions divided by the wall time of the loop.
"""
from __future__ import annotations

import heapq
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from .llama import GraphedDecode, LlamaShaped
from .runtime.kv_pool import KVPool, KVState

PAGE = 16


@dataclass
class AgentLoopConfig:
    sessions: int = 512
    steps: int = 10
    prefix_tokens: int = 4096
    question_tokens: int = 128
    decode_tokens: int = 32
    tool_ms: float = 100.0
    tool_len_mean: float = 120.0
    tool_len_cap: int = 1024
    spec_tokens: int = 4
    speculative: bool = True
    graphs: bool = True              # decode iterations replayed from CUDA graphs
    max_prefill_tokens: int = 16384
    # While sessions are decoding, a prefill batch waits until this many tokens are pending or
    # its oldest request has waited max_prefill_wait_ms: each forward reads all the weights, so
    # tiny prefill batches (a few returning tools at a time) cost a whole forward each.
    min_prefill_tokens: int = 2048
    max_prefill_wait_ms: float = 25.0
    seed: int = 0


@dataclass
class _Sess:
    idx: int
    state: KVState
    pos: int = 0
    step: int = 0
    phase: str = "prefill"          # prefill | decode | tool | done
    pending: List[int] = field(default_factory=list)
    decoded: int = 0
    last_token: int = 0
    spec_done: bool = False
    ready_at: float = 0.0
    pending_since: float = 0.0


@dataclass
class AgentLoopStats:
    sessions: int = 0
    steps_done: int = 0
    wall_s: float = 0.0
    steps_per_s: float = 0.0
    prefill_batches: int = 0
    decode_iters: int = 0
    spec_batches: int = 0
    spec_tokens: int = 0
    prefill_tokens: int = 0
    decode_tokens: int = 0
    gpu_busy_s: float = 0.0
    prefill_s: float = 0.0
    decode_s: float = 0.0
    spec_s: float = 0.0
    idle_waits: int = 0
    kernels: Optional[dict] = None     # per-kernel-class attribution (run(profile_ops=True))
    final_lengths: List[int] = field(default_factory=list)   # tokens per session at the end


class AgentLoop:
    PROFILE_SESSIONS = 64        # sessions in the attributed prefill batch
    PROFILE_PREFILL = 128        # new tokens per session in it (about one tool output)

    def __init__(self, model: LlamaShaped, cfg: AgentLoopConfig, session_ids: Optional[List[int]] = None,
                 device=None):
        self.model, self.cfg = model, cfg
        self.device = torch.device(device or model.device)
        self.ids = list(range(cfg.sessions)) if session_ids is None else list(session_ids)
        rng = np.random.default_rng(cfg.seed)
        # per (global session id, step) tool-output lengths and latencies: the same on every rank
        self.tool_len = np.minimum(rng.geometric(1.0 / cfg.tool_len_mean,
                                                 size=(cfg.sessions, cfg.steps)), cfg.tool_len_cap)
        self.tool_lat = rng.exponential(cfg.tool_ms / 1000.0, size=(cfg.sessions, cfg.steps))
        self.vocab = model.cfg.vocab
        self.template = [int(x) for x in rng.integers(0, self.vocab, size=cfg.spec_tokens)]
        n = len(self.ids)
        own = [cfg.question_tokens + int(self.tool_len[i].sum()) +
               cfg.steps * (cfg.decode_tokens + cfg.spec_tokens) for i in self.ids]
        # slack past the longest session: the per-kernel attribution forwards after the loop
        # append up to 2 decode tokens and one 128-token prefill chunk to a session
        max_len = cfg.prefix_tokens + max(own) + 64 + 2 + self.PROFILE_PREFILL
        self.n_prefix_pages = cfg.prefix_tokens // PAGE
        pages = self.n_prefix_pages + sum((o + PAGE - 1) // PAGE + 1 for o in own) + 16 + \
            n + min(n, self.PROFILE_SESSIONS) * (self.PROFILE_PREFILL // PAGE + 1)
        mc = model.cfg
        self.pool = KVPool(num_layers=mc.layers, num_heads=mc.q_heads, num_kv_heads=mc.kv_heads,
                           head_dim=mc.head_dim, max_seq_len=max_len, max_slots=n + 2,
                           dtype=torch.bfloat16, device=self.device, num_pages=pages + 1)
        self.rng = np.random.default_rng(cfg.seed + 17)
        self.root: Optional[KVState] = None
        self.gd: Optional[GraphedDecode] = None

    def _ids_tensor(self, toks: List[int]) -> torch.Tensor:
        return torch.tensor(toks, dtype=torch.long).to(self.device, non_blocking=True)

    def _run(self, sess: List[_Sess], chunks: List[List[int]], stats: AgentLoopStats) -> List[int]:
        toks = [t for ch in chunks for t in ch]
        t0 = time.perf_counter()
        nxt = self.model.forward(self._ids_tensor(toks), self.pool, [s.state for s in sess],
                                 [len(ch) for ch in chunks], n_prefix_pages=self.n_prefix_pages)
        out = nxt.tolist()                          # one host sync per batch
        stats.gpu_busy_s += time.perf_counter() - t0
        return out

    def setup(self) -> None:
        """System prompt prefilled once into a root session (forked to every session when the
        loop runs); with ``graphs``, a padding session and the decode graphs of every batch
        bucket up to the session count."""
        cfg, pool = self.cfg, self.pool
        self.root = pool.alloc()
        sys_prompt = [int(x) for x in self.rng.integers(0, self.vocab, size=cfg.prefix_tokens)]
        self._run([_Sess(-1, self.root)], [sys_prompt], AgentLoopStats())
        if cfg.graphs:
            pad = pool.pad_session(self.root, cfg.prefix_tokens)
            self.gd = GraphedDecode(self.model, pool, pad, self.n_prefix_pages)
            self.gd.prepare(len(self.ids))
        torch.cuda.synchronize(self.device)

    def _decode(self, sess: List[_Sess], stats: AgentLoopStats) -> List[int]:
        if self.gd is None:
            return self._run(sess, [[s.last_token] for s in sess], stats)
        t0 = time.perf_counter()
        nxt = self.gd.step([s.state for s in sess], [s.last_token for s in sess])
        out = nxt[:len(sess)].tolist()
        self.gd.raise_if_failed()
        stats.gpu_busy_s += time.perf_counter() - t0
        return out

    # -- per-kernel attribution ------------------------------------------------------------------
    def _op_work(self, T: int, n_out: int, attn_flops: float, attn_bytes: float) -> dict:
        """Algorithmic (FLOPs, HBM bytes) per op class of one forward of ``T`` new tokens
        (``n_out`` sessions' last positions go through the LM head), summed over the layers."""
        c = self.model.cfg
        d, f, V, L = c.d_model, c.ffn, c.vocab, c.layers
        nq, nkv = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
        qkv = nq + 2 * nkv

        def gemm(m, k, n):
            return 2.0 * m * k * n, 2.0 * (k * n + m * k + m * n)
        w = {"qkv_gemm": gemm(T, d, qkv), "o_gemm": gemm(T, nq, d),
             "gate_up_gemm": gemm(T, d, 2 * f), "down_gemm": gemm(T, f, d)}
        out = {k: (L * v[0], L * v[1]) for k, v in w.items()}
        out["qkv_rope_append"] = (0.0, L * 2.0 * T * (qkv + nq + 2 * nkv))
        out["attention"] = (attn_flops, attn_bytes)
        out["add_rmsnorm"] = (0.0, L * 2 * 4.0 * T * d * 2)
        out["swiglu"] = (0.0, L * 2.0 * T * 3 * f)
        out["lm_head"] = gemm(n_out, d, V)
        return out

    def _profile_ops(self, sessions: List["_Sess"], decode_steps: int = 2) -> dict:
        """Per-kernel-class time and roofline of one decode iteration over every session of this
        rank and of one prefill batch (``PROFILE_PREFILL`` new tokens for each of up to
        ``PROFILE_SESSIONS`` sessions, about one tool output each), both at the sessions' final
        lengths.  Eager forwards timed op by op with CUDA events; the stream is held by a
        device-side spin while the host enqueues, so host gaps are not charged."""
        from .analysis import kernel_roofline
        from .llama import OpTimer
        c, pool = self.model.cfg, self.pool
        kv_tok = 2 * c.kv_heads * c.head_dim * 2 * c.layers           # K+V bytes per token
        res = {}
        for phase in ("decode", "prefill"):
            chosen = sessions if phase == "decode" else sessions[:self.PROFILE_SESSIONS]
            states = [s.state for s in chosen]
            n = len(states)
            per = 1 if phase == "decode" else self.PROFILE_PREFILL
            reps = decode_steps if phase == "decode" else 1
            acc: dict = {}
            ctx = [st.current_len for st in states]
            for _ in range(reps):
                timer = OpTimer()
                toks = torch.randint(0, self.vocab, (n * per,), device=self.device)
                torch.cuda.synchronize(self.device)
                timer.start(hold_cycles=200_000_000)
                self.model.forward(toks, pool, states, [per] * n, n_prefix_pages=self.n_prefix_pages,
                                   timer=timer)
                torch.cuda.synchronize(self.device)
                for k, v in timer.totals().items():
                    acc[k] = acc.get(k, 0.0) + v / reps
            pre = self.n_prefix_pages * PAGE
            if phase == "decode":
                own = sum(max(0, L + 1 - pre) for L in ctx)
                a_bytes = float(kv_tok * (own + min(pre, max(ctx) + 1)))
                a_flops = 4.0 * c.q_heads * c.head_dim * c.layers * sum(L + 1 for L in ctx)
            else:
                a_bytes = float(kv_tok * (sum(max(0, L + per - pre) for L in ctx) + pre))
                pairs = sum(per * L + per * (per + 1) / 2 for L in ctx)
                a_flops = 4.0 * c.q_heads * c.head_dim * c.layers * pairs
            work = self._op_work(n * per, n, a_flops, a_bytes)
            total = sum(acc.values())
            ops = []
            for k, ms in sorted(acc.items(), key=lambda kv: -kv[1]):
                fl, by = work.get(k, (0.0, 0.0))
                r = kernel_roofline(k, fl, by, ms * 1e-3) if (fl or by) else {"kernel": k}
                r["ms"] = round(ms, 4)
                r["share"] = round(ms / total, 4) if total else None
                ops.append(r)
            res[phase] = {"sessions": n, "new_tokens": n * per, "ms": round(total, 3),
                          "mean_context": round(sum(ctx) / max(1, n), 1), "ops": ops}
        return res

    def run(self, profile_ops: bool = False) -> AgentLoopStats:
        cfg, pool = self.cfg, self.pool
        if self.root is None:
            self.setup()
        stats = AgentLoopStats(sessions=len(self.ids))
        t_start = time.perf_counter()
        root = self.root
        states = pool.fork(root, cfg.prefix_tokens, n=len(self.ids))
        sessions = [_Sess(i, st, k) for k, (i, st) in enumerate(zip(self.ids, states))]
        for s in sessions:
            s.pending = [int(x) for x in self.rng.integers(0, self.vocab, size=cfg.question_tokens)]
            s.pending_since = t_start
        tools: List = []                            # heap of (ready_at, idx in sessions)
        while True:
            now = time.perf_counter()
            while tools and tools[0][0] <= now:
                _, k = heapq.heappop(tools)
                s = sessions[k]
                out_len = int(self.tool_len[s.idx, s.step - 1])
                obs = [] if s.spec_done else list(self.template)
                s.pending = obs + [int(x) for x in self.rng.integers(0, self.vocab, size=out_len)]
                s.phase = "prefill"
                s.pending_since = now
            pre = [s for s in sessions if s.phase == "prefill"]
            dec = [s for s in sessions if s.phase == "decode"]
            if pre and dec:
                waited_ms = (now - min(s.pending_since for s in pre)) * 1000.0
                if (sum(len(s.pending) for s in pre) < cfg.min_prefill_tokens
                        and waited_ms < cfg.max_prefill_wait_ms):
                    pre = []                        # let more requests gather; decode meanwhile
            if pre:
                batch, budget = [], cfg.max_prefill_tokens
                for s in pre:
                    if batch and len(s.pending) > budget:
                        break
                    batch.append(s)
                    budget -= len(s.pending)
                t0 = time.perf_counter()
                nxt = self._run(batch, [s.pending for s in batch], stats)
                stats.prefill_s += time.perf_counter() - t0
                stats.prefill_batches += 1
                stats.prefill_tokens += sum(len(s.pending) for s in batch)
                for s, t in zip(batch, nxt):
                    s.pending, s.last_token, s.decoded, s.phase = [], t, 1, "decode"
                    s.spec_done = False
                continue
            if dec:
                t0 = time.perf_counter()
                nxt = self._decode(dec, stats)
                stats.decode_s += time.perf_counter() - t0
                stats.decode_iters += 1
                stats.decode_tokens += len(dec)
                now = time.perf_counter()
                for s, t in zip(dec, nxt):
                    s.last_token = t
                    s.decoded += 1
                    if s.decoded >= cfg.decode_tokens:
                        s.step += 1
                        stats.steps_done += 1
                        if s.step >= cfg.steps:
                            s.phase = "done"
                        else:
                            s.phase = "tool"
                            s.ready_at = now + float(self.tool_lat[s.idx, s.step - 1])
                            heapq.heappush(tools, (s.ready_at, s.pos))
                continue
            if not tools:
                break
            # idle window: speculative prefill of the observation template
            spec = [s for s in sessions if s.phase == "tool" and not s.spec_done] if cfg.speculative else []
            if spec:
                t0 = time.perf_counter()
                with torch.cuda.stream(pool.prefetch_stream):
                    self._run(spec, [list(self.template) for _ in spec], stats)
                torch.cuda.current_stream().wait_stream(pool.prefetch_stream)
                stats.spec_s += time.perf_counter() - t0
                for s in spec:
                    s.spec_done = True
                stats.spec_batches += 1
                stats.spec_tokens += len(spec) * cfg.spec_tokens
                continue
            stats.idle_waits += 1
            time.sleep(max(0.0, min(tools[0][0] - time.perf_counter(), 0.002)))
        torch.cuda.synchronize(self.device)
        stats.wall_s = time.perf_counter() - t_start
        stats.steps_per_s = stats.steps_done / stats.wall_s
        stats.final_lengths = [s.state.current_len for s in sessions]
        if profile_ops:                       # after the timed loop, on its final state
            stats.kernels = self._profile_ops(sessions)
        pool.release_all(states)
        return stats
