"""KV-fusion pass -- drop-in for the reference's ``passes/kv_fusion.py`` (``KVFusionPass``).

Same constructor (``min_prefix_len=8, min_steps=2``), same ``run(prog) -> PassResult``, same
inserted op: a ``KVFuseOp`` (phase FUSE, compiler-inserted) at the head of step 0's reason
region, carrying ``prefix_len`` = the model config's ``system_prompt_len`` (default 64, at
least ``min_prefix_len``) and the fused step ids.

What differs is when it fires and what the op means.  The reference decides at compile time
from the IR's KV-write positions (``passes/kv_fusion.py:57-107``) and only fires when two or
more steps write at position 0 -- which a built ReAct program never has (only step 0 starts at
0), so on real programs it changes nothing.  Here the prefix is shared by content at run time:
the pass fires on any program of at least ``min_steps`` steps whose system prompt is at least
``min_prefix_len`` tokens, and ``AgentExecutor`` turns the op into pool operations --
``KVPool.dedup_prefix`` maps the longest run of the prompt's leading pages whose token hashes
are already registered (by an earlier run) onto those pages before the first prefill, and
``KVPool.register_prefix`` publishes this run's first ``prefix_len`` tokens afterwards.  A
wrong ``prefix_len`` can only cost sharing, never share K/V of different tokens.  The step-0
KV writes stay in the program (the first run computes them); the op records them as the writes
later runs skip, so ``bytes_saved`` is the reference's figure.
"""
from __future__ import annotations

import time

from ..ir.dialect import AgentProgram, KVFuseOp
from .base import Pass, PassResult


class KVFusionPass(Pass):
    def __init__(self, min_prefix_len: int = 8, min_steps: int = 2):
        self.min_prefix_len = min_prefix_len
        self.min_steps = min_steps

    def run(self, prog: AgentProgram) -> PassResult:
        start = time.time()
        if prog.ops_by_type(KVFuseOp) or len(prog.steps) < self.min_steps:
            return self._result(prog, False, [], start)
        prefix_len = max(self.min_prefix_len, int(prog.model_config.get("system_prompt_len", 64)))
        step0 = min(prog.steps, key=lambda s: s.step_id)
        prefix_writes = [w for w in step0.kv_write_ops() if w.attrs.get("seq_pos", 0) == 0]
        steps = [s.step_id for s in prog.steps]
        op = KVFuseOp(prog.kv_state, steps, prefix_len, prefix_writes)
        step0.reason_region.insert(0, op)
        note = (f"fused steps {steps} prefix_len={prefix_len}: system-prompt pages shared by "
                f"content across runs (saved={op.bytes_saved() // 1024}KB per reuse)")
        return self._result(prog, True, [note], start)
