"""Speculative-prefill insertion -- drop-in for the reference's ``passes/spec_prefill.py``.

Same constructor (``min_idle_window_ms=30, confidence_threshold=0.5,
estimated_prefill_ms=15``), same ``run(prog) -> PassResult`` and the same inserted op: a
``SpeculativePrefillOp`` placed immediately before a tool call whose idle window can hold a
prefill, so the executor overlaps the next step's prompt prefill with the tool's host latency
(``passes/spec_prefill.py:59-124``).  The decision rules and the annotation text follow the
reference so that programs compile to the same IR:

* a tool call qualifies when its idle window is at least ``min_idle_window_ms`` and, after a
  20% margin on the prefill estimate, still holds one prefill;
* confidence that the prediction survives the tool result starts at 0.85, drops 0.05 per step
  index, gains 0.05 for search / lookup tools and loses 0.15 for execute / run tools, clamped
  to [0, 1] (``:126-159``); calls below ``confidence_threshold`` are skipped;
* one speculative op per step (the first qualifying call), never a second one in front of a
  call that already has one (idempotent).

What the op does at run time is this package's: ``runtime.executor.AgentExecutor`` forks the
session, prefills the model's predicted tokens on the pool's low-priority stream, and adopts
the branch on a hit or frees its pages on a miss.
"""
from __future__ import annotations

import time
from typing import List

from ..ir.dialect import (AgentProgram, AgentStepOp, SpeculativePrefillOp, TokenSeqType,
                          ToolCallOp, Value)
from .base import Pass, PassResult

SPEC_TOKENS = 64          # token-sequence length of the predicted prompt value


class SpecPrefillPass(Pass):
    def __init__(self, min_idle_window_ms: float = 30.0, confidence_threshold: float = 0.50,
                 estimated_prefill_ms: float = 15.0):
        self.min_idle_window_ms = min_idle_window_ms
        self.confidence_threshold = confidence_threshold
        self.estimated_prefill_ms = estimated_prefill_ms

    def run(self, prog: AgentProgram) -> PassResult:
        start = time.time()
        notes: List[str] = []
        for step in prog.steps:
            for tool in step.tool_ops():
                note = self._try_insert(prog, step, tool)
                if note is not None:
                    notes.append(note)
                    break
        return self._result(prog, bool(notes), notes, start)

    def _try_insert(self, prog: AgentProgram, step: AgentStepOp, tool: ToolCallOp):
        window = tool.idle_window_ms()
        if window < self.min_idle_window_ms or self._already_covered(step, tool):
            return None
        conf = self._estimate_confidence(step, tool, prog)
        if conf < self.confidence_threshold:
            return None
        if window - 0.2 * self.estimated_prefill_ms < self.estimated_prefill_ms:
            return None
        predicted = Value(f"spec_toks_step{step.step_id}",
                          TokenSeqType(SPEC_TOKENS, prog.model_config["vocab_size"]))
        op = SpeculativePrefillOp(predicted, prog.kv_state, prog.model_config, conf, tool)
        if not step.insert_before(tool, op):
            return None
        overlap = min(100, self.estimated_prefill_ms / window * 100)
        return (f"inserted spec_prefill in step {step.step_id} (confidence={conf:.2f}, "
                f"window={window:.0f}ms, est_overlap={overlap:.0f}%)")

    @staticmethod
    def _already_covered(step: AgentStepOp, tool: ToolCallOp) -> bool:
        act = step.act_region
        i = act.index(tool) if tool in act else -1
        return i > 0 and isinstance(act[i - 1], SpeculativePrefillOp)

    @staticmethod
    def _estimate_confidence(step: AgentStepOp, tool: ToolCallOp, prog: AgentProgram) -> float:
        conf = 0.85 - 0.05 * step.step_id
        name = tool.tool_name.lower()
        if "search" in name or "lookup" in name:
            conf += 0.05
        elif "execute" in name or "run" in name:
            conf -= 0.15
        return max(0.0, min(1.0, conf))
