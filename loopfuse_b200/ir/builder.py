"""Fluent builder for agent programs (ReAct steps), API-compatible with the reference.

``add_react_step`` lays out one step the way the reference builder does
(``ir/builder.py:40-100``): observe = prompt construction; reason = LLM
forward (PREFILL with ``system_prompt_len`` tokens on the first step, DECODE
of one token otherwise), a KV write at ``seq_pos = step_id * seq_len`` and an
argmax; act = action parse plus an optional tool call.
"""
from __future__ import annotations

from typing import Any, Dict, Optional

from .dialect import (AgentProgram, AgentStepOp, ArgmaxOp, KernelTarget, KVWriteOp,
                      LLMForwardOp, ParseActionOp, Phase, PromptConstructOp, TensorType,
                      TokenSeqType, ToolCallOp, Value)


class AgentProgramBuilder:
    def __init__(self, name: str, model_config: Dict[str, Any], kv_cache_config: Dict[str, Any]):
        self._prog = AgentProgram(name, model_config, kv_cache_config)
        self._cfg = model_config

    def add_react_step(self, step_id: int, tool_name: Optional[str] = "search",
                       tool_latency_ms: float = 100.0, is_first_step: bool = False,
                       system_prompt_len: int = 64) -> "AgentProgramBuilder":
        cfg, kv = self._cfg, self._prog.kv_state
        vocab = cfg["vocab_size"]
        prompt = PromptConstructOp(Value(f"obs_{step_id}", TokenSeqType(512, vocab)),
                                   Value(f"mem_{step_id}", TokenSeqType(512, vocab)),
                                   template="react_v1")
        phase = Phase.PREFILL if is_first_step else Phase.DECODE
        seq_len = system_prompt_len if is_first_step else 1
        fwd = LLMForwardOp(prompt.result(), kv, cfg, phase=phase, seq_len=seq_len)
        kv_shape = (cfg["num_layers"], cfg.get("num_kv_heads", cfg["num_heads"]), seq_len,
                    cfg["head_dim"])
        write = KVWriteOp(kv, Value(f"keys_{step_id}", TensorType(kv_shape, "fp16")),
                          Value(f"vals_{step_id}", TensorType(kv_shape, "fp16")),
                          seq_pos=step_id * seq_len, step_id=step_id)
        parse = ParseActionOp(Value(f"action_toks_{step_id}", TokenSeqType(64, vocab)),
                              action_schema="react_action_v1")
        act = [parse]
        if tool_name is not None:
            act.append(ToolCallOp(tool_name, parse.result(), estimated_latency_ms=tool_latency_ms,
                                  step_id=step_id))
        self._prog.add_step(AgentStepOp(step_id, observe_ops=[prompt],
                                        reason_ops=[fwd, write, ArgmaxOp(fwd.result())],
                                        act_ops=act))
        return self

    def add_custom_step(self, step: AgentStepOp) -> "AgentProgramBuilder":
        self._prog.add_step(step)
        return self

    def set_target(self, target: KernelTarget) -> "AgentProgramBuilder":
        self._prog.set_target(target)
        return self

    def build(self) -> AgentProgram:
        return self._prog
