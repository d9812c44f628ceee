"""Agent-program executor that actually dispatches the phase kernels.

Drop-in for the reference's ``runtime/executor.py``.  The reference walks the
steps and regions, times each op into a ``StepTrace`` and routes ops by type
(``:125-213``), but its LLM forward only synchronises (``:220-231``) and all
four ``_dispatch_*`` methods are ``pass`` (``:278-281``).  Here:

* ``_exec_llm_forward`` resolves the op's ``kernel_module``/``kernel_name``
  annotation (written by ``PhaseSelectPass``) to this package's sm_100a
  attention and runs the model's prefill (PREFILL ops) or greedy decode loop
  (DECODE ops, up to ``max_decode_tokens``) with it; KV lands in the paged pool.
* ``_dispatch_cuda`` is that path; TRITON / PALLAS / EAGER raise
  ``NotImplementedError`` -- no silent fallback.
* Speculative prefill (``:238-249``) runs the model's prefill of the predicted
  next-step tokens on the pool's low-priority stream while the tool call's
  host latency elapses, on a branch forked from the session (``KVPool.fork``
  shares the confirmed context).  The next PREFILL op compares its tokens with
  the predicted ones: a hit adopts the branch (``KVPool.adopt``) and skips the
  prefill, a miss releases the branch's pages.  Any other LLM op first waits
  for the speculation, since both streams update the pool's metadata.
* ``StepTrace`` keeps the reference's wall-clock fields and adds CUDA-event
  GPU times.
* A ``KVFuseOp`` (``passes.kv_fusion.KVFusionPass``) arms prefix sharing by
  content for the program's first prefill: the prompt's leading pages whose
  token hashes an earlier run registered are mapped onto that run's pages
  (``KVPool.dedup_prefix``), only the rest is prefilled, and this run's first
  ``prefix_len`` tokens are registered (``KVPool.register_prefix``).

Model contract (duck-typed): ``model.prefill(tokens, kv_state, attention)``
appends the tokens' K/V to the pool and returns last-position logits;
``model.decode(tokens, kv_state, attention)`` does the same for one token.
``attention`` is the resolved kernel.  ``model.prompt_tokens(step, observation)``
and ``model.spec_tokens(step)`` supply token ids when present.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

import torch

from ..ir.dialect import (AgentProgram, AgentStepOp, ArgmaxOp, KernelTarget, KVFuseOp,
                          KVWriteOp, LLMForwardOp, Op, ParseActionOp, Phase, PromptConstructOp,
                          SpeculativePrefillOp, ToolCallOp)
from ..passes.phase_select import PHASE_KERNEL_MAP, resolve_kernel
from .kv_pool import KVPool, KVState


@dataclass
class StepTrace:
    step_id: int
    prefill_ms: float = 0.0
    decode_ms: float = 0.0
    kv_write_ms: float = 0.0
    tool_io_ms: float = 0.0
    prompt_construct_ms: float = 0.0
    parse_action_ms: float = 0.0
    spec_prefill_ms: float = 0.0
    spec_prefill_hit: bool = False
    prefill_tokens: int = 0
    prefix_hit_tokens: int = 0                  # prompt tokens served from shared pages
    total_ms: float = 0.0
    gpu_prefill_ms: float = 0.0
    gpu_decode_ms: float = 0.0
    output_tokens: List[int] = field(default_factory=list)

    def gpu_active_ms(self) -> float:
        return self.prefill_ms + self.decode_ms + self.kv_write_ms

    def gpu_idle_ms(self) -> float:
        return self.tool_io_ms + self.prompt_construct_ms + self.parse_action_ms

    def idle_pct(self) -> float:
        return 0.0 if self.total_ms == 0 else 100.0 * self.gpu_idle_ms() / self.total_ms


@dataclass
class ExecutionResult:
    output: str
    step_traces: List[StepTrace]
    total_ms: float
    n_steps: int

    def phase_summary(self) -> Dict[str, float]:
        t = self.step_traces
        return {"prefill_ms": sum(x.prefill_ms for x in t), "decode_ms": sum(x.decode_ms for x in t),
                "kv_write_ms": sum(x.kv_write_ms for x in t),
                "tool_io_ms": sum(x.tool_io_ms for x in t),
                "prompt_ms": sum(x.prompt_construct_ms for x in t),
                "parse_ms": sum(x.parse_action_ms for x in t),
                "spec_ms": sum(x.spec_prefill_ms for x in t),
                "gpu_prefill_ms": sum(x.gpu_prefill_ms for x in t),
                "gpu_decode_ms": sum(x.gpu_decode_ms for x in t)}

    def avg_idle_pct(self) -> float:
        return sum(t.idle_pct() for t in self.step_traces) / max(1, len(self.step_traces))


class AgentExecutor:
    """Execute a compiled ``AgentProgram`` with a model whose attention runs on sm_100a."""

    def __init__(self, model: Any, kv_pool: KVPool, tools: Dict[str, Callable[[str], str]],
                 target: KernelTarget = KernelTarget.CUDA, device: str = "cuda",
                 max_decode_tokens: int = 64, prefix_cache: bool = True):
        self.model = model
        self.kv_pool = kv_pool
        self.tools = tools
        self.target = target
        self.device = device
        self.max_decode_tokens = max_decode_tokens
        self._dispatch = self._build_dispatch_table()
        self._last_token: Optional[int] = None
        self._spec: Optional[dict] = None
        self.prefix_cache = prefix_cache
        self._fuse_len = 0                          # prefix_len of the program's KVFuseOp

    # -- top level -------------------------------------------------------------
    def run(self, prog: AgentProgram, initial_input: str) -> ExecutionResult:
        state = self.kv_pool.allocate_slot()
        self._fuse_len = 0
        traces: List[StepTrace] = []
        output = ""
        t0 = time.perf_counter()
        try:
            obs = initial_input
            for step in prog.steps:
                trace = self._execute_step(step, state, obs, prog)
                traces.append(trace)
                if trace.output_tokens:
                    output = self._decode_tokens(trace.output_tokens)
                obs = output
                state.advance_step()
        finally:
            self._drop_speculation(state)
            self.kv_pool.release(state)
        return ExecutionResult(output, traces, (time.perf_counter() - t0) * 1000, len(traces))

    def _execute_step(self, step: AgentStepOp, kv_state: KVState, observation: str,
                      prog: AgentProgram) -> StepTrace:
        trace = StepTrace(step_id=step.step_id)
        t0 = time.perf_counter()
        for region in step.regions():
            for op in region:
                self._dispatch_op(op, kv_state, trace, observation, prog, step)
        trace.total_ms = (time.perf_counter() - t0) * 1000
        return trace

    def _dispatch_op(self, op: Op, kv_state: KVState, trace: StepTrace, observation: str,
                     prog: AgentProgram, step: Optional[AgentStepOp] = None) -> None:
        t0 = time.perf_counter()
        if isinstance(op, PromptConstructOp):
            self._exec_prompt_construct(op, observation)
            trace.prompt_construct_ms += (time.perf_counter() - t0) * 1000
        elif isinstance(op, LLMForwardOp):
            gpu_ms = self._dispatch[self.target](op, kv_state, prog, trace, step)
            dt = (time.perf_counter() - t0) * 1000
            if op.phase == Phase.PREFILL:
                trace.prefill_ms += dt
                trace.gpu_prefill_ms += gpu_ms
            else:
                trace.decode_ms += dt
                trace.gpu_decode_ms += gpu_ms
        elif isinstance(op, KVWriteOp):
            self._exec_kv_write(op, kv_state)
            trace.kv_write_ms += (time.perf_counter() - t0) * 1000
        elif isinstance(op, KVFuseOp):
            # Arms the content-addressed prefix sharing of the next (first) prefill.
            self._fuse_len = int(op.attrs.get("prefix_len", 0))
            trace.kv_write_ms += (time.perf_counter() - t0) * 1000
        elif isinstance(op, SpeculativePrefillOp):
            self._exec_spec_prefill(op, kv_state, prog, step)
            trace.spec_prefill_ms += (time.perf_counter() - t0) * 1000
        elif isinstance(op, ToolCallOp):
            self._exec_tool_call(op)
            trace.tool_io_ms += (time.perf_counter() - t0) * 1000
        elif isinstance(op, ArgmaxOp):
            pass                                    # fused into the decode loop
        elif isinstance(op, ParseActionOp):
            self._exec_parse_action(op)
            trace.parse_action_ms += (time.perf_counter() - t0) * 1000

    # -- op executors ------------------------------------------------------------
    def _exec_prompt_construct(self, op: PromptConstructOp, observation: str) -> str:
        return f"[{op.attrs.get('template', 'react_v1')}] Observation: {observation}\nThought:"

    def _kernel_for(self, op: LLMForwardOp) -> Callable:
        phase = op.phase or Phase.DECODE
        module = op.metadata.get("kernel_module")
        name = op.metadata.get("kernel_name")
        if module is None:                          # not annotated: use the selection table
            module, name, _ = PHASE_KERNEL_MAP[(self.target, phase)]
        return resolve_kernel(module, name, op.target or self.target)

    def _exec_llm_forward(self, op: LLMForwardOp, kv_state: KVState, prog: AgentProgram,
                          trace: StepTrace, step: Optional[AgentStepOp] = None) -> float:
        """Run the phase's kernel through the model; returns GPU milliseconds."""
        kernel = self._kernel_for(op)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        if op.phase == Phase.PREFILL:
            tokens = self._prompt_tokens(step, op)
            if not self._consume_speculation(kv_state, tokens, trace):
                fuse = self.prefix_cache and self._fuse_len >= 16 and kv_state.current_len == 0
                covered = 0
                if fuse:
                    # Leading pages another run already computed; one token is always left to
                    # prefill, since its logits start the decode.
                    covered = self.kv_pool.dedup_prefix([kv_state], [tokens[:-1].tolist()])[0]
                logits = self.model.prefill(tokens[covered:], kv_state, kernel)
                self._last_token = int(torch.argmax(logits[-1]).item())
                trace.prefill_tokens += int(tokens.numel()) - covered
                trace.prefix_hit_tokens += covered
                if fuse:
                    self.kv_pool.register_prefix(kv_state, tokens[: self._fuse_len].tolist())
        else:
            self._join_speculation()
            last = self._last_token if self._last_token is not None else 0
            out = []
            for _ in range(self.max_decode_tokens):
                if kv_state.current_len >= self.kv_pool.max_seq_len:
                    break
                logits = self.model.decode(torch.tensor([last], device=self.kv_pool.device),
                                           kv_state, kernel)
                last = int(torch.argmax(logits[-1]).item())
                out.append(last)
            self._last_token = last
            trace.output_tokens.extend(out)
        end.record()
        end.synchronize()
        return start.elapsed_time(end)

    def _prompt_tokens(self, step: Optional[AgentStepOp], op: LLMForwardOp) -> torch.Tensor:
        if hasattr(self.model, "prompt_tokens"):
            return self.model.prompt_tokens(step.step_id if step else 0, op.seq_len)
        return torch.zeros(op.seq_len, dtype=torch.long, device=self.kv_pool.device)

    def _exec_kv_write(self, op: KVWriteOp, kv_state: KVState) -> None:
        """KV is appended by the model's forward (fused into the attention step)."""
        return None

    def _exec_spec_prefill(self, op: SpeculativePrefillOp, kv_state: KVState,
                           prog: AgentProgram, step: Optional[AgentStepOp] = None) -> None:
        """Prefill the predicted next prompt on the low-priority stream, on a forked session."""
        if op.metadata.get("confidence", 0.0) < 0.5 or not hasattr(self.model, "spec_tokens"):
            return
        if not self.kv_pool._free_slots:
            return
        if self._spec is not None:                  # one speculation in flight at a time
            self._drop_speculation(kv_state)
        tokens = self.model.spec_tokens(step.step_id if step else 0)
        branch = self.kv_pool.fork(kv_state, kv_state.current_len, n=1)[0]
        kernel = self._kernel_for(LLMForwardOp(op.operands[0], op.operands[1], op.attrs,
                                               phase=Phase.PREFILL, seq_len=len(tokens)))
        done = torch.cuda.Event()
        # The branch's pages and the context it attends to were written on this stream.
        self.kv_pool.prefetch_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.kv_pool.prefetch_stream):
            logits = self.model.prefill(tokens, branch, kernel)
            done.record()
        self._spec = {"branch": branch, "tokens": tokens, "logits": logits, "event": done}

    def _consume_speculation(self, kv_state: KVState, tokens: torch.Tensor,
                             trace: StepTrace) -> bool:
        spec = self._spec
        if spec is None:
            return False
        self._spec = None
        hit = (spec["tokens"].shape == tokens.shape and
               bool(torch.equal(spec["tokens"].to(tokens.device), tokens)))
        torch.cuda.current_stream().wait_event(spec["event"])
        if not hit:
            self.kv_pool.release(spec["branch"])
            return False
        # Adopt the speculative branch: its pages already hold the prompt's K/V.
        self.kv_pool.adopt(kv_state, spec["branch"])
        self._last_token = int(torch.argmax(spec["logits"][-1]).item())
        trace.spec_prefill_hit = True
        return True

    def _join_speculation(self) -> None:
        """Order this stream's next pool operations after an in-flight speculative prefill:
        both streams update the same pool metadata."""
        if self._spec is not None:
            torch.cuda.current_stream().wait_event(self._spec["event"])

    def _drop_speculation(self, kv_state: KVState) -> None:
        if self._spec is not None:
            torch.cuda.current_stream().wait_event(self._spec["event"])
            self.kv_pool.release(self._spec["branch"])
            self._spec = None

    def _exec_tool_call(self, op: ToolCallOp) -> str:
        fn = self.tools.get(op.tool_name)
        if fn is None:
            return f"[tool '{op.tool_name}' not found]"
        try:
            return fn("")
        except Exception as e:                     # tool failures become observations
            return f"[tool error: {e}]"

    def _exec_parse_action(self, op: ParseActionOp) -> dict:
        return {"action": "unknown", "input": ""}

    def _decode_tokens(self, tokens: List[int]) -> str:
        return " ".join(str(t) for t in tokens)

    # -- dispatch ------------------------------------------------------------------
    def _build_dispatch_table(self) -> dict:
        return {KernelTarget.TRITON: self._dispatch_triton, KernelTarget.CUDA: self._dispatch_cuda,
                KernelTarget.PALLAS: self._dispatch_pallas, KernelTarget.EAGER: self._dispatch_eager}

    def _dispatch_cuda(self, op, kv_state, prog, trace, step=None) -> float:
        return self._exec_llm_forward(op, kv_state, prog, trace, step)

    def _unsupported(self, target: KernelTarget):
        raise NotImplementedError(f"target {target.value} does not execute in loopfuse_b200; "
                                  f"compile with KernelTarget.CUDA (sm_100a)")

    def _dispatch_triton(self, op, *args):
        self._unsupported(KernelTarget.TRITON)

    def _dispatch_pallas(self, op, *args):
        self._unsupported(KernelTarget.PALLAS)

    def _dispatch_eager(self, op, *args):
        self._unsupported(KernelTarget.EAGER)
