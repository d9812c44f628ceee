"""Agent-program IR: the types the kernel-selection pass and executor read.

This is the API host of ``Phase`` and ``KernelTarget``.  It keeps the
reference's public names, enum values, op names and cost estimators
(``ir/dialect.py:37-58, 90-110, 204-518`` of the reference) so that programs
built against the reference build the same way here and ``PhaseSelectPass``
annotates them identically.  The op classes carry only what the hot path and
its tests use: operands, results, ``phase``, ``target``, ``attrs`` and
``metadata``.

Added here: ``num_kv_heads`` on ``KVCacheType`` (defaults to
``num_heads``, so existing callers are unchanged) and the Llama-3-8B configs
used by the B200 workloads.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass
from enum import Enum
from typing import Any, Dict, List, Optional, Tuple

_BYTES = {"bf16": 2, "fp16": 2, "fp32": 4, "int8": 1, "int32": 4}


class Phase(Enum):
    """Execution phase of an op: the first key of kernel selection."""
    PREFILL = "prefill"
    DECODE = "decode"
    IO = "io"
    FUSE = "fuse"


class KernelTarget(Enum):
    """Backend a program is compiled for.  Only CUDA executes in this package."""
    TRITON = "triton"
    CUDA = "cuda"
    PALLAS = "pallas"
    EAGER = "eager"


class IRType:
    pass


@dataclass
class TensorType(IRType):
    shape: Tuple
    dtype: str

    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def bytes(self) -> int:
        return self.numel() * _BYTES.get(self.dtype, 2)

    def __repr__(self):
        return "tensor<" + "x".join(str(d) for d in self.shape) + f"x{self.dtype}>"


@dataclass
class KVCacheType(IRType):
    """KV cache of every layer; ``num_kv_heads`` < ``num_heads`` for GQA."""
    num_layers: int
    num_heads: int
    head_dim: int
    max_seq_len: int
    dtype: str = "bf16"
    num_kv_heads: Optional[int] = None

    @property
    def kv_heads(self) -> int:
        return self.num_kv_heads or self.num_heads

    def bytes_per_token(self) -> int:
        return 2 * self.num_layers * self.kv_heads * self.head_dim * _BYTES.get(self.dtype, 2)

    def total_bytes(self) -> int:
        return self.bytes_per_token() * self.max_seq_len

    def __repr__(self):
        return (f"kvcache<L={self.num_layers},H={self.num_heads},Hkv={self.kv_heads},"
                f"d={self.head_dim},seq={self.max_seq_len},{self.dtype}>")


@dataclass
class TokenSeqType(IRType):
    max_len: int
    vocab_size: int


@dataclass
class ScalarType(IRType):
    dtype: str


class Value:
    """A named, typed SSA value."""

    def __init__(self, name: str, type_: IRType, defining_op=None):
        self.name = name
        self.type = type_
        self.defining_op = defining_op

    def __repr__(self):
        return f"%{self.name}: {self.type}"


_ids = itertools.count()


class Op:
    """Base op: operands, typed results, attributes, phase/target and pass metadata."""

    def __init__(self, name: str, operands: List[Value], result_types: List[IRType],
                 attrs: Optional[Dict[str, Any]] = None):
        self.id = f"{next(_ids):08x}"
        self.name = name
        self.operands = operands
        self.results = [Value(f"{name.replace('.', '_')}_{self.id}_{i}", t, self)
                        for i, t in enumerate(result_types)]
        self.attrs: Dict[str, Any] = attrs or {}
        self.phase: Optional[Phase] = None
        self.target: Optional[KernelTarget] = None
        self.metadata: Dict[str, Any] = {}

    def result(self, idx: int = 0) -> Value:
        return self.results[idx]

    def is_compiler_inserted(self) -> bool:
        return bool(self.metadata.get("compiler_inserted", False))

    def estimated_flops(self) -> int:
        return 0

    def estimated_bytes(self) -> int:
        return 0

    def arithmetic_intensity(self) -> float:
        b = self.estimated_bytes()
        return float("inf") if b == 0 else self.estimated_flops() / b


class LLMForwardOp(Op):
    """One model forward pass in the PREFILL or DECODE phase.

    Cost model as in the reference (``ir/dialect.py:226-238``): FLOPs
    ``2 * seq * L * 12 d^2``; bytes = bf16 weights ``2 * L * 12 d^2 * 2`` plus
    the KV bytes of ``seq`` tokens.
    """

    def __init__(self, input_tokens: Value, kv_state: Value, model_config: Dict[str, Any],
                 phase: Phase = Phase.DECODE, seq_len: int = 1):
        super().__init__("llm.forward", [input_tokens, kv_state],
                         [TensorType((seq_len, model_config["vocab_size"]), "bf16")],
                         dict(model_config))
        self.phase = phase
        self.model_config = model_config
        self.seq_len = seq_len

    def estimated_flops(self) -> int:
        d = self.model_config.get("d_model", 768)
        n_layers = self.model_config.get("num_layers", 12)
        return 2 * self.seq_len * n_layers * 12 * d * d

    def estimated_bytes(self) -> int:
        d = self.model_config.get("d_model", 768)
        n_layers = self.model_config.get("num_layers", 12)
        kv_t = self.operands[1].type
        kv = kv_t.bytes_per_token() * self.seq_len if isinstance(kv_t, KVCacheType) else 0
        return 2 * n_layers * 12 * d * d * 2 + kv


class KVWriteOp(Op):
    def __init__(self, kv_state: Value, new_keys: Value, new_values: Value,
                 seq_pos: int, step_id: int = 0):
        super().__init__("kv.write", [kv_state, new_keys, new_values], [kv_state.type],
                         {"seq_pos": seq_pos, "step_id": step_id})
        self.phase = Phase.IO
        self.metadata["step_id"] = step_id

    def estimated_bytes(self) -> int:
        return sum(o.type.bytes() for o in self.operands[1:] if isinstance(o.type, TensorType))


class KVFuseOp(Op):
    """Compiler-inserted shared-prefix write; ``prefix_len`` drives ``KVPool.fork``."""

    def __init__(self, kv_state: Value, steps_to_fuse: List[int], prefix_len: int,
                 replaced_writes: List[KVWriteOp]):
        super().__init__("kv.fuse", [kv_state], [kv_state.type],
                         {"steps": steps_to_fuse, "prefix_len": prefix_len,
                          "n_fused": len(steps_to_fuse)})
        self.phase = Phase.FUSE
        self.metadata.update(compiler_inserted=True, fused_steps=steps_to_fuse,
                             shared_prefix_tokens=prefix_len, replaced_writes=replaced_writes)
        if replaced_writes:
            self.metadata["hbm_bytes_saved"] = (replaced_writes[0].estimated_bytes() * prefix_len
                                                * (len(steps_to_fuse) - 1))

    def bytes_saved(self) -> int:
        return self.metadata.get("hbm_bytes_saved", 0)


class ToolCallOp(Op):
    def __init__(self, tool_name: str, tool_input: Value, estimated_latency_ms: float = 100.0,
                 step_id: int = 0):
        super().__init__("tool.call", [tool_input], [TokenSeqType(512, 32000)],
                         {"tool": tool_name, "est_latency_ms": estimated_latency_ms,
                          "step_id": step_id})
        self.phase = Phase.IO
        self.metadata.update(gpu_idle=True, io_latency_ms=estimated_latency_ms)
        self.tool_name = tool_name

    def idle_window_ms(self) -> float:
        return self.metadata["io_latency_ms"]


class SpeculativePrefillOp(Op):
    def __init__(self, speculative_tokens: Value, kv_state: Value, model_config: Dict[str, Any],
                 confidence: float, overlapping_tool: Optional[ToolCallOp] = None):
        super().__init__("llm.spec_prefill", [speculative_tokens, kv_state],
                         [TensorType((1, model_config["vocab_size"]), "bf16")], dict(model_config))
        self.phase = Phase.PREFILL
        self.metadata.update(compiler_inserted=True, confidence=confidence,
                             overlap_with="tool.call")
        if overlapping_tool is not None:
            self.metadata["overlap_tool_id"] = overlapping_tool.id
            self.metadata["available_window_ms"] = overlapping_tool.idle_window_ms()


class PromptConstructOp(Op):
    def __init__(self, observation: Value, memory: Value, template: str):
        super().__init__("prompt.construct", [observation, memory], [TokenSeqType(2048, 32000)],
                         {"template": template})
        self.phase = Phase.IO
        self.metadata["gpu_idle"] = True


class ArgmaxOp(Op):
    def __init__(self, logits: Value):
        super().__init__("argmax", [logits], [ScalarType("int32")])
        self.phase = Phase.DECODE


class ParseActionOp(Op):
    def __init__(self, tokens: Value, action_schema: str):
        super().__init__("parse.action", [tokens], [TokenSeqType(256, 32000)],
                         {"schema": action_schema})
        self.phase = Phase.IO
        self.metadata["gpu_idle"] = True


class AgentStepOp(Op):
    """One Observe -> Reason -> Act iteration with three op regions."""

    def __init__(self, step_id: int, observe_ops=None, reason_ops=None, act_ops=None):
        super().__init__("agent.step", [], [], {"step_id": step_id})
        self.step_id = step_id
        self.observe_region: List[Op] = observe_ops or []
        self.reason_region: List[Op] = reason_ops or []
        self.act_region: List[Op] = act_ops or []

    def regions(self):
        return [self.observe_region, self.reason_region, self.act_region]

    def all_ops(self) -> List[Op]:
        return self.observe_region + self.reason_region + self.act_region

    def llm_ops(self):
        return [o for o in self.all_ops() if isinstance(o, LLMForwardOp)]

    def tool_ops(self):
        return [o for o in self.act_region if isinstance(o, ToolCallOp)]

    def kv_write_ops(self):
        return [o for o in self.all_ops() if isinstance(o, KVWriteOp)]

    def total_gpu_idle_ms(self) -> float:
        return sum(o.idle_window_ms() for o in self.tool_ops())

    def add_op(self, op: Op, region: str = "reason") -> "AgentStepOp":
        getattr(self, f"{region}_region").append(op)
        return self

    def insert_before(self, target: Op, new_op: Op) -> bool:
        for reg in self.regions():
            if target in reg:
                reg.insert(reg.index(target), new_op)
                return True
        return False

    def remove(self, op: Op) -> bool:
        for reg in self.regions():
            if op in reg:
                reg.remove(op)
                return True
        return False


class AgentProgram:
    """Compilation unit: steps, the shared KV-cache value, model config and target."""

    def __init__(self, name: str, model_config: Dict[str, Any], kv_cache_config: Dict[str, Any]):
        self.name = name
        self.model_config = model_config
        self.kv_cache_config = kv_cache_config
        self.steps: List[AgentStepOp] = []
        self.kv_state = Value("kv_cache", KVCacheType(
            num_layers=kv_cache_config["num_layers"], num_heads=kv_cache_config["num_heads"],
            head_dim=kv_cache_config["head_dim"], max_seq_len=kv_cache_config["max_seq_len"],
            dtype=kv_cache_config.get("dtype", "bf16"),
            num_kv_heads=kv_cache_config.get("num_kv_heads")))
        self.pass_annotations: List[str] = []
        self._target: Optional[KernelTarget] = None

    def add_step(self, step: AgentStepOp) -> "AgentProgram":
        self.steps.append(step)
        return self

    def set_target(self, target: KernelTarget) -> "AgentProgram":
        self._target = target
        for op in self.all_ops():
            if op.target is None:
                op.target = target
        return self

    @property
    def target(self) -> Optional[KernelTarget]:
        return self._target

    def all_ops(self) -> List[Op]:
        return [op for s in self.steps for op in s.all_ops()]

    def ops_by_type(self, t: type) -> List[Op]:
        return [o for o in self.all_ops() if isinstance(o, t)]

    def total_gpu_idle_ms(self) -> float:
        return sum(s.total_gpu_idle_ms() for s in self.steps)

    def add_annotation(self, msg: str) -> None:
        self.pass_annotations.append(msg)


GPT2_CONFIG = {"model_name": "gpt2", "d_model": 768, "num_layers": 12, "num_heads": 12,
               "head_dim": 64, "vocab_size": 50257, "max_seq_len": 1024}
GPT2_KV_CONFIG = {"num_layers": 12, "num_heads": 12, "head_dim": 64, "max_seq_len": 1024,
                  "dtype": "fp16"}
LLAMA3_8B_CONFIG = {"model_name": "llama-3-8b", "d_model": 4096, "num_layers": 32,
                    "num_heads": 32, "num_kv_heads": 8, "head_dim": 128, "ffn_dim": 14336,
                    "vocab_size": 128256, "max_seq_len": 32768}
LLAMA3_8B_KV_CONFIG = {"num_layers": 32, "num_heads": 32, "num_kv_heads": 8, "head_dim": 128,
                       "max_seq_len": 32768, "dtype": "bf16"}
