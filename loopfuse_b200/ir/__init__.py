from .dialect import (AgentProgram, AgentStepOp, ArgmaxOp, GPT2_CONFIG, GPT2_KV_CONFIG,
                      KernelTarget, KVCacheType, KVFuseOp, KVWriteOp, LLAMA3_8B_CONFIG,
                      LLAMA3_8B_KV_CONFIG, LLMForwardOp, Op, ParseActionOp, Phase,
                      PromptConstructOp, SpeculativePrefillOp, TensorType, TokenSeqType,
                      ToolCallOp, Value)
from .builder import AgentProgramBuilder
