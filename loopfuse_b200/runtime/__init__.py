from .kv_pool import KVPool, KVState
from .executor import AgentExecutor, ExecutionResult, StepTrace
