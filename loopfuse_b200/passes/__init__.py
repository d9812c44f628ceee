from .base import Pass, PassManager, PassResult
from .phase_select import PHASE_KERNEL_MAP, PhaseSelectPass, resolve_kernel
from .kv_fusion import KVFusionPass
from .spec_prefill import SpecPrefillPass
