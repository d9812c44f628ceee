"""``kernels.cuda.*`` entries of ``PHASE_KERNEL_MAP`` (reference ``passes/phase_select.py:60-69``)."""
from .async_prefill import agent_prefill_kernel
from .ring_kv_cache import ring_kv_decode_kernel, ring_kv_write
