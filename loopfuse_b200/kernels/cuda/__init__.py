"""``kernels.cuda.*`` entries of ``PHASE_KERNEL_MAP`` (reference ``passes/phase_select.py:60-69``).

Also the names the reference's package exports (``kernels/cuda/__init__.py``: ``is_available``,
``ring_kv_write``, ``async_zero_slot``), with the paged pool in place of the dense ring buffer.
"""
from .async_prefill import agent_prefill_kernel
from .ring_kv_cache import async_zero_slot, ring_kv_decode_kernel, ring_kv_write


def is_available() -> bool:
    """True when the sm_100a library loads and the current CUDA device is a compute-capability
    10.x GPU (reference ``kernels/cuda/_cuda_ext.py:55-57`` reports whether its extension
    compiled).  Nothing falls back when this is False: every op raises instead."""
    import torch

    from ... import _lib
    try:
        _lib.lib()
    except (_lib.LoopfuseError, OSError):
        return False
    return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10


__all__ = ["agent_prefill_kernel", "async_zero_slot", "is_available", "ring_kv_decode_kernel",
           "ring_kv_write"]
