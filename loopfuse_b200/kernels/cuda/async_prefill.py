"""``kernels.cuda.async_prefill.agent_prefill_kernel`` -> sm_100a tcgen05 prefill.

The reference's module of this name (``kernels/cuda/async_prefill.cu:56-236``)
does not compile and never computes softmax or P.V; the selection table still
names it for ``(KernelTarget.CUDA, Phase.PREFILL)``.  Here the name is bound to
the working kernel with the reference's prefill signature
``(q, k, v, causal=True)`` on ``[B, H, S, D]`` tensors.
"""
from ...attention import prefill_attention_fwd as agent_prefill_kernel

__all__ = ["agent_prefill_kernel"]
