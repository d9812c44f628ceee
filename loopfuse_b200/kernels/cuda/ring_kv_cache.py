"""``kernels.cuda.ring_kv_cache`` names -> sm_100a paged decode and pool append.

The reference's ring-buffer module (``kernels/cuda/ring_kv_cache.cu``,
bound by ``kernels/cuda/_cuda_ext.py:60-116``) does not compile.  Its selection
entry ``ring_kv_decode_kernel`` is bound to the paged split-KV decode, called
either as the reference's contiguous-cache ``(q, k, v)`` or, with a paged pool,
as ``(q, k_pages, v_pages, block_table, seq_lens, ...)``.  ``ring_kv_write``
appends to a ``KVPool`` session (there is no ring slot index any more).
"""
import torch

from ...attention import decode_attention_fwd, paged_decode


def ring_kv_decode_kernel(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *args, **kwargs):
    if args or "block_table" in kwargs:
        return paged_decode(q, k, v, *args, **kwargs)
    return decode_attention_fwd(q, k, v, **kwargs)


def ring_kv_write(pool, state, new_keys: torch.Tensor, new_values: torch.Tensor, stream=None):
    """Append ``[L, H, S_new, D]`` keys/values to ``state`` (replaces the slot-indexed write)."""
    return pool.write(state, new_keys, new_values, stream=stream)


def async_zero_slot(pool, state, stream=None) -> None:
    """The speculative-prefill hook that zeroed the next ring slot (reference
    ``kernels/cuda/_cuda_ext.py:93-116``, ``async_zero_next_slot_kernel``).

    A paged session reads only positions below its length, and its pages are reserved when
    tokens are appended, so there is nothing to clear: this checks its arguments and returns.
    The dense ring layout ``[slots, L, H, max_seq, D]`` is not supported; passing its tensors
    raises ``TypeError``."""
    from ...runtime.kv_pool import KVPool, KVState

    if not isinstance(pool, KVPool) or not isinstance(state, KVState):
        raise TypeError("async_zero_slot takes (KVPool, KVState): the paged pool replaces the "
                        "dense ring-buffer cache")
    pool.prefetch_next_slot(state)


__all__ = ["async_zero_slot", "ring_kv_decode_kernel", "ring_kv_write"]
