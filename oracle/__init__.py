"""CPU oracle for the loopfuse attention hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, what the
reference computes on its hot path so that the sm_100a kernels can be checked
against it.  It is imported by ``tests/``, by ``__graft_entry__.smoke()`` and by
the CPU-baseline / reference legs of ``bench.py`` -- never by the product
package ``loopfuse_b200``, which has no CPU fallback.

Contents
--------
attention  fp32 torch restatement of the reference's attention semantics:
           causal prefill (``kernels/triton/prefill_attn.py:35-168``), decode
           (``kernels/triton/decode_attn.py:57-171``), the reference's own
           decode check (``kernels/triton/decode_attn.py:178-184``) and its
           EAGER entry ``scaled_dot_product_attention``
           (``passes/phase_select.py:80-89``).
pool_spec  deterministic Python specification of the paged KV pool
           (alloc/append/fork/free, refcounts, FIFO free queue, block tables,
           prefix dedup).  The reference pool (``runtime/kv_pool.py:28-235``)
           is dense; its slot FIFO order (``:110``), append-at-``current_len``
           (``:142-145``) and error strings (``:106-109``, ``:136-139``) are
           kept, and the page-level behaviour is specified here.

Parity pinning: ``tests/golden/`` holds vectors produced by importing the
reference's Python code (script ``tests/golden/make_golden.py``); the CPU
tests check this oracle against them.
"""
