"""loopfuse_b200: sm_100a phase-specialised attention hot path behind loopfuse's API.

* ``loopfuse_b200.attention``: prefill (tcgen05/TMEM/TMA) and paged split-KV decode.
* ``loopfuse_b200.runtime``: device-resident paged ``KVPool`` and ``AgentExecutor``.
* ``loopfuse_b200.passes``: ``PhaseSelectPass`` / ``PHASE_KERNEL_MAP``.
* ``loopfuse_b200.ir``: the agent-program IR the pass and executor read.

The compute path is ``liblf_sm100.so`` (C ABI, ``include/loopfuse_b200.h``), built by
``python -m loopfuse_b200.build``.  Nothing here falls back to the CPU.
"""
__version__ = "0.1.0"
