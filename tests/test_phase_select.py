"""Kernel selection parity with the reference (golden annotations) and the no-fallback rule."""
import json
import os

import pytest

from loopfuse_b200.ir import GPT2_CONFIG, GPT2_KV_CONFIG, AgentProgramBuilder, KernelTarget, LLMForwardOp, Phase
from loopfuse_b200.ir.dialect import KVCacheType
from loopfuse_b200.passes import PHASE_KERNEL_MAP, PhaseSelectPass, resolve_kernel


def _prog(target):
    return (AgentProgramBuilder("t3", GPT2_CONFIG, GPT2_KV_CONFIG)
            .add_react_step(0, "search", 150.0, is_first_step=True)
            .add_react_step(1, "lookup", 80.0)
            .add_react_step(2, None)
            .set_target(target).build())


@pytest.mark.parametrize("target", list(KernelTarget))
def test_annotations_match_reference(golden_dir, target):
    ref = json.load(open(os.path.join(golden_dir, "phase_select.json")))[target.value]
    prog = _prog(target)
    res = PhaseSelectPass().run(prog)
    assert res.changed == ref["changed"]
    assert res.annotations == ref["annotations"]
    ops = prog.ops_by_type(LLMForwardOp)
    assert len(ops) == len(ref["ops"])
    for op, r in zip(ops, ref["ops"]):
        for key in ("kernel_module", "kernel_name", "kernel_notes", "is_compute_bound",
                    "arithmetic_intensity", "roofline_efficiency"):
            assert op.metadata[key] == r[key], key
        assert op.phase.value == r["phase"]
        assert op.estimated_flops() == r["estimated_flops"]
        assert op.estimated_bytes() == r["estimated_bytes"]


def test_kvcache_bytes(golden_dir):
    ref = json.load(open(os.path.join(golden_dir, "phase_select.json")))["kvcache_gpt2_fp16"]
    kv = KVCacheType(12, 12, 64, 1024, "fp16")
    assert kv.bytes_per_token() == ref["bytes_per_token"] == 36864
    assert kv.total_bytes() == ref["total_bytes"]
    assert KVCacheType(32, 32, 128, 4096, "bf16", num_kv_heads=8).bytes_per_token() == 2 * 32 * 8 * 128 * 2


def test_reference_phase_select_assertions():
    """The reference's TestPhaseSelectPass (tests/test_passes.py:100-140), restated."""
    prog = _prog(KernelTarget.TRITON)
    assert PhaseSelectPass().run(prog).changed
    for op in prog.ops_by_type(LLMForwardOp):
        assert {"kernel_module", "kernel_name", "is_compute_bound"} <= set(op.metadata)
        assert "triton" in op.metadata["kernel_module"]
        assert op.metadata["arithmetic_intensity"] >= 0
        if op.phase == Phase.DECODE:
            assert not op.metadata["is_compute_bound"]
    prog = _prog(KernelTarget.EAGER)
    PhaseSelectPass().run(prog)
    assert all("torch" in op.metadata["kernel_module"] for op in prog.ops_by_type(LLMForwardOp))


def test_cuda_names_resolve_to_sm100_ops():
    from loopfuse_b200.attention import prefill_attention_fwd
    from loopfuse_b200.kernels.cuda.ring_kv_cache import ring_kv_decode_kernel
    mod, fn, _ = PHASE_KERNEL_MAP[(KernelTarget.CUDA, Phase.PREFILL)]
    assert resolve_kernel(mod, fn) is prefill_attention_fwd
    mod, fn, _ = PHASE_KERNEL_MAP[(KernelTarget.CUDA, Phase.DECODE)]
    assert resolve_kernel(mod, fn) is ring_kv_decode_kernel


def test_cuda_package_exports_the_reference_names():
    """The reference's ``kernels/cuda/__init__.py`` exports ``is_available``, ``ring_kv_write``
    and ``async_zero_slot``; the same names import here.  Without a GPU nothing is available,
    and the dense ring-slot form of ``async_zero_slot`` is refused, not emulated."""
    import torch

    from loopfuse_b200.kernels import cuda as kc
    for name in ("is_available", "ring_kv_write", "async_zero_slot", "agent_prefill_kernel",
                 "ring_kv_decode_kernel"):
        assert callable(getattr(kc, name)), name
    if not torch.cuda.is_available():
        assert kc.is_available() is False
    ring = torch.zeros(2, 1, 1, 16, 64, dtype=torch.float16)
    with pytest.raises(TypeError, match="paged pool"):
        kc.async_zero_slot(ring, ring, 1)


@pytest.mark.gpu
def test_cuda_package_is_available_on_b200_and_zero_slot_leaves_the_pool_unchanged():
    import torch

    from loopfuse_b200.kernels import cuda as kc
    from loopfuse_b200.runtime.kv_pool import KVPool
    assert kc.is_available()
    pool = KVPool(num_layers=1, num_heads=2, head_dim=64, max_seq_len=64, max_slots=2,
                  dtype=torch.bfloat16, device="cuda")
    st = pool.alloc()
    k = torch.randn(1, 2, 20, 64, device="cuda").to(torch.bfloat16)
    kc.ring_kv_write(pool, st, k, -k)
    before = pool.snapshot()
    kc.async_zero_slot(pool, st)
    assert pool.snapshot() == before
    kr, vr = pool.read(st, 0)
    assert torch.equal(kr, k[0]) and torch.equal(vr, -k[0])


@pytest.mark.parametrize("target", [KernelTarget.TRITON, KernelTarget.PALLAS, KernelTarget.EAGER])
def test_other_targets_do_not_execute(target):
    for phase in (Phase.PREFILL, Phase.DECODE):
        mod, fn, _ = PHASE_KERNEL_MAP[(target, phase)]
        with pytest.raises(NotImplementedError):
            resolve_kernel(mod, fn, target)


def test_b200_profile_classifies_prefill_and_decode():
    prog = _prog(KernelTarget.CUDA)
    PhaseSelectPass(hardware="b200").run(prog)
    ops = prog.ops_by_type(LLMForwardOp)
    assert all(not op.metadata["is_compute_bound"] for op in ops if op.phase == Phase.DECODE)
