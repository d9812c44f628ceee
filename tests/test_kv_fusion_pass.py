"""KVFusionPass: the reference's pass contract (tests/test_passes.py:142-164 of the reference)
plus the run-time meaning this package gives the op."""
import copy

import pytest

from loopfuse_b200.ir.builder import AgentProgramBuilder
from loopfuse_b200.ir.dialect import GPT2_CONFIG, GPT2_KV_CONFIG, KernelTarget, KVFuseOp, Phase
from loopfuse_b200.passes import KVFusionPass, PassManager, PassResult, PhaseSelectPass


def _prog(n):
    b = AgentProgramBuilder(f"t{n}", GPT2_CONFIG, GPT2_KV_CONFIG)
    tools = ["search", "lookup", "calculator", "search"]
    for i in range(n):
        b.add_react_step(i, tools[i] if i < n - 1 else None, 100.0, is_first_step=(i == 0))
    return b.set_target(KernelTarget.TRITON).build()


def test_no_fusion_below_min_steps():
    assert not KVFusionPass(min_prefix_len=4, min_steps=10).run(_prog(3)).changed


def test_result_and_fuse_op_properties():
    prog = copy.deepcopy(_prog(5))
    r = KVFusionPass(min_prefix_len=4).run(prog)
    assert isinstance(r, PassResult) and r.changed
    ops = prog.ops_by_type(KVFuseOp)
    assert len(ops) == 1
    op = ops[0]
    assert op.phase == Phase.FUSE and op.is_compiler_inserted()
    assert op.attrs["prefix_len"] == 64 and op.attrs["steps"] == [0, 1, 2, 3, 4]
    assert prog.steps[0].reason_region[0] is op
    assert op.bytes_saved() > 0


def test_idempotent_and_prefix_from_config():
    prog = _prog(3)
    prog.model_config = dict(prog.model_config, system_prompt_len=512)
    assert KVFusionPass().run(prog).changed
    assert not KVFusionPass().run(prog).changed
    assert prog.ops_by_type(KVFuseOp)[0].attrs["prefix_len"] == 512


def test_pipeline_with_phase_select():
    prog = _prog(3)
    prog.set_target(KernelTarget.CUDA)
    results = PassManager([KVFusionPass(), PhaseSelectPass(hardware="b200")]).run(prog)
    assert [r.changed for r in results] == [True, True]
