"""Generate the golden fixtures in this folder from the reference's own code.

Run once, giving the path of a checkout of the reference (required):

    python tests/golden/make_golden.py <path to the loopfuse checkout>

The reference is a flat Python package (its root directory *is* the
``loopfuse`` package), so it is imported through a temporary directory holding
a ``loopfuse`` symlink to it.  Nothing here is needed at test time: the tests
read only the fixture files written below.

Fixtures
--------
kvpool_trace.json      a scripted session on ``loopfuse.runtime.kv_pool.KVPool``
                       (CPU, ``GPT2_KV_CONFIG``, 4 slots): slot ids, lengths,
                       error messages, ``stats()`` and read shapes.
phase_select.json      ``PhaseSelectPass`` annotations of the 3-step GPT-2
                       program (``tests/conftest.py:23-30`` of the reference)
                       for every ``KernelTarget``, plus IR byte arithmetic.
passes.json            ``SpecPrefillPass`` insertions and annotations on programs
                       with varied tool names and latencies (run twice, for
                       idempotence), ``PassManager.run_until_fixed_point`` result
                       flags, and ``RooflineAnalyzer(A100_SPEC)`` reports.
attention_fp16.npz     seeded MHA fp16 inputs and the reference's own checks:
                       ``_reference_decode_attn`` (``kernels/triton/
                       decode_attn.py:178-184``) and the fp32 SDPA causal
                       check of ``verify_prefill_kernel`` (``kernels/triton/
                       prefill_attn.py:180-182``).
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root: str):
    tmp = tempfile.mkdtemp(prefix="lf_ref_")
    os.symlink(os.path.abspath(ref_root), os.path.join(tmp, "loopfuse"))
    sys.path.insert(0, tmp)
    import loopfuse  # noqa: F401
    return tmp


def kvpool_trace():
    from loopfuse.runtime.kv_pool import KVPool
    from loopfuse.ir.dialect import GPT2_KV_CONFIG
    pool = KVPool.from_config(GPT2_KV_CONFIG, device="cpu", max_slots=4)
    ev = []
    nl, nh, hd = pool.num_layers, pool.num_heads, pool.head_dim
    st = [pool.allocate_slot() for _ in range(4)]
    ev.append({"op": "allocate x4", "slots": [s.slot_id for s in st]})
    try:
        pool.allocate_slot()
    except RuntimeError as e:
        ev.append({"op": "allocate (exhausted)", "error": str(e)})
    pool.release(st[1])
    pool.release(st[3])
    s_a = pool.allocate_slot()
    s_b = pool.allocate_slot()
    ev.append({"op": "release 1,3 then allocate x2", "slots": [s_a.slot_id, s_b.slot_id]})
    lens = []
    for n in (8, 4, 4, 4, 4):
        k = torch.zeros(nl, nh, n, hd, dtype=torch.float16)
        lens.append(pool.write(st[0], k, torch.zeros_like(k)))
    ev.append({"op": "write 8,4,4,4,4 to slot 0", "returned": lens,
               "current_len": st[0].current_len})
    try:
        k = torch.zeros(nl, nh, pool.max_seq_len, hd, dtype=torch.float16)
        pool.write(st[0], k, torch.zeros_like(k))
    except RuntimeError as e:
        ev.append({"op": "write max_seq_len more (overflow)", "error": str(e),
                   "current_len_after": st[0].current_len})
    k_in = torch.randn(nl, nh, 16, hd, dtype=torch.float16,
                       generator=torch.Generator().manual_seed(7))
    pool.write(s_a, k_in, k_in + 1)
    k0, v0 = pool.read(s_a, layer=0)
    ka, va = pool.read_all_layers(s_a)
    kr, _ = pool.read(s_a, layer=3, seq_start=4, seq_end=12)
    ev.append({"op": "read shapes", "read": list(k0.shape), "read_all": list(ka.shape),
               "read_range": list(kr.shape),
               "read_equal_input": bool(torch.equal(k0, k_in[0])),
               "read_range_equal_input": bool(torch.equal(kr, k_in[3, :, 4:12]))})
    s = st[0]
    s.advance_step()
    ev.append({"op": "advance_step", "step_id": s.step_id})
    ev.append({"op": "stats", "stats": pool.stats(), "hbm_usage_bytes": pool.hbm_usage_bytes()})
    pool.release(st[0])
    ev.append({"op": "stats after release", "stats": pool.stats()})
    return {"config": GPT2_KV_CONFIG, "max_slots": 4, "events": ev}


def phase_select():
    from loopfuse.ir.builder import AgentProgramBuilder
    from loopfuse.ir.dialect import (GPT2_CONFIG, GPT2_KV_CONFIG, KernelTarget, LLMForwardOp,
                                     KVCacheType)
    from loopfuse.passes.phase_select import PhaseSelectPass
    out = {}
    for tgt in KernelTarget:
        prog = (AgentProgramBuilder("t3", GPT2_CONFIG, GPT2_KV_CONFIG)
                .add_react_step(0, "search", 150.0, is_first_step=True)
                .add_react_step(1, "lookup", 80.0)
                .add_react_step(2, None)
                .set_target(tgt).build())
        res = PhaseSelectPass().run(prog)
        ops = []
        for op in prog.ops_by_type(LLMForwardOp):
            md = {k: op.metadata[k] for k in ("kernel_module", "kernel_name", "kernel_notes",
                                               "is_compute_bound", "arithmetic_intensity",
                                               "roofline_efficiency")}
            md["phase"] = op.phase.value
            md["seq_len"] = op.seq_len
            md["estimated_flops"] = op.estimated_flops()
            md["estimated_bytes"] = op.estimated_bytes()
            ops.append(md)
        out[tgt.value] = {"changed": res.changed, "annotations": res.annotations, "ops": ops}
    kv = KVCacheType(12, 12, 64, 1024, "fp16")
    out["kvcache_gpt2_fp16"] = {"bytes_per_token": kv.bytes_per_token(),
                                "total_bytes": kv.total_bytes()}
    return out


def _pass_programs():
    """(name, builder calls) of the programs the pass fixtures cover."""
    return [
        ("react3", [(0, "search", 150.0, True), (1, "lookup", 80.0, False), (2, None, 0.0, False)]),
        ("tools", [(0, "execute_code", 120.0, True), (1, "run_shell", 500.0, False),
                   (2, "web_search", 25.0, False), (3, "calculator", 40.0, False),
                   (4, "lookup_db", 18.0, False), (5, "search", 300.0, False)]),
        ("long", [(i, "search" if i % 2 else "fetch", 60.0 + 10 * i, i == 0) for i in range(12)]),
    ]


def _build(mod_builder, cfg, kv, steps, target):
    b = mod_builder.AgentProgramBuilder("p", cfg, kv)
    for sid, tool, lat, first in steps:
        b.add_react_step(sid, tool, lat, is_first_step=first)
    return b.set_target(target).build()


def passes():
    import loopfuse.ir.builder as builder
    from loopfuse.ir.dialect import GPT2_CONFIG, GPT2_KV_CONFIG, KernelTarget, SpeculativePrefillOp
    from loopfuse.passes.base import PassManager
    from loopfuse.passes.phase_select import PhaseSelectPass
    from loopfuse.passes.spec_prefill import SpecPrefillPass
    from loopfuse.analysis.roofline import A100_SPEC, RooflineAnalyzer
    out = {}
    for name, steps in _pass_programs():
        prog = _build(builder, GPT2_CONFIG, GPT2_KV_CONFIG, steps, KernelTarget.CUDA)
        p = SpecPrefillPass()
        r1, r2 = p.run(prog), p.run(prog)
        layout = [[[type(o).__name__ for o in reg]
                   for reg in (s.observe_region, s.reason_region, s.act_region)]
                  for s in prog.steps]
        spec_md = [{k: op.metadata[k] for k in ("confidence", "available_window_ms")}
                   for op in prog.ops_by_type(SpeculativePrefillOp)]
        fresh = _build(builder, GPT2_CONFIG, GPT2_KV_CONFIG, steps, KernelTarget.CUDA)
        fp = PassManager([SpecPrefillPass(), PhaseSelectPass()]).run_until_fixed_point(fresh, 4)
        roof = RooflineAnalyzer(A100_SPEC).analyze_program(
            _build(builder, GPT2_CONFIG, GPT2_KV_CONFIG, steps, KernelTarget.CUDA))
        out[name] = {
            "spec_first": {"changed": r1.changed, "annotations": r1.annotations},
            "spec_second": {"changed": r2.changed, "annotations": r2.annotations},
            "layout": layout, "spec_metadata": spec_md,
            "fixed_point": [[r.pass_name, r.changed] for r in fp],
            "roofline": {"points": [[pt.op_name, pt.phase.value if pt.phase else None, pt.flops,
                                     pt.bytes_accessed, pt.is_compute_bound,
                                     pt.achieved_efficiency, pt.bottleneck]
                                    for pt in roof.op_points],
                         "phase_summary": roof.phase_summary, "total_flops": roof.total_flops,
                         "total_bytes": roof.total_bytes, "gpu_idle_ms": roof.gpu_idle_ms,
                         "text": roof.phase_breakdown_str()},
        }
    return out


def attention_fp16():
    from loopfuse.kernels.triton.decode_attn import _reference_decode_attn
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(1234)
    arrays = {}
    # decode: the reference's MHA fp16 shape family, small enough to store
    q = torch.randn(1, 4, 1, 64, generator=g).half()
    k = torch.randn(1, 4, 80, 64, generator=g).half()
    v = torch.randn(1, 4, 80, 64, generator=g).half()
    arrays.update(dec_q=q, dec_k=k, dec_v=v, dec_out=_reference_decode_attn(q, k, v))
    # prefill: verify_prefill_kernel's oracle, causal, seq_q == seq_k
    q = torch.randn(1, 4, 48, 64, generator=g).half()
    k = torch.randn(1, 4, 48, 64, generator=g).half()
    v = torch.randn(1, 4, 48, 64, generator=g).half()
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)
    arrays.update(pre_q=q, pre_k=k, pre_v=v, pre_out_fp32=ref, pre_out=ref.half())
    return {name: t.numpy() for name, t in arrays.items()}


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the loopfuse checkout>")
    _import_reference(sys.argv[1])
    with open(os.path.join(HERE, "kvpool_trace.json"), "w") as f:
        json.dump(kvpool_trace(), f, indent=1)
    with open(os.path.join(HERE, "phase_select.json"), "w") as f:
        json.dump(phase_select(), f, indent=1)
    with open(os.path.join(HERE, "passes.json"), "w") as f:
        json.dump(passes(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "attention_fp16.npz"), **attention_fp16())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
