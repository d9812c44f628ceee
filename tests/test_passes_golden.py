"""SpecPrefillPass, PassManager.run_until_fixed_point and the roofline analyser against
fixtures generated from the reference's own passes (``tests/golden/make_golden.py``), plus the
B200 peaks the selection and the analyser classify against."""
import json
import os

import pytest

from loopfuse_b200.analysis import A100_SPEC, B200_SPEC, RooflineAnalyzer, kernel_roofline
from loopfuse_b200.ir import GPT2_CONFIG, GPT2_KV_CONFIG, AgentProgramBuilder, KernelTarget
from loopfuse_b200.ir.dialect import SpeculativePrefillOp
from loopfuse_b200.passes import PassManager, PhaseSelectPass, SpecPrefillPass
from loopfuse_b200.passes import phase_select
from loopfuse_b200.peaks import b200_peaks

PROGRAMS = {
    "react3": [(0, "search", 150.0, True), (1, "lookup", 80.0, False), (2, None, 0.0, False)],
    "tools": [(0, "execute_code", 120.0, True), (1, "run_shell", 500.0, False),
              (2, "web_search", 25.0, False), (3, "calculator", 40.0, False),
              (4, "lookup_db", 18.0, False), (5, "search", 300.0, False)],
    "long": [(i, "search" if i % 2 else "fetch", 60.0 + 10 * i, i == 0) for i in range(12)],
}


def _build(steps):
    b = AgentProgramBuilder("p", GPT2_CONFIG, GPT2_KV_CONFIG)
    for sid, tool, lat, first in steps:
        b.add_react_step(sid, tool, lat, is_first_step=first)
    return b.set_target(KernelTarget.CUDA).build()


@pytest.fixture(scope="module")
def golden(golden_dir):
    return json.load(open(os.path.join(golden_dir, "passes.json")))


@pytest.mark.parametrize("name", list(PROGRAMS))
def test_spec_prefill_pass_matches_reference(golden, name):
    ref = golden[name]
    prog = _build(PROGRAMS[name])
    p = SpecPrefillPass()
    r1, r2 = p.run(prog), p.run(prog)
    assert [r1.changed, r1.annotations] == [ref["spec_first"]["changed"], ref["spec_first"]["annotations"]]
    assert [r2.changed, r2.annotations] == [ref["spec_second"]["changed"], ref["spec_second"]["annotations"]]
    layout = [[[type(o).__name__ for o in reg] for reg in s.regions()] for s in prog.steps]
    assert layout == ref["layout"]
    md = [{k: op.metadata[k] for k in ("confidence", "available_window_ms")}
          for op in prog.ops_by_type(SpeculativePrefillOp)]
    assert md == ref["spec_metadata"]


@pytest.mark.parametrize("name", list(PROGRAMS))
def test_run_until_fixed_point_matches_reference(golden, name):
    res = PassManager([SpecPrefillPass(), PhaseSelectPass()]).run_until_fixed_point(
        _build(PROGRAMS[name]), 4)
    assert [[r.pass_name, r.changed] for r in res] == golden[name]["fixed_point"]


def test_fixed_point_stops_when_nothing_changes():
    prog = _build(PROGRAMS["react3"])
    res = PassManager([SpecPrefillPass()]).run_until_fixed_point(prog, 10)
    assert [r.changed for r in res] == [True, False]


@pytest.mark.parametrize("name", list(PROGRAMS))
def test_roofline_report_matches_reference(golden, name):
    ref = golden[name]["roofline"]
    rep = RooflineAnalyzer(A100_SPEC).analyze_program(_build(PROGRAMS[name]))
    pts = [[p.op_name, p.phase.value if p.phase else None, p.flops, p.bytes_accessed,
            p.is_compute_bound, p.achieved_efficiency, p.bottleneck] for p in rep.op_points]
    assert pts == ref["points"]
    assert rep.phase_summary == ref["phase_summary"]
    assert (rep.total_flops, rep.total_bytes, rep.gpu_idle_ms) == \
        (ref["total_flops"], ref["total_bytes"], ref["gpu_idle_ms"])
    assert rep.phase_breakdown_str() == ref["text"]


def test_b200_peaks_come_from_the_measurement_file():
    pk = b200_peaks()
    assert pk["hbm_gbs"] > 1000 and pk["bf16_tflops"] > 100
    assert B200_SPEC.hbm_bandwidth == pk["hbm_gbs"] * 1e9
    assert phase_select.B200_PEAK_FLOPS_BF16 == pk["bf16_tflops"] * 1e12
    assert abs(B200_SPEC.ridge_point - phase_select.B200_RIDGE_POINT) < 1e-9
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if os.path.exists(os.path.join(root, "MEASURED_PEAKS.json")):
        d = json.load(open(os.path.join(root, "MEASURED_PEAKS.json")))
        assert pk["source"] == "measured" and pk["hbm_gbs"] == float(d["hbm_gbs"])


def test_kernel_roofline_classifies_by_intensity():
    dec = kernel_roofline("decode", flops=7.1e10, nbytes=15.5e9, seconds=2.4e-3)
    assert dec["bound"] == "hbm" and 0 < dec["frac"] < 1.2
    pre = kernel_roofline("prefill", flops=1.0998e12, nbytes=6.7e8, seconds=0.95e-3)
    assert pre["bound"] == "tensor" and pre["unit"] == "TFLOP/s"
