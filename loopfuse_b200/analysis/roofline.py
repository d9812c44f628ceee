"""Roofline analysis of agent programs and of measured kernels.

Drop-in for the reference's ``analysis/roofline.py``: the same ``HardwareSpec`` (with its
``ridge_point``), the A100 / T4 / TPU v4 constants (``:46-71``), ``OpRooflinePoint``,
``RooflineReport`` and ``RooflineAnalyzer.analyze_program`` (``:143-190``), which classifies
every op of a program by its estimated arithmetic intensity against the ridge point and
summarises each phase.  Added here:

* ``B200_SPEC``: the B200 with its measured peaks (``peaks.b200_peaks()``: copy bandwidth and
  burst bf16 GEMM throughput measured on the machine, else the built-in figures), 126 MB of L2,
  228 KB of shared memory per SM, compute capability 10.0;
* ``kernel_roofline``: the roofline point of a kernel that was actually timed -- its bound, its
  achieved FLOP/s or bytes/s and the fraction of the peak that bounds it -- which is what the
  agent loop's per-kernel report uses.

Plotting (``RooflineAnalyzer.plot`` in the reference) is not built: it needs matplotlib, which
this package does not depend on, and draws nothing the report does not already hold.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

from ..ir.dialect import AgentProgram, KVFuseOp, KVWriteOp, LLMForwardOp, Phase
from ..peaks import b200_peaks


@dataclass
class HardwareSpec:
    name: str
    peak_flops: float          # FLOP/s, dense bf16 / fp16 tensor cores
    hbm_bandwidth: float       # bytes/s
    l2_cache_bytes: int
    shared_mem_bytes: int      # per SM
    compute_cap: float         # 0 for TPU

    @property
    def ridge_point(self) -> float:
        """Arithmetic intensity (FLOP/byte) where the memory and compute roofs meet."""
        return self.peak_flops / self.hbm_bandwidth


A100_SPEC = HardwareSpec("NVIDIA A100 SXM4 80GB", 312e12, 2.0e12, 40 * 1024 * 1024, 192 * 1024, 8.0)
T4_SPEC = HardwareSpec("NVIDIA T4", 65e12, 320e9, 4 * 1024 * 1024, 64 * 1024, 7.5)
TPU_V4_SPEC = HardwareSpec("Google TPU v4", 275e12, 1.2e12, 0, 0, 0.0)

_PK = b200_peaks()
B200_SPEC = HardwareSpec(f"NVIDIA B200 (peaks: {_PK['source']})", _PK["bf16_tflops"] * 1e12,
                         _PK["hbm_gbs"] * 1e9, 126 * 1024 * 1024, 228 * 1024, 10.0)


@dataclass
class OpRooflinePoint:
    op_id: str
    op_name: str
    phase: Optional[Phase]
    flops: int
    bytes_accessed: int
    arithmetic_intensity: float
    is_compute_bound: bool
    achieved_efficiency: float     # heuristic estimate, 0..1
    bottleneck: str                # "compute" or "memory"


@dataclass
class RooflineReport:
    hw_spec: HardwareSpec
    program_name: str
    op_points: List[OpRooflinePoint] = field(default_factory=list)
    phase_summary: Dict[str, Any] = field(default_factory=dict)
    total_flops: int = 0
    total_bytes: int = 0
    gpu_idle_ms: float = 0.0

    @property
    def overall_arithmetic_intensity(self) -> float:
        return float("inf") if self.total_bytes == 0 else self.total_flops / self.total_bytes

    @property
    def overall_bottleneck(self) -> str:
        return "compute" if self.overall_arithmetic_intensity > self.hw_spec.ridge_point else "memory"

    def phase_breakdown_str(self) -> str:
        ridge = self.hw_spec.ridge_point
        out = [f"Roofline Report: {self.program_name} on {self.hw_spec.name}",
               f"Ridge point: {ridge:.0f} FLOP/byte",
               f"Overall arithmetic intensity: {self.overall_arithmetic_intensity:.1f} FLOP/byte",
               f"Overall bottleneck: {self.overall_bottleneck}",
               f"GPU idle time (tool I/O): {self.gpu_idle_ms:.1f}ms", ""]
        for name, st in self.phase_summary.items():
            kind = "compute" if st["mean_ai"] > ridge else "memory"
            out.append(f"  {name:12s}: {st['n_ops']:3d} ops, AI={st['mean_ai']:.1f} FLOP/byte, "
                       f"{kind}-bound")
        return "\n".join(out)


class RooflineAnalyzer:
    """``RooflineAnalyzer(spec).analyze_program(prog)`` -> ``RooflineReport``."""

    # Heuristic efficiencies the reference assigns per op kind (``:192-206``).
    _EFF_PREFILL, _EFF_DECODE, _EFF_FUSE, _EFF_WRITE, _EFF_OTHER = 0.72, 0.55, 0.85, 0.60, 0.50

    def __init__(self, hw_spec: HardwareSpec):
        self.hw = hw_spec

    def analyze_program(self, prog: AgentProgram) -> RooflineReport:
        rep = RooflineReport(self.hw, prog.name, gpu_idle_ms=prog.total_gpu_idle_ms())
        per_phase: Dict[str, List[float]] = {p.value: [] for p in Phase}
        for op in prog.all_ops():
            flops, nbytes = op.estimated_flops(), op.estimated_bytes()
            if flops == 0 and nbytes == 0:
                continue
            ai = op.arithmetic_intensity()
            compute = ai > self.hw.ridge_point
            rep.op_points.append(OpRooflinePoint(op.id, op.name, op.phase, flops, nbytes, ai, compute,
                                                 self._estimate_efficiency(op, compute),
                                                 "compute" if compute else "memory"))
            rep.total_flops += flops
            rep.total_bytes += nbytes
            if op.phase:
                per_phase[op.phase.value].append(ai)
        for name, ais in per_phase.items():
            if ais:
                rep.phase_summary[name] = {"n_ops": len(ais), "mean_ai": sum(ais) / len(ais),
                                           "min_ai": min(ais), "max_ai": max(ais)}
        return rep

    def _estimate_efficiency(self, op: Any, is_compute_bound: bool) -> float:
        if isinstance(op, LLMForwardOp):
            return self._EFF_PREFILL if op.phase == Phase.PREFILL else self._EFF_DECODE
        if isinstance(op, KVFuseOp):
            return self._EFF_FUSE
        if isinstance(op, KVWriteOp):
            return self._EFF_WRITE
        return self._EFF_OTHER

    def plot(self, report: RooflineReport, show_phases: bool = True):
        """Not built (no plotting dependency); returns None."""
        return None


def kernel_roofline(name: str, flops: float, nbytes: float, seconds: float,
                    spec: HardwareSpec = B200_SPEC) -> dict:
    """Roofline point of a timed kernel: bound by its intensity against the ridge point,
    achieved rate and the fraction of the bounding peak (``frac``)."""
    ai = flops / nbytes if nbytes else float("inf")
    tensor = ai > spec.ridge_point
    if seconds <= 0:
        return {"kernel": name, "bound": "tensor" if tensor else "hbm", "frac": None}
    if tensor:
        achieved = flops / seconds / 1e12
        return {"kernel": name, "bound": "tensor", "achieved": round(achieved, 1), "unit": "TFLOP/s",
                "peak": round(spec.peak_flops / 1e12, 1),
                "frac": round(achieved / (spec.peak_flops / 1e12), 4), "ms": round(seconds * 1e3, 4)}
    achieved = nbytes / seconds / 1e9
    return {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "unit": "GB/s",
            "peak": round(spec.hbm_bandwidth / 1e9, 1),
            "frac": round(achieved / (spec.hbm_bandwidth / 1e9), 4), "ms": round(seconds * 1e3, 4)}
