"""Phase-specialised kernel selection: ``(KernelTarget, Phase) -> kernel``.

Drop-in for the reference's ``passes/phase_select.py``.  ``PHASE_KERNEL_MAP``
keeps every key and every ``(module, name, notes)`` string of the reference
(``:48-90``), so programs annotated here carry the same metadata.  What changes
is what the names *resolve to*: ``resolve_kernel`` maps the CUDA entries,
``kernels.cuda.async_prefill/agent_prefill_kernel`` and
``kernels.cuda.ring_kv_cache/ring_kv_decode_kernel``, onto this package's
sm_100a prefill and paged decode.  TRITON and PALLAS names stay selectable
(annotation only) but do not execute: this package has one backend and no CPU
fallback, and the EAGER entry is the test oracle, not a runtime path.

The roofline classification (``:130-144``) is kept with the reference's
A100 constants by default, so annotations match the reference bit for bit;
``PhaseSelectPass(hardware="b200")`` classifies against the B200's measured
peaks (``peaks.b200_peaks()``: the machine's measured copy bandwidth and
burst bf16 GEMM throughput, or the built-in figures measured on a B200 of the
build pool when no peaks file is present).
"""
from __future__ import annotations

import importlib
import time
from typing import Callable, List

from .base import Pass, PassResult
from ..ir.dialect import AgentProgram, KernelTarget, LLMForwardOp, Phase
from ..peaks import b200_peaks

A100_PEAK_FLOPS_BF16 = 312e12
A100_HBM_BANDWIDTH = 2.0e12
A100_RIDGE_POINT = A100_PEAK_FLOPS_BF16 / A100_HBM_BANDWIDTH
T4_PEAK_FLOPS_FP16 = 65e12
T4_HBM_BANDWIDTH = 320e9
T4_RIDGE_POINT = T4_PEAK_FLOPS_FP16 / T4_HBM_BANDWIDTH
_B200 = b200_peaks()
B200_PEAK_FLOPS_BF16 = _B200["bf16_tflops"] * 1e12
B200_HBM_BANDWIDTH = _B200["hbm_gbs"] * 1e9
B200_RIDGE_POINT = B200_PEAK_FLOPS_BF16 / B200_HBM_BANDWIDTH

PHASE_KERNEL_MAP = {
    (KernelTarget.TRITON, Phase.PREFILL): (
        "kernels.triton.prefill_attn", "prefill_attention_fwd",
        "large-tile GEMM, block=128x128, compute-optimized"),
    (KernelTarget.TRITON, Phase.DECODE): (
        "kernels.triton.decode_attn", "decode_attention_fwd",
        "streaming load, block=16x64, bandwidth-optimized"),
    (KernelTarget.CUDA, Phase.PREFILL): (
        "kernels.cuda.async_prefill", "agent_prefill_kernel",
        "async memcpy pipeline, double-buffered, warp-specialized"),
    (KernelTarget.CUDA, Phase.DECODE): (
        "kernels.cuda.ring_kv_cache", "ring_kv_decode_kernel",
        "ring-buffer KV, async prefetch, tensor core MMA"),
    (KernelTarget.PALLAS, Phase.PREFILL): (
        "kernels.pallas.agent_attn", "pallas_prefill_fwd",
        "TPU VMEM-resident QK^T, column-major K layout"),
    (KernelTarget.PALLAS, Phase.DECODE): (
        "kernels.pallas.agent_attn", "pallas_decode_fwd",
        "TPU streaming decode, HBM bandwidth optimized"),
    (KernelTarget.EAGER, Phase.PREFILL): (
        "torch.nn.functional", "scaled_dot_product_attention", "PyTorch eager baseline"),
    (KernelTarget.EAGER, Phase.DECODE): (
        "torch.nn.functional", "scaled_dot_product_attention",
        "PyTorch eager baseline (same kernel — the suboptimality we measure)"),
}

_PEAKS = {
    # hardware -> {target: (ridge FLOP/B, peak FLOP/s, peak B/s)}
    "a100": {KernelTarget.CUDA: (A100_RIDGE_POINT, A100_PEAK_FLOPS_BF16, A100_HBM_BANDWIDTH),
             KernelTarget.TRITON: (A100_RIDGE_POINT, A100_PEAK_FLOPS_BF16, A100_HBM_BANDWIDTH),
             KernelTarget.PALLAS: (200.0, 275e12, 1.2e12),
             KernelTarget.EAGER: (A100_RIDGE_POINT, A100_PEAK_FLOPS_BF16, A100_HBM_BANDWIDTH)},
    "b200": {t: (B200_RIDGE_POINT, B200_PEAK_FLOPS_BF16, B200_HBM_BANDWIDTH)
             for t in KernelTarget},
}


def resolve_kernel(module: str, name: str, target: KernelTarget = KernelTarget.CUDA) -> Callable:
    """Return the callable a ``(kernel_module, kernel_name)`` annotation names.

    Only CUDA annotations execute; they resolve inside ``loopfuse_b200``
    (``kernels.cuda.async_prefill`` -> ``loopfuse_b200.kernels.cuda.async_prefill``).
    Any other target raises ``NotImplementedError``: there is no silent
    fallback to another backend or to the CPU.
    """
    if target is not KernelTarget.CUDA or not module.startswith("kernels.cuda."):
        raise NotImplementedError(
            f"kernel {module}.{name} (target {target.value}) is not executable in "
            f"loopfuse_b200; only KernelTarget.CUDA runs (sm_100a)")
    mod = importlib.import_module("loopfuse_b200." + module)
    return getattr(mod, name)


class PhaseSelectPass(Pass):
    """Annotate every ``LLMForwardOp`` with its kernel and roofline class.

    Writes ``kernel_module``, ``kernel_name``, ``kernel_notes``,
    ``is_compute_bound``, ``arithmetic_intensity`` and
    ``roofline_efficiency`` into ``op.metadata`` and sets ``op.target``;
    unknown ``(target, phase)`` keys fall back to the EAGER entry, as in the
    reference (``:119-121``).
    """

    def __init__(self, hardware: str = "a100"):
        if hardware not in _PEAKS:
            raise ValueError(f"unknown hardware profile {hardware!r}")
        self.hardware = hardware

    def run(self, prog: AgentProgram) -> PassResult:
        start = time.time()
        target = prog.target or KernelTarget.EAGER
        n_pre = n_dec = 0
        changed = False
        for op in prog.ops_by_type(LLMForwardOp):
            phase = op.phase or Phase.DECODE
            key = (target, phase) if (target, phase) in PHASE_KERNEL_MAP else (KernelTarget.EAGER,
                                                                                 phase)
            module, fn, notes = PHASE_KERNEL_MAP[key]
            op.metadata.update(kernel_module=module, kernel_name=fn, kernel_notes=notes)
            op.target = target
            ridge, peak_flops, peak_bw = self._peaks(target)
            ai = op.arithmetic_intensity()
            compute_bound = ai > ridge
            op.metadata["is_compute_bound"] = compute_bound
            op.metadata["arithmetic_intensity"] = round(ai, 2)
            if compute_bound:
                eff = min(1.0, op.estimated_flops() / (peak_flops * 1e-3))
            else:
                eff = min(1.0, op.estimated_bytes() / (peak_bw * 1e-3))
            op.metadata["roofline_efficiency"] = round(eff, 3)
            if phase == Phase.PREFILL:
                n_pre += 1
            else:
                n_dec += 1
            changed = True
        ann: List[str] = [f"annotated {n_pre} PREFILL ops + {n_dec} DECODE ops "
                          f"for target={target.value}"]
        return self._result(prog, changed, ann, start)

    def _peaks(self, target: KernelTarget):
        table = _PEAKS[self.hardware]
        return table.get(target, table[KernelTarget.CUDA])

    def _ridge_point(self, target: KernelTarget) -> float:
        return self._peaks(target)[0]

    def _peak_flops(self, target: KernelTarget) -> float:
        return self._peaks(target)[1]

    def _peak_bandwidth(self, target: KernelTarget) -> float:
        return self._peaks(target)[2]
