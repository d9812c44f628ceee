"""Pass harness: ``Pass``, ``PassResult``, ``PassManager`` (reference ``passes/base.py:19-94``)."""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List, Optional

from ..ir.dialect import AgentProgram


@dataclass
class PassResult:
    pass_name: str
    changed: bool
    duration_ms: float
    annotations: List[str] = field(default_factory=list)


class Pass:
    @property
    def name(self) -> str:
        return type(self).__name__

    def run(self, prog: AgentProgram) -> PassResult:
        raise NotImplementedError

    def _result(self, prog: AgentProgram, changed: bool, annotations: List[str],
                start: float) -> PassResult:
        for a in annotations:
            prog.add_annotation(f"[{self.name}] {a}")
        return PassResult(self.name, changed, (time.time() - start) * 1000, annotations)


class PassManager:
    def __init__(self, passes: Optional[List[Pass]] = None):
        self.passes: List[Pass] = list(passes or [])

    def add_pass(self, p: Pass) -> "PassManager":
        self.passes.append(p)
        return self

    def run(self, prog: AgentProgram) -> List[PassResult]:
        return [p.run(prog) for p in self.passes]

    def run_until_fixed_point(self, prog: AgentProgram,
                              max_iterations: int = 10) -> List[PassResult]:
        """Run the pipeline repeatedly until a whole round changes nothing, at most
        ``max_iterations`` rounds (reference ``passes/base.py:81-94``); returns every result."""
        results: List[PassResult] = []
        for _ in range(max_iterations):
            round_results = self.run(prog)
            results.extend(round_results)
            if not any(r.changed for r in round_results):
                break
        return results
