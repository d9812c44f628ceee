"""B200 roofline denominators: measured copy bandwidth and dense bf16 GEMM throughput.

``b200_peaks()`` reads a peaks file written by a measurement run on the machine itself (a
STREAM-style ``copy_`` of 1 Gi bf16 elements for ``hbm_gbs``; a bf16 8192^3 ``matmul`` for
``bf16_tflops`` (best of 10, burst) and ``bf16_tflops_sustained`` (back to back for seconds,
under the power cap)).  It looks at ``$LOOPFUSE_B200_PEAKS`` first, then ``MEASURED_PEAKS.json``
at the repository root.  Without either it returns the figures such a run measured on a B200
of the build machine's pool (6546 GB/s, 1638 / 1375 TFLOP/s), marked ``source="built-in"``.
"""
from __future__ import annotations

import json
import os
from functools import lru_cache

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILT_IN = {"hbm_gbs": 6545.9, "bf16_tflops": 1637.7, "bf16_tflops_sustained": 1375.4}


@lru_cache(maxsize=None)
def b200_peaks() -> dict:
    for path in (os.environ.get("LOOPFUSE_B200_PEAKS"), os.path.join(_ROOT, "MEASURED_PEAKS.json")):
        if not path:
            continue
        try:
            with open(path) as f:
                d = json.load(f)
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                    "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained",
                                                         d["bf16_tflops"])),
                    "source": "measured", "path": path}
        except (OSError, KeyError, ValueError, TypeError):
            continue
    return dict(BUILT_IN, source="built-in")
