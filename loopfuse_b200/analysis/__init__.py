from .roofline import (A100_SPEC, B200_SPEC, T4_SPEC, TPU_V4_SPEC, HardwareSpec,
                       OpRooflinePoint, RooflineAnalyzer, RooflineReport, kernel_roofline)
