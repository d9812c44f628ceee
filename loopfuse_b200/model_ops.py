"""Decoder elementwise ops on the sm_100a library: residual add + RMSNorm and the SwiGLU gate.

Each is one bandwidth-bound kernel in place of the chain of torch elementwise passes a model
would otherwise run around its GEMMs (``lf_add_rmsnorm`` / ``lf_swiglu`` in
``include/loopfuse_b200.h``).  Rounding follows the eager torch sequence: the residual sum is
rounded to bf16, the normalised value is rounded to bf16 before the weight multiply, the SiLU
output is rounded to bf16 before the gate multiply.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import LoopfuseError


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cuda" or t.dtype != torch.bfloat16 or not t.is_contiguous():
        raise LoopfuseError(_lib.LF_EINVAL, f"{name} must be a contiguous CUDA bf16 tensor")


def add_rmsnorm(x: torch.Tensor, delta: Optional[torch.Tensor], w: Optional[torch.Tensor],
                eps: float, out: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """``x += delta`` (in place, when given), then ``rmsnorm(x) * w`` (when ``w`` is given).
    ``x, delta, out [rows, dim]``, ``w [dim]``."""
    _check(x, "x")
    rows, dim = x.shape[0], x.shape[-1]
    if delta is not None:
        _check(delta, "delta")
        if delta.shape != x.shape:
            raise LoopfuseError(_lib.LF_EINVAL, "add_rmsnorm: delta must match x")
    if w is not None:
        _check(w, "w")
        if out is None:
            out = torch.empty_like(x)
        _check(out, "out")
    _lib.call("lf_add_rmsnorm", x.data_ptr(), delta.data_ptr() if delta is not None else None,
              w.data_ptr() if w is not None else None, out.data_ptr() if out is not None else None,
              rows, dim, float(eps), _stream())
    return out


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``silu(gu[:, :F]) * gu[:, F:]`` for a fused ``[rows, 2F]`` gate|up projection."""
    _check(gu, "gu")
    rows, two_f = gu.shape
    out = torch.empty((rows, two_f // 2), dtype=gu.dtype, device=gu.device)
    _lib.call("lf_swiglu", gu.data_ptr(), out.data_ptr(), rows, two_f // 2, _stream())
    return out
