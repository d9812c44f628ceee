"""Decoder ops on the sm_100a library: residual add + RMSNorm, the SwiGLU gate, and a
weight-streaming tcgen05 GEMM for decode batches (``gemm_skinny``).

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


_SKINNY_MAX_M = 128
_skinny_ws: dict = {}


def _sm_count(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def skinny_workspace_bytes(m: int, n: int, k: int, sm_count: int) -> int:
    out = _lib.c_size_t(0)
    _lib.call("lf_gemm_skinny_workspace_size", int(m), int(n), int(k), int(sm_count),
              _lib.ctypes.byref(out))
    return int(out.value)


def gemm_skinny(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ w`` for a decode batch: ``x [M, K]`` (1 <= M <= 128), ``w [K, N]``, bf16, on the
    weight-streaming tcgen05 GEMM (``lf_gemm_skinny``).  Without ``workspace`` the partial-sum
    buffer is a per-device cache grown on demand (pass one explicitly inside a CUDA graph that
    must not allocate)."""
    _check(x, "x")
    _check(w, "w")
    m, k = x.shape
    k2, n = w.shape
    if k2 != k:
        raise LoopfuseError(_lib.LF_EINVAL, f"gemm_skinny: x is [{m}, {k}] but w is [{k2}, {n}]")
    if not 1 <= m <= _SKINNY_MAX_M:
        raise LoopfuseError(_lib.LF_EINVAL, f"gemm_skinny: M = {m} outside 1..{_SKINNY_MAX_M}")
    sms = _sm_count(x.device)
    need = skinny_workspace_bytes(m, n, k, sms)
    if workspace is None:
        key = x.device.index
        workspace = _skinny_ws.get(key)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=x.device)
            _skinny_ws[key] = workspace
    if workspace.numel() < need:
        raise LoopfuseError(_lib.LF_EINVAL, f"gemm_skinny: workspace of {workspace.numel()} bytes, "
                                            f"need {need}")
    if out is None:
        out = torch.empty((m, n), dtype=x.dtype, device=x.device)
    _check(out, "out")
    _lib.call("lf_gemm_skinny", x.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k,
              workspace.data_ptr(), workspace.numel(), sms, _stream())
    return out
