"""Decode-step glue kernels: fused residual-add + RMSNorm, fused SiLU * up.

Both replace short chains of torch elementwise kernels in the decoder layer
(model.py:115-122, :301-311, :333-343) with one launch each from
``libmi_paged.so``; they raise if the library is missing.
"""
from __future__ import annotations

import torch

from . import capi
from ._tensor import dtype_code, need_on, ptr, stream_of


def add_rmsnorm(x: torch.Tensor | None, residual: torch.Tensor, weight: torch.Tensor,
                eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual += x`` (in place, rounded to its dtype; skipped when ``x`` is
    None), then return ``F.rms_norm(residual, weight, eps)``.

    ``residual``/``x``/``out`` are contiguous ``[..., hidden]`` of one dtype;
    ``weight`` is ``[hidden]`` of the same dtype."""
    hidden = residual.shape[-1]
    if not residual.is_contiguous():
        raise ValueError("add_rmsnorm: residual must be contiguous")
    if weight.shape != (hidden,) or weight.dtype != residual.dtype:
        raise ValueError("add_rmsnorm: weight must be [hidden] with the residual's dtype")
    if x is not None and (x.shape != residual.shape or x.dtype != residual.dtype
                          or not x.is_contiguous()):
        raise ValueError("add_rmsnorm: x must match residual (shape, dtype, contiguous)")
    dev = residual.device
    need_on("weight", weight, dev)
    if x is not None:
        need_on("x", x, dev)
    rows = residual.numel() // hidden
    if out is None:
        out = torch.empty_like(residual)
    elif out.shape != residual.shape or out.dtype != residual.dtype or not out.is_contiguous():
        raise ValueError("add_rmsnorm: out must be contiguous with the residual's shape and dtype")
    need_on("out", out, dev)
    capi.call("mi_add_rmsnorm", ptr(x), ptr(residual), ptr(weight.contiguous()), ptr(out),
              rows, hidden, float(eps), dtype_code(residual.dtype), stream_of(residual))
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.silu(gate_up[..., :I]) * gate_up[..., I:]`` for contiguous
    ``[..., 2I]`` input (the fused gate/up GEMM output)."""
    if not gate_up.is_contiguous() or gate_up.shape[-1] % 2:
        raise ValueError("silu_mul: gate_up must be contiguous [..., 2*inter]")
    inter = gate_up.shape[-1] // 2
    rows = gate_up.numel() // (2 * inter)
    if out is None:
        out = torch.empty(*gate_up.shape[:-1], inter, dtype=gate_up.dtype,
                          device=gate_up.device)
    elif (out.shape != (*gate_up.shape[:-1], inter) or out.dtype != gate_up.dtype
          or not out.is_contiguous()):
        raise ValueError("silu_mul: out must be contiguous [..., inter] of gate_up's dtype")
    need_on("out", out, gate_up.device)
    capi.call("mi_silu_mul", ptr(gate_up), ptr(out), rows, inter, dtype_code(gate_up.dtype),
              stream_of(gate_up))
    return out
