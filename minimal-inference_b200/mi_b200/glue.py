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


_PROJ_STATUS: dict[int, torch.Tensor] = {}
PROJ_MAX_ROWS = 32


def proj_status(device: torch.device) -> torch.Tensor:
    """The int32 status word proj_small_m calls on ``device`` OR their
    MI_STATUS_* bits into (MI_STATUS_TIMEOUT: a bounded wait gave up)."""
    idx = device.index or 0
    st = _PROJ_STATUS.get(idx)
    if st is None:
        st = _PROJ_STATUS[idx] = torch.zeros(1, dtype=torch.int32, device=device)
    return st


def proj_small_m(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                 out: torch.Tensor | None = None,
                 status: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T (+ bias)`` for ``x`` of at most 32 rows: ``F.linear``
    at decode batch sizes, streaming ``weight`` ([n, k], the nn.Linear
    layout, rows contiguous) once from HBM (``mi_proj_small_m``).

    ``x`` is ``[..., k]`` with contiguous rows (row stride >= k), ``out`` (if
    given) ``[..., n]`` with contiguous rows; one dtype (bf16 / fp16)
    throughout; ``k`` a multiple of 64. ``status``: int32 device word for
    MI_STATUS_* bits (default: ``proj_status(device)``)."""
    k = x.shape[-1]
    n = weight.shape[0]
    x2 = x.reshape(-1, k)
    m = x2.shape[0]
    if m > PROJ_MAX_ROWS:
        raise ValueError(f"proj_small_m: {m} rows > {PROJ_MAX_ROWS}")
    if weight.dim() != 2 or weight.shape[1] != k or weight.stride(1) != 1:
        raise ValueError("proj_small_m: weight must be [n, k] with contiguous rows")
    if x2.stride(-1) != 1 or weight.dtype != x.dtype:
        raise ValueError("proj_small_m: x rows must be contiguous, of weight's dtype")
    if bias is not None and (bias.shape != (n,) or bias.dtype != x.dtype or bias.stride(0) != 1):
        raise ValueError("proj_small_m: bias must be a contiguous [n] of x's dtype")
    dev = x.device
    need_on("weight", weight, dev)
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=dev)
    elif out.shape != (*x.shape[:-1], n) or out.dtype != x.dtype:
        raise ValueError("proj_small_m: out must be [..., n] of x's dtype")
    y2 = out.view(-1, n)
    if y2.stride(-1) != 1:
        raise ValueError("proj_small_m: out rows must be contiguous")
    need_on("out", out, dev)
    if m == 0:
        return out
    capi.call("mi_proj_small_m", ptr(x2), x2.stride(0) if m > 1 else k, ptr(weight),
              weight.stride(0), ptr(bias), ptr(y2), y2.stride(0) if m > 1 else n, m, n, k,
              dtype_code(x.dtype), ptr(status if status is not None else proj_status(dev)),
              stream_of(x))
    return out
