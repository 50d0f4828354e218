"""Tensor -> C-ABI argument helpers (pointers, dtypes, the current stream)."""
from __future__ import annotations

import torch

from . import capi

_DTYPES = {torch.float32: capi.DTYPE_F32, torch.float16: capi.DTYPE_F16,
           torch.bfloat16: capi.DTYPE_BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """cudaStream_t of torch's current stream on ``t``'s device."""
    if not t.is_cuda:
        raise capi.MiError("mi_b200 ops need CUDA tensors (no CPU fallback)")
    return torch.cuda.current_stream(t.device).cuda_stream


def need_i32(name: str, t: torch.Tensor, device) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def check_pool(kv: torch.Tensor):
    """Validate a [P, 2, ps, Hkv, D] NHD pool; return (P, ps, Hkv, D)."""
    if kv.dim() != 5 or kv.shape[1] != 2:
        raise ValueError(f"paged kv cache must be [P, 2, page_size, Hkv, D], got {tuple(kv.shape)}")
    if not kv.is_contiguous():
        raise ValueError("paged kv cache must be contiguous")
    p, _, ps, hkv, d = kv.shape
    return p, ps, hkv, d


def need_on(name: str, t: torch.Tensor, device) -> torch.Tensor:
    """``t`` must live on ``device``: a kernel given another device's (or host)
    memory would read or write through a pointer it cannot use."""
    if t.device != torch.device(device):
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    return t


def check_rows(name: str, t: torch.Tensor, min_rows: int, row_shape: tuple, dtype: torch.dtype,
               device) -> torch.Tensor:
    """A caller-provided output the kernels write as dense rows: ``[>= min_rows,
    *row_shape]``, contiguous, of ``dtype`` on ``device``."""
    if (t.dim() != 1 + len(row_shape) or t.shape[0] < min_rows
            or tuple(t.shape[1:]) != tuple(row_shape)):
        raise ValueError(f"{name} must be [>= {min_rows}, {', '.join(map(str, row_shape))}], "
                         f"got {tuple(t.shape)}")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return need_on(name, t, device)

