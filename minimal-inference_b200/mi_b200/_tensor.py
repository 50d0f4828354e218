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
