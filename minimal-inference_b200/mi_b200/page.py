"""KV append (kernel 1): drop-in for ``flashinfer.page.append_paged_kv_cache``.

Same arguments and in-place semantics as the call at model.py:207-216
(FlashInfer page.py:280-290, NHD layout). Keyword-only extensions fuse the
RoPE of model.py:169-170 into the same launch: pass the model's cos/sin
tables and the raw (un-rotated) K; pass ``q``/``q_out`` to rotate the
queries too.
"""
from __future__ import annotations

import torch

from . import capi
from ._tensor import check_pool, dtype_code, need_i32, need_on, ptr, stream_of


def append_paged_kv_cache(append_key: torch.Tensor, append_value: torch.Tensor,
                          batch_indices: torch.Tensor, positions: torch.Tensor,
                          paged_kv_cache: torch.Tensor, kv_indices: torch.Tensor,
                          kv_indptr: torch.Tensor, kv_last_page_len: torch.Tensor,
                          kv_layout: str = "NHD", *, rope_cos: torch.Tensor | None = None,
                          rope_sin: torch.Tensor | None = None,
                          rope_positions: torch.Tensor | None = None,
                          q: torch.Tensor | None = None, q_out: torch.Tensor | None = None,
                          scratch_page: int = -1, status: torch.Tensor | None = None) -> None:
    """Append ``append_key``/``append_value`` ``[nnz, Hkv, D]`` into the pages.

    Token ``i`` of request ``batch_indices[i]`` at ``positions[i]`` lands on
    page ``kv_indices[kv_indptr[b] + pos // ps]``, slot ``pos % ps``. With
    ``rope_cos``/``rope_sin`` (``[max_pos, D]``, model dtype) K is rotated on
    the way (bit-identical to ``apply_rotary_emb``); with ``q``/``q_out``
    (``[nnz, Hq, D]``) the queries are rotated into ``q_out``.
    """
    if kv_layout != "NHD":
        raise ValueError("only the NHD layout (the reference's) is supported")
    dev = paged_kv_cache.device
    num_pages, ps, hkv, d = check_pool(paged_kv_cache)
    nnz = append_key.shape[0]
    if append_key.shape != (nnz, hkv, d) or append_value.shape != (nnz, hkv, d):
        raise ValueError(f"append_key/value must be [nnz, {hkv}, {d}], got "
                         f"{tuple(append_key.shape)} / {tuple(append_value.shape)}")
    if append_key.stride(-1) != 1 or append_value.stride(-1) != 1:
        raise ValueError("append_key/value need a unit stride on head_dim")
    dt = paged_kv_cache.dtype
    for name, t in (("append_key", append_key), ("append_value", append_value)):
        if t.dtype != dt or t.device != dev:
            raise ValueError(f"{name} must be {dt} on {dev}")
    for name, t in (("batch_indices", batch_indices), ("positions", positions),
                    ("kv_indices", kv_indices), ("kv_indptr", kv_indptr)):
        need_i32(name, t, dev)
    if batch_indices.numel() < nnz or positions.numel() < nnz:
        raise ValueError("batch_indices/positions shorter than nnz")
    rope_max = 0
    if rope_cos is not None or rope_sin is not None:
        if rope_cos is None or rope_sin is None:
            raise ValueError("pass both rope_cos and rope_sin")
        if rope_cos.dtype != dt or rope_sin.dtype != dt or rope_cos.shape[-1] != d:
            raise ValueError("rope tables must be [max_pos, head_dim] in the pool dtype")
        if not (rope_cos.is_contiguous() and rope_sin.is_contiguous()):
            raise ValueError("rope tables must be contiguous")
        need_on("rope_cos", rope_cos, dev)
        need_on("rope_sin", rope_sin, dev)
        rope_max = rope_cos.shape[0]
    if rope_positions is not None:
        need_i32("rope_positions", rope_positions, dev)
    hq = 0
    if q is not None:
        if q_out is None or rope_max == 0:
            raise ValueError("query rotation needs q_out and the rope tables")
        hq = q.shape[1]
        if q.shape != (nnz, hq, d) or q_out.shape != (nnz, hq, d):
            raise ValueError("q/q_out must be [nnz, Hq, D]")
        if q.stride(-1) != 1 or q_out.stride(-1) != 1 or q.dtype != dt or q_out.dtype != dt:
            raise ValueError("q/q_out need the pool dtype and a unit stride on head_dim")
        need_on("q", q, dev)
        need_on("q_out", q_out, dev)
    if status is not None:
        need_i32("status", status, dev)
    capi.call(
        "mi_append_paged_kv_cache",
        append_key.data_ptr(), append_key.stride(0), append_key.stride(1),
        append_value.data_ptr(), append_value.stride(0), append_value.stride(1),
        batch_indices.data_ptr(), positions.data_ptr(), nnz,
        paged_kv_cache.data_ptr(), num_pages, ps, hkv, d, dtype_code(dt),
        kv_indices.data_ptr(), kv_indptr.data_ptr(), kv_indptr.numel() - 1,
        ptr(rope_cos), ptr(rope_sin), rope_max, ptr(rope_positions),
        ptr(q), q.stride(0) if q is not None else 0, q.stride(1) if q is not None else 0,
        ptr(q_out), q_out.stride(0) if q is not None else 0,
        q_out.stride(1) if q is not None else 0, hq,
        scratch_page, ptr(status), stream_of(paged_kv_cache))
