"""Paged prefill attention (kernel 3): drop-in for FlashInfer's prefill wrapper.

``BatchPrefillWithPagedKVCacheWrapper`` keeps the shape of the FlashInfer
wrapper the reference drives (scheduler.py:530-534, :704-716, model.py:235):
ragged queries ``[total_q, Hq, D]`` split by ``qo_indptr``, causal with
bottom-right alignment. ``plan()`` only validates and records pointers.
"""
from __future__ import annotations

import math

import torch

from . import capi
from ._tensor import check_pool, check_rows, dtype_code, need_i32, need_on, ptr, stream_of


class BatchPrefillWithPagedKVCacheWrapper:
    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD", **_unused):
        if kv_layout != "NHD":
            raise ValueError("only the NHD layout (the reference's) is supported")
        if not float_workspace_buffer.is_cuda:
            raise capi.MiError("workspace must be a CUDA tensor (no CPU fallback)")
        self._ws = float_workspace_buffer
        # the tensor-core kernel keeps two work-item counters at the start of
        # the workspace; they must start at zero (each call leaves them so)
        nbytes = self._ws.numel() * self._ws.element_size()
        if nbytes >= 256:
            self._ws.view(torch.uint8)[:256].zero_()
        self._plan = None
        self.status = torch.zeros(1, dtype=torch.int32, device=self._ws.device)

    def plan(self, qo_indptr: torch.Tensor, paged_kv_indptr: torch.Tensor,
             paged_kv_indices: torch.Tensor, paged_kv_last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim_qk: int, page_size: int,
             head_dim_vo: int | None = None, custom_mask=None, packed_custom_mask=None,
             causal: bool = False, pos_encoding_mode: str = "NONE", window_left: int = -1,
             logits_soft_cap: float | None = None, q_data_type=torch.bfloat16,
             kv_data_type=None, sm_scale: float | None = None, **_unused):
        if pos_encoding_mode != "NONE":
            raise ValueError("only pos_encoding_mode='NONE' is supported")
        if custom_mask is not None or packed_custom_mask is not None:
            raise ValueError("custom masks are not supported")
        if window_left != -1 or logits_soft_cap not in (None, 0.0):
            raise ValueError("sliding window / logits soft cap are not supported")
        if head_dim_vo not in (None, head_dim_qk):
            raise ValueError("head_dim_vo must equal head_dim_qk")
        if num_qo_heads % num_kv_heads:
            raise ValueError("num_qo_heads must be a multiple of num_kv_heads")
        dev = self._ws.device
        for name, t in (("qo_indptr", qo_indptr), ("paged_kv_indptr", paged_kv_indptr),
                        ("paged_kv_indices", paged_kv_indices),
                        ("paged_kv_last_page_len", paged_kv_last_page_len)):
            need_i32(name, t, dev)
        if qo_indptr.numel() != paged_kv_indptr.numel():
            raise ValueError("qo_indptr and paged_kv_indptr must have batch+1 entries each")
        self._plan = dict(qo=qo_indptr, indptr=paged_kv_indptr, indices=paged_kv_indices,
                          last=paged_kv_last_page_len, batch=qo_indptr.numel() - 1,
                          hq=num_qo_heads, hkv=num_kv_heads, d=head_dim_qk, ps=page_size,
                          causal=bool(causal),
                          scale=sm_scale if sm_scale is not None else
                          1.0 / math.sqrt(head_dim_qk))

    def run(self, q: torch.Tensor, paged_kv_cache: torch.Tensor, out: torch.Tensor | None = None,
            lse: torch.Tensor | None = None, return_lse: bool = False):
        """``q [total_q, Hq, D]`` -> ``out [total_q, Hq, D]`` (and ``lse``)."""
        pl = self._plan
        if pl is None:
            raise RuntimeError("plan() must be called before run()")
        num_pages, ps, hkv, d = check_pool(paged_kv_cache)
        if (ps, hkv, d) != (pl["ps"], pl["hkv"], pl["d"]):
            raise ValueError("paged kv cache geometry differs from plan()")
        total_q = q.shape[0]
        if q.dim() != 3 or q.shape[1] != pl["hq"] or q.shape[2] != d:
            raise ValueError(f"q must be [total_q, {pl['hq']}, {d}], got {tuple(q.shape)}")
        if q.stride(-1) != 1 or q.dtype != paged_kv_cache.dtype:
            raise ValueError("q needs the pool dtype and a unit stride on head_dim")
        dev = self._ws.device
        need_on("q", q, dev)
        need_on("paged_kv_cache", paged_kv_cache, dev)
        if out is None:
            out = torch.empty((total_q, pl["hq"], d), dtype=q.dtype, device=q.device)
        else:
            check_rows("out", out, total_q, (pl["hq"], d), q.dtype, dev)
        if lse is not None:
            check_rows("lse", lse, total_q, (pl["hq"],), torch.float32, dev)
        elif return_lse:
            lse = torch.empty((total_q, pl["hq"]), dtype=torch.float32, device=q.device)
        ws_bytes = self._ws.numel() * self._ws.element_size()
        capi.call(
            "mi_paged_prefill",
            q.data_ptr(), q.stride(0), q.stride(1), pl["qo"].data_ptr(), total_q,
            paged_kv_cache.data_ptr(), num_pages, ps, hkv, d, dtype_code(q.dtype),
            pl["indptr"].data_ptr(), pl["indices"].data_ptr(), pl["last"].data_ptr(),
            pl["batch"], pl["hq"], int(pl["causal"]), pl["scale"], out.data_ptr(), ptr(lse),
            self._ws.data_ptr(), ws_bytes, self.status.data_ptr(), stream_of(q))
        return (out, lse) if return_lse else out

    def check_status(self) -> None:
        w = int(self.status.item())
        if w:
            self.status.zero_()
            raise capi.MiError(f"paged prefill device status: {capi.status_names(w)}")
