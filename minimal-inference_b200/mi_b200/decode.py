"""Paged decode attention (kernel 2): drop-in for FlashInfer's decode wrapper.

``BatchDecodeWithPagedKVCacheWrapper`` keeps the shape of the FlashInfer
wrapper the reference constructs and drives (scheduler.py:535-539,
:905-916, model.py:235): ``plan()`` records the CSR page table, ``run(q,
kv_data)`` computes attention. ``plan()`` does no host work beyond
validation (the kernel plans its split-K on the device), so it may run
inside or outside a CUDA graph and never synchronises.
"""
from __future__ import annotations

import math

import torch

from . import capi
from ._tensor import check_pool, check_rows, dtype_code, need_i32, need_on, ptr, stream_of


class BatchDecodeWithPagedKVCacheWrapper:
    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, **_unused):
        if kv_layout != "NHD":
            raise ValueError("only the NHD layout (the reference's) is supported")
        if not float_workspace_buffer.is_cuda:
            raise capi.MiError("workspace must be a CUDA tensor (no CPU fallback)")
        if float_workspace_buffer.data_ptr() % 256:
            raise ValueError("workspace must be 256-byte aligned")
        self._ws = float_workspace_buffer
        # split-K counters must start at zero; every launch leaves them at zero
        self._ws.zero_()
        self._plan = None
        self.status = torch.zeros(1, dtype=torch.int32, device=self._ws.device)

    def plan(self, indptr: torch.Tensor, indices: torch.Tensor, last_page_len: torch.Tensor,
             num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
             pos_encoding_mode: str = "NONE", window_left: int = -1,
             logits_soft_cap: float | None = None, q_data_type=torch.bfloat16,
             kv_data_type=None, data_type=None, sm_scale: float | None = None, **_unused):
        if pos_encoding_mode != "NONE":
            raise ValueError("only pos_encoding_mode='NONE' is supported (RoPE is applied "
                             "by the append kernel)")
        if window_left != -1 or logits_soft_cap not in (None, 0.0):
            raise ValueError("sliding window / logits soft cap are not supported")
        if num_qo_heads % num_kv_heads:
            raise ValueError("num_qo_heads must be a multiple of num_kv_heads")
        dev = self._ws.device
        for name, t in (("indptr", indptr), ("indices", indices),
                        ("last_page_len", last_page_len)):
            need_i32(name, t, dev)
        batch = indptr.numel() - 1
        need = capi.lib().mi_paged_decode_workspace_size(batch, num_qo_heads, num_kv_heads,
                                                          head_dim)
        if need > self._ws.numel() * self._ws.element_size():
            raise capi.MiError(f"decode workspace too small: need {need} bytes")
        self._plan = dict(indptr=indptr, indices=indices, last=last_page_len, batch=batch,
                          hq=num_qo_heads, hkv=num_kv_heads, d=head_dim, ps=page_size,
                          scale=sm_scale if sm_scale is not None else 1.0 / math.sqrt(head_dim))

    def run(self, q: torch.Tensor, paged_kv_cache: torch.Tensor, out: torch.Tensor | None = None,
            lse: torch.Tensor | None = None, return_lse: bool = False):
        """``q [B, Hq, D]`` -> ``out [B, Hq, D]`` (and ``lse [B, Hq]``)."""
        pl = self._plan
        if pl is None:
            raise RuntimeError("plan() must be called before run()")
        num_pages, ps, hkv, d = check_pool(paged_kv_cache)
        if (ps, hkv, d) != (pl["ps"], pl["hkv"], pl["d"]):
            raise ValueError("paged kv cache geometry differs from plan()")
        b = pl["batch"]
        if q.dim() != 3 or q.shape[0] < b or q.shape[1] != pl["hq"] or q.shape[2] != d:
            raise ValueError(f"q must be [{b}, {pl['hq']}, {d}], got {tuple(q.shape)}")
        if q.stride(-1) != 1 or q.dtype != paged_kv_cache.dtype:
            raise ValueError("q needs the pool dtype and a unit stride on head_dim")
        dev = self._ws.device
        need_on("q", q, dev)
        need_on("paged_kv_cache", paged_kv_cache, dev)
        if out is None:
            out = torch.empty((b, pl["hq"], d), dtype=q.dtype, device=q.device)
        else:
            check_rows("out", out, b, (pl["hq"], d), q.dtype, dev)
        if lse is not None:
            check_rows("lse", lse, b, (pl["hq"],), torch.float32, dev)
        elif return_lse:
            lse = torch.empty((b, pl["hq"]), dtype=torch.float32, device=q.device)
        capi.call(
            "mi_paged_decode",
            q.data_ptr(), q.stride(0), q.stride(1),
            paged_kv_cache.data_ptr(), num_pages, ps, hkv, d, dtype_code(q.dtype),
            pl["indptr"].data_ptr(), pl["indices"].data_ptr(), pl["last"].data_ptr(), b,
            pl["hq"], pl["scale"], out.data_ptr(), ptr(lse),
            self._ws.data_ptr(), self._ws.numel() * self._ws.element_size(),
            self.status.data_ptr(), stream_of(q))
        return (out, lse) if return_lse else out

    def run_with_append(self, q: torch.Tensor, paged_kv_cache: torch.Tensor,
                        append_key: torch.Tensor, append_value: torch.Tensor,
                        rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                        out: torch.Tensor | None = None,
                        status: torch.Tensor | None = None,
                        positions: torch.Tensor | None = None,
                        scratch_page: int = -1) -> torch.Tensor:
        """A decode step with its append fused in (extension, no FlashInfer
        counterpart): ``q`` are the raw queries ``[B, Hq, D]``,
        ``append_key``/``append_value`` the raw new K / V ``[B, Hkv, D]`` of
        each request's token at position ``kv_len - 1`` (the planned page
        table already counts it). Same pages and output, bit for bit, as
        ``append_paged_kv_cache(k, v, arange(B), kv_len - 1, ..., rope tables,
        q=q, q_out=q_rot)`` followed by ``run(q_rot)``; shapes the fused kernel
        does not cover take exactly those two calls, with ``positions`` and
        ``scratch_page`` passed to the append when given (a scheduler's
        padded lanes have no pages and append into its scratch page; the
        fused kernel leaves such lanes out). Device-side problems are
        flagged in ``status`` (default: this wrapper's)."""
        pl = self._plan
        if pl is None:
            raise RuntimeError("plan() must be called before run_with_append()")
        num_pages, ps, hkv, d = check_pool(paged_kv_cache)
        if (ps, hkv, d) != (pl["ps"], pl["hkv"], pl["d"]):
            raise ValueError("paged kv cache geometry differs from plan()")
        b, dt, dev = pl["batch"], paged_kv_cache.dtype, self._ws.device
        need_on("paged_kv_cache", paged_kv_cache, dev)
        for name, t, heads in (("q", q, pl["hq"]), ("append_key", append_key, hkv),
                               ("append_value", append_value, hkv)):
            if t.dim() != 3 or t.shape[0] < b or t.shape[1] != heads or t.shape[2] != d:
                raise ValueError(f"{name} must be [{b}, {heads}, {d}], got {tuple(t.shape)}")
            if t.stride(-1) != 1 or t.dtype != dt:
                raise ValueError(f"{name} needs the pool dtype and a unit stride on head_dim")
            need_on(name, t, dev)
        for name, t in (("rope_cos", rope_cos), ("rope_sin", rope_sin)):
            if t.dim() != 2 or t.shape[1] != d or t.dtype != dt or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous [max_pos, {d}] table of {dt}")
            need_on(name, t, dev)
        if rope_cos.shape != rope_sin.shape:
            raise ValueError("rope_cos and rope_sin differ in shape")
        if out is None:
            out = torch.empty((b, pl["hq"], d), dtype=dt, device=dev)
        else:
            check_rows("out", out, b, (pl["hq"], d), dt, dev)
        st = self.status if status is None else need_i32("status", status, dev)
        lib = capi.lib()
        rc = lib.mi_paged_decode_append(
            q.data_ptr(), q.stride(0), q.stride(1),
            append_key.data_ptr(), append_key.stride(0), append_key.stride(1),
            append_value.data_ptr(), append_value.stride(0), append_value.stride(1),
            rope_cos.data_ptr(), rope_sin.data_ptr(), rope_cos.shape[0],
            paged_kv_cache.data_ptr(), num_pages, ps, hkv, d, dtype_code(dt),
            pl["indptr"].data_ptr(), pl["indices"].data_ptr(), pl["last"].data_ptr(), b,
            pl["hq"], pl["scale"], out.data_ptr(), None,
            self._ws.data_ptr(), self._ws.numel() * self._ws.element_size(), st.data_ptr(),
            stream_of(q))
        if rc == capi.ERR_UNSUPPORTED:
            from .page import append_paged_kv_cache
            if positions is None:
                npages = pl["indptr"][1:b + 1] - pl["indptr"][:b]
                positions = ((npages - 1) * ps + pl["last"][:b] - 1).clamp(min=0)
                positions = positions.to(torch.int32)
            q_rot = torch.empty((b, pl["hq"], d), dtype=dt, device=dev)
            append_paged_kv_cache(append_key[:b], append_value[:b],
                                  torch.arange(b, dtype=torch.int32, device=dev), positions,
                                  paged_kv_cache, pl["indices"], pl["indptr"], pl["last"],
                                  rope_cos=rope_cos, rope_sin=rope_sin, q=q[:b], q_out=q_rot,
                                  scratch_page=scratch_page, status=st)
            return self.run(q_rot, paged_kv_cache, out=out)
        if rc != 0:
            msg = lib.mi_last_error().decode(errors="replace")
            raise capi.MiError(f"mi_paged_decode_append failed (code {rc}): {msg}")
        return out

    def check_status(self) -> None:
        """Synchronise and raise if a launch flagged a device-side problem."""
        w = int(self.status.item())
        if w:
            self.status.zero_()
            raise capi.MiError(f"paged decode device status: {capi.status_names(w)}")
