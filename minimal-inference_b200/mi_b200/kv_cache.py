"""Paged KV cache with a device-side page pool (kernel 4).

``PagedKVCache`` keeps the reference's interface and layout
(scheduler.py:168-221): per-layer ``kv_data[P, 2, ps, Hkv, D]`` (NHD, K at
index 0), ``P = max_batch * ceil(max_seq/ps)``, page ``P-1`` reserved as the
scratch page, FIFO allocation, zero-on-release. The free list lives on the
GPU (``free_ring`` + ``pool_ctrl``) and is driven by the library's pool
kernels, so page tables come out identical to the reference's while the
decode step's page growth can run inside a CUDA graph.

Two ways to use it:

* the reference's list API -- ``allocate_pages(n) -> list[int]`` and
  ``release_pages(pages)`` (one launch for all pages and layers). These read
  the popped ids back to the host, i.e. they synchronise.
* the slot API the graph-captured scheduler uses -- each request owns a
  slot row of ``page_table`` on the device; ``slot_alloc`` (admission),
  ``step_prepare`` (page growth + CSR for a step) and ``slot_release``
  (retire) never synchronise.

The host keeps an exact mirror of the free-page count (``num_free_pages``),
so admission control and the out-of-pages error (scheduler.py:208-214) need
no device read.
"""
from __future__ import annotations

import math

import torch

from . import capi
from ._tensor import stream_of


class _FreeCount:
    """``len()``-able stand-in for the reference's ``free_pages`` deque."""

    def __init__(self, cache: "PagedKVCache"):
        self._c = cache

    def __len__(self) -> int:
        return self._c.num_free_pages


class PagedKVCache:
    def __init__(self, config, max_batch_size: int, max_seq_len: int, page_size: int,
                 device, dtype: torch.dtype, num_layers: int | None = None,
                 num_kv_heads: int | None = None):
        device = torch.device(device)
        if device.type != "cuda":
            raise capi.MiError("PagedKVCache lives on a CUDA device (no CPU fallback)")
        self.page_size = page_size
        self.num_layers = config.num_hidden_layers if num_layers is None else num_layers
        self.num_kv_heads = config.num_key_value_heads if num_kv_heads is None else num_kv_heads
        self.head_dim = config.head_dim
        self.device, self.dtype = device, dtype
        self.max_batch_size = max_batch_size
        self.max_pages_per_seq = math.ceil(max_seq_len / page_size)
        self.max_num_pages = max_batch_size * self.max_pages_per_seq
        self.kv_data: list[torch.Tensor] = [
            torch.zeros(self.max_num_pages, 2, page_size, self.num_kv_heads, self.head_dim,
                        device=device, dtype=dtype)
            for _ in range(self.num_layers)
        ]
        self.scratch_page = self.max_num_pages - 1
        self.page_bytes = 2 * page_size * self.num_kv_heads * self.head_dim * \
            torch.empty((), dtype=dtype).element_size()
        self.layer_ptrs = torch.tensor([t.data_ptr() for t in self.kv_data], dtype=torch.int64,
                                       device=device)
        i32 = dict(dtype=torch.int32, device=device)
        self.free_ring = torch.empty(self.max_num_pages, **i32)
        self.pool_ctrl = torch.zeros(4, **i32)
        self.page_table = torch.full((max_batch_size, self.max_pages_per_seq), -1, **i32)
        self.slot_num_pages = torch.zeros(max_batch_size, **i32)
        self.status = torch.zeros(1, **i32)
        capi.call("mi_page_pool_init", self.free_ring.data_ptr(), self.pool_ctrl.data_ptr(),
                  self.max_num_pages, stream_of(self.free_ring))
        self.num_free_pages = self.max_num_pages - 1
        self.free_pages = _FreeCount(self)

    # ---- reference list API ---------------------------------------------
    def allocate_pages(self, num_pages: int) -> list[int]:
        """Pop ``num_pages`` pages FIFO (scheduler.py:208-214); synchronises."""
        if self.num_free_pages < num_pages:
            raise RuntimeError(
                f"Cannot allocate {num_pages} pages, only {self.num_free_pages} free")
        if num_pages == 0:
            return []
        counts = torch.tensor([num_pages], dtype=torch.int32, device=self.device)
        out = torch.empty(num_pages, dtype=torch.int32, device=self.device)
        capi.call("mi_page_alloc", self.free_ring.data_ptr(), self.pool_ctrl.data_ptr(),
                  self.max_num_pages, counts.data_ptr(), 1, out.data_ptr(),
                  self.status.data_ptr(), stream_of(out))
        self.num_free_pages -= num_pages
        return out.tolist()

    def release_pages(self, page_indices) -> None:
        """Zero the pages in every layer, then free them (scheduler.py:216-221)."""
        pages = [int(p) for p in page_indices]
        if not pages:
            return
        t = torch.tensor(pages, dtype=torch.int32, device=self.device)
        capi.call("mi_page_release", self.free_ring.data_ptr(), self.pool_ctrl.data_ptr(),
                  self.max_num_pages, t.data_ptr(), len(pages), self.layer_ptrs.data_ptr(),
                  self.num_layers, self.page_bytes, self.status.data_ptr(), stream_of(t))
        self.num_free_pages += len(pages)

    # ---- slot API (no host synchronisation) --------------------------------
    def slot_alloc(self, slots: torch.Tensor, counts: torch.Tensor, total: int) -> None:
        """Admission: pop ``counts[i]`` pages into slot ``slots[i]`` (device int32)."""
        if self.num_free_pages < total:
            raise RuntimeError(
                f"Cannot allocate {total} pages, only {self.num_free_pages} free")
        capi.call("mi_slot_alloc", self.free_ring.data_ptr(), self.pool_ctrl.data_ptr(),
                  self.max_num_pages, self.page_table.data_ptr(), self.slot_num_pages.data_ptr(),
                  self.max_batch_size, self.max_pages_per_seq, slots.data_ptr(),
                  counts.data_ptr(), slots.numel(), self.status.data_ptr(), stream_of(slots))
        self.num_free_pages -= total

    def slot_release(self, slots: torch.Tensor, total_pages: int) -> None:
        """Retire: zero every page of ``slots`` in every layer and free them."""
        capi.call("mi_slot_release", self.free_ring.data_ptr(), self.pool_ctrl.data_ptr(),
                  self.max_num_pages, self.page_table.data_ptr(), self.slot_num_pages.data_ptr(),
                  self.max_batch_size, self.max_pages_per_seq, slots.data_ptr(), slots.numel(),
                  self.layer_ptrs.data_ptr(), self.num_layers, self.page_bytes,
                  self.status.data_ptr(), stream_of(slots))
        self.num_free_pages += total_pages

    def step_prepare(self, lane_slots: torch.Tensor, lane_positions: torch.Tensor,
                     kv_indptr: torch.Tensor, kv_indices: torch.Tensor,
                     kv_last_page_len: torch.Tensor, append_positions: torch.Tensor,
                     grow: bool = True) -> None:
        """Page growth + CSR metadata of one step, all on the device.

        Graph-capturable. The caller accounts for grown pages in
        ``num_free_pages`` (it knows positions on the host).
        """
        capi.call("mi_step_prepare", self.free_ring.data_ptr(), self.pool_ctrl.data_ptr(),
                  self.max_num_pages, self.page_table.data_ptr(), self.slot_num_pages.data_ptr(),
                  self.max_batch_size, self.max_pages_per_seq, lane_slots.data_ptr(),
                  lane_positions.data_ptr(), lane_slots.numel(), self.page_size, int(grow),
                  kv_indptr.data_ptr(), kv_indices.data_ptr(), kv_indices.numel(),
                  kv_last_page_len.data_ptr(), append_positions.data_ptr(),
                  self.status.data_ptr(), stream_of(lane_slots))

    def slot_pages(self, slot: int) -> list[int]:
        """Pages held by ``slot`` (reads the device table; synchronises)."""
        n = int(self.slot_num_pages[slot].item())
        return self.page_table[slot, :n].tolist()

    def check_status(self) -> None:
        w = int(self.status.item())
        if w:
            self.status.zero_()
            if w == 1:
                raise RuntimeError("page pool exhausted on the device (OUT_OF_PAGES)")
            raise capi.MiError(f"page pool device status: {capi.status_names(w)}")
