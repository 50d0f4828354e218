"""Fused all-reduce for tensor-parallel decode steps (NVLink peer memory).

``PeerAllReduce`` owns one symmetric buffer per rank (a plain device
allocation of the same size on every rank, mapped into every other rank with
CUDA IPC handles: NVLink P2P mappings, never bound to an NVLink multicast
object, so a rank that ends cannot leave a multicast object behind that
other ranks' GPUs still use): a flag array and
one ``[max_rows, hidden]`` region per call site (two per decoder layer: after
``o_proj`` and after ``down_proj``, plus nothing for the final norm, which
reuses the last ``down_proj`` site). The row-parallel GEMM of a call site
writes its partial straight into its region; ``reduce_add_norm`` then runs
``mi_allreduce_add_rmsnorm``: the all-reduce over peer memory, the residual
add and the RMSNorm in one launch (model.py:115-122, :333-343 after the
sharded projections). Calls with more rows than ``max_rows`` (prefill) take
the NCCL all-reduce instead.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import capi
from ._tensor import check_rows, dtype_code, stream_of

MAX_ROWS = 256          # the kernel's flag slots per rank
_FLAG_BYTES_PER_RANK = MAX_ROWS * 4


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerAllReduce:
    def __init__(self, group, device, dtype: torch.dtype, hidden: int, num_sites: int,
                 max_rows: int = 64):
        if max_rows > MAX_ROWS:
            raise ValueError(f"max_rows {max_rows} > {MAX_ROWS}")
        if hidden % 8:
            raise ValueError("hidden must be a multiple of 8")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device)
        self.dtype, self.hidden, self.max_rows = dtype, hidden, max_rows
        elt = torch.empty((), dtype=dtype).element_size()
        self.flag_off = 0
        self.site_bytes = _align(max_rows * hidden * elt)
        self.data_off0 = _align(self.world * _FLAG_BYTES_PER_RANK)
        total = self.data_off0 + num_sites * self.site_bytes
        self.buf = torch.zeros(total, dtype=torch.uint8, device=self.device)
        self._opened = []       # peer allocations mapped into this process
        self.peer_bases = None
        lib = capi.lib()
        handle = ctypes.create_string_buffer(capi.IPC_HANDLE_BYTES)
        offset = ctypes.c_int64(0)
        capi.call("mi_ipc_export", self.buf.data_ptr(), ctypes.addressof(handle),
                  ctypes.addressof(offset))
        mine = (bytes(handle.raw), int(offset.value))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        bases = []
        try:
            for q, (h, off) in enumerate(everyone):
                if q == self.rank:
                    bases.append(self.buf.data_ptr())
                    continue
                hb = ctypes.create_string_buffer(h, capi.IPC_HANDLE_BYTES)
                base = ctypes.c_void_p(0)
                rc = lib.mi_ipc_open(ctypes.addressof(hb), ctypes.addressof(base))
                if rc != 0:
                    raise capi.MiError(f"mi_ipc_open of rank {q}'s buffer failed: "
                                       f"{lib.mi_last_error().decode(errors='replace')}")
                self._opened.append(base.value)
                bases.append(base.value + off)
        except Exception:
            self._close_mappings()
            raise
        self.peer_bases = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.counters = torch.zeros(MAX_ROWS, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.num_sites = num_sites
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)          # every rank's flags are zero before first use

    def _close_mappings(self) -> None:
        lib = capi.lib()
        while self._opened:
            lib.mi_ipc_close(self._opened.pop())

    def close(self) -> None:
        """Unmap the peers' buffers once no rank uses them any more (collective:
        every rank calls it). This rank's own buffer is freed only after every
        peer has unmapped it."""
        if self.peer_bases is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)     # no rank still reads or writes a peer's buffer
        self._close_mappings()
        dist.barrier(group=self.group)     # every mapping of this rank's buffer is gone
        self.peer_bases = None

    def usable(self, rows: int) -> bool:
        return 0 < rows <= self.max_rows

    def site(self, i: int, rows: int) -> torch.Tensor:
        """This rank's region of call site ``i`` as a ``[rows, hidden]`` tensor."""
        if not 0 <= i < self.num_sites:
            raise IndexError(f"call site {i} of {self.num_sites}")
        start = self.data_off0 + i * self.site_bytes
        elt = torch.empty((), dtype=self.dtype).element_size()
        return self.buf[start:start + rows * self.hidden * elt].view(self.dtype).view(
            rows, self.hidden)

    def reduce_add_norm(self, i: int, rows: int, residual: torch.Tensor, weight: torch.Tensor,
                        eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
        """residual += all-reduce(site i partial); return rms_norm(residual) * weight."""
        if not self.usable(rows):
            raise ValueError(f"rows {rows} outside (0, {self.max_rows}]")
        if not 0 <= i < self.num_sites:
            raise IndexError(f"call site {i} of {self.num_sites}")
        if residual.shape[-1] != self.hidden or residual.numel() != rows * self.hidden:
            raise ValueError("residual must hold rows x hidden elements")
        check_rows("residual", residual.reshape(rows, self.hidden) if residual.is_contiguous()
                   else residual, rows, (self.hidden,), self.dtype, self.device)
        check_rows("weight", weight.unsqueeze(0), 1, (self.hidden,), self.dtype, self.device)
        if out is None:
            out = torch.empty_like(residual)
        elif out.shape != residual.shape:
            raise ValueError("out must have the residual's shape")
        else:
            check_rows("out", out.reshape(rows, self.hidden) if out.is_contiguous() else out,
                       rows, (self.hidden,), self.dtype, self.device)
        capi.call("mi_allreduce_add_rmsnorm", self.peer_bases.data_ptr(),
                  self.data_off0 + i * self.site_bytes, self.flag_off,
                  self.counters.data_ptr(), self.rank, self.world, residual.data_ptr(),
                  weight.data_ptr(), out.data_ptr(), rows, self.hidden, float(eps),
                  dtype_code(self.dtype), self.status.data_ptr(), stream_of(residual))
        return out

    def check_status(self) -> None:
        w = int(self.status.item())
        if w:
            self.status.zero_()
            raise capi.MiError(f"peer all-reduce device status: {capi.status_names(w)}")
