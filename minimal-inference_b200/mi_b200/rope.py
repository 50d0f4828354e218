"""RoPE cos/sin tables.

The fused append kernel rotates K (and, in the same launch, Q) from these
tables, so they must hold the very bits the reference's tables hold: built in
fp32 on the CPU exactly as ``precompute_rope`` does (``model.py:79-89``:
``inv_freq = 1/theta**(arange(0,D,2)/D)``, ``outer(t, inv_freq)``, the two
halves concatenated, ``cos``/``sin``), then cast to the model dtype the way
``Model.to(dtype)`` casts the registered buffers.
"""
from __future__ import annotations

import torch


def rope_tables(head_dim: int, max_pos: int, theta: float,
                dtype: torch.dtype = torch.float32, device="cpu"):
    """``(cos, sin)`` of shape ``[max_pos, head_dim]`` in ``dtype`` on ``device``."""
    # built on the host whatever the default device is (e.g. a meta-device
    # model construction)
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device="cpu").float() / head_dim))
    t = torch.arange(max_pos, dtype=torch.float32, device="cpu")
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    cos, sin = emb.cos(), emb.sin()
    return (cos.to(dtype).to(device).contiguous(),
            sin.to(dtype).to(device).contiguous())
