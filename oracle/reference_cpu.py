"""CPU port of the reference's own decode-attention path -- TEST/BASELINE ONLY.

The reference runs on the CPU through its padded path (the scheduler picks it
whenever the device is not CUDA, scheduler.py:504): a per-slot padded cache
``[Bmax, Hkv, max_seq, D]`` (``BatchedKVCache``, scheduler.py:98-160) and
PyTorch SDPA (``Attention._pytorch_attention``, model.py:254-298). This module
restates one layer of one decode step of that path so ``bench.py`` can time
it on the GPU box's host cores as the CPU baseline (``--impl reference`` and
the ``cpu_baseline`` key). It follows, per step:

1. ``get_batch_caches`` + trim: ``k[slots][:, :, :max_kv_len].contiguous()``
   (scheduler.py:786-791, :143-147);
2. the per-lane write of the new K/V at each position (model.py:269-277);
3. GQA by ``repeat_interleave`` (model.py:287-288);
4. SDPA with the per-lane length mask (scheduler.py:793-800, model.py:293-295);
5. write-back of the new entries into the master cache
   (scheduler.py:811, :149-160).

Only ``bench.py``'s CPU legs and ``tests/`` use it.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


class PaddedDecodeLayer:
    """One layer's padded KV cache and its decode step, as the reference runs it."""

    def __init__(self, batch: int, hkv: int, max_seq: int, d: int, dtype=torch.bfloat16):
        self.k = torch.zeros(batch, hkv, max_seq, d, dtype=dtype)
        self.v = torch.zeros(batch, hkv, max_seq, d, dtype=dtype)
        self.dtype = dtype

    def fill(self, lens, seed: int = 0) -> None:
        """Random contents for the first ``lens[b]`` positions of each slot."""
        g = torch.Generator().manual_seed(seed)
        for b, n in enumerate(lens):
            self.k[b, :, :n] = torch.randn(self.k.shape[1], n, self.k.shape[3], generator=g)
            self.v[b, :, :n] = torch.randn(self.v.shape[1], n, self.v.shape[3], generator=g)

    def step(self, slots: list[int], positions: list[int], q: torch.Tensor, k_new: torch.Tensor,
             v_new: torch.Tensor) -> torch.Tensor:
        """q ``[B, Hq, 1, D]``, k/v ``[B, Hkv, 1, D]`` -> out ``[B, 1, Hq*D]``."""
        bsz, hq = q.shape[0], q.shape[1]
        groups = hq // self.k.shape[1]
        max_kv = max(positions) + 1
        kb = self.k[slots][:, :, :max_kv].contiguous()
        vb = self.v[slots][:, :, :max_kv].contiguous()
        mask = torch.zeros(bsz, 1, 1, max_kv, dtype=self.dtype)
        for i, pos in enumerate(positions):
            if pos + 1 < max_kv:
                mask[i, 0, 0, pos + 1:] = float("-inf")
        for i, pos in enumerate(positions):
            kb[i, :, pos, :] = k_new[i, :, 0, :]
            vb[i, :, pos, :] = v_new[i, :, 0, :]
        k = kb.repeat_interleave(groups, dim=1)
        v = vb.repeat_interleave(groups, dim=1)
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=False)
        for i, (slot, pos) in enumerate(zip(slots, positions)):
            self.k[slot, :, pos, :] = kb[i, :, pos, :]
            self.v[slot, :, pos, :] = vb[i, :, pos, :]
        return out.transpose(1, 2).contiguous().view(bsz, 1, -1)
