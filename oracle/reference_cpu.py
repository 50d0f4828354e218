"""CPU port of the reference's own decode-attention path -- TEST/BASELINE ONLY.

The reference runs on the CPU through its padded path (the scheduler picks it
whenever the device is not CUDA, scheduler.py:504): a per-slot padded cache
``[Bmax, Hkv, max_seq, D]`` (``BatchedKVCache``, scheduler.py:98-160) and
PyTorch SDPA (``Attention._pytorch_attention``, model.py:254-298). This module
restates that path -- one layer of one decode step, and the whole model -- so
``bench.py`` can time it on the GPU box's host cores as the CPU baseline
(``--impl reference`` and the ``cpu_baseline`` key). Per decode step it
follows:

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


class PaddedReferenceModel:
    """The reference's whole padded CPU forward (prefill and batched decode),
    over the reference-named parameters of a model (``state_dict`` names of
    model.py:125-373: ``embed_tokens``, ``layers.N.self_attn.{q,k,v,o}_proj``,
    ``layers.N.mlp.{gate,up,down}_proj``, the norms, ``lm_head`` or tied
    embeddings).

    Per layer (model.py:333-343): pre-norm attention + residual, pre-norm
    SwiGLU MLP + residual. Attention (model.py:152-170, :254-298): q/k/v
    projections, rotate-half RoPE from the fp32 tables of ``precompute_rope``
    (model.py:79-107) indexed by position, the padded cache write, GQA by
    ``repeat_interleave`` and SDPA. Prefill (one request, scheduler.py:
    654-682) writes the prompt into its slot and masks causally (model.py:
    399-418); a decode step (scheduler.py:765-833) gathers and trims the
    batch's caches, writes each lane's token, masks each lane past its
    position and writes the new entries back. Returns the logits of the last
    position of each sequence.
    """

    def __init__(self, params: dict, cfg, max_batch: int, max_seq: int,
                 dtype=torch.float32):
        p = {k: v.detach().to("cpu", dtype) for k, v in params.items()}
        self.p, self.cfg, self.dtype = p, cfg, dtype
        self.n_layers = cfg.num_hidden_layers
        hkv, d = cfg.num_key_value_heads, cfg.head_dim
        self.caches = [(torch.zeros(max_batch, hkv, max_seq, d, dtype=dtype),
                        torch.zeros(max_batch, hkv, max_seq, d, dtype=dtype))
                       for _ in range(self.n_layers)]
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2).float() / d))
        freqs = torch.outer(torch.arange(cfg.max_position_embeddings, dtype=torch.float32),
                            inv_freq)
        emb = torch.cat([freqs, freqs], dim=-1)
        self.cos, self.sin = emb.cos().to(dtype), emb.sin().to(dtype)
        self.lm_head = p.get("lm_head.weight", p["embed_tokens.weight"])

    def _linear(self, x, name):
        b = self.p.get(name + ".bias")
        return F.linear(x, self.p[name + ".weight"], b)

    def _rms(self, x, name):
        w = self.p[name + ".weight"]
        return F.rms_norm(x, w.shape, w, self.cfg.rms_norm_eps)

    @staticmethod
    def _rope(x, cos, sin):
        half = x.shape[-1] // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return x * cos.unsqueeze(1) + rot * sin.unsqueeze(1)

    def _forward(self, ids, pos_ids, attend):
        cfg = self.cfg
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        bsz, seq = ids.shape
        h = self.p["embed_tokens.weight"][ids]
        cos, sin = self.cos[pos_ids], self.sin[pos_ids]
        for li in range(self.n_layers):
            pre = f"layers.{li}."
            x = self._rms(h, pre + "input_layernorm")
            q = self._linear(x, pre + "self_attn.q_proj").view(bsz, seq, hq, d).transpose(1, 2)
            k = self._linear(x, pre + "self_attn.k_proj").view(bsz, seq, hkv, d).transpose(1, 2)
            v = self._linear(x, pre + "self_attn.v_proj").view(bsz, seq, hkv, d).transpose(1, 2)
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            k, v, mask = attend(li, k, v)
            k = k.repeat_interleave(hq // hkv, dim=1)
            v = v.repeat_interleave(hq // hkv, dim=1)
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=False)
            o = o.transpose(1, 2).contiguous().view(bsz, seq, -1)
            h = h + self._linear(o, pre + "self_attn.o_proj")
            x = self._rms(h, pre + "post_attention_layernorm")
            gate = self._linear(x, pre + "mlp.gate_proj")
            up = self._linear(x, pre + "mlp.up_proj")
            h = h + self._linear(F.silu(gate) * up, pre + "mlp.down_proj")
        h = self._rms(h[:, -1:], "norm")
        return F.linear(h, self.lm_head)[:, 0]

    @torch.no_grad()
    def prefill(self, slot: int, prompt: list[int]) -> torch.Tensor:
        """One request's prompt into its slot; logits of its last token."""
        n = len(prompt)
        ids = torch.tensor([prompt])
        pos_ids = torch.arange(n).unsqueeze(0)
        mask = torch.triu(torch.full((n, n), float("-inf"), dtype=self.dtype), 1)[None, None]

        def attend(li, k, v):
            kc, vc = self.caches[li]
            kc[slot:slot + 1, :, :n] = k
            vc[slot:slot + 1, :, :n] = v
            return kc[slot:slot + 1, :, :n], vc[slot:slot + 1, :, :n], mask
        return self._forward(ids, pos_ids, attend)[0]

    @torch.no_grad()
    def decode(self, slots: list[int], positions: list[int], tokens: list[int]) -> torch.Tensor:
        """One decode step of a batch; logits ``[B, vocab]``."""
        bsz = len(slots)
        ids = torch.tensor(tokens).unsqueeze(1)
        pos_ids = torch.tensor(positions).unsqueeze(1)
        max_kv = max(positions) + 1
        trimmed = [(kc[slots][:, :, :max_kv].contiguous(), vc[slots][:, :, :max_kv].contiguous())
                   for kc, vc in self.caches]
        mask = torch.zeros(bsz, 1, 1, max_kv, dtype=self.dtype)
        for i, pos in enumerate(positions):
            if pos + 1 < max_kv:
                mask[i, 0, 0, pos + 1:] = float("-inf")

        def attend(li, k, v):
            kb, vb = trimmed[li]
            for i, pos in enumerate(positions):
                kb[i, :, pos, :] = k[i, :, 0, :]
                vb[i, :, pos, :] = v[i, :, 0, :]
            return kb, vb, mask
        logits = self._forward(ids, pos_ids, attend)
        for li, (kc, vc) in enumerate(self.caches):
            kb, vb = trimmed[li]
            for i, (slot, pos) in enumerate(zip(slots, positions)):
                kc[slot, :, pos, :] = kb[i, :, pos, :]
                vc[slot, :, pos, :] = vb[i, :, pos, :]
        return logits
