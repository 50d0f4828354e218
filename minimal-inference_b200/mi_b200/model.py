"""Qwen2 / Mistral transformer on the B200 paged-KV path.

Same module tree and parameter names as the reference (``model.py:37-435``)
so checkpoints and seeded random weights load unchanged, and the same call
signatures:

* ``Attention.forward(x, cos, sin, mask, kv_cache=None, position_ids=None,
  attn_backend=None)`` (model.py:152-161)
* ``Model.forward(input_ids, kv_caches=None, position_ids=None,
  attention_mask=None, attn_backend=None) -> logits`` (model.py:375-393)

The attention step goes through the library kernels: one fused append launch
applies RoPE to Q and K (the reference's ``apply_rotary_emb`` rounding,
bit-identical) and scatters K/V into the layer's pages; then paged decode or
paged prefill attention with native GQA (no head padding). There is no padded
CPU path: ``attn_backend`` is required. GEMMs stay in torch (cuBLAS); Q/K/V and
gate/up run as one GEMM each over fused weight views. Each residual add runs
fused with the RMSNorm that follows it, and SiLU(gate) * up is one kernel
(``glue``), so a decoder layer is five GEMMs, two attention-path launches and
three glue launches.
"""
from __future__ import annotations

import dataclasses
import json
import os

import torch
import torch.nn as nn
import torch.nn.functional as F

from .glue import add_rmsnorm, silu_mul
from .page import append_paged_kv_cache
from .rope import rope_tables


@dataclasses.dataclass
class ModelConfig:
    hidden_size: int = 896
    num_attention_heads: int = 14
    num_key_value_heads: int = 2
    head_dim: int = 64
    num_hidden_layers: int = 24
    intermediate_size: int = 4864
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = True
    attn_bias: bool = True

    @classmethod
    def from_pretrained(cls, model_path: str) -> "ModelConfig":
        """HuggingFace ``config.json`` -> config (model.py:52-71)."""
        with open(os.path.join(model_path, "config.json")) as f:
            raw = json.load(f)
        return cls(
            hidden_size=raw["hidden_size"],
            num_attention_heads=raw["num_attention_heads"],
            num_key_value_heads=raw["num_key_value_heads"],
            head_dim=raw.get("head_dim", raw["hidden_size"] // raw["num_attention_heads"]),
            num_hidden_layers=raw["num_hidden_layers"],
            intermediate_size=raw["intermediate_size"],
            vocab_size=raw["vocab_size"],
            rms_norm_eps=raw.get("rms_norm_eps", 1e-6),
            rope_theta=raw.get("rope_theta", 1_000_000.0),
            max_position_embeddings=raw.get("max_position_embeddings", 32768),
            tie_word_embeddings=raw.get("tie_word_embeddings", True),
            attn_bias=raw.get("attention_bias", raw.get("model_type", "") != "mistral"),
        )


# BASELINE shapes (configs 1, 3, 4, 5)
PRESETS = {
    "qwen2.5-0.5b": ModelConfig(),
    "mistral-7b": ModelConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8,
                              head_dim=128, num_hidden_layers=32, intermediate_size=14336,
                              vocab_size=32768, rms_norm_eps=1e-5, rope_theta=1e6,
                              tie_word_embeddings=False, attn_bias=False),
    "qwen2.5-7b": ModelConfig(hidden_size=3584, num_attention_heads=28, num_key_value_heads=4,
                              head_dim=128, num_hidden_layers=28, intermediate_size=18944,
                              vocab_size=152064, tie_word_embeddings=False, attn_bias=True),
    "qwen2.5-72b": ModelConfig(hidden_size=8192, num_attention_heads=64, num_key_value_heads=8,
                               head_dim=128, num_hidden_layers=80, intermediate_size=29568,
                               vocab_size=152064, tie_word_embeddings=False, attn_bias=True),
}


def _fuse_rows(params) -> torch.Tensor:
    """Concatenate parameters along dim 0 and re-point each at its slice."""
    fused = torch.cat([p.data for p in params]).contiguous()
    off = 0
    for p in params:
        n = p.shape[0]
        p.data = fused[off:off + n]
        off += n
    return fused


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.rms_norm(x, self.weight.shape, self.weight, self.eps)


class Attention(nn.Module):
    def __init__(self, config: ModelConfig, num_heads: int | None = None,
                 num_kv_heads: int | None = None):
        super().__init__()
        self.num_heads = num_heads or config.num_attention_heads
        self.num_kv_heads = num_kv_heads or config.num_key_value_heads
        self.head_dim = config.head_dim
        self.num_groups = self.num_heads // self.num_kv_heads
        self.q_proj = nn.Linear(config.hidden_size, self.num_heads * self.head_dim,
                                bias=config.attn_bias)
        self.k_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim,
                                bias=config.attn_bias)
        self.v_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim,
                                bias=config.attn_bias)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, config.hidden_size, bias=False)
        self._qkv_w = None
        self._qkv_b = None

    def fuse(self) -> None:
        """One [Hq+2Hkv]*D x hidden weight so Q, K, V come from one GEMM.

        The q/k/v parameters become views into the fused buffer (no second
        copy of the weights)."""
        projs = (self.q_proj, self.k_proj, self.v_proj)
        with torch.no_grad():
            self._qkv_w = _fuse_rows([p.weight for p in projs])
            self._qkv_b = (_fuse_rows([p.bias for p in projs])
                           if self.q_proj.bias is not None else None)

    def forward(self, x, cos, sin, mask, kv_cache=None, position_ids=None, attn_backend=None):
        if attn_backend is None:
            raise RuntimeError("mi_b200 has no padded/CPU attention path: pass attn_backend")
        bsz, seq_len, _ = x.shape
        n = bsz * seq_len
        hq, hkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        if self._qkv_w is None:
            self.fuse()
        qkv = F.linear(x.reshape(n, -1), self._qkv_w, self._qkv_b)   # [n, (hq+2hkv)*d]
        q = qkv[:, :hq * d].view(n, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].view(n, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(n, hkv, d)
        be = attn_backend
        layer = be.next_layer()
        kv_data = be.paged_kv_cache.kv_data[layer]
        q_rot = be.q_buffer(n, hq, d, x.dtype)
        # RoPE on Q and K + K/V scatter into the pages: one launch
        # (model.py:169-170, :203-216)
        append_paged_kv_cache(k, v, be.batch_indices, be.positions, kv_data,
                              be.kv_page_indices, be.kv_page_indptr, be.kv_last_page_len,
                              rope_cos=be.rope_cos, rope_sin=be.rope_sin, q=q, q_out=q_rot,
                              scratch_page=be.paged_kv_cache.scratch_page, status=be.status)
        out = be.wrapper.run(q_rot, kv_data, out=be.out_buffer(n, hq, d, x.dtype))
        return self.o_proj(out.view(bsz, seq_len, hq * d))


class MLP(nn.Module):
    """SwiGLU (model.py:301-311); gate and up run as one GEMM."""

    def __init__(self, config: ModelConfig, intermediate_size: int | None = None):
        super().__init__()
        inter = intermediate_size or config.intermediate_size
        self.gate_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.down_proj = nn.Linear(inter, config.hidden_size, bias=False)
        self._gu_w = None

    def fuse(self) -> None:
        with torch.no_grad():
            self._gu_w = _fuse_rows([self.gate_proj.weight, self.up_proj.weight])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._gu_w is None:
            self.fuse()
        return self.down_proj(silu_mul(F.linear(x, self._gu_w)))


class DecoderLayer(nn.Module):
    def __init__(self, config: ModelConfig, **shard):
        super().__init__()
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.self_attn = Attention(config, shard.get("num_heads"), shard.get("num_kv_heads"))
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.mlp = MLP(config, shard.get("intermediate_size"))

    def forward(self, x, cos, sin, mask, kv_cache=None, position_ids=None, attn_backend=None):
        """Reference signature (model.py:322-343); returns the new residual."""
        h = x.contiguous().clone()
        h.add_(self.residual_step(h, None, position_ids, attn_backend))
        return h

    def residual_step(self, h, pending, position_ids, attn_backend):
        """One layer on the residual stream ``h`` (updated in place).

        ``pending`` is the previous layer's MLP output not yet added to ``h``
        (None for the first layer); the add runs fused into this layer's input
        RMSNorm. Returns this layer's MLP output, likewise not yet added."""
        y = add_rmsnorm(pending, h, self.input_layernorm.weight, self.input_layernorm.eps)
        a = self.self_attn(y, None, None, None, None, position_ids, attn_backend)
        y = add_rmsnorm(a, h, self.post_attention_layernorm.weight,
                        self.post_attention_layernorm.eps)
        return self.mlp(y)


class Model(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.lm_head = (None if config.tie_word_embeddings else
                        nn.Linear(config.hidden_size, config.vocab_size, bias=False))
        # fp32 tables built exactly as model.py:79-89, cast with the model
        cos, sin = rope_tables(config.head_dim, config.max_position_embeddings,
                               config.rope_theta)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)

    def prepare(self) -> "Model":
        """Build the fused GEMM weights (after weights are loaded/initialised)."""
        for layer in self.layers:
            layer.self_attn.fuse()
            layer.mlp.fuse()
        return self

    def forward(self, input_ids, kv_caches=None, position_ids=None, attention_mask=None,
                attn_backend=None, *, logits_rows: torch.Tensor | None = None):
        """Logits ``[B, S, V]`` (model.py:375-435). ``logits_rows`` (extension):
        flat token indices whose logits are wanted; returns ``[1, len, V]``."""
        if attn_backend is None:
            raise RuntimeError("mi_b200 has no padded/CPU attention path: pass attn_backend")
        h = self.embed_tokens(input_ids)          # residual stream, updated in place
        attn_backend.rope_cos = self.cos_cached
        attn_backend.rope_sin = self.sin_cached
        pending = None
        for layer in self.layers:
            pending = layer.residual_step(h, pending, position_ids, attn_backend)
        # last residual add + final norm; the norm is per row, so selecting
        # rows after it equals selecting before
        h = add_rmsnorm(pending, h, self.norm.weight, self.norm.eps)
        if logits_rows is not None:
            h = h.reshape(-1, h.shape[-1])[logits_rows].unsqueeze(0)
        if self.lm_head is not None:
            return self.lm_head(h)
        return F.linear(h, self.embed_tokens.weight)
