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

Tensor parallelism (``tp_size > 1``, one process per GPU over NCCL): each rank
holds ``Hq/tp`` query heads and ``Hkv/tp`` KV heads (its own page pools, the
same page tables on every rank), ``intermediate/tp`` MLP columns and
``vocab/tp`` rows of the LM head. Q/K/V and gate/up are column-parallel;
``o_proj`` and ``down_proj`` are row-parallel and followed by one all-reduce
each, inside the decode CUDA graph; the logits are all-gathered at the end.
Attention needs no exchange: GQA groups never straddle ranks.
"""
from __future__ import annotations

import dataclasses
import json
import os

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .glue import PROJ_MAX_ROWS, add_rmsnorm, proj_small_m, silu_mul
from .page import append_paged_kv_cache
from .weights import load_weights  # noqa: F401  (server.py imports it from the model module)
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


def _fuse_rows_t(params) -> torch.Tensor:
    """Concatenate [n_i, K] weights along dim 0, store the result transposed
    ([K, sum n_i], contiguous) and re-point each parameter at its (transposed)
    slice. A decode-sized ``x @ W^T`` then runs as a plain ``x @ Wt``, for which
    cuBLAS picks faster kernels at a few rows (measured on B200: Mistral-7B's
    QKV 18.7 -> 12.8 us, o_proj 12.2 -> 10.3 us, gate/up 41.9 -> 37.2 us at 32
    tokens). Parameter names and shapes stay the reference's."""
    fused_t = torch.cat([p.data for p in params]).t().contiguous()
    off = 0
    for p in params:
        n = p.shape[0]
        p.data = fused_t[:, off:off + n].t()
        off += n
    return fused_t


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
        self._qkv_wt = None
        self._qkv_b = None
        self._o_wt = None

    def fuse(self) -> None:
        """One hidden x [Hq+2Hkv]*D weight (stored transposed) so Q, K, V come
        from one GEMM; o_proj's weight stored transposed as well.

        The parameters become views into these buffers (no second copy of the
        weights)."""
        projs = (self.q_proj, self.k_proj, self.v_proj)
        with torch.no_grad():
            self._qkv_wt = _fuse_rows_t([p.weight for p in projs])
            self._qkv_b = (_fuse_rows([p.bias for p in projs])
                           if self.q_proj.bias is not None else None)
            self._o_wt = _fuse_rows_t([self.o_proj.weight])

    def forward(self, x, cos, sin, mask, kv_cache=None, position_ids=None, attn_backend=None,
                *, proj_out: torch.Tensor | None = None):
        """``proj_out`` (extension): ``[tokens, hidden]`` buffer the o_proj GEMM
        writes into (the tensor-parallel peer all-reduce reads it from there)."""
        if attn_backend is None:
            raise RuntimeError("mi_b200 has no padded/CPU attention path: pass attn_backend")
        bsz, seq_len, _ = x.shape
        n = bsz * seq_len
        hq, hkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        if self._qkv_wt is None:
            self.fuse()
        x2 = x.reshape(n, -1)
        qkv = (torch.addmm(self._qkv_b, x2, self._qkv_wt) if self._qkv_b is not None
               else torch.mm(x2, self._qkv_wt))                        # [n, (hq+2hkv)*d]
        q = qkv[:, :hq * d].view(n, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].view(n, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(n, hkv, d)
        be = attn_backend
        layer = be.next_layer()
        kv_data = be.paged_kv_cache.kv_data[layer]
        if be.mode == "decode" and seq_len == 1:
            # one new token per request: its append (RoPE on Q and K, K/V into
            # the pages; model.py:169-170, :203-216) runs inside the decode
            # kernel (model.py:235)
            out = be.wrapper.run_with_append(
                q, kv_data, k, v, be.rope_cos, be.rope_sin,
                out=be.out_buffer(n, hq, d, x.dtype), status=be.status,
                positions=be.positions, scratch_page=be.paged_kv_cache.scratch_page)
        else:
            q_rot = be.q_buffer(n, hq, d, x.dtype)
            # RoPE on Q and K + K/V scatter into the pages: one launch
            # (model.py:169-170, :203-216)
            append_paged_kv_cache(k, v, be.batch_indices, be.positions, kv_data,
                                  be.kv_page_indices, be.kv_page_indptr, be.kv_last_page_len,
                                  rope_cos=be.rope_cos, rope_sin=be.rope_sin, q=q, q_out=q_rot,
                                  scratch_page=be.paged_kv_cache.scratch_page, status=be.status)
            out = be.wrapper.run(q_rot, kv_data, out=be.out_buffer(n, hq, d, x.dtype))
        if proj_out is not None:
            torch.mm(out.view(n, hq * d), self._o_wt, out=proj_out)
            return proj_out.view(bsz, seq_len, -1)
        return torch.mm(out.view(n, hq * d), self._o_wt).view(bsz, seq_len, -1)


def _streams_weight(x2: torch.Tensor, w: torch.Tensor) -> bool:
    """Whether ``x2 @ w.T`` runs on the small-M projection kernel
    (``glue.proj_small_m``): decode-sized rows, 16-bit types, K a multiple
    of 64, aligned rows."""
    return (x2.shape[0] <= PROJ_MAX_ROWS and x2.is_cuda and w.dtype == x2.dtype
            and x2.dtype in (torch.bfloat16, torch.float16) and w.shape[1] % 64 == 0
            and w.stride(1) == 1 and w.stride(0) % 8 == 0 and x2.stride(-1) == 1
            and (x2.shape[0] <= 1 or x2.stride(0) % 8 == 0)
            and x2.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0)


class MLP(nn.Module):
    """SwiGLU (model.py:301-311); gate and up run as one GEMM."""

    def __init__(self, config: ModelConfig, intermediate_size: int | None = None):
        super().__init__()
        inter = intermediate_size or config.intermediate_size
        self.gate_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, inter, bias=False)
        self.down_proj = nn.Linear(inter, config.hidden_size, bias=False)
        self._gu_wt = None

    def fuse(self) -> None:
        # gate/up stored transposed (see _fuse_rows_t); down_proj keeps the
        # reference layout, which cuBLAS already runs best at decode sizes
        with torch.no_grad():
            self._gu_wt = _fuse_rows_t([self.gate_proj.weight, self.up_proj.weight])

    def forward(self, x: torch.Tensor, *, proj_out: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> torch.Tensor:
        """``proj_out`` (extension): ``[tokens, hidden]`` buffer down_proj
        writes into; ``status``: device status word of the small-M kernel."""
        if self._gu_wt is None:
            self.fuse()
        act = silu_mul(torch.mm(x.reshape(-1, x.shape[-1]), self._gu_wt)).view(
            *x.shape[:-1], -1)
        a2 = act.view(-1, act.shape[-1])
        w = self.down_proj.weight
        if _streams_weight(a2, w):  # decode: the weight streamed once (mi_proj_small_m)
            y = proj_small_m(a2, w, out=proj_out, status=status)
            return y.view(*act.shape[:-1], -1)
        if proj_out is not None:  # down_proj straight into a peer all-reduce region
            torch.mm(a2, w.t(), out=proj_out)
            return proj_out.view(*act.shape[:-1], -1)
        return self.down_proj(act)


class DecoderLayer(nn.Module):
    def __init__(self, config: ModelConfig, tp_size: int = 1, tp_group=None, **shard):
        super().__init__()
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.self_attn = Attention(config, shard.get("num_heads"), shard.get("num_kv_heads"))
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.mlp = MLP(config, shard.get("intermediate_size"))
        self.tp_size, self.tp_group = tp_size, tp_group
        self.layer_idx = 0
        self.comm = None  # PeerAllReduce, when the fused decode all-reduce is enabled

    def _reduce(self, x: torch.Tensor) -> torch.Tensor:
        """Sum of the row-parallel partial outputs over the tensor-parallel ranks."""
        if self.tp_size > 1:
            dist.all_reduce(x, group=self.tp_group)
        return x

    def forward(self, x, cos, sin, mask, kv_cache=None, position_ids=None, attn_backend=None):
        """Reference signature (model.py:322-343); returns the new residual."""
        h = x.contiguous().clone()
        x_out, site = self.residual_step(h, None, position_ids, attn_backend)
        add_norm(self.comm, (x_out, site), h, self.input_layernorm)  # only for the add
        return h

    def residual_step(self, h, pending, position_ids, attn_backend):
        """One layer on the residual stream ``h`` (updated in place).

        ``pending`` is the previous layer's MLP output not yet added to ``h``
        (None for the first layer) as ``(tensor, site)``: site None means the
        tensor is complete, else it is this rank's partial in peer all-reduce
        region ``site``. The add (and the reduction) runs fused into this
        layer's input RMSNorm. Returns this layer's MLP output, likewise."""
        rows = h.numel() // h.shape[-1]
        peer = self.comm is not None and self.comm.usable(rows)
        y = add_norm(self.comm, pending, h, self.input_layernorm)
        site_a, site_m = 2 * self.layer_idx, 2 * self.layer_idx + 1
        a = self.self_attn(y, None, None, None, None, position_ids, attn_backend,
                           proj_out=self.comm.site(site_a, rows) if peer else None)
        y = add_norm(self.comm, (a, site_a) if peer else (self._reduce(a), None), h,
                     self.post_attention_layernorm)
        m = self.mlp(y, proj_out=self.comm.site(site_m, rows) if peer else None,
                     status=getattr(attn_backend, "status", None))
        return (m, site_m) if peer else (self._reduce(m), None)


def add_norm(comm, pending, h: torch.Tensor, norm: "RMSNorm") -> torch.Tensor:
    """``h += pending`` (all-reduced first when it is a peer partial), then
    ``norm(h)``; see ``DecoderLayer.residual_step``."""
    if pending is None:
        return add_rmsnorm(None, h, norm.weight, norm.eps)
    x, site = pending
    if site is None:
        return add_rmsnorm(x, h, norm.weight, norm.eps)
    rows = h.numel() // h.shape[-1]
    return comm.reduce_add_norm(site, rows, h, norm.weight, norm.eps)


def tp_shard_sizes(config: ModelConfig, tp_size: int) -> dict:
    """Per-rank head / column counts; raises if ``tp_size`` does not divide them."""
    dims = {"num_heads": config.num_attention_heads, "num_kv_heads": config.num_key_value_heads,
            "intermediate_size": config.intermediate_size, "vocab_size": config.vocab_size}
    for k, v in dims.items():
        if v % tp_size:
            raise ValueError(f"tensor parallel size {tp_size} does not divide {k}={v}")
    return {k: v // tp_size for k, v in dims.items()}


def tp_shard_spec(name: str):
    """``(dim, kind)`` of parameter ``name`` under tensor parallelism, or None
    if every rank holds all of it. kind: "col" (output rows split) or "row"
    (input columns split, output summed by all-reduce)."""
    leaf = name.split(".")
    if len(leaf) >= 4 and leaf[0] == "layers":
        mod, proj = leaf[2], leaf[3]
        if mod == "self_attn" and proj in ("q_proj", "k_proj", "v_proj"):
            return 0, "col"
        if mod == "self_attn" and proj == "o_proj" and leaf[-1] == "weight":
            return 1, "row"
        if mod == "mlp" and proj in ("gate_proj", "up_proj"):
            return 0, "col"
        if mod == "mlp" and proj == "down_proj":
            return 1, "row"
    if name == "lm_head.weight":
        return 0, "col"
    return None


def gather_vocab_logits(local: torch.Tensor, tp_size: int, group=None) -> torch.Tensor:
    """``[..., V/tp]`` vocab shards of every rank -> ``[..., V]`` on every rank."""
    if tp_size == 1:
        return local
    lead, vl = local.shape[:-1], local.shape[-1]
    flat = local.reshape(-1, vl).contiguous()
    out = torch.empty(tp_size * flat.shape[0], vl, dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    full = out.view(tp_size, flat.shape[0], vl).permute(1, 0, 2).reshape(flat.shape[0], -1)
    return full.reshape(*lead, tp_size * vl)


class Model(nn.Module):
    def __init__(self, config: ModelConfig, tp_rank: int = 0, tp_size: int = 1, tp_group=None):
        super().__init__()
        self.config = config
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        shard = {}
        vocab_local = config.vocab_size
        if tp_size > 1:
            sizes = tp_shard_sizes(config, tp_size)
            shard = {k: sizes[k] for k in ("num_heads", "num_kv_heads", "intermediate_size")}
            vocab_local = sizes["vocab_size"]
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(config, tp_size, tp_group, **shard)
                                     for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.lm_head = (None if config.tie_word_embeddings else
                        nn.Linear(config.hidden_size, vocab_local, bias=False))
        self.vocab_local = vocab_local
        self.comm = None
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

    def enable_peer_allreduce(self, max_rows: int = 64) -> "Model":
        """Decode steps of up to ``max_rows`` tokens reduce the row-parallel
        partials over NVLink peer memory, fused with the residual add and
        RMSNorm (``tp_comm.PeerAllReduce``); longer forwards keep NCCL."""
        if self.tp_size == 1:
            return self
        from .tp_comm import PeerAllReduce
        self.requires_grad_(False)  # the projections write into the peer buffers (out=)
        dtype = self.norm.weight.dtype
        self.comm = PeerAllReduce(self.tp_group or torch.distributed.group.WORLD,
                                  self.norm.weight.device, dtype, self.config.hidden_size,
                                  2 * len(self.layers), max_rows)
        for i, layer in enumerate(self.layers):
            layer.layer_idx = i
            layer.comm = self.comm
        return self

    @classmethod
    def create(cls, config: ModelConfig, device, dtype: torch.dtype, seed: int | None = None,
               tp_rank: int = 0, tp_size: int = 1, tp_group=None) -> "Model":
        """Allocate the model (this rank's shard) directly on ``device`` in
        ``dtype`` -- no host copy, so 70B-class shapes need no host memory --
        optionally fill it with the seeded random weights of
        ``weights.init_random_weights`` (each rank keeps its slices of the same
        full tensors), and fuse the GEMM weights."""
        from .weights import init_random_weights

        with torch.device("meta"):
            model = cls(config, tp_rank, tp_size, tp_group)
        model = model.to(dtype=dtype).to_empty(device=device)
        cos, sin = rope_tables(config.head_dim, config.max_position_embeddings,
                               config.rope_theta)
        model.cos_cached = cos.to(dtype).to(device)
        model.sin_cached = sin.to(dtype).to(device)
        if seed is not None:
            init_random_weights(model, seed, generator_device=torch.device(device).type)
        model.requires_grad_(False)  # an inference model (GEMMs may write into given buffers)
        return model.eval().prepare()

    def _lm_head_weight(self) -> torch.Tensor:
        if self.lm_head is not None:
            return self.lm_head.weight
        w = self.embed_tokens.weight               # tied: this rank's vocab rows
        return w if self.tp_size == 1 else w.narrow(0, self.tp_rank * self.vocab_local,
                                                    self.vocab_local)

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
        h = add_norm(self.comm, pending, h, self.norm)
        if logits_rows is not None:
            h = h.reshape(-1, h.shape[-1])[logits_rows].unsqueeze(0)
        return gather_vocab_logits(F.linear(h, self._lm_head_weight()), self.tp_size,
                                   self.tp_group)
