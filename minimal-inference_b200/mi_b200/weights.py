"""Seeded random initialisation and safetensors loading for the model shapes.

The benchmark configurations use random-init weights (there are no
checkpoints on the GPU boxes). ``init_random_weights`` is deterministic and
depends only on parameter names and shapes, so a module tree with the
reference's parameter names (``model.py:125-373``) gets bit-identical weights
whichever implementation holds them. That is how parity fixtures made from the
reference model line up with this package's model.
"""
from __future__ import annotations

import glob
import os

import torch


@torch.no_grad()
def init_random_weights(model: torch.nn.Module, seed: int, std: float = 0.02,
                        generator_device: str = "cpu") -> None:
    """N(0, std) for every parameter except RMSNorm weights, which stay 1.0.

    Parameters are visited in sorted-name order; each draws
    ``torch.randn(shape, generator=g) * std`` in fp32 from one generator seeded
    with ``seed`` and is then cast into the parameter's dtype/device. On a
    tensor-parallel shard (``model.tp_size > 1``) each split parameter draws
    its full shape and keeps the rank's slice, so every rank holds slices of
    the very tensors an unsharded model gets.
    ``generator_device="cuda"`` draws on the GPU instead (fast for 7B+ shapes;
    not bit-identical to the CPU stream).
    """
    from .model import tp_shard_spec

    tp_size, tp_rank = getattr(model, "tp_size", 1), getattr(model, "tp_rank", 0)
    g = torch.Generator(device=generator_device)
    g.manual_seed(seed)
    for name, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
        if name.endswith("norm.weight"):
            p.fill_(1.0)
            continue
        spec = tp_shard_spec(name) if tp_size > 1 else None
        shape = list(p.shape)
        if spec is not None:  # draw the full tensor, keep this rank's slice
            shape[spec[0]] *= tp_size
        w = torch.randn(tuple(shape), generator=g, dtype=torch.float32, device=generator_device)
        if spec is not None:
            n = p.shape[spec[0]]
            w = w.narrow(spec[0], tp_rank * n, n)
        w.mul_(std)
        p.copy_(w)
        del w


def load_weights(model: torch.nn.Module, model_path: str, device="cpu",
                 dtype: torch.dtype = torch.bfloat16) -> None:
    """Load a HuggingFace safetensors checkpoint (``model.py:443-474``).

    Strips the ``model.`` prefix, keeps ``lm_head.weight`` only when the model
    has an untied head, casts to ``dtype`` and loads non-strictly.
    """
    from safetensors.torch import load_file

    files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"No safetensors files found in {model_path}")
    state: dict[str, torch.Tensor] = {}
    for f in files:
        state.update(load_file(f, device=str(device)))
    cleaned: dict[str, torch.Tensor] = {}
    has_head = getattr(model, "lm_head", None) is not None
    for key, t in state.items():
        if key == "lm_head.weight":
            if has_head:
                cleaned[key] = t.to(dtype)
            continue
        cleaned[key.removeprefix("model.")] = t.to(dtype)
    missing, unexpected = model.load_state_dict(cleaned, strict=False)
    real_missing = [k for k in missing if "cached" not in k]
    if real_missing:
        print(f"load_weights: {len(real_missing)} model parameters absent from the "
              f"checkpoint (left as they were): {real_missing}")
    if unexpected:
        print(f"load_weights: {len(unexpected)} checkpoint tensors with no model parameter "
              f"(ignored): {unexpected}")
