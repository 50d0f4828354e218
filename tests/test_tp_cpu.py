"""Tensor-parallel host logic on the CPU (no GPU): shard specs, the sharded
random init, and the column/row-parallel split with its all-reduce and the
vocab all-gather, run as two gloo ranks against the unsharded model."""
import multiprocessing as mp

import pytest
import torch

from mi_b200.model import Model, tp_shard_sizes, tp_shard_spec
from mi_b200.weights import init_random_weights
from tests.tp_workers import TINY, tp_decomposition


def test_shard_specs():
    assert tp_shard_spec("layers.3.self_attn.q_proj.weight") == (0, "col")
    assert tp_shard_spec("layers.3.self_attn.k_proj.bias") == (0, "col")
    assert tp_shard_spec("layers.0.self_attn.o_proj.weight") == (1, "row")
    assert tp_shard_spec("layers.0.mlp.gate_proj.weight") == (0, "col")
    assert tp_shard_spec("layers.0.mlp.down_proj.weight") == (1, "row")
    assert tp_shard_spec("lm_head.weight") == (0, "col")
    for name in ("embed_tokens.weight", "norm.weight", "layers.1.input_layernorm.weight"):
        assert tp_shard_spec(name) is None


def test_shard_sizes_qwen72b_and_rejects():
    from mi_b200.model import PRESETS
    cfg = PRESETS["qwen2.5-72b"]
    for tp in (2, 4, 8):
        s = tp_shard_sizes(cfg, tp)
        assert s["num_heads"] * tp == 64 and s["num_kv_heads"] * tp == 8
        assert s["num_heads"] // s["num_kv_heads"] == 8          # GQA group kept whole
        assert s["intermediate_size"] * tp == 29568 and s["vocab_size"] * tp == 152064
    with pytest.raises(ValueError):
        tp_shard_sizes(cfg, 16)                                   # 8 KV heads


def test_sharded_init_holds_slices_of_the_full_weights():
    full = Model(TINY)
    init_random_weights(full, 7)
    fp = dict(full.named_parameters())
    for rank in range(2):
        m = Model(TINY, rank, 2)
        init_random_weights(m, 7)
        for name, p in m.named_parameters():
            spec = tp_shard_spec(name)
            want = fp[name]
            if spec is not None:
                n = p.shape[spec[0]]
                want = want.narrow(spec[0], rank * n, n)
            assert torch.equal(p, want), name


def test_tp2_gloo_matches_dense_model(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = str(tmp_path / "gloo_rendezvous")
    procs = [ctx.Process(target=tp_decomposition, args=(r, 2, init_file, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in results.items():
        assert errs.pop("logits_shape") is True
        for k, e in errs.items():
            assert e < 1e-4, (rank, k, e)
