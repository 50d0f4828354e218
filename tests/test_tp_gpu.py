"""Tensor-parallel decode on two GPUs (NCCL) against one GPU.

Qwen2.5-0.5B shape cut to 4 layers (14 Q / 2 KV heads -> 7 / 1 per rank,
group 7 kept whole), seeded random weights from ``Model.create``, in fp32 so
that the comparison is not lost in bf16 rounding (in bf16 the row-parallel
o_proj / down_proj round each rank's partial sum before the all-reduce adds
them, which moves logits by about one ulp). The one-GPU run's greedy tokens
are teacher-forced into the two-rank run, so both see the same sequences.
Both ranks must produce identical logits (they all-gather the same vocab
shards), and every prefill and decode logits row must match the one-GPU run
within max-abs 1e-3.
"""
import multiprocessing as mp

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_tp2_decode_matches_single_gpu(tmp_path):
    from mi_b200.model import Model
    from tests.tp_workers import _gpu_small_cfg, run_scheduler_logits, tp_gpu_decode

    cfg = _gpu_small_cfg()
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (37, 128, 70, 200)]
    max_new = 12
    dev = torch.device("cuda", 0)
    model = Model.create(cfg, dev, torch.float32, seed=21)
    toks1, logs1 = run_scheduler_logits(model, cfg, dev, prompts, max_new)
    del model
    torch.cuda.empty_cache()

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = str(tmp_path / "nccl_rendezvous")
    procs = [ctx.Process(target=tp_gpu_decode, args=(r, 2, init_file, prompts, max_new, toks1, q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, toks, logs = q.get(timeout=600)
        got[rank] = (toks, logs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got[0][0] == toks1 and got[1][0] == toks1
    l0, l1 = got[0][1], got[1][1]
    assert len(l0) == len(logs1) == len(l1)
    worst = 0.0
    for (k, ids, a), (_, ids0, b0), (_, ids1, b1) in zip(logs1, l0, l1):
        assert ids == ids0 == ids1
        assert torch.equal(b0, b1)                    # ranks agree bit for bit
        worst = max(worst, float((a - b0).abs().max()))
    assert worst <= 1e-3, worst


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_tp2_peer_allreduce_matches_nccl(tmp_path):
    """The fused peer-memory all-reduce + residual add + RMSNorm of decode
    steps against the NCCL all-reduce + add_rmsnorm path, bf16, both ranks:
    logits within one bf16 rounding of the (small) logits, ranks identical."""
    from tests.tp_workers import _gpu_small_cfg, tp_gpu_peer_vs_nccl

    cfg = _gpu_small_cfg()
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (20, 64, 130)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = str(tmp_path / "nccl_rendezvous")
    procs = [ctx.Process(target=tp_gpu_peer_vs_nccl, args=(r, 2, init_file, prompts, 10, q))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, ta, la, tb, lb = q.get(timeout=600)
        got[rank] = (ta, la, tb, lb)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ta, la, tb, lb = got[0]
    assert tb == ta and got[1][2] == ta
    worst = 0.0
    for (ka, ia, xa), (kb, ib, xb), (_, _, xb1) in zip(la, lb, got[1][3]):
        assert ka == kb and ia == ib
        assert torch.equal(xb, xb1)
        if ka == "decode":        # prefill rows take the NCCL path in both runs
            worst = max(worst, float((xa - xb).abs().max()))
        else:
            assert torch.equal(xa, xb)
    assert worst <= 2.0 ** -4, worst
