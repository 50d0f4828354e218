"""Rank bodies for the tensor-parallel CPU tests (spawned gloo processes)."""
import os

import torch
import torch.distributed as dist
import torch.nn.functional as F

from mi_b200.model import Model, ModelConfig, gather_vocab_logits
from mi_b200.weights import init_random_weights

TINY = ModelConfig(hidden_size=64, num_attention_heads=8, num_key_value_heads=2, head_dim=8,
                   num_hidden_layers=2, intermediate_size=96, vocab_size=128,
                   tie_word_embeddings=False, attn_bias=True)


def _mlp(m, x):
    return m.down_proj(F.silu(m.gate_proj(x)) * m.up_proj(x))


@torch.no_grad()
def tp_decomposition(rank: int, world: int, init_file: str, out_q) -> None:
    """Each rank's shard, combined through the collectives the model uses,
    against the unsharded model's dense math on the same seeded weights."""
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank,
                            world_size=world)
    try:
        cfg = TINY
        full = Model(cfg)
        init_random_weights(full, 7)
        shard = Model(cfg, rank, world, dist.group.WORLD)
        init_random_weights(shard, 7)
        g = torch.Generator().manual_seed(3)
        x = torch.randn(5, cfg.hidden_size, generator=g)
        d = cfg.head_dim
        errs = {}
        for li in range(cfg.num_hidden_layers):
            fa, sa = full.layers[li].self_attn, shard.layers[li].self_attn
            for proj, heads in (("q_proj", sa.num_heads), ("k_proj", sa.num_kv_heads),
                                ("v_proj", sa.num_kv_heads)):
                want = getattr(fa, proj)(x)[:, rank * heads * d:(rank + 1) * heads * d]
                errs[f"{li}.{proj}"] = float((getattr(sa, proj)(x) - want).abs().max())
            att = torch.randn(5, cfg.num_attention_heads * d, generator=g)
            cols = slice(rank * sa.num_heads * d, (rank + 1) * sa.num_heads * d)
            red = shard.layers[li]._reduce(sa.o_proj(att[:, cols].contiguous()))
            errs[f"{li}.o_proj"] = float((red - fa.o_proj(att)).abs().max())
            red = shard.layers[li]._reduce(_mlp(shard.layers[li].mlp, x))
            errs[f"{li}.mlp"] = float((red - _mlp(full.layers[li].mlp, x)).abs().max())
        h = torch.randn(2, 3, cfg.hidden_size, generator=g)
        got = gather_vocab_logits(F.linear(h, shard._lm_head_weight()), world)
        errs["logits"] = float((got - full.lm_head(h)).abs().max())
        errs["logits_shape"] = tuple(got.shape) == (2, 3, cfg.vocab_size)
        out_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# GPU: tensor-parallel decode through the scheduler (NCCL, one GPU per rank)
# ---------------------------------------------------------------------------
def _gpu_small_cfg():
    from mi_b200.model import PRESETS
    import dataclasses
    return dataclasses.replace(PRESETS["qwen2.5-0.5b"], num_hidden_layers=4)


def run_scheduler_logits(model, cfg, dev, prompts, max_new, teacher=None):
    """Greedy decode of ``prompts`` through the scheduler (CUDA graphs on);
    returns (tokens per request, [(kind, ids, logits rows)])."""
    from mi_b200.scheduler import Request, Scheduler

    sched = Scheduler(model, cfg, dev, next(model.parameters()).dtype, max_batch_size=8,
                      max_seq_len=512,
                      page_size=16, eos_token_ids=set(), teacher_tokens=teacher)
    sched.record_logits = True
    reqs = [Request(f"r{i}", p, max_new, 0.0) for i, p in enumerate(prompts)]
    for r in reqs:
        sched.submit_request(r)
    steps = 0
    while any(r.status.value != "finished" for r in reqs) and steps < 200:
        sched.step()
        steps += 1
    toks = {r.request_id: list(r.generated_tokens) for r in reqs}
    logs = sched.step_logits
    sched.close()
    return toks, logs


def _nccl_init(rank: int, world: int, init_file: str):
    from datetime import timedelta
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    return dev


@torch.no_grad()
def tp_gpu_decode(rank: int, world: int, init_file: str, prompts, max_new, teacher,
                  out_q) -> None:
    from mi_b200.model import Model

    dev = _nccl_init(rank, world, init_file)
    try:
        cfg = _gpu_small_cfg()
        model = Model.create(cfg, dev, torch.float32, seed=21, tp_rank=rank, tp_size=world,
                             tp_group=dist.group.WORLD)
        toks, logs = run_scheduler_logits(model, cfg, dev, prompts, max_new, teacher)
        out_q.put((rank, toks, [(k, ids, rows) for k, ids, rows in logs]))
    finally:
        dist.destroy_process_group()


@torch.no_grad()
def tp_gpu_peer_vs_nccl(rank: int, world: int, init_file: str, prompts, max_new, out_q) -> None:
    """bf16 TP decode twice on the same model: NCCL all-reduce, then the fused
    peer-memory all-reduce (teacher-forced with the first run's tokens)."""
    from mi_b200.model import Model

    dev = _nccl_init(rank, world, init_file)
    try:
        cfg = _gpu_small_cfg()
        model = Model.create(cfg, dev, torch.bfloat16, seed=21, tp_rank=rank, tp_size=world,
                             tp_group=dist.group.WORLD)
        toks_a, logs_a = run_scheduler_logits(model, cfg, dev, prompts, max_new)
        model.enable_peer_allreduce(max_rows=8)
        toks_b, logs_b = run_scheduler_logits(model, cfg, dev, prompts, max_new, teacher=toks_a)
        torch.cuda.synchronize()
        model.comm.check_status()
        model.comm.close()
        out_q.put((rank, toks_a, logs_a, toks_b, logs_b))
    finally:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# GPU: IPC mapping between two processes on one GPU
# ---------------------------------------------------------------------------
class _Cai:
    """A raw device pointer as a torch-readable array (``__cuda_array_interface__``)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


def ipc_child(handle: bytes, offset: int, n: int, q) -> None:
    """Child of the one-GPU IPC test: map the parent's buffer, read its first
    half, write a pattern into its second half, unmap."""
    import ctypes

    import torch as t
    from mi_b200 import capi

    try:
        t.cuda.set_device(0)
        t.zeros(1, device="cuda")                     # context up before the mapping
        lib = capi.lib()
        hb = ctypes.create_string_buffer(handle, capi.IPC_HANDLE_BYTES)
        base = ctypes.c_void_p(0)
        rc = lib.mi_ipc_open(ctypes.addressof(hb), ctypes.addressof(base))
        if rc != 0:
            q.put(("error", lib.mi_last_error().decode()))
            return
        view = t.as_tensor(_Cai(base.value + offset, n), device="cuda")
        seen = view[: n // 2].cpu().numpy().tobytes()
        view[n // 2:].copy_(t.arange(n - n // 2, device="cuda").to(t.uint8) ^ 0x5A)
        t.cuda.synchronize()
        del view
        rc = lib.mi_ipc_close(base)
        q.put(("ok", seen, rc))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put(("error", repr(e)))
