#!/usr/bin/env python
"""Benchmark of the B200 paged-KV hot path.

Workload ("step"): the attention half of one Mistral-7B-shape decode step at
BASELINE config 2 -- for each of 32 layers, one fused KV-append (RoPE on K
and Q, scatter of the new token into its page) and one paged decode
attention over 32 requests with contexts U[256, 4096] (seeded), 32 Q / 8 KV
heads, head_dim 128, page_size 16, bf16, a 10240-page pool per layer with
random non-contiguous page tables. Each layer has its own pool, so a step
streams ~9 GB of distinct KV data (inputs far larger than the 126 MB L2).

Prints ONE JSON line (rank 0): value = algorithmic GB/s of the whole job
(all ranks' bytes / max-over-ranks device time), the decode kernel's roofline
against the measured HBM copy bandwidth (its launch duration from a loop of
back-to-back decode launches in the same timed window), an end-to-end figure through the
public API with host buffers, the CPU baseline (the reference's own padded
CPU path, ported in oracle/reference_cpu.py) and SM clocks sampled during
the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU. The headline is config 2 split
by KV head: every GPU holds 8/N of the KV heads of every page and decodes
them with their query heads (strong scaling; attention needs no exchange
between heads). Beside it: ``replicas`` (every GPU runs the whole step on its
own pools: weak scaling, no collective) and ``tp_decode`` (
Qwen2.5-72B-shape decode at batch 64, tensor parallel over the N GPUs, with
the decode all-reduce named). N = 1 adds the reference's CPU path
(``cpu_baseline``), the Mistral-7B-shape decode (config 3), the prefill
kernel on config 3's prompts, Qwen2.5-7B serving under churn (config 4) and
config 1's decode step beside the reference's CPU step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "minimal-inference_b200"))
sys.path.insert(0, REPO)

# Under torchrun: NCCL's communicator-init log (ranks, devices, transports)
# on stderr, set before torch loads NCCL; stdout keeps the one JSON line.
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

METRIC = "paged decode attn HBM GB/s (% of peak); Mistral-7B-shape decode tok/s @B=32"
CFG = dict(batch=32, hq=32, hkv=8, head_dim=128, page_size=16, ctx_lo=256, ctx_hi=4096,
           num_pages=10240, layers=32, seed=0)
FALLBACK_HBM_GBS = 6650.0


def config2_lens(seed=0, batch=32, lo=256, hi=4096):
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=batch).tolist()


def decode_bytes(lens, c=CFG) -> int:
    """Algorithmic bytes of one paged decode launch (K+V of every context
    token, q read, out write, page ids, indptr + last_page_len)."""
    hkv, d, hq, b = c["hkv"], c["head_dim"], c["hq"], len(lens)
    kv = sum(lens) * hkv * d * 2 * 2
    qo = 2 * b * hq * d * 2
    meta = sum(math.ceil(L / c["page_size"]) for L in lens) * 4 + (2 * b + 1) * 4
    return kv + qo + meta


def append_bytes(b, c=CFG) -> int:
    """Algorithmic bytes of one fused append launch (read raw q/k/v and two
    RoPE table rows, write rotated q and the K/V rows, token metadata)."""
    hq, hkv, d = c["hq"], c["hkv"], c["head_dim"]
    return (b * (hq + 2 * hkv) * d * 2 + b * 2 * d * 2 + b * (hq + 2 * hkv) * d * 2
            + b * 2 * 4)


def read_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, TypeError, ValueError):  # absent or malformed: the fallback
        return FALLBACK_HBM_GBS, "fallback"


def read_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    p = os.path.join(REPO, "profiles", "decode_sk_config2.md")
    try:
        with open(p) as f:
            m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.5)

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU legs: the reference's own padded CPU path (ported in oracle/)
# ---------------------------------------------------------------------------
def cpu_reference_steps(lens, steps, budget_s=20.0, dtype_name="bfloat16"):
    """Time single-layer decode steps of the reference's CPU path.

    Returns (GB/s of algorithmic decode bytes, seconds, threads, sample text).
    The batch is cut to a prefix of the requests when the full batch would
    not fit ``budget_s`` for ``steps`` steps. Bytes count the K/V, q and out
    elements at the run's element size.
    """
    import torch
    from oracle.reference_cpu import PaddedDecodeLayer
    c = CFG
    dt = getattr(torch, dtype_name)
    elt = torch.empty((), dtype=dt).element_size()
    threads = torch.get_num_threads()
    b = len(lens)
    layer = PaddedDecodeLayer(b, c["hkv"], c["ctx_hi"] + 1, c["head_dim"], dt)
    layer.fill([L - 1 for L in lens], seed=1)
    g = torch.Generator().manual_seed(2)
    q = torch.randn(b, c["hq"], 1, c["head_dim"], generator=g).to(dt)
    kn = torch.randn(b, c["hkv"], 1, c["head_dim"], generator=g).to(dt)
    vn = torch.randn(b, c["hkv"], 1, c["head_dim"], generator=g).to(dt)
    pos = [L - 1 for L in lens]
    t0 = time.perf_counter()
    layer.step(list(range(b)), pos, q, kn, vn)  # warm-up + per-step estimate
    est = time.perf_counter() - t0
    nb = b
    if est * steps > budget_s:
        nb = max(1, int(b * budget_s / (est * steps)))
    slots = list(range(nb))
    t0 = time.perf_counter()
    for _ in range(steps):
        layer.step(slots, pos[:nb], q[:nb], kn[:nb], vn[:nb])
    secs = time.perf_counter() - t0
    sub = lens[:nb]
    elems = sum(sub) * c["hkv"] * c["head_dim"] * 2 + 2 * nb * c["hq"] * c["head_dim"]
    nbytes = decode_bytes(sub) + (elt - 2) * elems  # decode_bytes counts 2-byte elements
    gbs = nbytes * steps / secs / 1e9
    sample = (f"{steps} single-layer decode steps of the reference CPU path (padded cache + "
              f"SDPA, {dtype_name}) over the first {nb} of the {b} config-2 requests")
    return gbs, secs, threads, sample


# ---------------------------------------------------------------------------
# Mistral-7B-shape continuous-batching decode @ B=32
# ---------------------------------------------------------------------------
def model_decode(dev, batch=32, out_tokens=50, seed=3):
    """Decode tok/s of the Mistral-7B shape (random bf16 weights) at batch 32.

    32 requests with prompts U[128, 1024] of random ids, 50 output tokens
    each (1 from prefill + 49 decode steps), page_size 16, CUDA-graph decode
    through this package's Scheduler. T2T follows the reference's definition
    (scheduler.py:984-995, benchmark.py:57-62): per request, the time between
    its first and last token divided by (tokens - 1); tok/s = batch / T2T.
    """
    import torch
    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Request, Scheduler
    cfg = PRESETS["mistral-7b"]
    model = Model.create(cfg, dev, torch.bfloat16, seed=seed)
    rng = np.random.default_rng(seed)
    lens = rng.integers(128, 1025, batch).tolist()
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in lens]
    sched = Scheduler(model, cfg, dev, torch.bfloat16, max_batch_size=batch,
                      max_seq_len=1024 + out_tokens + 16, page_size=16, eos_token_ids=set())
    # warm-up request set (fills caches / allocator paths), then the measured one
    for rep in range(2):
        reqs = [Request(f"w{rep}_{i}", p, out_tokens if rep else 4, 0.0)
                for i, p in enumerate(prompts)]
        for r in reqs:
            sched.submit_request(r)
        torch.cuda.synchronize()
        step_ms = []
        t_start = time.perf_counter()
        while sched.active_requests or sched.waiting_queue:
            t0 = time.perf_counter()
            sched.step()
            step_ms.append((time.perf_counter() - t0) * 1e3)
        total_s = time.perf_counter() - t_start
    t2t = [(r.last_token_time - r.prefill_done_time) / (len(r.generated_tokens) - 1)
           for r in reqs]
    t2t_ms = statistics.mean(t2t) * 1e3
    decode_steps = step_ms[1:]  # the first step holds the prefill
    out = {"metric": "Mistral-7B-shape decode tok/s @B=32 (config 3)",
           "value": round(batch / (t2t_ms / 1e3), 1), "unit": "tok/s",
           "t2t_ms": round(t2t_ms, 3),
           "decode_step_ms_median": round(statistics.median(decode_steps), 3),
           "decode_step_ms_mean": round(statistics.mean(decode_steps), 3),
           "decode_step_ms_p90_max": [round(float(np.percentile(decode_steps, 90)), 3),
                                      round(max(decode_steps), 3)],
           "decode_step_ms_first5": [round(x, 3) for x in decode_steps[:5]],
           "first_step_ms (prefill of all 32 + 1 decode)": round(step_ms[0], 2),
           "wall_s": round(total_s, 3), "batch": batch, "output_tokens": out_tokens,
           "prompt_lens": "U[128,1024] seeded", "weights": "random N(0,0.02) bf16",
           "cuda_graph_decode": True}
    del sched, model
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
def churn_requests(n, vocab, seed=11, p_lo=64, p_hi=2048, o_lo=16, o_hi=512):
    """BASELINE config 4's request stream: prompts U[p_lo, p_hi] of random ids,
    output lengths U[o_lo, o_hi], seeded."""
    rng = np.random.default_rng(seed)
    return [(rng.integers(0, vocab, int(rng.integers(p_lo, p_hi + 1))).tolist(),
             int(rng.integers(o_lo, o_hi + 1))) for _ in range(n)]


def churn_measure(dev, n_req=160, name=None) -> dict:
    """Qwen2.5-7B-shape serving under churn.

    max_batch 48, max_seq 4096, page_size 16; 48 requests start, and a new
    one (prompt U[64,2048], output U[16,512], seeded) is submitted whenever
    one finishes, until ``n_req`` requests have been served, so admissions,
    prefills, page growth and retirements interleave and the pool fragments.
    Random bf16 weights, greedy, EOS disabled (outputs run to their drawn
    length). Reports generated tokens per second of the whole run, the
    reference-definition T2T and TTFT, the decode step time, and whether
    every page came back to the pool.
    """
    import torch
    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Request, Scheduler

    name = name or "qwen2.5-7b"
    cfg = PRESETS[name]
    model = Model.create(cfg, dev, torch.bfloat16, seed=7)
    sched = Scheduler(model, cfg, dev, torch.bfloat16, max_batch_size=48, max_seq_len=4096,
                      page_size=16, eos_token_ids=set())
    stream = churn_requests(n_req, cfg.vocab_size)
    # warm-up: a few short requests through every path (graph replay included)
    warm = [Request(f"w{i}", p[:64], 4, 0.0) for i, (p, _) in enumerate(stream[:8])]
    for r in warm:
        sched.submit_request(r)
    while sched.active_requests or sched.waiting_queue:
        sched.step()
    torch.cuda.synchronize()
    reqs, nxt = [], 0

    def submit(k):
        nonlocal nxt
        for _ in range(k):
            if nxt >= n_req:
                return
            prompt, out_len = stream[nxt]
            r = Request(f"r{nxt}", prompt, out_len, 0.0)
            r.submit_time = time.perf_counter()
            reqs.append(r)
            sched.submit_request(r)
            nxt += 1

    clocks = ClockSampler(dev.index or 0)
    t0 = time.perf_counter()
    submit(48)
    steps, step_ms, min_free = 0, [], sched.kv_cache.num_free_pages
    while sched.active_requests or sched.waiting_queue or nxt < n_req:
        done_before = sum(1 for r in reqs if r.status.value == "finished")
        ts = time.perf_counter()
        sched.step()
        step_ms.append((time.perf_counter() - ts) * 1e3)
        steps += 1
        min_free = min(min_free, sched.kv_cache.num_free_pages)
        done = sum(1 for r in reqs if r.status.value == "finished")
        submit(done - done_before)   # a new request whenever a slot frees
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    sched.kv_cache.check_status()
    gen = sum(len(r.generated_tokens) for r in reqs)
    t2t = [(r.last_token_time - r.prefill_done_time) / (len(r.generated_tokens) - 1)
           for r in reqs if len(r.generated_tokens) > 1]
    ttft = [r.prefill_done_time - r.submit_time for r in reqs]
    complete = all(len(r.generated_tokens) == stream[i][1] for i, r in enumerate(reqs))
    pages_back = int(sched.kv_cache.pool_ctrl[1].item()) == sched.kv_cache.max_num_pages - 1
    pool_pages = sched.kv_cache.max_num_pages
    sched.close()
    del sched, model
    torch.cuda.empty_cache()
    return {"metric": f"{name} serving under churn: generated tok/s (config 4)",
            "value": round(gen / wall, 1), "unit": "tok/s", "steps": steps,
            "warmup_requests": len(warm),
            "decode_step_ms_median": round(statistics.median(step_ms), 3),
            "model": name, "max_batch": 48, "max_seq_len": 4096, "requests": n_req,
            "prompt_lens": "U[64,2048] seeded", "output_lens": "U[16,512] seeded",
            "page_size": 16, "weights": "random N(0,0.02) bf16",
            "t2t_ms_mean": round(statistics.mean(t2t) * 1e3, 3),
            "ttft_ms_mean": round(statistics.mean(ttft) * 1e3, 1),
            "generated_tokens": gen, "wall_s": round(wall, 3),
            "min_free_pages": min_free, "pool_pages": pool_pages,
            "all_outputs_complete": complete, "all_pages_returned": pages_back,
            "clocks": clk}


def run_churn(args):
    """``--workload config4``: ``churn_measure`` on its own (``--batch``
    requests, default 160)."""
    import torch
    dev = torch.device("cuda", dist_env()[2])
    torch.cuda.set_device(dev)
    r = churn_measure(dev, n_req=args.batch or 160, name=args.model)
    line = {"metric": r["metric"], "value": r["value"], "unit": "tok/s", "n_gpus": 1,
            "steps": r["steps"], "warmup": r["warmup_requests"],
            "ms_per_step": r["decode_step_ms_median"], "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "continuous batching with a new request whenever one "
                                   "finishes", "model": r["model"], "max_batch": 48,
                       "max_seq_len": 4096, "requests": r["requests"],
                       "prompt_lens": r["prompt_lens"], "output_lens": r["output_lens"],
                       "page_size": 16, "weights": r["weights"]},
            **{k: r[k] for k in ("t2t_ms_mean", "ttft_ms_mean", "generated_tokens", "wall_s",
                                 "min_free_pages", "pool_pages", "all_outputs_complete",
                                 "all_pages_returned", "clocks")}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
def tp_decode(args, rank, world, local, dev, batch=64, steps=128, allreduce=None,
              name=None) -> dict:
    """Qwen2.5-72B-shape continuous-batching decode with
    tensor parallelism over the ranks of the (already initialised) process
    group, one rank per GPU.

    ``batch`` requests, prompts U[512, 4096] of random ids (seeded, the same on
    every rank), ``steps + 1`` output tokens each (1 from prefill), page size
    16, greedy sampling, CUDA-graph decode with the two all-reduces per layer
    captured in the graph. Random bf16 weights (``Model.create``: each rank
    keeps its slices of the same seeded tensors). T2T follows the reference's
    definition (per request, time between its first and last token over
    tokens - 1, averaged); every timing is the max over ranks. Returns the
    measured numbers (every rank; the same on all).
    """
    import torch
    import torch.distributed as dist

    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Request, Scheduler

    group = dist.group.WORLD if world > 1 else None
    name = name or "qwen2.5-72b"
    cfg = PRESETS[name]
    lo, hi = 512, 4096
    t0 = time.perf_counter()
    model = Model.create(cfg, dev, torch.bfloat16, seed=5, tp_rank=rank, tp_size=world,
                         tp_group=group)
    allreduce = allreduce or "auto"
    if allreduce == "auto":
        allreduce = "peer" if world <= 4 else "nccl"
    if world > 1 and allreduce == "peer":
        model.enable_peer_allreduce(max_rows=batch)
    torch.cuda.synchronize()
    init_s = time.perf_counter() - t0
    rng = np.random.default_rng(5)
    lens = rng.integers(lo, hi + 1, batch).tolist()
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in lens]
    t0 = time.perf_counter()
    sched = Scheduler(model, cfg, dev, torch.bfloat16, max_batch_size=batch,
                      max_seq_len=hi + steps, page_size=16, eos_token_ids=set(),
                      max_prefill_tokens=16384)
    torch.cuda.synchronize()
    capture_s = time.perf_counter() - t0

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    reqs = [Request(f"r{i}", p, steps + 1, 0.0) for i, p in enumerate(prompts)]
    for r in reqs:
        sched.submit_request(r)
    clocks = ClockSampler(local)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    t0 = time.perf_counter()
    sched.step()                                   # admit + prefill all + first decode
    torch.cuda.synchronize()
    first_s = time.perf_counter() - t0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    n_dec = 0
    while sched.active_requests or sched.waiting_queue:
        sched.step()
        n_dec += 1
    ev1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    dec_ms = ev0.elapsed_time(ev1) / max(n_dec, 1)
    t2t = statistics.mean((r.last_token_time - r.prefill_done_time)
                          / (len(r.generated_tokens) - 1) for r in reqs) * 1e3
    t2t, dec_ms, first_s, init_s, capture_s = max_over_ranks(
        [t2t, dec_ms, first_s, init_s, capture_s])
    ok = all(len(r.generated_tokens) == steps + 1 for r in reqs)
    sched.close()
    if model.comm is not None:
        model.comm.check_status()
        model.comm.close()
    del sched, model
    torch.cuda.empty_cache()
    return {"metric": f"{name} decode tok/s @B={batch}, tensor parallel (config 5)",
            "value": round(batch / (dec_ms / 1e3), 1), "unit": "tok/s",
            "decode_step_ms": round(dec_ms, 3), "t2t_ms": round(t2t, 3),
            "t2t_tok_s": round(batch / (t2t / 1e3), 1),
            "t2t_note": ("reference definition (per request, first to last token): includes "
                         "the wait of early-prefilled requests for the later prefill chunks"),
            "parallelism": f"tp{world}", "decode_allreduce": allreduce if world > 1 else "none",
            "model": name, "batch": batch, "decode_steps": steps,
            "prompt_lens": f"U[{lo},{hi}] seeded", "weights": "random N(0,0.02) bf16",
            "first_step_s (prefill of all + 1 decode)": round(first_s, 3),
            "model_init_s": round(init_s, 2), "graph_capture_s": round(capture_s, 2),
            "decode_steps_timed": n_dec, "all_requests_complete": ok, "clocks": clk}


def run_tp_decode(args):
    """``--workload config5``: ``tp_decode`` at the launch's N on its own."""
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    active = nccl_group(dev, 300) if world > 1 else 1
    batch, steps = args.batch or 64, args.decode_steps or 128
    r = tp_decode(args, rank, world, local, dev, batch=batch, steps=steps,
                  allreduce=args.allreduce, name=args.model)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": r["metric"], "value": r["t2t_tok_s"], "unit": "tok/s", "n_gpus": world,
        "gpus_active": active,
        "steps": steps, "warmup": 0, "ms_per_step": r["decode_step_ms"], "t2t_ms": r["t2t_ms"],
        "decode_step_tok_s": r["value"], "t2t_note": r["t2t_note"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "BASELINE config 5: continuous-batching decode, all requests "
                               "admitted at once, greedy", "model": r["model"],
                   "global_batch": batch, "seq_len": f"prompts {r['prompt_lens']} + {steps} decode",
                   "parallelism": r["parallelism"], "page_size": 16, "weights": r["weights"],
                   "decode_allreduce": r["decode_allreduce"]},
        "first_step_s (prefill of all + 1 decode)": r["first_step_s (prefill of all + 1 decode)"],
        "model_init_s": r["model_init_s"], "graph_capture_s": r["graph_capture_s"],
        "decode_steps_timed": r["decode_steps_timed"],
        "all_requests_complete": r["all_requests_complete"], "clocks": r["clocks"],
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
DECODE_SHAPES = [  # (batch, Q heads, KV heads, ctx lo, ctx hi, note)
    (32, 32, 8, 256, 4096, "config 2"),
    (64, 32, 8, 512, 4096, ""),
    (64, 64, 8, 512, 4096, "Qwen2.5-72B, one GPU's worth of heads"),
    (64, 32, 4, 512, 4096, "Qwen2.5-72B at TP 2"),
    (64, 16, 2, 512, 4096, "Qwen2.5-72B at TP 4"),
    (64, 8, 1, 512, 4096, "Qwen2.5-72B at TP 8"),
    (32, 28, 4, 256, 4096, "Qwen2.5-7B (group 7)"),
    (32, 16, 4, 256, 4096, "config 2 head-sharded over 2 GPUs: one GPU's heads"),
    (32, 8, 2, 256, 4096, "config 2 head-sharded over 4 GPUs: one GPU's heads"),
    (32, 4, 1, 256, 4096, "config 2 head-sharded over 8 GPUs: one GPU's heads"),
]


def run_decode_shapes(args):
    """Paged decode alone across the head/batch shapes of configs 2-5.

    Per shape: seeded contexts, random non-contiguous page tables, as many
    distinct layer pools as fit in ~6 GB (so back-to-back launches never hit
    in L2), decode launches back to back through the C ABI, CUDA events around
    the loop. Prints one JSON line per shape (bytes = K/V of all contexts).
    """
    import torch
    from mi_b200 import capi

    dev = torch.device("cuda", dist_env()[2])
    torch.cuda.set_device(dev)
    lib = capi.lib()
    ps, d = 16, 128
    ws = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    peak, _ = read_peak()
    for (b, hq, hkv, lo, hi, note) in DECODE_SHAPES:
        lens = np.random.default_rng(0).integers(lo, hi + 1, b).tolist()
        P = sum(math.ceil(n / ps) for n in lens) + 16
        L = max(2, min(16, int(6e9 // (P * 2 * ps * hkv * d * 2))))
        pools = [torch.empty(P, 2, ps, hkv, d, device=dev, dtype=torch.bfloat16).normal_()
                 for _ in range(L)]
        perm = np.random.default_rng(1).permutation(P - 1)
        indptr, indices, last, k0 = [0], [], [], 0
        for n in lens:
            k = math.ceil(n / ps)
            indices += perm[k0:k0 + k].tolist()
            k0 += k
            indptr.append(len(indices))
            last.append(n % ps or ps)
        i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
        ip, ind, lp = i32(indptr), i32(indices), i32(last)
        q = torch.randn(b, hq, d, device=dev, dtype=torch.bfloat16)
        out = torch.empty_like(q)

        def dec(pool):
            return lib.mi_paged_decode(
                q.data_ptr(), q.stride(0), q.stride(1), pool.data_ptr(), P, ps, hkv, d,
                capi.DTYPE_BF16, ip.data_ptr(), ind.data_ptr(), lp.data_ptr(), b, hq,
                1 / math.sqrt(d), out.data_ptr(), None, ws.data_ptr(), ws.numel(),
                st.data_ptr(), stream)
        rc = 0
        for i in range(max(args.warmup, 3) * L):
            rc |= dec(pools[i % L])
        torch.cuda.synchronize()
        reps = max(2, 200 // L)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for pool in pools:
                rc |= dec(pool)
        e1.record()
        torch.cuda.synchronize()
        if rc or int(st.item()):
            raise capi.MiError(f"decode failed: rc={rc} status={int(st.item())}")
        us = e0.elapsed_time(e1) * 1e3 / (reps * L)
        byt = sum(lens) * hkv * d * 2 * 2
        print(json.dumps({"batch": b, "q_heads": hq, "kv_heads": hkv, "ctx": f"U[{lo},{hi}]",
                          "mb_per_launch": round(byt / 1e6, 1), "us_per_launch": round(us, 2),
                          "gbs": round(byt / us / 1e3, 1), "frac": round(byt / us / 1e3 / peak, 4),
                          "layer_pools": L, "note": note}), flush=True)
        del pools
        torch.cuda.empty_cache()


def prefill_flops(lens, hq=32, d=128) -> int:
    """Causal prefill attention flops: sum_r 4*Hq*D*L_r(L_r+1)/2 (QK^T + PV)."""
    return sum(4 * hq * d * n * (n + 1) // 2 for n in lens)


CONFIG1_PROMPT_LENS = (37, 128, 255, 500)


def config1_prompts(vocab, seed=1):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).tolist() for n in CONFIG1_PROMPT_LENS]


def cpu_reference_config1(steps=8, seed=1234):
    """The reference's CPU decode step at BASELINE config 1 (Qwen2.5-0.5B
    shape, fp32, seeded weights, the 4 prompts of 37/128/255/500 tokens),
    through the port of its whole padded forward (oracle/reference_cpu.py):
    prefill of the 4 prompts, then ``steps`` batched decode steps. Returns
    (mean ms per decode step, sample text)."""
    import torch
    from mi_b200.model import PRESETS, Model
    from mi_b200.weights import init_random_weights
    from oracle.reference_cpu import PaddedReferenceModel
    cfg = PRESETS["qwen2.5-0.5b"]
    model = Model(cfg)
    init_random_weights(model, seed)
    ref = PaddedReferenceModel(model.state_dict(), cfg, max_batch=4,
                               max_seq=max(CONFIG1_PROMPT_LENS) + steps + 2)
    del model
    prompts = config1_prompts(cfg.vocab_size)
    tokens = []
    for slot, pr in enumerate(prompts):
        tokens.append(int(ref.prefill(slot, pr).argmax()))
    positions = [len(pr) for pr in prompts]
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        logits = ref.decode(list(range(4)), positions, tokens)
        times.append((time.perf_counter() - t0) * 1e3)
        tokens = logits.argmax(-1).tolist()
        positions = [p_ + 1 for p_ in positions]
    ms = statistics.mean(times[1:]) if len(times) > 1 else times[0]
    return ms, (f"{steps} batched decode steps (B=4, greedy) after the prefill of prompts "
                f"{list(CONFIG1_PROMPT_LENS)}, fp32, {torch.get_num_threads()} threads; "
                "mean of all but the first")


def config1_measure(dev, cpu_ms=None) -> dict:
    """BASELINE config 1 on one GPU: Qwen2.5-0.5B shape, fp32, the 4 prompts,
    50 output tokens each, CUDA-graph decode; the median decode step beside
    the reference's CPU decode step on the same workload (``cpu_ms``, timed
    by the caller, or here when not given)."""
    import torch
    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Request, Scheduler
    cfg = PRESETS["qwen2.5-0.5b"]
    model = Model.create(cfg, dev, torch.float32, seed=1234)
    prompts = config1_prompts(cfg.vocab_size)
    sched = Scheduler(model, cfg, dev, torch.float32, max_batch_size=4, max_seq_len=1024,
                      page_size=16, eos_token_ids=set())
    for rep in range(2):   # warm-up set, then the measured one
        reqs = [Request(f"c{rep}_{i}", p_, 50 if rep else 4, 0.0) for i, p_ in enumerate(prompts)]
        for r in reqs:
            sched.submit_request(r)
        torch.cuda.synchronize()
        step_ms = []
        while sched.active_requests or sched.waiting_queue:
            t0 = time.perf_counter()
            sched.step()
            step_ms.append((time.perf_counter() - t0) * 1e3)
    gpu_ms = statistics.median(step_ms[1:])
    sched.close()
    del sched, model
    torch.cuda.empty_cache()
    sample = "timed by the caller (cpu_baseline.config1_decode_step_ms)"
    if cpu_ms is None:
        cpu_ms, sample = cpu_reference_config1()
    return {"metric": "config 1 decode step (Qwen2.5-0.5B shape, fp32, B=4)",
            "value": round(gpu_ms, 3), "unit": "ms", "higher_is_better": False,
            "cuda_graph_decode": True, "decode_steps": len(step_ms) - 1,
            "cpu_reference_ms": round(cpu_ms, 2), "cpu_sample": sample,
            "speedup_vs_cpu_reference": round(cpu_ms / gpu_ms, 1)}


def run_config1(args):
    """``--workload config1``: ``config1_measure`` on its own."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = config1_measure(dev)
    print(json.dumps({**r, "n_gpus": 1}), flush=True)


def prefill_measure(dev, layers=8, steps=5, warmup=3) -> dict:
    """Kernel 3 on its own: ragged causal paged prefill of config 3's prompts.

    32 requests, prompts U[128, 1024] (seeded), Mistral-7B attention shape
    (32 Q / 8 KV heads, head_dim 128), bf16, page_size 16, random
    non-contiguous page tables, K/V already in the pages (as after the append
    of the same step). One launch per layer, each layer with its own pool;
    ``steps`` passes over ``layers`` pools back to back, CUDA events around
    the whole loop. Reports tensor TFLOP/s against the measured dense bf16
    peak (the burst figure: the kernel is timed alone).
    """
    import torch
    from mi_b200.prefill import BatchPrefillWithPagedKVCacheWrapper

    hq, hkv, d, ps = 32, 8, 128, 16
    L = min(layers, 8)
    rng = np.random.default_rng(3)
    lens = rng.integers(128, 1025, 32).tolist()
    npages = [math.ceil(n / ps) for n in lens]
    P = sum(npages) + 1
    perm = np.random.default_rng(4).permutation(P - 1)
    indptr, indices, last, qo, k0 = [0], [], [], [0], 0
    for n, k in zip(lens, npages):
        indices.extend(perm[k0:k0 + k].tolist())
        k0 += k
        indptr.append(len(indices))
        last.append(n % ps or ps)
        qo.append(qo[-1] + n)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    ip, ind, lp, qo_t = i32(indptr), i32(indices), i32(last), i32(qo)
    g = torch.Generator(device=dev).manual_seed(7)
    pools = [torch.randn(P, 2, ps, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
             for _ in range(L)]
    q = torch.randn(qo[-1], hq, d, device=dev, dtype=torch.bfloat16, generator=g)
    out = torch.empty_like(q)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device=dev)
    w = BatchPrefillWithPagedKVCacheWrapper(ws)
    w.plan(qo_t, ip, ind, lp, hq, hkv, d, ps, causal=True, q_data_type=torch.bfloat16)
    for i in range(max(warmup, 3)):
        for pool in pools:
            w.run(q, pool, out=out)
    torch.cuda.synchronize()
    w.check_status()
    K = max(1, min(steps, 20))
    clocks = ClockSampler(dev.index or 0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        for pool in pools:
            w.run(q, pool, out=out)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    w.check_status()
    ms = e0.elapsed_time(e1) / (K * L)
    fl = prefill_flops(lens, hq, d)
    tflops = fl / (ms / 1e3) / 1e12
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
        kind = "measured"
    except (OSError, KeyError, TypeError, ValueError):  # absent or malformed: the fallback
        peak, kind = 1590.0, "fallback"
    del pools
    torch.cuda.empty_cache()
    return {"metric": "paged prefill attention TFLOP/s (config-3 prompts)",
            "value": round(tflops, 1), "unit": "TFLOP/s", "steps": K,
            "warmup": max(warmup, 3), "ms_per_launch": round(ms, 4),
            "workload": ("ragged causal paged prefill, 32 requests, prompts U[128,1024] seeded, "
                         "32 Q / 8 KV heads, head_dim 128, page_size 16"),
            "tokens": qo[-1], "layers_pools": L,
            "roofline": {"bound": "tensor", "kernel": "prefill_tc2_kernel",
                         "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4), "peak_kind": f"{kind} (burst)",
                         "algorithmic_flops": fl, "avg_launch_us": round(ms * 1e3, 2)},
            "clocks": clk, "gpu_launches": K * L}


def run_prefill(args):
    """``--workload prefill``: ``prefill_measure`` on its own."""
    import torch
    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    r = prefill_measure(dev, layers=args.layers, steps=args.steps, warmup=args.warmup)
    line = {"metric": r["metric"], "value": r["value"], "unit": "TFLOP/s", "n_gpus": 1,
            "steps": r["steps"], "warmup": r["warmup"], "ms_per_step": r["ms_per_launch"],
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": r["workload"], "tokens": r["tokens"],
                       "layers_pools": r["layers_pools"]},
            "roofline": r["roofline"], "clocks": r["clocks"], "gpu_launches": r["gpu_launches"]}
    print(json.dumps(line), flush=True)


PROJ_SHAPES = {"qkv": (6144, 4096), "o_proj": (4096, 4096), "gate_up": (28672, 4096),
               "down_proj": (4096, 14336), "lm_head": (32768, 4096)}  # Mistral-7B [N, K]


def run_proj(args):
    """``--workload proj``: the decode step's projections at 32 rows
    (Mistral-7B shapes), this package's small-M projection kernel
    (``glue.proj_small_m``) beside cuBLAS (``F.linear`` on the nn.Linear
    layout and ``x @ Wt`` on the transposed one). Each measurement is 30
    (add+RMSNorm -> projection) pairs captured in one CUDA graph, the order
    of a decode step, over weight copies larger than L2 together, minus the
    RMSNorm alone; CUDA events around 5 replays. ``--proj-shape`` limits the
    run to one shape (for a profiler)."""
    import torch
    from mi_b200 import glue
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    m = 32

    def graph_us(fns, reps=30):
        for f in fns:
            f()
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for f in fns:
                f()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(reps):
                fns[i % len(fns)]()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (5 * reps)

    shapes = {args.proj_shape: PROJ_SHAPES[args.proj_shape]} if args.proj_shape else PROJ_SHAPES
    out = {}
    for name, (n, k) in shapes.items():
        size = n * k * 2
        copies = max(2, math.ceil(400e6 / size))
        ws = [(torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
        res = torch.randn(m, k, device=dev).to(torch.bfloat16)
        nw = torch.ones(k, device=dev, dtype=torch.bfloat16)
        xn = torch.empty(m, k, device=dev, dtype=torch.bfloat16)
        y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)

        def norm():
            glue.add_rmsnorm(None, res, nw, 1e-6, out=xn)
        t_norm = graph_us([norm])
        t_mi = graph_us([lambda w=w: (norm(), glue.proj_small_m(xn, w, out=y)) for w in ws]) - t_norm
        row = {"mi_us": round(t_mi, 2), "mi_TBs": round(size / t_mi / 1e6, 2)}
        if not args.proj_shape:
            wts = [w.t().contiguous() for w in ws]
            t_lin = graph_us([lambda w=w: (norm(), torch.nn.functional.linear(xn, w))
                              for w in ws]) - t_norm
            t_mm = graph_us([lambda w=w: (norm(), torch.mm(xn, w, out=y)) for w in wts]) - t_norm
            row.update({"cublas_linear_us": round(t_lin, 2), "cublas_wt_us": round(t_mm, 2)})
            del wts
        out[name] = row
        del ws
        torch.cuda.empty_cache()
    st = int(glue.proj_status(dev).item())
    print(json.dumps({"workload": "proj", "rows": m, "dtype": "bf16", "shapes_NK": PROJ_SHAPES,
                      "status": st, "results": out,
                      "timing": "30 add+RMSNorm -> projection pairs per CUDA graph, minus the "
                                "RMSNorm alone; weights cycled over copies larger than L2"}),
          flush=True)


def run_model_step(args):
    """``--workload model-step``: config 3 (Mistral-7B shape, 32 requests)
    stepped to a steady decode, then one decode step between
    ``cudaProfilerStart`` / ``cudaProfilerStop`` (for a profiler's
    ``--profile-from-start off``); prints the steady step times."""
    import torch
    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Request, Scheduler
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = PRESETS["mistral-7b"]
    model = Model.create(cfg, dev, torch.bfloat16, seed=3)
    rng = np.random.default_rng(3)
    lens = rng.integers(128, 1025, 32).tolist()
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in lens]
    sched = Scheduler(model, cfg, dev, torch.bfloat16, max_batch_size=32,
                      max_seq_len=1024 + 66, page_size=16, eos_token_ids=set())
    for i, p in enumerate(prompts):
        sched.submit_request(Request(f"r{i}", p, 40, 0.0))
    for _ in range(10):
        sched.step()
    torch.cuda.synchronize()
    times = []
    for _ in range(5):
        t0 = time.perf_counter()
        sched.step()
        torch.cuda.synchronize()
        times.append(round((time.perf_counter() - t0) * 1e3, 3))
    torch.cuda.profiler.start()
    sched.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"workload": "model-step", "steady_decode_step_ms": times}), flush=True)


def run_flashinfer_context(args):
    """Context, not a baseline arm: the reference's own GPU path for one
    config-2 layer on this GPU -- stock ``flashinfer.page.append_paged_kv_cache``
    plus ``BatchDecodeWithPagedKVCacheWrapper`` constructed and planned as the
    reference does (scheduler.py:535-539, :905-916; model.py:207-216, :235) --
    over the same pools, page tables and contexts as ``run_config2`` (8 layer
    pools, ~5 GB, so every launch reads from HBM). The reference's RoPE
    (torch elementwise ops) and per-step ``plan()`` are not counted."""
    import torch
    try:
        import flashinfer
    except ImportError as e:
        print(json.dumps({"workload": "flashinfer-context", "unavailable": str(e)}), flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = CFG
    b, hq, hkv, d, ps, P, L = (c["batch"], c["hq"], c["hkv"], c["head_dim"], c["page_size"],
                               c["num_pages"], 8)
    lens = config2_lens(c["seed"], b, c["ctx_lo"], c["ctx_hi"])
    perm = np.random.default_rng(c["seed"]).permutation(P - 1)
    indptr, indices, last, k0 = [0], [], [], 0
    for n in lens:
        k = math.ceil(n / ps)
        indices.extend(perm[k0:k0 + k].tolist())
        k0 += k
        indptr.append(len(indices))
        last.append(n % ps or ps)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    ip, ind, lp = i32(indptr), i32(indices), i32(last)
    g = torch.Generator(device=dev).manual_seed(1234)
    pools = [torch.randn(P, 2, ps, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
             for _ in range(L)]
    q = torch.randn(b, hq, d, device=dev, dtype=torch.bfloat16, generator=g)
    kn = torch.randn(b, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
    vn = torch.randn(b, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
    bi = torch.arange(b, dtype=torch.int32, device=dev)
    pos = i32([n - 1 for n in lens])
    t0 = time.perf_counter()
    ws = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    w = flashinfer.decode.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="NHD")
    w.plan(indptr=ip, indices=ind, last_page_len=lp, num_qo_heads=hq, num_kv_heads=hkv,
           head_dim=d, page_size=ps, pos_encoding_mode="NONE", q_data_type=torch.bfloat16,
           data_type=torch.bfloat16)

    def layer(pool):
        flashinfer.page.append_paged_kv_cache(kn, vn, bi, pos, pool, ind, ip, lp, kv_layout="NHD")
        return w.run(q, pool)

    for _ in range(max(args.warmup, 3)):
        for pool in pools:
            layer(pool)
    torch.cuda.synchronize()
    setup_s = time.perf_counter() - t0

    def timed(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for pool in pools:
                fn(pool)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * L)

    reps = max(1, min(args.steps, 20))
    clocks = ClockSampler(0)
    us_pair = timed(layer, reps)
    us_dec = timed(lambda pool: w.run(q, pool), reps)
    clk = clocks.stop()
    peak, kind = read_peak()
    byt = decode_bytes(lens)
    print(json.dumps({
        "workload": "flashinfer-context", "metric": "reference GPU path (FlashInfer) at config 2",
        "flashinfer": flashinfer.__version__, "append_plus_decode_us": round(us_pair, 2),
        "decode_us": round(us_dec, 2), "decode_gbs": round(byt / us_dec / 1e3, 1),
        "decode_frac": round(byt / us_dec / 1e3 / peak, 4), "peak_kind": kind,
        "setup_s (JIT / module load, plan, warm-up)": round(setup_s, 1), "layer_pools": L,
        "reps": reps, "clocks": clk,
        "note": "context only; the reference's RoPE ops and per-step plan() are not counted"}),
        flush=True)


# ---------------------------------------------------------------------------
def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=CFG["layers"],
                    help="layer pools per step (32 = Mistral-7B; fewer only for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--shard", choices=["auto", "replicas", "heads"], default="auto",
                    help="config 2 on N GPUs: the KV heads split over the GPUs (strong "
                         "scaling; the default for N > 1, with the replicas split reported "
                         "beside it) or N replicas (weak scaling)")
    ap.add_argument("--no-tp", action="store_true",
                    help="N > 1: skip the Qwen2.5-72B tensor-parallel decode (config 5)")
    ap.add_argument("--tp-steps", type=int, default=48,
                    help="N > 1: decode steps of the config-5 measurement")
    ap.add_argument("--no-extra", action="store_true",
                    help="N = 1: skip the prefill, churn (config 4) and config-1 measurements")
    ap.add_argument("--churn-requests", type=int, default=96,
                    help="N = 1: requests served in the churn (config 4) measurement")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the Mistral-7B-shape decode measurement (config 3)")
    ap.add_argument("--workload",
                    choices=["config2", "config1", "config4", "config5", "prefill",
                             "decode-shapes", "flashinfer-context", "proj", "model-step"],
                    default="config2",
                    help="config5: Qwen2.5-72B tensor-parallel decode over the launch's GPUs; "
                         "prefill: the paged prefill kernel alone on config 3's prompts")
    ap.add_argument("--model", default=None, help="config5: model preset (default qwen2.5-72b)")
    ap.add_argument("--proj-shape", choices=sorted(PROJ_SHAPES), default=None,
                    help="proj: one projection shape only (no cuBLAS timings)")
    ap.add_argument("--batch", type=int, default=None,
                    help="config5: requests (default 64); config4: requests served (default 160)")
    ap.add_argument("--decode-steps", type=int, default=None,
                    help="config5: decode steps per request (default 128)")
    ap.add_argument("--allreduce", choices=["auto", "peer", "nccl"], default="auto",
                    help="config5: decode-step all-reduce: fused over NVLink peer memory "
                         "(with the residual add and RMSNorm), NCCL, or auto (peer up to "
                         "4 GPUs, NCCL beyond: there NCCL's in-switch reduction wins)")
    return ap.parse_args()


def nccl_group(dev, timeout_s: int):
    """The NCCL process group for N > 1 ranks (its init log is switched on
    at the top of this file) and the number of distinct GPUs taking part
    (device UUIDs gathered from every rank)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=dev)
    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    uuids = [None] * dist.get_world_size()
    dist.all_gather_object(uuids, uuid)
    return len(set(uuids))


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    steps, warm = max(args.steps, 1), max(args.warmup, 0)
    lens = config2_lens(CFG["seed"])
    # warm-up steps untimed; the timed run is bounded to ~2 minutes in total
    if warm:
        cpu_reference_steps(lens, warm, budget_s=20.0)  # untimed warm-up
    gbs, dt, threads, sample = cpu_reference_steps(lens, steps, budget_s=100.0)
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm,
        "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(shard="replicas", world=1):
    c = CFG
    heads = shard == "heads" and world > 1
    return {"workload": "BASELINE config 2: Mistral-7B-shape paged KV append + decode "
                        "attention, 32 layers per step, B=32, ctx U[256,4096] seeded, "
                        "random non-contiguous page tables",
            "model": "Mistral-7B attention shape (32 Q / 8 KV heads, head_dim 128)",
            "global_batch": c["batch"], "seq_len": f"U[{c['ctx_lo']},{c['ctx_hi']}]",
            "layers_per_step": c["layers"], "page_size": c["page_size"],
            "pages_per_layer_pool": c["num_pages"],
            "parallelism": (f"heads{world}: each GPU holds {c['hkv'] // world} of the "
                            f"{c['hkv']} KV heads of every page" if heads else "replicas"),
            "l2": "inputs larger than L2: each step streams 32 distinct layer pools "
                  "(~285 MB of KV per layer)"}


def run_config2(args, rank, world, local, dev, heads: bool, with_e2e: bool = True) -> dict:
    """BASELINE config 2 on this rank: the timed steps, the roofline loops and
    (optionally) the end-to-end graph. Returns the measured numbers; the
    caller assembles the JSON line. ``heads``: this rank holds KV heads
    [rank * 8/N, (rank+1) * 8/N) of every page (and their query heads)."""
    import torch
    import torch.distributed as dist

    from mi_b200.decode import BatchDecodeWithPagedKVCacheWrapper
    from mi_b200.rope import rope_tables

    c = dict(CFG)
    c["layers"] = args.layers
    if heads:
        # head-sharded config 2: rank r decodes KV heads [r * hkv/N, (r+1) * hkv/N)
        # (and their query heads) of every request; no exchange between ranks
        if CFG["hkv"] % world:
            raise SystemExit(f"--shard heads needs {CFG['hkv']} KV heads divisible by {world}")
        c["hq"], c["hkv"] = CFG["hq"] // world, CFG["hkv"] // world
    b, hq, hkv, d, ps, P, L = (c["batch"], c["hq"], c["hkv"], c["head_dim"], c["page_size"],
                               c["num_pages"], c["layers"])
    lens = config2_lens(c["seed"], b, c["ctx_lo"], c["ctx_hi"])
    rng = np.random.default_rng(c["seed"])
    perm = rng.permutation(P - 1)
    indptr, indices, last, k0 = [0], [], [], 0
    for n in lens:
        np_ = math.ceil(n / ps)
        indices.extend(perm[k0:k0 + np_].tolist())
        k0 += np_
        indptr.append(len(indices))
        last.append(n % ps or ps)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    indptr_t, indices_t, last_t = i32(indptr), i32(indices), i32(last)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    pools = [torch.randn(P, 2, ps, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
             for _ in range(L)]
    q_raw = torch.randn(b, hq, d, device=dev, dtype=torch.bfloat16, generator=g)
    k_new = torch.randn(b, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
    v_new = torch.randn(b, hkv, d, device=dev, dtype=torch.bfloat16, generator=g)
    out = torch.empty(b, hq, d, device=dev, dtype=torch.bfloat16)
    cos, sin = rope_tables(d, 32768, 1e6, torch.bfloat16, dev)
    ws = torch.zeros(128 * 1024 * 1024, dtype=torch.uint8, device=dev)
    dec = BatchDecodeWithPagedKVCacheWrapper(ws)
    dec.plan(indptr_t, indices_t, last_t, hq, hkv, d, ps, q_data_type=torch.bfloat16)

    def layer_step(pool, ev=None):
        """One layer through the public API (validating wrappers): the decode
        step with its append (RoPE, K/V into the pages) fused in."""
        dec.run_with_append(q_raw, pool, k_new, v_new, cos, sin, out=out)

    # The timed loop calls the C ABI directly with arguments validated once by
    # the calls above, so host-side Python never limits the device time.
    from mi_b200 import capi
    lib = capi.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws_bytes = ws.numel()
    status = dec.status

    def raw_args(pool):
        return (q_raw.data_ptr(), q_raw.stride(0), q_raw.stride(1),
                k_new.data_ptr(), k_new.stride(0), k_new.stride(1),
                v_new.data_ptr(), v_new.stride(0), v_new.stride(1),
                cos.data_ptr(), sin.data_ptr(), cos.shape[0],
                pool.data_ptr(), P, ps, hkv, d, capi.DTYPE_BF16,
                indptr_t.data_ptr(), indices_t.data_ptr(), last_t.data_ptr(), b, hq,
                1.0 / math.sqrt(d), out.data_ptr(), None, ws.data_ptr(), ws_bytes,
                status.data_ptr(), stream)

    args_per_layer = [raw_args(pl) for pl in pools]
    step_fn = lib.mi_paged_decode_append

    def raw_step(layer):
        return step_fn(*args_per_layer[layer])

    # The same layer as two calls (the append kernel rotating q and writing
    # K/V, then the plain decode), timed in the same window for comparison.
    q_rot = torch.empty_like(q_raw)
    bidx_t = torch.arange(b, dtype=torch.int32, device=dev)
    pos_t = i32([n - 1 for n in lens])

    def two_call_args(pool):
        app = (k_new.data_ptr(), k_new.stride(0), k_new.stride(1),
               v_new.data_ptr(), v_new.stride(0), v_new.stride(1),
               bidx_t.data_ptr(), pos_t.data_ptr(), b,
               pool.data_ptr(), P, ps, hkv, d, capi.DTYPE_BF16,
               indices_t.data_ptr(), indptr_t.data_ptr(), b,
               cos.data_ptr(), sin.data_ptr(), cos.shape[0], None,
               q_raw.data_ptr(), q_raw.stride(0), q_raw.stride(1),
               q_rot.data_ptr(), q_rot.stride(0), q_rot.stride(1), hq,
               -1, status.data_ptr(), stream)
        de = (q_rot.data_ptr(), q_rot.stride(0), q_rot.stride(1),
              pool.data_ptr(), P, ps, hkv, d, capi.DTYPE_BF16,
              indptr_t.data_ptr(), indices_t.data_ptr(), last_t.data_ptr(), b, hq,
              1.0 / math.sqrt(d), out.data_ptr(), None, ws.data_ptr(), ws_bytes,
              status.data_ptr(), stream)
        return app, de

    two_call_per_layer = [two_call_args(pl) for pl in pools]

    def two_call_step(layer):
        app, de = two_call_per_layer[layer]
        return lib.mi_append_paged_kv_cache(*app) | lib.mi_paged_decode(*de)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(max(args.warmup, 3)):
        for layer in range(L):
            layer_step(pools[layer])
    torch.cuda.synchronize()
    dec.check_status()

    # ---- device-resident timed region ----------------------------------------
    # K steps of L layers (append + decode per layer), no events between the
    # launches: an event record between two kernels would break the
    # programmatic-dependent-launch overlap they have in a model step.
    K = args.steps
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record()
    rc = 0
    for _ in range(K):
        for layer in range(L):
            rc |= raw_step(layer)
    t_end.record()
    # Launch duration for the roofline: the step's one launch pair (fused
    # decode + split-K merge) back to back over the layer pools (each pool is
    # read once per pass, and the L pools together are far larger than L2),
    # bracketed by one event pair.
    kd = max(1, min(K, 20))
    d_start, d_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d_start.record()
    for _ in range(kd):
        for layer in range(L):
            rc |= raw_step(layer)
    d_end.record()
    # the two-call form of the same layers (append kernel, then plain decode)
    c_start, c_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c_start.record()
    for _ in range(kd):
        for layer in range(L):
            rc |= two_call_step(layer)
    c_end.record()
    if rc:
        raise capi.MiError(f"launch failed in the timed loop: {lib.mi_last_error().decode()}")
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms_total = max_over_ranks(t_start.elapsed_time(t_end))
    dec_ms = max_over_ranks(d_start.elapsed_time(d_end)) / (kd * L)
    two_call_ms = max_over_ranks(c_start.elapsed_time(c_end)) / (kd * L)
    dec.check_status()

    step_bytes = L * (decode_bytes(lens, c) + append_bytes(b, c))  # this rank's bytes
    ms_per_step = ms_total / K
    value = world * step_bytes * K / (ms_total / 1e3) / 1e9
    peak, peak_kind = read_peak()
    achieved = (decode_bytes(lens, c) + append_bytes(b, c)) / (dec_ms / 1e3) / 1e9
    traffic = read_traffic()

    # ---- end to end through the public API with host buffers -----------------
    # Every step copies each layer's q / k_new / v_new in from pinned host
    # memory and each layer's attention output back out, and the host waits
    # for the step's last output. Serving form: one CUDA graph per step (the
    # model's decode step is a graph too) in which a copy stream brings the
    # layers' inputs in ahead of the compute stream and a second copy stream
    # drains each layer's output as soon as its decode is done. The eager form
    # (same calls issued one by one on one stream) is reported beside it.
    e2e = None
    if with_e2e:
        nq, nk = b * hq * d, b * hkv * d
        seg = nq + 2 * nk
        in_h = torch.randn(L, seg, dtype=torch.bfloat16).pin_memory()
        o_h = torch.empty(L, b, hq, d, dtype=torch.bfloat16).pin_memory()
        in_d = torch.empty(L, seg, dtype=torch.bfloat16, device=dev)
        out_d = torch.empty(L, b, hq, d, dtype=torch.bfloat16, device=dev)
        views = [(in_d[i, :nq].view(b, hq, d), in_d[i, nq:nq + nk].view(b, hkv, d),
                  in_d[i, nq + nk:].view(b, hkv, d)) for i in range(L)]
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(L)]
        ev_out = [torch.cuda.Event() for _ in range(L)]

        def e2e_step():
            cs = torch.cuda.current_stream(dev)
            h2d.wait_stream(cs)
            d2h.wait_stream(cs)
            with torch.cuda.stream(h2d):
                for i in range(L):
                    in_d[i].copy_(in_h[i], non_blocking=True)
                    ev_in[i].record(h2d)
            for i in range(L):
                cs.wait_event(ev_in[i])
                qv, kv, vv = views[i]
                dec.run_with_append(qv, pools[i], kv, vv, cos, sin, out=out_d[i])
                ev_out[i].record(cs)
                d2h.wait_event(ev_out[i])
                with torch.cuda.stream(d2h):
                    o_h[i].copy_(out_d[i], non_blocking=True)
            cs.wait_stream(h2d)
            cs.wait_stream(d2h)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                e2e_step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        # thread-local capture: the process group's watchdog thread may query
        # its CUDA events while this thread captures
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            e2e_step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        dec.check_status()
        ke = max(1, min(K, 50))

        def timed(step_fn):
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(ke):
                step_fn()
                torch.cuda.current_stream(dev).synchronize()  # the caller reads the step's result
            e1.record()
            torch.cuda.synchronize()
            barrier()
            return max_over_ranks(e0.elapsed_time(e1)) / ke

        e2e_ms = timed(graph.replay)

        def eager_step():
            for i in range(L):
                qv, kv, vv = views[i]
                in_d[i].copy_(in_h[i], non_blocking=True)
                dec.run_with_append(qv, pools[i], kv, vv, cos, sin, out=out_d[i])
                o_h[i].copy_(out_d[i], non_blocking=True)

        eager_ms = timed(eager_step)
        dec.check_status()
        del graph
        gbs = lambda ms: round(world * step_bytes / (ms / 1e3) / 1e9, 2)  # noqa: E731
        e2e = {"value": gbs(e2e_ms), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
               "h2d_bytes_per_step": L * seg * 2, "d2h_bytes_per_step": L * nq * 2,
               "timing": (f"CUDA events around {ke} steps, host synchronised after each; "
                          "one CUDA graph per step: per-layer H2D of q/k_new/v_new from "
                          "pinned memory on a copy stream, append + decode through the "
                          "public wrappers on the compute stream, per-layer D2H of the "
                          "output on a second copy stream"),
               "eager": {"value": gbs(eager_ms), "ms_per_step": round(eager_ms, 4),
                         "timing": "same calls issued one by one on one stream"}}

    return {"value": value, "ms_per_step": ms_per_step, "K": K, "L": L,
            "peak": peak, "peak_kind": peak_kind, "achieved": achieved, "traffic": traffic,
            "algorithmic_bytes": decode_bytes(lens, c) + append_bytes(b, c),
            "dec_ms": dec_ms, "two_call_ms": two_call_ms, "kd": kd, "clocks": clk, "e2e": e2e}


def cpu_baseline_line(lens) -> dict:
    """The reference's own CPU path on this host (rank 0, N = 1)."""
    gbs, _, threads, sample = cpu_reference_steps(lens, 8, budget_s=20.0)
    cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": sample}
    # the same path in fp32 (the reference's CPU dtype for config 1)
    gbs32, _, _, sample32 = cpu_reference_steps(lens, 4, budget_s=10.0, dtype_name="float32")
    cpu["fp32"] = {"value": round(gbs32, 3), "unit": "GB/s", "sample": sample32}
    # the reference's whole CPU decode step at config 1 (its own workload)
    c1_ms, c1_sample = cpu_reference_config1()
    cpu["config1_decode_step_ms"] = {"value": round(c1_ms, 2), "unit": "ms", "sample": c1_sample}
    return cpu


def roofline_obj(r: dict, heads: bool) -> dict:
    return {"bound": "hbm", "kernel": "decode_sk_kernel (append fused in)",
            "achieved": round(r["achieved"], 1), "peak": r["peak"], "unit": "GB/s",
            "frac": round(r["achieved"] / r["peak"], 4), "peak_kind": r["peak_kind"],
            "traffic": r["traffic"] if not heads else None,
            "algorithmic_bytes": r["algorithmic_bytes"],
            "avg_launch_us": round(r["dec_ms"] * 1e3, 2),
            "two_call_us": round(r["two_call_ms"] * 1e3, 2),
            "timing": (f"CUDA events around {r['kd'] * r['L']} back-to-back launch pairs "
                       "(fused append + decode, split-K merge) over the layer pools; "
                       "two_call_us: the same layers as the append kernel followed by "
                       "the plain decode pair, timed right after"),
            "gpu_launches_roofline_loop": 2 * r["kd"] * r["L"]}


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "config5":
        run_tp_decode(args)
        return
    if args.workload == "config4":
        run_churn(args)
        return
    if args.workload == "prefill":
        run_prefill(args)
        return
    if args.workload == "decode-shapes":
        run_decode_shapes(args)
        return
    if args.workload == "config1":
        run_config1(args)
        return
    if args.workload == "flashinfer-context":
        run_flashinfer_context(args)
        return
    if args.workload == "proj":
        run_proj(args)
        return
    if args.workload == "model-step":
        run_model_step(args)
        return
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    active = nccl_group(dev, 180) if world > 1 else 1
    heads = world > 1 and args.shard != "replicas"
    if heads and CFG["hkv"] % world:
        raise SystemExit(f"head sharding needs {CFG['hkv']} KV heads divisible by {world}")
    lens = config2_lens(CFG["seed"])
    r = run_config2(args, rank, world, local, dev, heads, with_e2e=not args.no_e2e)

    # ---- N > 1: the other split of config 2, and the tensor-parallel model ----
    replicas = tp = None
    if world > 1 and heads:
        torch.cuda.empty_cache()
        rr = run_config2(args, rank, world, local, dev, False, with_e2e=False)
        replicas = {"value": round(rr["value"], 2), "unit": "GB/s",
                    "ms_per_step": round(rr["ms_per_step"], 4), "scaling": "weak",
                    "parallelism": "replicas: every GPU runs the whole config-2 step on its own "
                                   "pools (no collective)",
                    "roofline": roofline_obj(rr, False), "clocks": rr["clocks"]}
        torch.cuda.empty_cache()
    if world > 1 and not args.no_tp:
        tp = tp_decode(args, rank, world, local, dev, batch=64, steps=args.tp_steps)
        torch.cuda.empty_cache()

    # ---- N = 1: CPU baseline and the other single-GPU workloads (rank 0) -------
    cpu = model_line = prefill = churn = c1 = None
    if rank == 0 and world == 1:
        if not args.no_cpu_baseline:
            cpu = cpu_baseline_line(lens)
        torch.cuda.empty_cache()
        if not args.no_model:
            model_line = model_decode(dev)
        if not args.no_extra:
            prefill = prefill_measure(dev, layers=8, steps=5, warmup=3)
            churn = churn_measure(dev, n_req=args.churn_requests)
            c1 = config1_measure(dev, cpu_ms=(cpu or {}).get("config1_decode_step_ms",
                                                             {}).get("value"))

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(r["value"], 2), "unit": "GB/s", "n_gpus": world,
        "gpus_active": active, "steps": r["K"], "warmup": max(args.warmup, 3), "ms_per_step": round(r["ms_per_step"], 4),
        "higher_is_better": True, "scaling": "strong" if heads else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload_config("heads" if heads else "replicas", world),
        "roofline": roofline_obj(r, heads),
        "cpu_baseline": cpu, "e2e": r["e2e"], "clocks": r["clocks"],
        "gpu_launches": 2 * r["K"] * r["L"],
        "model_decode": model_line,
    }
    if replicas is not None:
        line["replicas"] = replicas
    if tp is not None:
        line["tp_decode"] = tp
    for key, val in (("prefill", prefill), ("churn", churn), ("config1", c1)):
        if val is not None:
            line[key] = val
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
