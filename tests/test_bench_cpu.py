"""bench.py's CPU-side contract: the reference arm's JSON line, the rank rule
under torchrun, and the algorithmic byte / flop counts the roofline uses."""
import json
import os
import subprocess
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402


def _run(args, env_extra=None, timeout=240):
    env = dict(os.environ, **(env_extra or {}))
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args],
                       capture_output=True, text=True, timeout=timeout, env=env, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_reference_arm_prints_one_contract_line():
    out = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    lines = [l for l in out.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["config"]["workload"].startswith("BASELINE config 2")


def test_reference_arm_other_ranks_do_nothing():
    out = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"],
               {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=60)
    assert out.strip() == ""


def test_decode_bytes_formula():
    lens = [1, 16, 17, 300]
    c = dict(bench.CFG)
    hkv, hq, d = c["hkv"], c["hq"], c["head_dim"]
    want = (sum(lens) * hkv * d * 2 * 2 + 2 * len(lens) * hq * d * 2
            + sum((n + 15) // 16 for n in lens) * 4 + (2 * len(lens) + 1) * 4)
    assert bench.decode_bytes(lens) == want


def test_prefill_flops_formula():
    assert bench.prefill_flops([1, 3], hq=2, d=4) == 4 * 2 * 4 * (1 + 6)


def test_seeded_workloads_are_deterministic_and_in_range():
    a, b = bench.config2_lens(0), bench.config2_lens(0)
    assert a == b and len(a) == 32 and min(a) >= 256 and max(a) <= 4096
    s1 = bench.churn_requests(20, 1000)
    s2 = bench.churn_requests(20, 1000)
    assert [len(p) for p, _ in s1] == [len(p) for p, _ in s2]
    assert all(64 <= len(p) <= 2048 and 16 <= n <= 512 for p, n in s1)
    assert all(0 <= t < 1000 for p, _ in s1 for t in p)


def test_head_sharded_config_names_its_split_and_bytes_add_up():
    """--shard heads: each of N GPUs holds Hkv/N KV heads of every page, so
    the per-rank algorithmic bytes of the KV stream are 1/N of the whole."""
    assert bench.workload_config()["parallelism"] == "replicas"
    assert bench.workload_config("heads", 4)["parallelism"].startswith("heads4: each GPU holds 2")
    assert bench.workload_config("heads", 1)["parallelism"] == "replicas"
    lens = bench.config2_lens()
    full = bench.decode_bytes(lens)
    quarter = bench.decode_bytes(lens, dict(bench.CFG, hq=8, hkv=2))
    kv_full = sum(lens) * 8 * 128 * 2 * 2
    assert full - quarter > 0.74 * kv_full   # the KV bytes shrink 4x; q/out and metadata stay small
