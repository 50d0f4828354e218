"""Pin the CPU oracle against fixtures produced by the reference itself.

The fixtures in ``tests/golden`` come from running the reference's own code on
the CPU (``tests/golden/make_golden.py``). These tests need no GPU.
"""
import json
import os

import numpy as np
import pytest

from oracle import paged_oracle as po

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _vals(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return bits.astype(np.float32)
    if dtype == "bfloat16":
        return po.bf16_bits_to_f32(bits)
    return bits.view(np.float16).astype(np.float32)


@pytest.fixture(scope="module")
def rope_fx():
    return np.load(os.path.join(GOLDEN, "rope.npz"))


@pytest.fixture(scope="module")
def attn_fx():
    return np.load(os.path.join(GOLDEN, "attn.npz"))


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("d", [64, 128])
def test_rope_bit_exact(rope_fx, dtype, d):
    key = f"{dtype}_d{d}"
    x = _vals(rope_fx[f"{key}_x"], dtype)
    cos = _vals(rope_fx[f"{key}_cos"], dtype)[:, None, :]
    sin = _vals(rope_fx[f"{key}_sin"], dtype)[:, None, :]
    want = _vals(rope_fx[f"{key}_y"], dtype)
    got = po.apply_rope(x, cos, sin, dtype)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_rope_single_fp32_evaluation_is_not_exact(rope_fx):
    """The three roundings matter: one fused fp32 evaluation differs."""
    key = "bfloat16_d128"
    x = _vals(rope_fx[f"{key}_x"], "bfloat16")
    cos = _vals(rope_fx[f"{key}_cos"], "bfloat16")[:, None, :]
    sin = _vals(rope_fx[f"{key}_sin"], "bfloat16")[:, None, :]
    want = _vals(rope_fx[f"{key}_y"], "bfloat16")
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], -1)
    once = po.bf16_round(x * cos + rot * sin)
    assert not np.array_equal(once, want)


def test_rope_tables_match_reference_rows(rope_fx):
    torch = pytest.importorskip("torch")
    from mi_b200.rope import rope_tables
    for dtype, tdt in (("bfloat16", torch.bfloat16), ("float32", torch.float32)):
        for d in (64, 128):
            key = f"{dtype}_d{d}"
            cos, sin = rope_tables(d, 32768, 1e6, tdt)
            pos = rope_fx[f"{key}_pos"]
            c = cos[pos].float().numpy()
            s = sin[pos].float().numpy()
            assert np.array_equal(c, _vals(rope_fx[f"{key}_cos"], dtype))
            assert np.array_equal(s, _vals(rope_fx[f"{key}_sin"], dtype))


def _attn_cases(fx):
    keys = sorted({k.split("__")[0] for k in fx.files})
    return keys


@pytest.mark.parametrize("case", ["float32_g7", "float32_g4", "bfloat16_g7", "bfloat16_g4"])
def test_paged_oracle_matches_reference_padded_path(attn_fx, case):
    """Oracle append + paged attention == reference padded SDPA path.

    Page contents gathered through the reference's page tables must equal the
    reference's padded cache bit for bit; attention outputs must agree within
    fp32 / bf16 tolerance.
    """
    fx = {k.split("__", 1)[1]: attn_fx[k] for k in attn_fx.files if k.startswith(case + "__")}
    dtype = case.split("_")[0]
    hq, hkv, d, ps, b, steps = (int(v) for v in fx["meta"])
    num_pages = int(fx["num_pages"][0])
    kv = np.zeros((num_pages, 2, ps, hkv, d), np.float32)
    tol = 2e-5 if dtype == "float32" else 2e-2
    for r in range(b):
        q = _vals(fx[f"pre{r}_q"], dtype)
        k = _vals(fx[f"pre{r}_k"], dtype)
        v = _vals(fx[f"pre{r}_v"], dtype)
        L = q.shape[0]
        # prefill appends go to request 0 of a 1-request CSR (scheduler.py:719-720)
        po.append_paged_kv(kv, k, v, np.zeros(L, np.int32), np.arange(L, dtype=np.int32),
                           fx[f"pre{r}_indices"], fx[f"pre{r}_indptr"], ps)
        o, _ = po.prefill_attention(q, np.array([0, L]), kv, fx[f"pre{r}_indptr"],
                                    fx[f"pre{r}_indices"], fx[f"pre{r}_last"], ps, causal=True)
        np.testing.assert_allclose(o, fx[f"pre{r}_o"], atol=tol, rtol=0)
    for s in range(steps):
        q = _vals(fx[f"dec{s}_q"], dtype)
        k = _vals(fx[f"dec{s}_k"], dtype)
        v = _vals(fx[f"dec{s}_v"], dtype)
        pos = fx[f"dec{s}_pos"]
        po.append_paged_kv(kv, k, v, np.arange(b, dtype=np.int32), pos, fx[f"dec{s}_indices"],
                           fx[f"dec{s}_indptr"], ps)
        o, _ = po.decode_attention(q, kv, fx[f"dec{s}_indptr"], fx[f"dec{s}_indices"],
                                   fx[f"dec{s}_last"], ps)
        np.testing.assert_allclose(o, fx[f"dec{s}_o"], atol=tol, rtol=0)
    # page contents, gathered through the last step's page table, equal the
    # reference's padded cache bit for bit
    kc = _vals(fx["final_kc"], dtype)
    vc = _vals(fx["final_vc"], dtype)
    s = steps - 1
    lens = fx["final_len"]
    for r in range(b):
        kk, vv = po.gather_kv(kv, fx[f"dec{s}_indptr"], fx[f"dec{s}_indices"], fx[f"dec{s}_last"],
                              ps, r)
        n = int(lens[r])
        assert kk.shape[0] == n
        assert np.array_equal(kk.transpose(1, 0, 2).view(np.uint32),
                              kc[r, :, :n].view(np.uint32))
        assert np.array_equal(vv.transpose(1, 0, 2).view(np.uint32),
                              vc[r, :, :n].view(np.uint32))


def _trace_events(log):
    """Group the reference's recorded events per scheduler step."""
    steps, cur = [], None
    for ev in log:
        if ev["event"] == "step":
            cur = {"alloc": [], "plan_prefill": [], "plan_decode": [], "release": []}
            steps.append(cur)
        else:
            cur[ev["event"]].append(ev)
    return steps


@pytest.mark.parametrize("case", ["churn", "seqcap"])
def test_scheduler_page_tables_match_reference_trace(case):
    with open(os.path.join(GOLDEN, "sched_trace.json")) as f:
        fx = json.load(f)[case]
    c = fx["config"]
    ref_steps = _trace_events(fx["log"])
    sim = po.simulate_page_tables(c["prompts"], c["max_new"], c["max_batch"], c["max_seq"], 16)
    assert len(sim) == len(ref_steps)
    for ref, mine in zip(ref_steps, sim):
        # admissions: one prefill plan per admitted request, pages in FIFO order
        assert len(ref["plan_prefill"]) == len(mine["admitted"])
        for pl, (_, pages) in zip(ref["plan_prefill"], mine["admitted"]):
            assert pl["indices"] == pages
        if mine["decode"] is None:
            assert ref["plan_decode"] == []
        else:
            (pl,) = ref["plan_decode"]
            assert pl["indptr"] == mine["decode"]["indptr"]
            assert pl["indices"] == mine["decode"]["indices"]
            assert pl["last_page_len"] == mine["decode"]["last_page_len"]
        assert [e["pages"] for e in ref["release"]] == [p for _, p in mine["released"]]


def test_pool_exhaustion_raises_like_reference():
    pool = po.PagePoolOracle(max_batch_size=2, max_seq_len=32, page_size=16)
    assert pool.max_num_pages == 4 and pool.scratch_page == 3
    assert pool.allocate_pages(2) == [0, 1]
    pool.release_pages([1])
    assert pool.allocate_pages(1) == [2]
    assert pool.allocate_pages(1) == [1]
    with pytest.raises(RuntimeError):
        pool.allocate_pages(1)


def test_graph_padding_routes_padded_lanes_to_scratch():
    indptr, indices, last = po.build_csr([[4, 9], [2]], [20, 3], 16)
    ip, ind, lp, pos, bi = po.pad_decode_batch(indptr, indices, last,
                                               np.array([19, 2], np.int32), 4, 11, 16)
    assert ip.tolist() == [0, 2, 3, 3, 3]
    assert lp.tolist() == [4, 3, 1, 1]
    pages, slots = po.append_targets(bi, pos, ind, ip, 16, scratch_page=11)
    assert pages.tolist() == [9, 2, 11, 11]
    assert slots.tolist() == [3, 2, 0, 0]
    # without the scratch rule a padded lane reads indices[total_pages]: here
    # the buffer holds the scratch page there, as the reference intends
    pages2, _ = po.append_targets(bi, pos, ind, ip, 16)
    assert pages2.tolist() == [9, 2, 11, 11]


def test_csr_last_page_len_rule():
    _, _, last = po.build_csr([[0], [1], [2, 3], []], [16, 1, 17, 0], 16)
    assert last.tolist() == [16, 1, 1, 0]
