"""GPU parity of the four hot-path kernels against the CPU oracle.

Every call goes through the C ABI (libmi_paged.so via ctypes). Bars:
page contents and page tables bit-exact; attention outputs within
max-abs 2e-2 (bf16/fp16) or 1e-4 (fp32) of the fp32 oracle.
"""
import json
import math
import os

import numpy as np
import pytest

from oracle import paged_oracle as po
from tests.gpu_cases import config2_lens, paged_case

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = {"bfloat16": 2e-2, "float16": 2e-2, "float32": 1e-4}
DEV = "cuda"


def tdt(name):
    return getattr(torch, name)


def to_dev(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(tdt(dtype))
    return t.to(DEV)


def i32(x):
    return torch.as_tensor(np.asarray(x, dtype=np.int32)).to(DEV)


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw bits of a device tensor as a uint32/uint16 numpy array."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.numpy().view(np.uint32)
    return t.view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def oracle_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "float32":
        return np.ascontiguousarray(x, np.float32).view(np.uint32)
    if dtype == "bfloat16":
        return po.f32_to_bf16_bits(x)
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def decode_ws():
    return torch.zeros(64 * 1024 * 1024, dtype=torch.uint8, device=DEV)


# --------------------------------------------------------------------------
# (1) append
# --------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (14, 2, 64), (7, 1, 32)])
def test_append_rope_bit_exact(dtype, hq, hkv, d):
    from mi_b200.page import append_paged_kv_cache
    from mi_b200.rope import rope_tables
    lens = [1, 15, 16, 17, 33, 300]
    c = paged_case(1, lens, hq, hkv, d, dtype=dtype)
    rng = np.random.default_rng(2)
    b = len(lens)
    # decode-style append: the last position of each request
    pos = np.asarray([L - 1 for L in lens], np.int32)
    kraw = po.round_to(rng.standard_normal((b, hkv, d), dtype=np.float32) * 3, dtype)
    v = po.round_to(rng.standard_normal((b, hkv, d), dtype=np.float32), dtype)
    qraw = po.round_to(rng.standard_normal((b, hq, d), dtype=np.float32) * 3, dtype)
    cos, sin = rope_tables(d, 4096, 1e6, tdt(dtype))
    cos_h, sin_h = cos.float().numpy(), sin.float().numpy()
    want = c["pool"].copy()
    po.append_paged_kv_rope(want, kraw, v, np.arange(b), pos, c["indices"], c["indptr"], 16,
                            cos_h, sin_h, dtype)
    q_rot = po.apply_rope(qraw, cos_h[pos][:, None], sin_h[pos][:, None], dtype)
    pool = to_dev(c["pool"], dtype)
    q_out = torch.empty(b, hq, d, dtype=tdt(dtype), device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    append_paged_kv_cache(to_dev(kraw, dtype), to_dev(v, dtype), i32(np.arange(b)), i32(pos),
                          pool, i32(c["indices"]), i32(c["indptr"]), i32(c["last"]),
                          rope_cos=cos.to(DEV), rope_sin=sin.to(DEV), q=to_dev(qraw, dtype),
                          q_out=q_out, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert np.array_equal(bits(pool), oracle_bits(want, dtype))
    assert np.array_equal(bits(q_out), oracle_bits(q_rot, dtype))


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_append_prefill_style_and_strided_inputs(dtype):
    """A whole prompt appended for one request, K/V read from a fused QKV buffer."""
    from mi_b200.page import append_paged_kv_cache
    hq, hkv, d, L = 8, 2, 64, 100
    c = paged_case(3, [L], hq, hkv, d, dtype=dtype)
    rng = np.random.default_rng(4)
    qkv = po.round_to(rng.standard_normal((L, (hq + 2 * hkv) * d), dtype=np.float32), dtype)
    qkv_t = to_dev(qkv, dtype)
    k_view = qkv_t[:, hq * d:(hq + hkv) * d].view(L, hkv, d)
    v_view = qkv_t[:, (hq + hkv) * d:].view(L, hkv, d)
    pool = to_dev(c["pool"], dtype)
    append_paged_kv_cache(k_view, v_view, i32(np.zeros(L)), i32(np.arange(L)), pool,
                          i32(c["indices"]), i32(c["indptr"]), i32(c["last"]))
    want = c["pool"].copy()
    k = qkv[:, hq * d:(hq + hkv) * d].reshape(L, hkv, d)
    vv = qkv[:, (hq + hkv) * d:].reshape(L, hkv, d)
    po.append_paged_kv(want, k, vv, np.zeros(L, np.int64), np.arange(L), c["indices"],
                       c["indptr"], 16)
    torch.cuda.synchronize()
    assert np.array_equal(bits(pool), oracle_bits(want, dtype))


def test_append_padding_lanes_go_to_scratch_page():
    from mi_b200.page import append_paged_kv_cache
    hkv, d = 2, 64
    c = paged_case(5, [20, 3], 4, hkv, d)
    scratch = c["P"] - 1
    ip, ind, lp, pos, bi = po.pad_decode_batch(c["indptr"], c["indices"], c["last"],
                                               np.array([19, 2], np.int32), 4, scratch, 64)
    rng = np.random.default_rng(6)
    k = po.round_to(rng.standard_normal((4, hkv, d), dtype=np.float32), "bfloat16")
    v = po.round_to(rng.standard_normal((4, hkv, d), dtype=np.float32), "bfloat16")
    # padding lanes all carry token 0 at position 0 (scheduler.py:887-896), so
    # they write identical rows to the same scratch slot
    k[3], v[3] = k[2], v[2]
    want = c["pool"].copy()
    po.append_paged_kv(want, k, v, bi, pos, ind, ip, 16, scratch_page=scratch)
    pool = to_dev(c["pool"], "bfloat16")
    # the static indices buffer past the real prefix holds a stale real page
    # id here; the kernel must still route padding lanes to the scratch page
    stale = ind.copy()
    stale[len(c["indices"]):] = c["indices"][0]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    append_paged_kv_cache(to_dev(k, "bfloat16"), to_dev(v, "bfloat16"), i32(bi), i32(pos), pool,
                          i32(stale), i32(ip), i32(lp), scratch_page=scratch, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert np.array_equal(bits(pool), oracle_bits(want, "bfloat16"))


def test_append_flags_bad_page_without_writing():
    from mi_b200.page import append_paged_kv_cache
    c = paged_case(7, [5], 4, 2, 64)
    bad = c["indices"].copy()
    bad[0] = c["P"] + 100  # outside the pool
    pool = to_dev(c["pool"], "bfloat16")
    before = bits(pool).copy()
    k = torch.ones(1, 2, 64, dtype=torch.bfloat16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    append_paged_kv_cache(k, k, i32([0]), i32([4]), pool, i32(bad), i32(c["indptr"]),
                          i32(c["last"]), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 2  # MI_STATUS_BAD_PAGE
    assert np.array_equal(bits(pool), before)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("d", [64, 128])
def test_rope_golden_through_append_kernel(dtype, d):
    """The reference's apply_rotary_emb outputs (fixture) come out of the kernel."""
    from mi_b200.page import append_paged_kv_cache
    from mi_b200.rope import rope_tables
    fx = np.load(os.path.join(GOLDEN, "rope.npz"))
    key = f"{dtype}_d{d}"
    xb, yb, pos = fx[f"{key}_x"], fx[f"{key}_y"], fx[f"{key}_pos"]
    n, h, _ = xb.shape
    if dtype == "float32":
        x = xb
    elif dtype == "bfloat16":
        x = po.bf16_bits_to_f32(xb)
    else:
        x = xb.view(np.float16).astype(np.float32)
    cos, sin = rope_tables(d, 32768, 1e6, tdt(dtype))
    ps = 16
    npg = math.ceil(n / ps)
    pool = torch.zeros(npg + 1, 2, ps, h, d, dtype=tdt(dtype), device=DEV)
    indptr, indices, last = po.build_csr([list(range(npg))], [n], ps)
    xt = to_dev(x, dtype)
    append_paged_kv_cache(xt, xt, i32(np.zeros(n)), i32(np.arange(n)), pool, i32(indices),
                          i32(indptr), i32(last), rope_cos=cos.to(DEV), rope_sin=sin.to(DEV),
                          rope_positions=i32(pos))
    torch.cuda.synchronize()
    got = pool[:npg, 0].reshape(npg * ps, h, d)[:n]
    assert np.array_equal(bits(got), yb.view(np.uint32) if dtype == "float32" else yb)


# --------------------------------------------------------------------------
# (2) decode
# --------------------------------------------------------------------------


def run_decode(c, ws=None):
    from mi_b200.decode import BatchDecodeWithPagedKVCacheWrapper
    w = BatchDecodeWithPagedKVCacheWrapper(ws if ws is not None else decode_ws())
    w.plan(i32(c["indptr"]), i32(c["indices"]), i32(c["last"]), c["hq"], c["hkv"], c["d"],
           c["ps"], q_data_type=tdt(c["dtype"]))
    out, lse = w.run(to_dev(c["q"], c["dtype"]), to_dev(c["pool"], c["dtype"]), return_lse=True)
    torch.cuda.synchronize()
    w.check_status()
    return f32(out), f32(lse)


def check_decode(c, ws=None):
    out, lse = run_decode(c, ws)
    want, wlse = po.decode_attention(c["q"], c["pool"], c["indptr"], c["indices"], c["last"],
                                     c["ps"])
    tol = TOL[c["dtype"]]
    np.testing.assert_allclose(out, want, atol=tol, rtol=0)
    fin = np.isfinite(wlse)
    assert np.array_equal(np.isfinite(lse), fin)
    np.testing.assert_allclose(lse[fin], wlse[fin], atol=max(tol, 1e-3), rtol=0)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (28, 4, 128), (14, 2, 64), (64, 8, 128),
                                      (8, 8, 128), (16, 1, 64), (32, 16, 128), (8, 1, 128)])
def test_decode_ragged_edges(dtype, hq, hkv, d):
    lens = [0, 1, 15, 16, 17, 31, 32, 33, 250, 1023]
    check_decode(paged_case(11, lens, hq, hkv, d, dtype=dtype))


@pytest.mark.parametrize("batch", [1, 3, 33])
def test_decode_batch_sizes(batch):
    lens = np.random.default_rng(batch).integers(1, 700, batch).tolist()
    check_decode(paged_case(12 + batch, lens, 32, 8, 128))


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_decode_score_spikes(dtype):
    """Keys scoring far above every other key of their request (about 23 in
    exp2 units after the scale, against about 4), early, mid-tile and deep
    into long contexts: the running max jumps inside a 16-key tile, across
    tiles and across the split-K runs merged at the end."""
    hq, hkv, d = 32, 8, 128
    lens = [700, 3000, 40, 1]
    c = paged_case(71, lens, hq, hkv, d, dtype=dtype)
    rng = np.random.default_rng(72)
    u = rng.standard_normal(d).astype(np.float32)
    u /= np.linalg.norm(u)
    pool = c["pool"].copy()
    for r, spikes in enumerate([[3, 301, 650], [17, 1800, 1801, 2999], [39], []]):
        for pos in spikes:
            page = c["tables"][r][pos // c["ps"]]
            pool[page, 0, pos % c["ps"]] = po.round_to(np.tile(60.0 * u, (hkv, 1)), dtype)
    c["pool"] = pool
    c["q"] = po.round_to(rng.standard_normal((len(lens), hq, d)).astype(np.float32) + 3.0 * u,
                         dtype)
    check_decode(c)


def test_decode_split_k_long_contexts():
    """Few long requests: many chunks per (request, head), merged on device."""
    check_decode(paged_case(13, [4096, 4095, 1, 2049], 32, 8, 128))


def test_decode_config2_full_size():
    """B=32, ctx U[256,4096], 10240-page pool, random tables."""
    c = paged_case(0, config2_lens(0), 32, 8, 128, num_pages=10240)
    check_decode(c)


def test_decode_workspace_reuse_and_page_size_8():
    ws = decode_ws()
    for seed in range(3):
        check_decode(paged_case(20 + seed, [700, 5, 1400], 32, 8, 128), ws)
    check_decode(paged_case(30, [37, 64, 129], 14, 2, 64, page_size=8))
    check_decode(paged_case(31, [37, 64, 129, 1000], 32, 8, 128, page_size=32))


def _append_then_decode_vs_fused(seed, lens, hq, hkv, d, ps, dtype):
    """(pool, out) of append (RoPE) + decode and of the fused decode step on
    the same inputs."""
    from mi_b200.decode import BatchDecodeWithPagedKVCacheWrapper
    from mi_b200.page import append_paged_kv_cache
    from mi_b200.rope import rope_tables
    c = paged_case(seed, lens, hq, hkv, d, page_size=ps, dtype=dtype)
    rng = np.random.default_rng(seed + 1)
    b = len(lens)
    raw = lambda h: to_dev(po.round_to(rng.standard_normal((b, h, d), dtype=np.float32),  # noqa: E731
                                       dtype), dtype)
    q, k, v = raw(hq), raw(hkv), raw(hkv)
    cos, sin = rope_tables(d, 8192, 1e6, tdt(dtype), DEV)
    ip, ind, last = i32(c["indptr"]), i32(c["indices"]), i32(c["last"])
    pools, outs = [], []
    for fused in (False, True):
        pool = to_dev(c["pool"], dtype)
        w = BatchDecodeWithPagedKVCacheWrapper(torch.zeros(64 << 20, dtype=torch.uint8,
                                                           device=DEV))
        w.plan(ip, ind, last, hq, hkv, d, ps)
        if fused:
            out = w.run_with_append(q, pool, k, v, cos, sin)
        else:
            q_rot = torch.empty_like(q)
            append_paged_kv_cache(k, v, i32(list(range(b))), i32([n - 1 for n in lens]), pool,
                                  ind, ip, last, rope_cos=cos, rope_sin=sin, q=q, q_out=q_rot)
            out = w.run(q_rot, pool)
        torch.cuda.synchronize()
        w.check_status()
        pools.append(pool)
        outs.append(out)
    return pools, outs


@pytest.mark.parametrize("hq,hkv,d,ps", [(32, 8, 128, 16), (28, 4, 128, 16), (16, 2, 128, 32),
                                         (8, 1, 64, 16), (14, 2, 64, 16)])
def test_decode_append_matches_append_then_decode(hq, hkv, d, ps):
    """The fused decode step (the new token's RoPE'd K and V written into its
    page by the decode kernel, q rotated as it is loaded) leaves the same
    page bits and returns the same output bits as the append kernel followed
    by decode: one-token requests, tokens at page starts and ends, long and
    short contexts, requests cut across stream-K runs."""
    lens = [1, 16, 17, 300, 1024, 33, 4000, 129, 2, 640]
    (pa, pb), (oa, ob) = _append_then_decode_vs_fused(62, lens, hq, hkv, d, ps, "bfloat16")
    assert torch.equal(pa.view(torch.int16), pb.view(torch.int16))
    assert torch.equal(oa.view(torch.int16), ob.view(torch.int16))


def _assert_pool_bits(pool: torch.Tensor, want: np.ndarray, dtype: str, block: int = 512):
    """Every page of the device pool equals the oracle's, bit for bit (in
    blocks of pages, to bound host memory at full size)."""
    for p0 in range(0, want.shape[0], block):
        got = bits(pool[p0:p0 + block])
        exp = oracle_bits(want[p0:p0 + block], dtype)
        if not np.array_equal(got, exp):
            bad = np.argwhere(got != exp)[0]
            raise AssertionError(f"page {p0 + bad[0]} differs from the oracle at {tuple(bad)}")


def _fused_step_vs_oracle(seed, lens, hq, hkv, d, ps, dtype, num_pages=None):
    """The fused decode step (run_with_append) against the oracle's RoPE
    append (model.py:169-170, :207-216) followed by its paged decode
    (model.py:235): pages bit-exact, output within the dtype's tolerance."""
    from mi_b200.decode import BatchDecodeWithPagedKVCacheWrapper
    from mi_b200.rope import rope_tables
    c = paged_case(seed, lens, hq, hkv, d, page_size=ps, dtype=dtype, num_pages=num_pages)
    rng = np.random.default_rng(seed + 7)
    b = len(lens)
    raw = lambda h: po.round_to(rng.standard_normal((b, h, d), dtype=np.float32), dtype)  # noqa: E731
    q, k, v = raw(hq), raw(hkv), raw(hkv)
    cos, sin = rope_tables(d, 8192, 1e6, tdt(dtype))
    cos_h, sin_h = cos.float().numpy(), sin.float().numpy()
    pos = np.asarray(lens, np.int64) - 1          # each request's new token is its last
    want_pool = c["pool"]                           # updated in place by the oracle below
    pool = to_dev(want_pool, dtype)
    po.append_paged_kv_rope(want_pool, k, v, np.arange(b), pos, c["indices"], c["indptr"], ps,
                            cos_h, sin_h, dtype)
    q_rot = po.apply_rope(q, cos_h[pos][:, None, :], sin_h[pos][:, None, :], dtype)
    want_out, _ = po.decode_attention(q_rot, want_pool, c["indptr"], c["indices"], c["last"], ps)

    w = BatchDecodeWithPagedKVCacheWrapper(torch.zeros(64 << 20, dtype=torch.uint8, device=DEV))
    w.plan(i32(c["indptr"]), i32(c["indices"]), i32(c["last"]), hq, hkv, d, ps,
           q_data_type=tdt(dtype))
    out = w.run_with_append(to_dev(q, dtype), pool, to_dev(k, dtype), to_dev(v, dtype),
                            cos.to(DEV), sin.to(DEV))
    torch.cuda.synchronize()
    w.check_status()
    _assert_pool_bits(pool, want_pool, dtype)
    err = float(np.abs(f32(out) - want_out).max())
    assert err <= TOL[dtype], err


# new tokens at slot 0 (len % 16 == 1) and at the last slot of a 16-token page
# (len % 16 == 0), one-token requests, and contexts long enough to be cut
# across stream-K runs next to ones wholly inside a run
FUSED_LENS = [1, 16, 17, 300, 1024, 33, 4000, 129, 2, 640, 48, 4097]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("ps", [8, 16, 32])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (28, 4, 128)])
def test_decode_append_matches_oracle(dtype, ps, hq, hkv, d):
    """Groups 4 and 7 at head_dim 128, page sizes 8 (outside the fused
    kernel: the two calls), 16 and 32, bf16 and fp16."""
    _fused_step_vs_oracle(70 + ps, FUSED_LENS, hq, hkv, d, ps, dtype)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("hq,hkv,d", [(8, 1, 64), (14, 2, 64), (16, 1, 128), (64, 8, 128)])
def test_decode_append_matches_oracle_other_heads(dtype, hq, hkv, d):
    _fused_step_vs_oracle(90 + hq, FUSED_LENS[:9], hq, hkv, d, 16, dtype)


def test_decode_append_config2_full_size_matches_oracle():
    """BASELINE config 2 at full size: B=32, ctx U[256,4096], random tables
    in a 10240-page pool, bf16; the kernel the bench times."""
    _fused_step_vs_oracle(0, config2_lens(0), 32, 8, 128, 16, "bfloat16", num_pages=10240)


def test_decode_append_outside_the_fused_kernel_takes_the_two_calls():
    """fp32 is outside the fused kernel: run_with_append makes the append and
    decode calls itself, with the same result."""
    (pa, pb), (oa, ob) = _append_then_decode_vs_fused(64, [5, 70, 300], 8, 2, 64, 16, "float32")
    assert torch.equal(pa, pb)
    assert torch.equal(oa, ob)


def test_decode_bad_page_is_flagged():
    from mi_b200 import capi
    c = paged_case(40, [40, 40], 32, 8, 128)
    c["indices"] = c["indices"].copy()
    c["indices"][1] = 10 ** 6
    with pytest.raises(capi.MiError, match="BAD_PAGE"):
        run_decode(c)


# --------------------------------------------------------------------------
# (3) prefill
# --------------------------------------------------------------------------


def run_prefill(c, qo_lens, q, causal=True):
    from mi_b200.prefill import BatchPrefillWithPagedKVCacheWrapper
    w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=DEV))
    qo = np.concatenate([[0], np.cumsum(qo_lens)]).astype(np.int32)
    w.plan(i32(qo), i32(c["indptr"]), i32(c["indices"]), i32(c["last"]), c["hq"], c["hkv"],
           c["d"], c["ps"], causal=causal, q_data_type=tdt(c["dtype"]))
    out, lse = w.run(to_dev(q, c["dtype"]), to_dev(c["pool"], c["dtype"]), return_lse=True)
    torch.cuda.synchronize()
    w.check_status()
    return qo, f32(out), f32(lse)


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("hq,hkv,d", [(32, 8, 128), (14, 2, 64), (28, 4, 128)])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_ragged(dtype, hq, hkv, d, causal):
    kv_lens = [37, 128, 1, 200, 300]
    qo_lens = [37, 128, 1, 50, 0]  # request 3 continues after a 150-token prefix
    c = paged_case(50, kv_lens, hq, hkv, d, dtype=dtype)
    rng = np.random.default_rng(51)
    q = po.round_to(rng.standard_normal((sum(qo_lens), hq, d), dtype=np.float32), dtype)
    qo, out, lse = run_prefill(c, qo_lens, q, causal)
    want, wlse = po.prefill_attention(q, qo, c["pool"], c["indptr"], c["indices"], c["last"],
                                      16, causal=causal)
    np.testing.assert_allclose(out, want, atol=TOL[dtype], rtol=0)
    np.testing.assert_allclose(lse, wlse, atol=max(TOL[dtype], 1e-3), rtol=0)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_prefill_score_spikes_take_the_rescale_path(dtype):
    """Keys that outscore every earlier key of their rows by far more than
    2^8 (in exp2 units), in a first K/V tile's later chunks (past the first
    32 keys, whose max seeds an item's one pass) and in later tiles (past
    the running max): the softmax redoes those tiles in two passes and
    rescales O in TMEM. The result still matches the oracle."""
    hq, hkv, d = 32, 8, 128
    lens = [600, 260, 300]
    c = paged_case(61, lens, hq, hkv, d, dtype=dtype)
    rng = np.random.default_rng(62)
    u = rng.standard_normal(d).astype(np.float32)
    u /= np.linalg.norm(u)
    pool = c["pool"].copy()
    # q . spike = (3 + N(0,1)) * 60: about 23 in exp2 units after the
    # 1/sqrt(d) scale, against about 4 for the largest ordinary key; the
    # third request's one spike opens its second K/V tile
    for r, spikes in enumerate([[100, 300, 301, 520], [90, 200], [130]]):
        for pos in spikes:
            page = c["tables"][r][pos // c["ps"]]
            pool[page, 0, pos % c["ps"]] = po.round_to(np.tile(60.0 * u, (hkv, 1)), dtype)
    c["pool"] = pool
    q = po.round_to(rng.standard_normal((sum(lens), hq, d)).astype(np.float32) + 3.0 * u, dtype)
    qo, out, lse = run_prefill(c, lens, q)
    want, wlse = po.prefill_attention(q, qo, c["pool"], c["indptr"], c["indices"], c["last"],
                                      16, causal=True)
    np.testing.assert_allclose(out, want, atol=TOL[dtype], rtol=0)
    np.testing.assert_allclose(lse, wlse, atol=max(TOL[dtype], 1e-3), rtol=0)


@pytest.mark.parametrize("ws_bytes", [1 << 20, 16])
def test_prefill_repeated_calls_share_workspace(ws_bytes):
    """The persistent tensor-core prefill hands out work items through counters
    in the workspace: three calls in a row on one workspace must each cover
    every item (each call leaves the counters at zero); a workspace too small
    for the counters selects the round-robin assignment instead."""
    from mi_b200.prefill import BatchPrefillWithPagedKVCacheWrapper
    kv_lens = [700, 37, 1300, 256, 90, 513]
    hq, hkv, d, dtype = 32, 8, 128, "bfloat16"
    c = paged_case(53, kv_lens, hq, hkv, d, dtype=dtype)
    rng = np.random.default_rng(54)
    q = po.round_to(rng.standard_normal((sum(kv_lens), hq, d), dtype=np.float32), dtype)
    qo = np.concatenate([[0], np.cumsum(kv_lens)]).astype(np.int32)
    want, _ = po.prefill_attention(q, qo, c["pool"], c["indptr"], c["indices"], c["last"], 16,
                                   causal=True)
    w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(ws_bytes, dtype=torch.uint8, device=DEV))
    w.plan(i32(qo), i32(c["indptr"]), i32(c["indices"]), i32(c["last"]), hq, hkv, d, c["ps"],
           causal=True, q_data_type=tdt(dtype))
    qd, pool = to_dev(q, dtype), to_dev(c["pool"], dtype)
    for _ in range(3):
        out = torch.full_like(qd, float("nan"))
        w.run(qd, pool, out=out)
        torch.cuda.synchronize()
        w.check_status()
        np.testing.assert_allclose(f32(out), want, atol=TOL[dtype], rtol=0)


@pytest.mark.parametrize("case", ["ties", "over_sort_limit"])
def test_prefill_request_order_covers_every_request(case):
    """The tensor-core prefill takes requests longest first (batches up to
    128; larger ones keep their order): with many equal lengths, and with a
    batch past that limit, every output row must still be written once and
    match the oracle (the output starts as NaN)."""
    rng = np.random.default_rng(57)
    if case == "ties":
        kv_lens = [64, 130, 64, 1, 130, 64, 200, 1, 64, 130, 33, 64, 1, 200, 64, 33]
    else:
        kv_lens = rng.integers(1, 48, 140).tolist()
    hq, hkv, d, dtype = 32, 8, 128, "bfloat16"
    c = paged_case(58, kv_lens, hq, hkv, d, dtype=dtype)
    q = po.round_to(rng.standard_normal((sum(kv_lens), hq, d), dtype=np.float32), dtype)
    qo = np.concatenate([[0], np.cumsum(kv_lens)]).astype(np.int32)
    want, _ = po.prefill_attention(q, qo, c["pool"], c["indptr"], c["indices"], c["last"], 16,
                                   causal=True)
    from mi_b200.prefill import BatchPrefillWithPagedKVCacheWrapper
    w = BatchPrefillWithPagedKVCacheWrapper(torch.zeros(1 << 20, dtype=torch.uint8, device=DEV))
    w.plan(i32(qo), i32(c["indptr"]), i32(c["indices"]), i32(c["last"]), hq, hkv, d, c["ps"],
           causal=True, q_data_type=tdt(dtype))
    qd = to_dev(q, dtype)
    out = torch.full_like(qd, float("nan"))
    w.run(qd, to_dev(c["pool"], dtype), out=out)
    torch.cuda.synchronize()
    w.check_status()
    np.testing.assert_allclose(f32(out), want, atol=TOL[dtype], rtol=0)


def test_prefill_qo_indptr_past_q_is_flagged_and_stays_in_bounds():
    """A qo_indptr that claims more query rows than q holds (request 1: 80
    rows, q has 30 of them) is clamped on the device and flagged
    BAD_POSITION: nothing is written past total_q (a guard region behind
    ``out`` stays zero) and request 0, wholly inside q, is still exact."""
    from mi_b200 import capi
    from mi_b200.prefill import BatchPrefillWithPagedKVCacheWrapper
    hq, hkv, d, dtype = 32, 8, 128, "bfloat16"
    c = paged_case(55, [40, 80], hq, hkv, d, dtype=dtype)
    total_q = 70
    rng = np.random.default_rng(56)
    q = po.round_to(rng.standard_normal((total_q, hq, d), dtype=np.float32), dtype)
    w = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=DEV))
    w.plan(i32(np.array([0, 40, 120], np.int32)), i32(c["indptr"]), i32(c["indices"]),
           i32(c["last"]), hq, hkv, d, c["ps"], causal=True, q_data_type=tdt(dtype))
    out_full = torch.zeros(total_q + 64, hq, d, dtype=tdt(dtype), device=DEV)
    w.run(to_dev(q, dtype), to_dev(c["pool"], dtype), out=out_full[:total_q])
    torch.cuda.synchronize()
    with pytest.raises(capi.MiError, match="BAD_POSITION"):
        w.check_status()
    assert not bool(out_full[total_q:].any())
    want, _ = po.prefill_attention(q[:40], np.array([0, 40], np.int32), c["pool"],
                                   c["indptr"][:2], c["indices"], c["last"][:1], 16, causal=True)
    np.testing.assert_allclose(f32(out_full[:40]), want, atol=TOL[dtype], rtol=0)


# --------------------------------------------------------------------------
# the reference's own attention path, replayed through the GPU kernels
# --------------------------------------------------------------------------


@pytest.mark.parametrize("case", ["float32_g7", "float32_g4", "bfloat16_g7", "bfloat16_g4"])
def test_reference_attention_fixture_on_gpu(case):
    from mi_b200.decode import BatchDecodeWithPagedKVCacheWrapper
    from mi_b200.page import append_paged_kv_cache
    from mi_b200.prefill import BatchPrefillWithPagedKVCacheWrapper
    fx_all = np.load(os.path.join(GOLDEN, "attn.npz"))
    fx = {k.split("__", 1)[1]: fx_all[k] for k in fx_all.files if k.startswith(case + "__")}
    dtype = case.split("_")[0]
    hq, hkv, d, ps, b, steps = (int(v) for v in fx["meta"])

    def vals(x):
        return x if dtype == "float32" else po.bf16_bits_to_f32(x)

    pool = torch.zeros(int(fx["num_pages"][0]), 2, ps, hkv, d, dtype=tdt(dtype), device=DEV)
    tol = 2e-4 if dtype == "float32" else 2e-2
    pre = BatchPrefillWithPagedKVCacheWrapper(torch.empty(1 << 20, dtype=torch.uint8, device=DEV))
    dec = BatchDecodeWithPagedKVCacheWrapper(decode_ws())
    for r in range(b):
        q, k, v = (to_dev(vals(fx[f"pre{r}_{n}"]), dtype) for n in "qkv")
        L = q.shape[0]
        ip, ind, last = (i32(fx[f"pre{r}_{n}"]) for n in ("indptr", "indices", "last"))
        append_paged_kv_cache(k, v, i32(np.zeros(L)), i32(np.arange(L)), pool, ind, ip, last)
        pre.plan(i32([0, L]), ip, ind, last, hq, hkv, d, ps, causal=True)
        o = pre.run(q, pool)
        np.testing.assert_allclose(f32(o), fx[f"pre{r}_o"], atol=tol, rtol=0)
    for s in range(steps):
        q, k, v = (to_dev(vals(fx[f"dec{s}_{n}"]), dtype) for n in "qkv")
        ip, ind, last = (i32(fx[f"dec{s}_{n}"]) for n in ("indptr", "indices", "last"))
        append_paged_kv_cache(k, v, i32(np.arange(b)), i32(fx[f"dec{s}_pos"]), pool, ind, ip, last)
        dec.plan(ip, ind, last, hq, hkv, d, ps)
        o = dec.run(q, pool)
        np.testing.assert_allclose(f32(o), fx[f"dec{s}_o"], atol=tol, rtol=0)
    # page contents equal the reference's padded cache, bit for bit
    s = steps - 1
    kc, vc = fx["final_kc"], fx["final_vc"]
    host = f32(pool) if dtype == "float32" else po.bf16_bits_to_f32(bits(pool))
    for r in range(b):
        kk, vv = po.gather_kv(host, fx[f"dec{s}_indptr"], fx[f"dec{s}_indices"],
                              fx[f"dec{s}_last"], ps, r)
        n = int(fx["final_len"][r])
        for got, ref in ((kk, kc), (vv, vc)):
            want = ref[r, :, :n]
            want = np.ascontiguousarray(want).view(np.uint32) if dtype == "float32" else want
            assert np.array_equal(oracle_bits(got.transpose(1, 0, 2), dtype), want)


# --------------------------------------------------------------------------
# (4) page pool
# --------------------------------------------------------------------------


class _Cfg:
    num_hidden_layers = 3
    num_key_value_heads = 2
    head_dim = 64


def test_pool_list_api_matches_reference_fifo():
    from mi_b200.kv_cache import PagedKVCache
    kv = PagedKVCache(_Cfg, max_batch_size=3, max_seq_len=64, page_size=16, device=DEV,
                      dtype=torch.bfloat16)
    ref = po.PagePoolOracle(3, 64, 16)
    assert kv.max_num_pages == ref.max_num_pages == 12 and kv.scratch_page == 11
    for layer in kv.kv_data:
        layer.fill_(1.0)
    seq = [("a", 3), ("a", 4), ("r", [2, 0]), ("a", 2), ("r", [5, 1, 6]), ("a", 4), ("a", 2)]
    for op, arg in seq:
        if op == "a":
            assert kv.allocate_pages(arg) == ref.allocate_pages(arg)
        else:
            kv.release_pages(arg)
            ref.release_pages(arg)
            for layer in kv.kv_data:
                assert float(layer[arg].float().abs().sum()) == 0.0
        assert len(kv.free_pages) == len(ref.free_pages)
    with pytest.raises(RuntimeError):
        kv.allocate_pages(len(ref.free_pages) + 1)
    torch.cuda.synchronize()
    assert int(kv.status.item()) == 0
    # the scratch page is never handed out nor zeroed
    assert float(kv.kv_data[0][kv.scratch_page].float().mean()) == 1.0


def test_slot_api_replays_reference_scheduler_trace():
    """Admission / growth / retire through the device pool reproduce the
    reference scheduler's own page tables (tests/golden/sched_trace.json)."""
    from mi_b200.kv_cache import PagedKVCache
    with open(os.path.join(GOLDEN, "sched_trace.json")) as f:
        fx = json.load(f)["churn"]
    cfg = fx["config"]
    kv = PagedKVCache(_Cfg, max_batch_size=cfg["max_batch"], max_seq_len=cfg["max_seq"],
                      page_size=16, device=DEV, dtype=torch.bfloat16)
    sim = po.simulate_page_tables(cfg["prompts"], cfg["max_new"], cfg["max_batch"],
                                  cfg["max_seq"], 16)
    slot_of: dict[int, int] = {}
    free_slots = list(range(cfg["max_batch"]))
    cap = kv.max_num_pages
    lanes = 4
    for st in sim:
        for rid, pages in st["admitted"]:
            s = free_slots.pop(0)
            slot_of[rid] = s
            n = len(pages)
            kv.slot_alloc(i32([s]), i32([n]), n)
            assert kv.slot_pages(s) == pages
        if st["decode"] is not None:
            ids, pos = st["decode"]["ids"], st["decode"]["positions"]
            n = len(ids)
            ls = [slot_of[r] for r in ids] + [-1] * (lanes - n)
            lp = pos + [0] * (lanes - n)
            ip = torch.zeros(lanes + 1, dtype=torch.int32, device=DEV)
            ind = torch.full((cap,), -7, dtype=torch.int32, device=DEV)
            last = torch.zeros(lanes, dtype=torch.int32, device=DEV)
            ap = torch.zeros(lanes, dtype=torch.int32, device=DEV)
            kv.step_prepare(i32(ls), i32(lp), ip, ind, last, ap)
            ipl = ip.tolist()
            assert ipl[:n + 1] == st["decode"]["indptr"]
            assert ipl[n + 1:] == [ipl[n]] * (lanes - n)          # padding: 0 pages
            assert ind[:ipl[n]].tolist() == st["decode"]["indices"]
            assert last.tolist() == st["decode"]["last_page_len"] + [1] * (lanes - n)
            assert ap.tolist() == pos + [0] * (lanes - n)
        if st["released"]:
            for rid, pages in st["released"]:
                assert kv.slot_pages(slot_of[rid]) == pages
            kv.slot_release(i32([slot_of[r] for r, _ in st["released"]]),
                            sum(len(p) for _, p in st["released"]))
            for r, _ in st["released"]:
                free_slots.append(slot_of.pop(r))
            free_slots.sort()
    torch.cuda.synchronize()
    assert int(kv.status.item()) == 0
    # every request retired: the device free list is full again (the host
    # mirror did not see the pages grown inside step_prepare, so read the device)
    ref = po.PagePoolOracle(cfg["max_batch"], cfg["max_seq"], 16)
    assert int(kv.pool_ctrl[1].item()) == len(ref.free_pages)


def test_step_prepare_out_of_pages_sets_status_and_keeps_tables():
    from mi_b200.kv_cache import PagedKVCache
    kv = PagedKVCache(_Cfg, max_batch_size=2, max_seq_len=32, page_size=16, device=DEV,
                      dtype=torch.bfloat16)  # 4 pages, 3 usable
    kv.slot_alloc(i32([0, 1]), i32([2, 1]), 3)
    ip = torch.zeros(3, dtype=torch.int32, device=DEV)
    ind = torch.zeros(4, dtype=torch.int32, device=DEV)
    last = torch.zeros(2, dtype=torch.int32, device=DEV)
    ap = torch.zeros(2, dtype=torch.int32, device=DEV)
    kv.step_prepare(i32([0, 1]), i32([20, 16]), ip, ind, last, ap)  # slot 1 needs a 2nd page
    torch.cuda.synchronize()
    assert int(kv.status.item()) & 1
    assert kv.slot_num_pages.tolist() == [2, 1]
    with pytest.raises(RuntimeError):
        kv.check_status()
