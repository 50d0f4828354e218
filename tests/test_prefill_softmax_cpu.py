"""The prefill kernel's per-tile softmax, restated on the CPU.

prefill_tc2_kernel (minimal-inference_b200/csrc/prefill_tc2.cu) takes a
query row's keys 128 per K/V tile, in four 32-key chunks, in one pass
against a base max mb (the running max; in an item's first tile the max of
its first chunk). Chunk c's P = 2^(s * scale_log2 - mb) is stored in the
16-bit input type over S columns already read, unless a key of the chunk
lies more than kRescaleLog2 = 8 above mb: from the first such chunk on the
tile takes two passes against m_new = max(mb, the later chunks' max), and
the P already stored (at most 2^8, so it fits fp16) is rebased by
2^(mb - m_new). The running (m, l, O) follow with O rescaled by the same
factor. This restatement follows those steps for single rows (fp32
arithmetic, 16-bit P) and checks them against exact softmax attention on
rows whose scores jump far above every earlier key, where the redo runs.
"""
import numpy as np
import pytest

from oracle import paged_oracle as po

RESCALE_LOG2 = 8.0
CHUNK, TILE = 32, 128


def _row(s, v, scale_log2, dtype, plant=None):
    """Attention of one query row over its visible keys: scores s [L] (raw
    q.k), values v [L, d]. Returns the output and how many tiles took the
    two-pass redo. plant="redo_over_p": the redo starts at chunk 0 and reads
    the first 64 keys' scores from columns the one pass has overwritten with
    P (a mistake the checks must catch)."""
    m, l, o = -np.inf, 0.0, np.zeros(v.shape[1], np.float64)
    redos = 0
    for j, t0 in enumerate(range(0, len(s), TILE)):
        st, vt = s[t0:t0 + TILE], v[t0:t0 + TILE]
        chunks = [st[c:c + CHUNK] for c in range(0, len(st), CHUNK)]
        mb = m if j > 0 else chunks[0].max() * scale_log2
        stored, total, first_bad = [], 0.0, None
        for c, sc in enumerate(chunks):
            if sc.max() * scale_log2 > mb + RESCALE_LOG2:
                first_bad = c
                break
            p = np.exp2(sc * scale_log2 - mb)
            assert p.max() <= 2.0 ** RESCALE_LOG2        # the rebase below cannot overflow
            stored.append(po.round_to(p.astype(np.float32), dtype))
            total += p.sum()
        corr, m_new = 1.0, mb
        if first_bad is not None and plant == "redo_over_p":
            # the one pass wrote every chunk's P as bf16 pairs over the first
            # 64 columns; the redo reads each pair back as an fp32 score,
            # whose value is about the pair's second P
            redos += 1
            p_all = po.round_to(np.exp2(st * scale_log2 - mb).astype(np.float32), "bfloat16")
            seen = np.array([p_all[2 * i + 1] if 2 * i + 1 < len(st) else 0.0
                             for i in range(min(len(st), 2 * CHUNK))])
            st = np.concatenate([seen, st[len(seen):]])
            mt = st.max() * scale_log2
            m_new = max(m, mt) if (mt > m + RESCALE_LOG2 or m == -np.inf) else m
            corr = 1.0 if m_new == m else np.exp2(m - m_new)
            p = np.exp2(st * scale_log2 - m_new)
            stored, total = [po.round_to(p.astype(np.float32), dtype)], p.sum()
        elif first_bad is not None:
            redos += 1
            mt = max(sc.max() for sc in chunks[first_bad:]) * scale_log2
            m_new = max(mb, mt) if mt > mb + RESCALE_LOG2 else mb
            corr = np.exp2(mb - m_new)
            total *= corr
            stored = [po.round_to((p * corr).astype(np.float32), dtype) for p in stored]
            for sc in chunks[first_bad:]:
                p = np.exp2(sc * scale_log2 - m_new)
                stored.append(po.round_to(p.astype(np.float32), dtype))
                total += p.sum()
        pt = np.concatenate(stored).astype(np.float64)
        l = l * corr + total if j > 0 else total
        o = (o * corr if j > 0 else 0.0) + pt @ vt
        m = m_new
    return o / l, redos


def _exact(s, v, scale_log2):
    w = np.exp2((s - s.max()) * scale_log2)
    return (w / w.sum()) @ v


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("seed", range(6))
def test_rows_with_score_spikes_match_exact_softmax(dtype, seed):
    rng = np.random.default_rng(seed)
    d = 32
    scale_log2 = np.log2(np.e) / np.sqrt(d)
    redos = 0
    for _ in range(40):
        L = int(rng.integers(1, 700))
        s = rng.standard_normal(L) * np.sqrt(d)
        # jumps far above every earlier key, anywhere in a tile: in its
        # first chunk (past an earlier tile's max), its later chunks, and
        # past the first chunk that seeds an item's first tile
        for pos in rng.choice(L, size=min(L, int(rng.integers(0, 4))), replace=False):
            s[pos] += rng.uniform(10.0, 200.0) / scale_log2
        v = po.round_to(rng.standard_normal((L, d)).astype(np.float32), dtype).astype(np.float64)
        out, r = _row(s, v, scale_log2, dtype)
        redos += r
        np.testing.assert_allclose(out, _exact(s, v, scale_log2), atol=2e-2, rtol=0)
    assert redos > 0


def test_a_redo_over_overwritten_scores_is_caught():
    rng = np.random.default_rng(11)
    d = 32
    scale_log2 = np.log2(np.e) / np.sqrt(d)
    caught = 0
    for _ in range(20):
        L = 300
        s = rng.standard_normal(L) * np.sqrt(d)
        s[200:202] += 40.0 / scale_log2           # past the first tile: a redo in tile 1
        v = rng.standard_normal((L, d))
        out, redos = _row(s, v, scale_log2, "bfloat16", plant="redo_over_p")
        assert redos == 1
        caught += not np.allclose(out, _exact(s, v, scale_log2), atol=2e-2, rtol=0)
    assert caught > 0


def test_rows_without_spikes_need_no_redo():
    rng = np.random.default_rng(7)
    d = 128
    scale_log2 = np.log2(np.e) / np.sqrt(d)
    for _ in range(20):
        L = int(rng.integers(1, 1100))
        s = rng.standard_normal(L) * np.sqrt(d)
        v = rng.standard_normal((L, d))
        out, redos = _row(s, v, scale_log2, "bfloat16")
        assert redos == 0
        np.testing.assert_allclose(out, _exact(s, v, scale_log2), atol=2e-2, rtol=0)
