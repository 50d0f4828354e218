"""The stream-K decode's cost-balanced split, restated on the CPU.

``decode_sk.cu`` cuts the requests' concatenated pages into one run per CTA
in virtual units of a quarter page, charging every non-empty request's start
``c4`` units (``vsplit_run`` / ``vsplit_page``); the split-K merge kernel
derives each request's covering runs from the same numbers. These tests
restate both formulas and check, over random batches with empty requests,
that the runs partition the pages, that the merge's run range of every
request is exactly the set of CTAs that own its pages, and that the partial
slots ``cta + b`` of the non-direct segments never collide.
"""
import math

import numpy as np
import pytest


def vsplit_total(ip, c4):
    nz = sum(1 for b in range(len(ip) - 1) if ip[b + 1] > ip[b])
    return 4 * (ip[-1] - ip[0]) + c4 * nz


def vsplit_page(ip, c4, x):
    """First page (from indptr[0]) whose virtual start is >= x."""
    base0, nzpre, best = ip[0], 0, None
    for b in range(len(ip) - 1):
        np_ = ip[b + 1] - ip[b]
        vs = 4 * (ip[b] - base0) + c4 * nzpre
        if np_ > 0 and vs <= x:
            best = (b, vs)
        if np_ > 0:
            nzpre += 1
    if best is None:
        return 0
    b, vs = best
    local = x - vs - c4
    j = 0 if local <= 0 else min(ip[b + 1] - ip[b], (local + 3) // 4)
    return ip[b] - base0 + j


def vsplit_run(ip, c4, grid, cta):
    vt = vsplit_total(ip, c4)
    rv = max(4, -(-vt // grid))
    x0 = min(vt, cta * rv)
    x1 = min(vt, x0 + rv)
    return vsplit_page(ip, c4, x0), vsplit_page(ip, c4, x1)


def merge_runs(ip, c4, grid, b):
    """(first run, number of runs) of request b, as the merge kernel derives them."""
    base0 = ip[0]
    nz_before = sum(1 for r in range(b) if ip[r + 1] > ip[r])
    vt = vsplit_total(ip, c4)
    np_ = ip[b + 1] - ip[b]
    if vt <= 0 or np_ <= 0:
        return 0, 0
    rv = max(4, -(-vt // grid))
    v0 = 4 * (ip[b] - base0) + c4 * nz_before + c4
    first = v0 // rv
    return first, (v0 + 4 * (np_ - 1)) // rv - first + 1


def _batches():
    rng = np.random.default_rng(0)
    yield [0] * 5                                      # nothing to do
    yield [1]
    yield [0, 3, 0, 0, 7, 0]
    for _ in range(40):
        b = int(rng.integers(1, 70))
        pages = rng.integers(0, 300, b)
        pages[rng.random(b) < 0.2] = 0                  # empty requests (padding lanes)
        yield pages.tolist()


@pytest.mark.parametrize("c4", [0, 1, 9, 75, 600])
@pytest.mark.parametrize("grid", [1, 7, 148])
def test_runs_partition_pages_and_match_the_merge(c4, grid):
    for pages in _batches():
        ip = [5] + list(5 + np.cumsum(pages))           # indptr may start past 0
        total = ip[-1] - ip[0]
        runs = [vsplit_run(ip, c4, grid, i) for i in range(grid)]
        # contiguous, in order, covering [0, total) exactly once
        assert runs[0][0] == 0 and runs[-1][1] == total
        for (lo, hi), (lo2, _) in zip(runs, runs[1:]):
            assert lo <= hi == lo2
        owner = np.empty(total, np.int64)
        for i, (lo, hi) in enumerate(runs):
            owner[lo:hi] = i
        slots = set()
        for b in range(len(pages)):
            s, e = ip[b] - ip[0], ip[b + 1] - ip[0]
            first, nch = merge_runs(ip, c4, grid, b)
            if e == s:
                assert nch == 0
                continue
            ctas = sorted(set(owner[s:e].tolist()))
            assert ctas == list(range(first, first + nch)), (pages, b)
            if nch > 1:                                  # partials: one slot per covering run
                for cta in ctas:
                    assert cta + b not in slots
                    slots.add(cta + b)
                    assert cta + b < grid + len(pages)


def test_request_starts_take_pages_from_their_runs():
    """With c4 > 0 a run holding more request starts gets fewer pages; with
    c4 = 0 the runs differ by at most one page (the last run holds the
    remainder)."""
    pages = [137] * 8 + [2] * 40 + [137] * 8
    ip = [0] + list(np.cumsum(pages))
    grid = 20
    flat = [hi - lo for lo, hi in (vsplit_run(ip, 0, grid, i) for i in range(grid))]
    assert max(flat[:-1]) - min(flat[:-1]) <= 1 and flat[-1] <= max(flat)
    c4 = 9
    runs = [vsplit_run(ip, c4, grid, i) for i in range(grid)]
    starts = [sum(1 for b in range(len(pages)) if lo <= ip[b] < hi) for lo, hi in runs]
    sizes = [hi - lo for lo, hi in runs]
    busy = max(range(grid), key=lambda i: starts[i])
    quiet = min(range(grid), key=lambda i: starts[i])
    assert starts[busy] > starts[quiet] and sizes[busy] < sizes[quiet]
    # cost (pages + c4/4 per start) is balanced to within a page and a start
    cost = [sz + c4 / 4 * st for sz, st in zip(sizes, starts)][:-1]
    assert max(cost) - min(cost) <= 1 + math.ceil(c4 / 4)
