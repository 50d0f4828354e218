"""The prefill kernel's work queue, restated on the CPU.

prefill_tc2_kernel (minimal-inference_b200/csrc/prefill_tc2.cu) hands out
work items (request, KV head, query chunk of 2 Tq tokens) from a counter.
Its prologue ranks the requests by query length (longest first, ties by
index; batches up to 128 keep that order, larger ones their own) and takes
the prefix of item counts over that order; item k maps, by a binary search
over the prefix, to a request, and inside the request to its chunks last
(heaviest) first with all KV heads of a chunk together. This restatement
follows the kernel's arithmetic and checks that the queue is a bijection
onto every (request, head, chunk), and that each request's chunk index
never increases along the queue.
"""
import math
import random

import pytest

SORT_BATCH = 128


def queue(qo_lens, hkv, tq2):
    batch = len(qo_lens)
    order = [0] * batch
    for i, li in enumerate(qo_lens):
        rank = i
        if batch <= SORT_BATCH:
            rank = sum(1 for j, lj in enumerate(qo_lens) if lj > li or (lj == li and j < i))
        order[rank] = i
    pre = [0]
    for pos in range(batch):
        pre.append(pre[-1] + math.ceil(qo_lens[order[pos]] / tq2))
    items = []
    for k in range(pre[batch] * hkv):
        lo, hi = 0, batch - 1           # last position with pre[pos] * hkv <= k
        while lo < hi:
            mid = (lo + hi + 1) >> 1
            if pre[mid] * hkv <= k:
                lo = mid
            else:
                hi = mid - 1
        ntq = pre[lo + 1] - pre[lo]
        rem = k - pre[lo] * hkv
        items.append((order[lo], rem % hkv, ntq - 1 - rem // hkv))
    return items, order


def _check(qo_lens, hkv, tq2):
    items, order = queue(qo_lens, hkv, tq2)
    want = {(b, h, c) for b, L in enumerate(qo_lens) for h in range(hkv)
            for c in range(math.ceil(L / tq2))}
    assert len(items) == len(want) and set(items) == want
    last = {}
    for b, _, c in items:
        assert c <= last.get(b, c)
        last[b] = c
    if len(qo_lens) <= SORT_BATCH:
        assert [qo_lens[b] for b in order] == sorted(qo_lens, reverse=True)
    return items


@pytest.mark.parametrize("seed", range(40))
def test_queue_covers_every_item_once(seed):
    rnd = random.Random(seed)
    batch = rnd.choice([1, 2, 7, 32, 100, 128, 129, 200])
    lens = [rnd.choice([0, 1, 31, 32, 33, 64, 65, 200, rnd.randrange(1, 1100)])
            for _ in range(batch)]
    _check(lens, rnd.choice([1, 2, 4, 8]), rnd.choice([32, 64, 128, 256]))


def test_config3_prompts_start_with_the_longest_requests_heaviest_chunks():
    rnd = random.Random(3)
    lens = [rnd.randrange(128, 1025) for _ in range(32)]
    items = _check(lens, 8, 64)
    longest = max(range(32), key=lambda b: (lens[b], -b))
    assert items[:8] == [(longest, h, math.ceil(lens[longest] / 64) - 1) for h in range(8)]


def test_a_batch_above_the_sort_limit_keeps_its_order():
    lens = [3] * 64 + [500] * 65
    items, order = queue(lens, 1, 64)
    assert order == list(range(129))
    _check(lens, 1, 64)
