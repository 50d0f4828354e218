"""The two-query-tile prefill kernel's mbarrier protocol, checked on the CPU.

A model of prefill_tc2_kernel (minimal-inference_b200/csrc/prefill_tc2.cu) in
the discrete-event form of tests/barrier_model.py: the producer warp, the
MMA thread, the softmax warps of tile A and of tile B (each group as one
role) and the epilogue warps yield the kernel's waits, arrivals, TMA copies
and tensor-core products / commits in the kernel's order, with the kernel's
counters (work items, Q loads, K/V stages, tiles, O buffers, hand-off
slots). Random work-item sequences, items without keys included, must finish
without deadlock or phase aliasing, and a planted wrong wait must be caught.
The model follows the kernel: a change to one of its waits or commits goes
here too.
"""
import random

import pytest

from tests.barrier_model import Bar, run

NK, NV = 2, 2


def _model(items, plant=None):
    bars = {}

    def bar(name, count):
        bars[name] = Bar(name, count)

    for i in range(2):
        bar(f"it_full{i}", 1)
        bar(f"it_empty{i}", 3)      # the MMA thread and the two softmax groups
        bar(f"q_full{i}", 1)
        bar(f"q_empty{i}", 1)
        bar(f"k_full{i}", 1)
        bar(f"k_empty{i}", 1)
        bar(f"v_full{i}", 1)
        bar(f"v_empty{i}", 1)
        bar(f"s_full{i}", 1)
        bar(f"p_full{i}", 1)        # the tile's softmax group
        bar(f"pv_done{i}", 1)
        bar(f"o_full{i}", 1)
        bar(f"o_free{i}", 1)        # the epilogue
        bar(f"l_ready{2 * i}", 1)
        bar(f"l_ready{2 * i + 1}", 1)
        bar(f"h_free{2 * i}", 1)
        bar(f"h_free{2 * i + 1}", 1)
    bar("drain", 1)
    records = list(items) + [None]  # tiles per item; None: the end record
    ring = [None, None]

    def producer():
        gt = qc = 0
        for it, n in enumerate(records):
            slot = it & 1
            if it >= 2:
                yield ("wait", f"it_empty{slot}", (it >> 1) - 1)
            ring[slot] = n
            yield ("arrive", f"it_full{slot}")
            if n is None:
                break
            if n == 0:
                continue
            for x in range(2):
                if qc >= 1:
                    yield ("wait", f"q_empty{x}", qc - 1)
                yield ("tma", f"q_full{x}")
            qc += 1

            def issue(g, which):
                nst = NV if which else NK
                kind = "v" if which else "k"
                if g >= nst:
                    yield ("wait", f"{kind}_empty{g % nst}", g // nst - 1)
                yield ("tma", f"{kind}_full{g % nst}")
            for j in range(n):                      # K0, V0, K1, V1, ..., K(n-1), V(n-1)
                if j > 0:
                    yield from issue(gt - 1, 1)
                yield from issue(gt, 0)
                gt += 1
            yield from issue(gt - 1, 1)
        # drain: the last copies have landed
        if qc >= 1:
            for x in range(2):
                yield ("wait", f"q_full{x}", qc - 1)
        for t in range(max(0, gt - NK), gt):
            yield ("wait", f"k_full{t % NK}", t // NK)
        for t in range(max(0, gt - NV), gt):
            yield ("wait", f"v_full{t % NV}", t // NV)

    def mma():
        gt = oc = 0
        issued = False
        for it in range(len(records)):
            slot = it & 1
            yield ("wait", f"it_full{slot}", it >> 1)
            n = ring[slot]
            yield ("arrive", f"it_empty{slot}")
            if n is None:
                break
            if n == 0:
                continue
            for x in range(2):
                yield ("wait", f"q_full{x}", oc)
                if x == 0:
                    yield ("wait", f"k_full{gt % NK}", gt // NK)
                if gt >= 1 and plant != "no_pv_wait_at_item_start":
                    yield ("wait", f"pv_done{x}", gt - 1)
                yield ("mma", f"S{x}")
                yield ("commit", f"s_full{x}")
                issued = True
                if n == 1:
                    yield ("commit", f"q_empty{x}")
            yield ("commit", f"k_empty{gt % NK}")
            for j in range(n):
                t = gt + j
                for x in range(2):
                    yield ("wait", f"p_full{x}", t)
                    if x == 0:
                        yield ("wait", f"v_full{t % NV}", t // NV)
                    if j == 0 and oc >= 1:
                        yield ("wait", f"o_free{x}", oc - 1)
                    yield ("mma", f"PV{x}")
                    yield ("commit", f"pv_done{x}")
                    if x == 1:
                        yield ("commit", f"v_empty{t % NV}")
                    if j + 1 == n:
                        yield ("commit", f"o_full{x}")
                    if j + 1 < n:
                        if x == 0:
                            yield ("wait", f"k_full{(t + 1) % NK}", (t + 1) // NK)
                        yield ("wait", f"pv_done{x}", t)
                        yield ("mma", f"S{x}")
                        yield ("commit", f"s_full{x}")
                        if x == 1:
                            yield ("commit", f"k_empty{(t + 1) % NK}")
                        if j + 2 == n:
                            yield ("commit", f"q_empty{x}")
            gt += n
            oc += 1
        if issued:
            yield ("commit", "drain")
            yield ("wait", "drain", 0)

    def softmax(x):
        gt = oc = 0
        for it in range(len(records)):
            slot = it & 1
            yield ("wait", f"it_full{slot}", it >> 1)
            n = ring[slot]
            yield ("arrive", f"it_empty{slot}")
            if n is None:
                if x == 0:                           # the end record for the epilogue
                    hs = oc & 1
                    if oc >= 2:
                        yield ("wait", f"h_free{hs * 2 + x}", (oc >> 1) - 1)
                    yield ("arrive", f"l_ready{hs * 2 + x}")
                break
            if n == 0:
                continue
            for j in range(n):
                yield ("wait", f"s_full{x}", gt)
                if j > 0:
                    yield ("tmem", f"O{x}")          # O rescaled when the row max moved
                yield ("arrive", f"p_full{x}")
                gt += 1
            hs = oc & 1
            if oc >= 2:
                wait_on = (f"o_free{x}", oc - 2) if plant == "slot_wait_on_o_free" else \
                    (f"h_free{hs * 2 + x}", (oc >> 1) - 1)
                yield ("wait", *wait_on)
            yield ("arrive", f"l_ready{hs * 2 + x}")
            oc += 1

    n_keyed = sum(1 for n in items if n)

    def epilogue():
        for oc in range(n_keyed + 1):
            slot = oc & 1
            for x in range(2):
                yield ("wait", f"l_ready{slot * 2 + x}", oc >> 1)
                if x == 0 and oc == n_keyed:
                    return                           # the end record
                if plant != "epilogue_reads_o_early":
                    yield ("wait", f"o_full{x}", oc)
                yield ("tmem", f"O{x}")                  # O read for the output
                yield ("arrive", f"o_free{x}")
                yield ("arrive", f"h_free{slot * 2 + x}")

    roles = {"producer": producer(), "mma": mma(), "softmax_a": softmax(0),
             "softmax_b": softmax(1), "epilogue": epilogue()}
    return bars, roles


def _items(rnd, count):
    return [rnd.choice([0, 1, 1, 2, 3, 4, 7]) for _ in range(count)]


# S_x is written over P_x, which the tile's P V reads from TMEM; a P V and an
# S accumulate into different TMEM columns, so nothing orders them but the
# pv_done wait
HAZARDS = {"S0": {"PV0"}, "S1": {"PV1"}}
# O_x is written by the tile's P V products and read or rescaled by the
# softmax and epilogue warps
TMEM_HAZARDS = {"O0": {"PV0"}, "O1": {"PV1"}}


@pytest.mark.parametrize("seed", range(60))
def test_random_item_sequences_finish(seed):
    rnd = random.Random(seed)
    items = _items(rnd, rnd.randrange(0, 9))
    bars, roles = _model(items)
    run(bars, roles, seed, hazards=HAZARDS, tmem_hazards=TMEM_HAZARDS)


def test_an_epilogue_read_before_o_full_is_caught():
    """The epilogue reading O_x without waiting for the item's last P_x V:
    on some schedule that product is still writing O_x."""
    caught = 0
    for seed in range(200):
        bars, roles = _model([2, 1, 3], plant="epilogue_reads_o_early")
        try:
            run(bars, roles, seed, hazards=HAZARDS, tmem_hazards=TMEM_HAZARDS)
        except AssertionError as e:
            caught += "accessed while" in str(e)
    assert caught > 0


def test_a_first_s_without_the_pv_wait_is_caught():
    """An item's first S_x issued without waiting for the previous item's
    last P_x V: on some schedule that P V is still in flight when S_x
    overwrites P_x."""
    caught = 0
    for seed in range(200):
        bars, roles = _model([2, 1, 3, 1], plant="no_pv_wait_at_item_start")
        try:
            run(bars, roles, seed, hazards=HAZARDS, tmem_hazards=TMEM_HAZARDS)
        except AssertionError as e:
            assert "in flight" in str(e)
            caught += 1
    assert caught > 0


def test_a_slot_wait_on_a_per_item_barrier_is_caught():
    """The hand-off slot waited for on a barrier that completes every item
    (o_free) instead of every other item: when the epilogue runs two items
    ahead the parity wait names the wrong completion. The checker must see it
    on some schedule."""
    caught = 0
    for seed in range(200):
        bars, roles = _model([3, 1, 2, 1, 2], plant="slot_wait_on_o_free")
        try:
            run(bars, roles, seed)
        except AssertionError:
            caught += 1
    assert caught > 0
