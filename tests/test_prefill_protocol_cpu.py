"""The tensor-core prefill kernel's mbarrier protocol, checked on the CPU.

A model of prefill_tc_kernel (minimal-inference_b200/csrc/prefill_tc.cu) in
the discrete-event form of tests/barrier_model.py: the producer warp, the
MMA thread, the 8 softmax warps and the 4 epilogue warps yield the kernel's
waits, arrivals, TMA copies and tensor-core products / commits in the
kernel's order, with the kernel's counters (work items, Q buffers, K/V
stages, S tiles, O buffers). Random work-item sequences, items without keys
included, must finish without deadlock or phase aliasing. The model follows
the kernel: a change to one of the kernel's waits or commits goes here too.
"""
import random

from tests.barrier_model import Bar, run

NQ, NK, NV = 2, 2, 2


def _model(items, seed):
    rnd = random.Random(seed)
    bars = {}

    def bar(name, count):
        bars[name] = Bar(name, count)

    for i in range(2):
        bar(f"q_full{i}", 1)
        bar(f"q_empty{i}", 1)
        bar(f"k_full{i}", 1)
        bar(f"k_empty{i}", 1)
        bar(f"v_full{i}", 1)
        bar(f"v_empty{i}", 1)
        bar(f"o_full{i}", 1)
        bar(f"o_free{i}", 4)    # the epilogue warps
        bar(f"l_ready{i}", 8)   # the softmax warps
        bar(f"it_full{i}", 1)
        bar(f"it_empty{i}", 9)  # the MMA thread and the softmax warps
    bar("s_full", 1)
    bar("s_free", 8)
    bar("p_full", 8)
    bar("o_done", 1)
    bar("xch", 8)
    records = list(items) + [None]   # tiles per item; None: the end record
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
                return
            if n == 0:
                continue
            qb = qc % NQ
            if qc >= NQ:
                yield ("wait", f"q_empty{qb}", qc // NQ - 1)
            yield ("tma", f"q_full{qb}")
            qc += 1

            def issue(g, which):
                nst = NV if which else NK
                kind = "v" if which else "k"
                if g >= nst:
                    yield ("wait", f"{kind}_empty{g % nst}", g // nst - 1)
                yield ("tma", f"{kind}_full{g % nst}")
            for j in range(n):                  # K0, K1, V0, K2, V1, ..., V(n-1)
                yield from issue(gt, 0)
                if j > 0:
                    yield from issue(gt - 1, 1)
                gt += 1
            yield from issue(gt - 1, 1)

    def mma():
        state = {"it": 0}

        def next_item():
            while True:
                it = state["it"]
                yield ("wait", f"it_full{it & 1}", it >> 1)
                n = ring[it & 1]
                yield ("arrive", f"it_empty{it & 1}")
                state["it"] = it + 1
                if n is None:
                    return None
                if n > 0:
                    return n

        def qk(t, qb):
            yield ("mma", "S")
            yield ("commit", "s_full")
            yield ("commit", f"k_empty{t % NK}")

        gt = qc = oc = 0
        cur = yield from next_item()
        if cur is not None:
            yield ("wait", "q_full0", 0)
            yield ("wait", "k_full0", 0)
            yield from qk(0, 0)
            if cur == 1:
                yield ("commit", "q_empty0")
        last_gt = -1
        while cur is not None:
            ob = oc & 1
            nxt = None
            for j in range(cur):
                ahead, cross = j + 1 < cur, False
                if not ahead:
                    nxt = yield from next_item()
                    ahead = cross = nxt is not None
                if ahead:
                    qn = qc + 1 if cross else qc
                    yield ("wait", "s_free", gt)
                    if cross:
                        yield ("wait", f"q_full{qn % NQ}", qn // NQ)
                    yield ("wait", f"k_full{(gt + 1) % NK}", (gt + 1) // NK)
                    yield from qk(gt + 1, qn % NQ)
                    if (nxt == 1) if cross else (j + 2 == cur):
                        yield ("commit", f"q_empty{qn % NQ}")
                yield ("wait", "p_full", gt)
                yield ("wait", f"v_full{gt % NV}", gt // NV)
                if j == 0 and oc >= 2:
                    yield ("wait", f"o_free{ob}", (oc >> 1) - 1)
                yield ("mma", "PV")
                yield ("commit", f"v_empty{gt % NV}")
                yield ("commit", "o_done")
                if j + 1 == cur:
                    yield ("commit", f"o_full{ob}")
                last_gt = gt
                gt += 1
            qc += 1
            oc += 1
            cur = nxt
        if last_gt >= 0:
            yield ("wait", "o_done", last_gt)

    def softmax():
        gt = oc = 0

        def hand_off(ob):
            if oc >= 2:
                yield ("wait", f"o_free{ob}", (oc >> 1) - 1)
            yield ("arrive", f"l_ready{ob}")

        it = 0
        while True:
            yield ("wait", f"it_full{it & 1}", it >> 1)
            n = ring[it & 1]
            yield ("arrive", f"it_empty{it & 1}")
            it += 1
            if n is None:
                yield from hand_off(oc & 1)
                return
            if n == 0:
                continue
            for _ in range(n):
                yield ("wait", "s_full", gt)
                yield ("arrive", "s_free")
                yield ("arrive", "xch")
                yield ("wait", "xch", gt)
                if gt > 0:
                    yield ("wait", "o_done", gt - 1)
                yield ("arrive", "p_full")
                gt += 1
            yield from hand_off(oc & 1)
            oc += 1

    n_keys = sum(1 for n in items if n)

    def epilogue():
        for oc in range(n_keys + 1):
            ob = oc & 1
            yield ("wait", f"l_ready{ob}", oc >> 1)
            if oc == n_keys:          # the end record
                return
            yield ("wait", f"o_full{ob}", oc >> 1)
            yield ("arrive", f"o_free{ob}")

    roles = {"producer": producer(), "mma": mma()}
    roles.update({f"softmax{w}": softmax() for w in range(8)})
    roles.update({f"epilogue{w}": epilogue() for w in range(4)})
    run(bars, roles, seed)


def test_prefill_protocol_has_no_deadlock_or_phase_aliasing():
    rnd = random.Random(0)
    for trial in range(400):
        items = [rnd.choice([0, 1, 1, 2, 3, 4, 5, 8]) for _ in range(rnd.randint(0, 8))]
        _model(items, trial)


def test_model_catches_a_wait_on_the_wrong_completion():
    """The checker itself: a protocol whose consumer waits one completion too
    far ahead must fail (here: a single-slot ring waited with the slot's
    use count instead of the previous use's)."""
    bars = {"full": Bar("full", 1), "empty": Bar("empty", 1)}

    def prod():
        for k in range(4):
            if k >= 1:
                yield ("wait", "empty", k)      # should be k - 1
            yield ("arrive", "full")

    def cons():
        for k in range(4):
            yield ("wait", "full", k)
            yield ("arrive", "empty")

    try:
        run(bars, {"p": prod(), "c": cons()}, 0)
    except AssertionError:
        return
    raise AssertionError("the planted wrong wait went unnoticed")
