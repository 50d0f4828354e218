"""The stream-K decode kernel's mbarrier protocol, checked on the CPU.

A model of decode_sk_kernel (minimal-inference_b200/csrc/decode_sk.cu) in the
discrete-event form of tests/barrier_model.py: the producer warp fills a ring
of S stages (full / empty barriers, the copies completing in any order,
stages whose tiles are all bad pages completing on the producer's arrival
alone) and ends with a sentinel stage; each of the 8 consumer warps takes
every stage and releases it, and at a segment's end the warps of one KV
head combine through the shared scratch behind hsync / hdone. Random stage
sequences must finish without deadlock or phase aliasing for every head
count and ring depth the kernel uses. The model follows the kernel: a change
to one of the kernel's waits or arrivals goes here too.
"""
import random

import pytest

from tests.barrier_model import Bar, run

NC = 8  # consumer warps


def _model(stages, S, hkv, seed):
    """stages: list of (segment_ends, has_copy) per stage."""
    subs = NC // hkv
    bars = {}
    for s in range(S):
        bars[f"full{s}"] = Bar(f"full{s}", 1)
        bars[f"empty{s}"] = Bar(f"empty{s}", NC)
    for h in range(hkv):
        bars[f"hsync{h}"] = Bar(f"hsync{h}", subs)
        bars[f"hdone{h}"] = Bar(f"hdone{h}", subs)
    recs = [None] * S

    def producer():
        k = 0
        for seg_end, has_copy in stages:
            s = k % S
            if k >= S:
                yield ("wait", f"empty{s}", k // S - 1)
            recs[s] = seg_end
            # arrive.expect_tx + the copies: the phase completes when the
            # bytes land (or at once when every tile of the stage is bad)
            yield ("tma", f"full{s}") if has_copy else ("arrive", f"full{s}")
            k += 1
        s = k % S                                # the end-of-run sentinel
        if k >= S:
            yield ("wait", f"empty{s}", k // S - 1)
        recs[s] = "end"
        yield ("arrive", f"full{s}")
        # no copy in flight at exit: the issues after the sentinel's slot
        for kk in range(max(0, k - S + 1), k):
            yield ("wait", f"full{kk % S}", kk // S)

    def consumer(w):
        h = w // subs
        segments = 0
        k = 0
        while True:
            s = k % S
            yield ("wait", f"full{s}", k // S)
            rec = recs[s]
            if rec == "end":
                return
            yield ("arrive", f"empty{s}")
            k += 1
            if not rec:
                continue
            # end of a run segment: combine the warps of this head
            if subs > 1 and segments > 0:
                yield ("wait", f"hdone{h}", segments - 1)
            segments += 1
            if subs > 1:
                yield ("arrive", f"hsync{h}")
                yield ("wait", f"hsync{h}", segments - 1)
                yield ("arrive", f"hdone{h}")

    roles = {"producer": producer()}
    roles.update({f"consumer{w}": consumer(w) for w in range(NC)})
    run(bars, roles, seed)


@pytest.mark.parametrize("hkv", [1, 2, 4, 8])
@pytest.mark.parametrize("S", [2, 3])
def test_decode_protocol_has_no_deadlock_or_phase_aliasing(hkv, S):
    rnd = random.Random(hkv * 10 + S)
    for trial in range(150):
        n = rnd.randint(0, 12)
        stages = [(rnd.random() < 0.35, rnd.random() < 0.9) for _ in range(n)]
        if stages:
            stages[-1] = (True, stages[-1][1])   # a run ends with a segment end
        _model(stages, S, hkv, trial)
