"""A small discrete-event model of a kernel's mbarrier protocol (test helper).

Roles (warps, or one thread) are generators that yield the kernel's
synchronisation steps in program order:

* ``("wait", bar, n)``    wait for completion ``n`` of ``bar`` (the kernel
                          waits on parity ``n & 1``);
* ``("arrive", bar)``     one arrival;
* ``("tma", bar)``        an asynchronous copy that completes on ``bar``
                          at any later time, in any order;
* ``("mma", tag)``        a tensor-core product, and
* ``("commit", bar)``     an arrival on ``bar`` once every product the same
                          role issued before it has completed (each role's
                          products complete in its issue order; two roles'
                          products in any interleaving), and
* ``("tmem", region)``    a read or write of a TMEM region by the role's own
                          threads.

``run`` interleaves the roles and the asynchronous completions at random.
It raises ``AssertionError`` on a deadlock (nothing can move), on a wait
that passes on another completion than the one it names (phase aliasing:
a parity wait cannot tell completion ``n`` from ``n - 1`` or ``n + 2``) and
on arrivals beyond a barrier's count. ``hazards`` maps a product tag to the
tags of products it overwrites the operands of (products on different
accumulators need not run in issue order): issuing it while one of those is
still in flight raises too, and ``tmem_hazards`` maps a TMEM region to the
tags of the products that write it: a ``tmem`` access to it while one of
those is in flight (any role's) raises.
"""
from __future__ import annotations

import random


class Bar:
    def __init__(self, name: str, count: int):
        self.name, self.count, self.arrived, self.done = name, count, 0, 0

    def arrive(self) -> None:
        self.arrived += 1
        assert self.arrived <= self.count, f"{self.name}: arrivals beyond its count"
        if self.arrived == self.count:
            self.arrived = 0
            self.done += 1


def run(bars: dict, roles: dict, seed: int, max_steps: int = 10 ** 6,
        hazards: dict | None = None, tmem_hazards: dict | None = None) -> None:
    rnd = random.Random(seed)
    pending = []     # barriers with an asynchronous copy in flight
    products = {}    # per issuing role, in order: ("mma", tag) / ("commit", bar)
    action = {name: None for name in roles}
    alive = set(roles)
    for _ in range(max_steps):
        queues = [q for q in products.values() if q]
        if not (alive or pending or queues):
            return
        progress = False
        order = sorted(alive)
        rnd.shuffle(order)
        for name in order:
            act = action[name]
            while True:
                if act is None:
                    try:
                        act = next(roles[name])
                    except StopIteration:
                        alive.discard(name)
                        progress = True
                        break
                kind = act[0]
                if kind == "wait":
                    bar, n = bars[act[1]], act[2]
                    if (bar.done & 1) != (n & 1):
                        assert bar.done == n + 1, (
                            f"{name}: wait on {act[1]} for completion {n} passed at {bar.done}")
                        act, progress = None, True
                        continue
                    assert bar.done <= n, (
                        f"{name}: wait on {act[1]} for completion {n} aliased at {bar.done}")
                    break
                if kind == "tmem":
                    writers = (tmem_hazards or {}).get(act[1], ())
                    busy = [a[1] for q in products.values() for a in q
                            if a[0] == "mma" and a[1] in writers]
                    assert not busy, f"{name}: {act[1]} accessed while {busy[0]} is in flight"
                elif kind == "arrive":
                    bars[act[1]].arrive()
                elif kind == "tma":
                    pending.append(act[1])
                else:
                    queue = products.setdefault(name, [])
                    if kind == "mma" and hazards:
                        busy = [a[1] for a in queue if a[0] == "mma" and a[1] in hazards.get(act[1], ())]
                        assert not busy, f"{name}: {act[1]} issued while {busy[0]} is in flight"
                    queue.append(act)
                act, progress = None, True
                if rnd.random() < 0.3:
                    break
            action[name] = act
        if pending and rnd.random() < 0.5:
            bars[pending.pop(rnd.randrange(len(pending)))].arrive()
            progress = True
        queues = [q for q in products.values() if q]
        if queues and rnd.random() < 0.5:
            act = rnd.choice(queues).pop(0)
            if act[0] == "commit":
                bars[act[1]].arrive()
            progress = True
        if not progress and not pending and not any(products.values()):
            raise AssertionError(f"deadlock: {({n: action[n] for n in alive})}")
    raise AssertionError("no end within the step limit")
