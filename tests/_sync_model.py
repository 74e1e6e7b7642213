# SPDX-License-Identifier: Apache-2.0
"""A small model checker for the mbarrier protocols of the tensor-core kernels.

Roles are Python generators that yield the operations one warp role issues,
in program order:

* ``("wait", bar, m)``: wait for completion number m (0-based) of ``bar``;
* ``("arrive", bar, n)``: n arrivals (a commit, a TMA completion or a
  warpgroup's arrivals, taken at the moment of issue);
* ``("write", buf, tag, readers)``, ``("read", buf, tag)``,
  ``("read_write", buf, old, new)``: buffer contents and the readers they owe.

``simulate`` runs the roles under a random interleaving and raises
``Violation`` on a deadlock, a buffer hazard, arrivals of two phases mixed, or
a parity wait that would be ambiguous on the hardware: a waiter for
completion m must find the barrier at m or m + 1 completions, and the barrier
must not reach m + 2 while it waits.
"""
import random


class Violation(AssertionError):
    pass


class Bar:
    def __init__(self, count):
        self.count, self.arrived, self.done = count, 0, 0

    def arrive(self, n):
        self.arrived += n
        if self.arrived > self.count:
            raise Violation("arrivals of two phases mixed")
        if self.arrived == self.count:
            self.arrived, self.done = 0, self.done + 1


class Buf:
    """Content tag plus the readers the content still owes."""

    def __init__(self, name):
        self.name, self.tag, self.pending = name, None, 0

    def write(self, tag, readers):
        if self.pending:
            raise Violation(f"{self.name}: {tag} overwrites {self.tag} before its readers")
        self.tag, self.pending = tag, readers

    def read(self, tag):
        if self.tag != tag or self.pending == 0:
            raise Violation(f"{self.name}: read of {tag} finds {self.tag} (pending {self.pending})")
        self.pending -= 1



def simulate(roles, bars, seed):
    rng = random.Random(seed)
    bufs = {}

    def buf(name):
        return bufs.setdefault(name, Buf(name))

    pending, waiting = {}, {}

    def advance(name):
        try:
            pending[name] = next(roles[name])
        except StopIteration:
            pending[name] = None

    for name in roles:
        advance(name)
    while True:
        live = [n for n, op in pending.items() if op is not None]
        if not live:
            return
        ready = []
        for n in live:
            op = pending[n]
            if op[0] != "wait":
                ready.append(n)
                continue
            b, m = bars[op[1]], op[2]
            if n not in waiting:
                if not (m <= b.done <= m + 1):
                    raise Violation(f"{n} waits for completion {m} of {op[1]} at {b.done}")
                waiting[n] = (op[1], m)
            if b.done > m:
                ready.append(n)
        if not ready:
            raise Violation("deadlock: " + ", ".join(f"{n}: {pending[n]}" for n in live))
        n = rng.choice(ready)
        op = pending[n]
        kind = op[0]
        if kind == "wait":
            waiting.pop(n, None)
        elif kind == "arrive":
            b = bars[op[1]]
            b.arrive(op[2])
            for w, (bn, m) in waiting.items():
                if bn == op[1] and b.done >= m + 2:
                    raise Violation(f"{w} still waits for completion {m} of {bn} at {b.done}")
        elif kind == "write":
            buf(op[1]).write(op[2], op[3])
        elif kind == "read":
            buf(op[1]).read(op[2])
        elif kind == "read_write":
            buf(op[1]).read(op[2])
            buf(op[1]).write(op[3], 1)
        advance(n)
