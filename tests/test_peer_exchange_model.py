# SPDX-License-Identifier: Apache-2.0
"""Model check of the NVLink peer exchange of decode partials (the mailbox
protocol of kotflash_b200/csrc/decode.cu: ``merge_put_kernel`` /
``peer_put_kernel`` and ``peer_merge_kernel``).

Each of W ranks runs a sequence of decode calls in stream order.  Call e of
rank r:

* put: reads the epoch from its own mailbox (completed calls + 1), stores its
  partial rows into slot r of half ``e & 1`` of every rank's mailbox, then
  adds its row count to each receiver's counter of that half (a release per
  receiver once all its stores are issued);
* merge: reads the epoch, waits until its own counter of half ``e & 1``
  equals ``W * rows * ((e + 1) >> 1)`` (an equality test: an overshoot by a
  later call's rows would make it spin until the bounded wait gives up),
  merges the W slots and advances the epoch.

Rows are one unit here.  The model runs the ranks under random interleavings
for 2-8 ranks and several calls, and checks: no deadlock, no overshoot while
a merge waits, the epoch each kernel reads is its own call number, and no
slot is overwritten before the receiver's merge of the previous use of that
half has read it.  A variant whose mailboxes have a single half (no
alternation by epoch parity) must fail.
"""
import random

import pytest

from _sync_model import Buf, Violation


def rank_program(r, world, calls, halves):
    for e in range(1, calls + 1):
        # put
        epoch = yield ("read_epoch", r)
        if epoch != e:
            raise Violation(f"rank {r} put of call {e} reads epoch {epoch}")
        h = e % halves if halves == 2 else 0
        for p in range(world):
            yield ("store", p, h, r, e)
        for p in range(world):
            yield ("add", p, h)
        # merge
        epoch = yield ("read_epoch", r)
        if epoch != e:
            raise Violation(f"rank {r} merge of call {e} reads epoch {epoch}")
        target = world * ((e + 1) >> 1) if halves == 2 else world * e
        yield ("wait_eq", r, h, target)
        for q in range(world):
            yield ("load", r, h, q, e)
        yield ("advance_epoch", r, e)


def run(world, calls, seed, halves=2):
    rng = random.Random(seed)
    ctrl = [0] * world
    counter = {(p, h): 0 for p in range(world) for h in range(2)}
    slots = {}
    progs = {r: rank_program(r, world, calls, halves) for r in range(world)}
    pending, waiting = {}, {}

    def slot(p, h, q):
        return slots.setdefault((p, h, q), Buf(f"mailbox {p} half {h} slot {q}"))

    def step(r, value=None):
        try:
            pending[r] = progs[r].send(value)
        except StopIteration:
            pending[r] = None

    for r in progs:
        step(r)
    while True:
        live = [r for r, op in pending.items() if op is not None]
        if not live:
            return
        ready = []
        for r in live:
            op = pending[r]
            if op[0] == "wait_eq":
                _, p, h, target = op
                c = counter[(p, h)]
                if c > target:
                    raise Violation(f"rank {r}: counter {c} passed its target {target}")
                if c == target:
                    ready.append(r)
            else:
                ready.append(r)
        if not ready:
            raise Violation("deadlock: " + ", ".join(f"{r}: {pending[r]}" for r in live))
        r = rng.choice(ready)
        op = pending[r]
        kind = op[0]
        if kind == "read_epoch":
            step(r, ctrl[op[1]] + 1)
            continue
        if kind == "store":
            _, p, h, q, e = op
            slot(p, h, q).write(e, 1)
        elif kind == "add":
            _, p, h = op
            counter[(p, h)] += 1
            for w, wop in pending.items():
                if wop is not None and wop[0] == "wait_eq" and (wop[1], wop[2]) == (p, h) and counter[(p, h)] > wop[3]:
                    raise Violation(f"rank {w}: counter passed its target while it waited")
        elif kind == "load":
            _, p, h, q, e = op
            slot(p, h, q).read(e)
        elif kind == "advance_epoch":
            ctrl[op[1]] = op[2]
        step(r)


def test_peer_exchange_is_safe_for_2_to_8_ranks():
    for world in (2, 3, 4, 8):
        for seed in range(80):
            run(world, calls=6, seed=1000 * world + seed)


def test_single_half_mailbox_fails():
    with pytest.raises(Violation):
        for seed in range(200):
            run(4, calls=5, seed=seed, halves=1)
