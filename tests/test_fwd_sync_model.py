# SPDX-License-Identifier: Apache-2.0
"""Model check of the forward kernel's synchronisation (kotflash_b200/csrc/fwd_sm100.cu).

The roles of a forward CTA (TMA producer, one MMA issuer per Q tile, one
softmax warpgroup per Q tile) are restated as small sequential programs over
the kernel's mbarriers, in the order the kernel issues them, and run under
many random interleavings for random sequences of work items (one or two
tiles, one to six K/V blocks).  Each run checks:

* no deadlock: every role finishes;
* every parity wait is unambiguous: a role waiting for completion number m of
  a barrier finds the barrier at m or m + 1 completed phases when it starts
  waiting, and the barrier never reaches m + 2 while the role still waits
  (an mbarrier parity wait cannot tell those cases apart);
* no buffer hazard: S, P, O of each tile and every K/V ring slot are read
  only after the intended write and overwritten only after their readers.

MMAs and TMA copies complete in issue order here (the hardware guarantees
this per issuing thread for tcgen05.commit); a commit or a TMA completion is
an arrival at the moment of issue, and softmax warpgroups (128 arrivals in
the kernel) arrive as one.  A variant with one score buffer shared by the two
tiles, and one load barrier for both, fails the parity check: that is the
form a measured experiment ran into.
"""
import random

import pytest

from _sync_model import Bar, Violation, simulate

STAGES = 3


def producer(items):
    g = 0
    for it, (nt, nblk) in enumerate(items):
        if it > 0:
            yield ("wait", "q_empty", it - 1)
        for t in range(nt):
            yield ("write", f"Q{t}", it, 1 + (nblk - 1))  # read by every QK^T of the tile
        yield ("arrive", "q_full", 1)
        for j in range(nblk):
            gj, s = g + j, (g + j) % STAGES
            if gj >= STAGES:
                yield ("wait", f"k_empty{s}", gj // STAGES - 1)
            yield ("write", f"K{s}", gj, nt)
            yield ("arrive", f"k_full{s}", 1)
            if gj >= STAGES:
                yield ("wait", f"v_empty{s}", gj // STAGES - 1)
            yield ("write", f"V{s}", gj, nt)
            yield ("arrive", f"v_full{s}", 1)
        g += nblk


def content_order(items):
    """(tile, that tile's load index) of every S content, in issue order."""
    order, loads = [], [0, 0]
    for nt, nblk in items:
        for j in range(nblk):
            for t in range(nt):
                order.append((t, loads[t]))
                loads[t] += 1
    return order


def issuer(t, items, shared_s):
    g = jt = cs = 0
    contents = content_order(items)
    for it, (nt, nblk) in enumerate(items):
        if t < nt:
            rel = 1 if nt == 2 else 2
            sbuf = "S" if shared_s else f"S{t}"

            def s_ready(j):
                if not shared_s:
                    return [] if j == 0 else [("wait", f"s_free{t}", jt + j - 1)]
                c = cs + (2 * j + t if nt == 2 else j)
                if c == 0:
                    return []
                if shared_s == "per_tile":
                    # wait for the load of content c - 1 on the barrier of the tile that loaded it
                    owner, index = contents[c - 1]
                    return [("wait", f"s_free{owner}", index)]
                return [("wait", "s_free", c - 1)]

            def qk(j, gj):
                s = gj % STAGES
                ops = [("read", f"Q{t}", it), ("read", f"K{s}", gj), ("write", sbuf, (it, t, j), 1),
                       ("arrive", f"s_full{t}", 1)]
                if j == nblk - 1:
                    ops.append(("arrive", "q_empty", rel))
                ops.append(("arrive", f"k_empty{s}", rel))
                return ops

            yield ("wait", "q_full", it)
            yield ("wait", f"k_full{g % STAGES}", g // STAGES)
            yield from s_ready(0)
            yield from qk(0, g)
            for j in range(nblk):
                gj, s = g + j, (g + j) % STAGES
                if j + 1 < nblk:
                    yield from s_ready(j + 1)
                    yield ("wait", f"k_full{(gj + 1) % STAGES}", (gj + 1) // STAGES)
                    yield from qk(j + 1, gj + 1)
                yield ("wait", f"v_full{s}", gj // STAGES)
                yield ("wait", f"p_full{t}", jt + j)
                yield ("read", f"V{s}", gj)
                yield ("read", f"P{t}", (it, j))
                # PV of the first block overwrites O (no accumulation)
                yield ("write", f"O{t}", (it, j), 1) if j == 0 else ("read_write", f"O{t}", (it, j - 1), (it, j))
                yield ("arrive", f"pv_done{t}", 1)
                yield ("arrive", f"v_empty{s}", rel)
            yield ("arrive", f"o_final{t}", 1)
            jt += nblk
        g += nblk
        cs += nt * nblk


def softmax(t, items, shared_s):
    jt = vt = jturn = 0
    sbuf = "S" if shared_s else f"S{t}"
    for it, (nt, nblk) in enumerate(items):
        if t >= nt:
            continue
        for j in range(nblk):
            yield ("wait", f"s_full{t}", jt + j)
            yield ("read", sbuf, (it, t, j))
            yield ("arrive", "s_free" if shared_s is True else f"s_free{t}", 1)
            if nt == 2 and (t == 1 or j > 0):
                yield ("wait", f"turn{t}", jturn + j - (0 if t == 1 else 1))
            if nt == 2:
                yield ("arrive", f"turn{1 - t}", 1)
            if j > 0:
                yield ("wait", f"pv_done{t}", jt + j - 1)
            yield ("write", f"P{t}", (it, j), 1)
            yield ("arrive", f"p_full{t}", 1)
        yield ("wait", f"o_final{t}", vt)
        yield ("read", f"O{t}", (it, nblk - 1))
        jt += nblk
        vt += 1
        if nt == 2:
            jturn += nblk


def run(items, seed, shared_s=False):
    bars = {"q_full": Bar(1), "q_empty": Bar(2), "s_free": Bar(1)}
    for s in range(STAGES):
        bars.update({f"k_full{s}": Bar(1), f"k_empty{s}": Bar(2), f"v_full{s}": Bar(1), f"v_empty{s}": Bar(2)})
    for t in range(2):
        bars.update({f"s_full{t}": Bar(1), f"s_free{t}": Bar(1), f"p_full{t}": Bar(1), f"pv_done{t}": Bar(1),
                     f"o_final{t}": Bar(1), f"turn{t}": Bar(1)})
    roles = {"producer": producer(items)}
    for t in range(2):
        roles[f"issuer{t}"] = issuer(t, items, shared_s)
        roles[f"softmax{t}"] = softmax(t, items, shared_s)
    simulate(roles, bars, seed)


def random_items(rng, n, tiles=(2,)):
    return [(rng.choice(tiles), rng.randint(1, 6)) for _ in range(n)]


def test_two_tile_item_sequences_are_deadlock_free_and_parity_safe():
    rng = random.Random(7)
    for case in range(60):
        items = random_items(rng, rng.randint(1, 5))
        for seed in range(15):
            run(items, seed=1000 * case + seed)


def test_one_item_per_cta_and_single_tile_items_last():
    rng = random.Random(8)
    for case in range(40):
        items = random_items(rng, 1, tiles=(1, 2))
        if case % 2:
            items = random_items(rng, rng.randint(1, 3)) + [(1, rng.randint(1, 6)) for _ in range(rng.randint(1, 2))]
        for seed in range(15):
            run(items, seed=1000 * case + seed)


def test_fixed_cases():
    for items in ([(2, 1)], [(1, 1)], [(2, 1), (2, 1), (1, 1)], [(2, 6), (2, 2), (1, 3)], [(1, 5)]):
        for seed in range(40):
            run(items, seed=seed)


def test_single_tile_item_before_a_two_tile_item_breaks_parity():
    """The tile-1 issuer skips a single-tile item without waiting, so at the
    next two-tile item it can wait for Q-load completion it + 1 while the
    barrier has not completed load it: the parity wait returns at once.  The
    launcher therefore gives every CTA one item when a launch has single-tile
    items and more items than SMs (``launch_fwd``)."""
    failures = 0
    for items in ([(1, 3), (2, 3)], [(1, 1), (2, 2), (2, 1)], [(1, 4), (1, 2), (2, 5)]):
        for seed in range(20):
            try:
                run(items, seed=seed)
            except Violation:
                failures += 1
    assert failures > 0


def test_shared_score_buffer_breaks_the_parity_invariant():
    rng = random.Random(11)
    failures = 0
    for case in range(20):
        items = [(2, rng.randint(2, 6)) for _ in range(rng.randint(1, 3))]
        for seed in range(10):
            try:
                run(items, seed=100 * case + seed, shared_s=True)
            except Violation:
                failures += 1
    assert failures > 0


def test_shared_score_buffer_with_a_load_barrier_per_tile_passes():
    """The repaired form of the shared-buffer variant: each tile's softmax
    arrives on its own load barrier, and the issuer of content c waits for
    the load of content c - 1 on the barrier of the tile that loaded it (a
    waiter is then never two phases ahead of that barrier)."""
    rng = random.Random(12)
    for case in range(40):
        items = random_items(rng, rng.randint(1, 4))
        for seed in range(15):
            run(items, seed=1000 * case + seed, shared_s="per_tile")


def test_model_catches_a_missing_wait():
    # dropping the softmax's wait for the previous PV lets P be overwritten early
    global softmax
    original = softmax

    def no_pv_wait(t, items, shared_s):
        for op in original(t, items, shared_s):
            if op[0] == "wait" and op[1].startswith("pv_done"):
                continue
            yield op

    softmax = no_pv_wait
    try:
        with pytest.raises(Violation):
            for seed in range(200):
                run([(2, 4), (2, 3)], seed=seed)
    finally:
        softmax = original
