# SPDX-License-Identifier: Apache-2.0
"""Model check of the tensor-core decode kernel's synchronisation
(``decode_tc_kernel`` in kotflash_b200/csrc/decode.cu).

One split CTA walks ``n_tiles`` 64-key tiles.  Roles, in the kernel's issue
order over its mbarriers:

* producer: K and V of tile t into ring stage ``t % kTcStages`` (``full``)
  once the stage's previous tile was released (``empty``);
* MMA issuer: S(0) = Q K(0)^T, then per tile S(t + 1) into the other S buffer
  before O += P(t) V(t) (after ``p_full``), releasing the stage (``empty``)
  and signalling ``pv_done``; ``o_done`` at the end.  P(t) lies over S(t),
  and S(t + 1) overwrites P(t - 1), which PV(t - 1), issued earlier by the
  same thread, has read;
* softmax warps: S(t) -> P(t) in place (``s_full`` / ``p_full``); when the
  running maximum jumps they rescale O, after waiting for PV(t - 1)
  (``pv_done`` completion t - 1: S(t) was committed after PV(t - 2), so the
  barrier is never two phases short of it); the epilogue after ``o_done``.

The checks are those of ``_sync_model`` (no deadlock, no buffer hazard, no
ambiguous parity wait), with the rescale taken on a random subset of tiles.
"""
import random

import pytest

from _sync_model import Bar, Violation, simulate

STAGES = 4


def producer(n):
    for t in range(n):
        s = t % STAGES
        if t >= STAGES:
            yield ("wait", f"empty{s}", t // STAGES - 1)
        yield ("write", f"KV{s}", t, 2)  # read by QK^T(t) and PV(t)
        yield ("arrive", f"full{s}", 1)


def issuer(n):
    def qk(t):
        yield ("read", f"KV{t % STAGES}", t)
        yield ("write", f"S{t & 1}", ("S", t), 1)
        yield ("arrive", f"s_full{t & 1}", 1)

    yield ("wait", "q_ready", 0)
    yield ("wait", "full0", 0)
    yield from qk(0)
    for t in range(n):
        s = t % STAGES
        if t + 1 < n:
            yield ("wait", f"full{(t + 1) % STAGES}", (t + 1) // STAGES)
            yield from qk(t + 1)
        yield ("wait", f"p_full{t & 1}", t >> 1)
        yield ("read", f"S{t & 1}", ("P", t))
        yield ("read", f"KV{s}", t)
        yield ("write", "O", ("O", t), 1) if t == 0 else ("read_write", "O", ("O", t - 1), ("O", t))
        yield ("arrive", f"empty{s}", 1)
        yield ("arrive", "pv_done", 1)
    yield ("arrive", "o_done", 1)


def softmax(n, rescale):
    yield ("arrive", "q_ready", 1)
    for t in range(n):
        yield ("wait", f"s_full{t & 1}", t >> 1)
        yield ("read_write", f"S{t & 1}", ("S", t), ("P", t))
        if t > 0 and rescale[t]:
            yield ("wait", "pv_done", t - 1)
            yield ("read_write", "O", ("O", t - 1), ("O", t - 1))
        yield ("arrive", f"p_full{t & 1}", 1)
    yield ("wait", "o_done", 0)
    yield ("read", "O", ("O", n - 1))


def run(n, seed):
    rng = random.Random(seed)
    rescale = [rng.random() < 0.3 for _ in range(n)]
    bars = {"q_ready": Bar(1), "pv_done": Bar(1), "o_done": Bar(1)}
    for s in range(STAGES):
        bars.update({f"full{s}": Bar(1), f"empty{s}": Bar(1)})
    for b in range(2):
        bars.update({f"s_full{b}": Bar(1), f"p_full{b}": Bar(1)})
    roles = {"producer": producer(n), "issuer": issuer(n), "softmax": softmax(n, rescale)}
    simulate(roles, bars, seed)


def test_tc_decode_protocol_is_deadlock_free_and_parity_safe():
    for n in range(1, 14):
        for seed in range(60):
            run(n, seed=1000 * n + seed)


def test_model_catches_a_missing_stage_release_wait():
    # a producer that reuses a ring stage without waiting for ``empty``
    # overwrites K/V that PV has not read yet
    def eager(n):
        for op in producer(n):
            if op[0] != "wait":
                yield op

    with pytest.raises(Violation):
        for seed in range(200):
            rng = random.Random(seed)
            bars = {"q_ready": Bar(1), "pv_done": Bar(1), "o_done": Bar(1)}
            for s in range(STAGES):
                bars.update({f"full{s}": Bar(1), f"empty{s}": Bar(1)})
            for b in range(2):
                bars.update({f"s_full{b}": Bar(1), f"p_full{b}": Bar(1)})
            simulate({"producer": eager(9), "issuer": issuer(9),
                      "softmax": softmax(9, [rng.random() < 0.3 for _ in range(9)])}, bars, seed)
