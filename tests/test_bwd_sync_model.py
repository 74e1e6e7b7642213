# SPDX-License-Identifier: Apache-2.0
"""Model check of the backward kernel's synchronisation (kotflash_b200/csrc/bwd_sm100.cu).

One key-block CTA of ``bwd_kernel`` walks ``nsteps`` 64-row query steps.  Its
roles, restated in the kernel's issue order over its mbarriers:

* producer: K/V once (``kv_full``), then per step Q, dO and the row
  statistics into ring stage ``s % kStages`` (``qdo_full``), after the stage's
  previous use was released (``qdo_empty``);
* score issuer: S^T(s) into TMEM buffer ``s & 1`` once P^T(s - 2) has been
  read (``p_free``), dP^T(s) into the other buffer pair once dQ^T(s - 2) has
  been drained (``ds_free``);
* gradient issuer: dV += P^T dO after ``p_ready``; dK += dS^T Q after
  ``ds_ready``, which also releases the Q/dO stage; dQ^T(s) over this step's
  dS^T in TMEM (same thread, after dK read it) for the drain (``dq_full``);
  ``mma_done`` at the end;
* P/dS warpgroups: statistics from the stage, S^T -> P^T in place
  (``p_ready``), dP^T -> dS^T in place plus dS^T into shared memory
  (``ds_ready``); the dK/dV epilogue after ``mma_done``;
* dQ drain: reads dQ^T (``dq_full``) and frees the buffer (``ds_free``).

The checks are the ones of ``_sync_model``: no deadlock, no buffer hazard,
no ambiguous parity wait, for 1 to 12 steps under random interleavings.
"""
import pytest

from _sync_model import Bar, Violation, simulate

K_STAGES = 3


def producer(nsteps):
    yield ("arrive", "kv_full", 1)
    for s in range(nsteps):
        st = s % K_STAGES
        if s >= K_STAGES:
            yield ("wait", f"qdo_empty{st}", s // K_STAGES - 1)
        # readers: S^T, dP^T, dV, dK and the P/dS warpgroups' statistics
        yield ("write", f"QDO{st}", s, 5)
        yield ("arrive", f"qdo_full{st}", 1)


def score_issuer(nsteps, skip_ds_free=False):
    yield ("wait", "kv_full", 0)
    for s in range(nsteps):
        st, buf = s % K_STAGES, s & 1
        yield ("wait", f"qdo_full{st}", s // K_STAGES)
        if s >= 2:
            yield ("wait", f"p_free{buf}", (s - 2) >> 1)
        yield ("read", f"QDO{st}", s)
        yield ("write", f"S{buf}", ("S", s), 1)
        yield ("arrive", f"s_ready{buf}", 1)
        if s >= 2 and not skip_ds_free:
            yield ("wait", f"ds_free{buf}", (s - 2) >> 1)
        yield ("read", f"QDO{st}", s)
        yield ("write", f"DP{buf}", ("dP", s), 1)
        yield ("arrive", f"dp_ready{buf}", 1)


def gradient_issuer(nsteps):
    yield ("wait", "kv_full", 0)
    for s in range(nsteps):
        st, buf = s % K_STAGES, s & 1
        yield ("wait", f"p_ready{buf}", s >> 1)
        yield ("read", f"S{buf}", ("P", s))
        yield ("read", f"QDO{st}", s)
        yield ("arrive", f"p_free{buf}", 1)
        yield ("wait", f"ds_ready{buf}", s >> 1)
        yield ("read", f"DP{buf}", ("dS", s))
        yield ("read", f"QDO{st}", s)
        yield ("arrive", f"qdo_empty{st}", 1)
        yield ("read", f"sdS{buf}", ("dS", s))
        yield ("write", f"DP{buf}", ("dQ", s), 1)
        yield ("arrive", f"dq_full{buf}", 1)
    yield ("arrive", "mma_done", 1)


def p_ds_warps(nsteps):
    for s in range(nsteps):
        st, buf = s % K_STAGES, s & 1
        yield ("wait", f"qdo_full{st}", s // K_STAGES)
        yield ("read", f"QDO{st}", s)
        yield ("wait", f"s_ready{buf}", s >> 1)
        yield ("read_write", f"S{buf}", ("S", s), ("P", s))
        yield ("arrive", f"p_ready{buf}", 1)
        yield ("wait", f"dp_ready{buf}", s >> 1)
        yield ("read_write", f"DP{buf}", ("dP", s), ("dS", s))
        yield ("write", f"sdS{buf}", ("dS", s), 1)
        yield ("arrive", f"ds_ready{buf}", 1)
    if nsteps > 0:
        yield ("wait", "mma_done", 0)


def dq_drain(nsteps):
    for s in range(nsteps):
        buf = s & 1
        yield ("wait", f"dq_full{buf}", s >> 1)
        yield ("read", f"DP{buf}", ("dQ", s))
        yield ("arrive", f"ds_free{buf}", 1)


def run(nsteps, seed, skip_ds_free=False):
    bars = {"kv_full": Bar(1), "mma_done": Bar(1)}
    for st in range(K_STAGES):
        bars.update({f"qdo_full{st}": Bar(1), f"qdo_empty{st}": Bar(1)})
    for b in range(2):
        bars.update({f"s_ready{b}": Bar(1), f"p_ready{b}": Bar(1), f"p_free{b}": Bar(1), f"dp_ready{b}": Bar(1),
                     f"ds_ready{b}": Bar(1), f"dq_full{b}": Bar(1), f"ds_free{b}": Bar(1)})
    roles = {"producer": producer(nsteps), "score_issuer": score_issuer(nsteps, skip_ds_free),
             "gradient_issuer": gradient_issuer(nsteps), "p_ds": p_ds_warps(nsteps), "dq_drain": dq_drain(nsteps)}
    simulate(roles, bars, seed)


def test_backward_protocol_is_deadlock_free_and_parity_safe():
    for nsteps in range(1, 13):
        for seed in range(60):
            run(nsteps, seed=100 * nsteps + seed)


def test_model_catches_a_missing_ds_free_wait():
    # without waiting for the drain, dP^T(s + 2) can overwrite dQ^T(s) before it is read
    with pytest.raises(Violation):
        for seed in range(300):
            run(6, seed=seed, skip_ds_free=True)
