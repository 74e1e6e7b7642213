# SPDX-License-Identifier: Apache-2.0
"""The LM training A/B (the reference's benchmarks/benchmark_tinystories_training.py
shape, on the seeded synthetic token stream): from identical weights and
paired batches, the kernels and PyTorch SDPA on expanded K/V start from the
same evaluation loss (the reference's 0.02 criterion), both learn, and both
stay finite and close."""
import pytest

import bench

pytestmark = pytest.mark.gpu


def test_lm_training_ab_short():
    res = bench.bench_story_lm_ab(seq=512, batch=2, steps=6, warmup=1)
    ours, sdpa = res["kotflash_b200"], res["sdpa_expanded"]
    print("[parity] lm a/b", {k: res[k] for k in ("initial_eval_loss_abs_delta", "final_eval_loss_abs_delta")},
          ours, sdpa)
    assert ours["finite"] and sdpa["finite"]
    assert res["initial_eval_loss_abs_delta"] <= 0.02
    assert res["final_eval_loss_abs_delta"] <= 0.05
    for r in (ours, sdpa):
        assert r["final_eval_loss"] < r["initial_eval_loss"]
