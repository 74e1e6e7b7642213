# SPDX-License-Identifier: Apache-2.0
"""The forward kernel's fp32-pipe exponential (exp2_poly2: Cody-Waite split
into rint(x) and f in [-0.5, 0.5], degree-3 relative-minimax polynomial for
2^f, exponent-field add) against exp2 in float64, over the argument range the
softmax feeds it, through the kf_selftest_exp2_poly entry point."""
import pytest
import torch

from kotflash_b200 import _ext

pytestmark = pytest.mark.gpu

MAX_REL_ERR = 1.5e-4  # the fit's stated bound is 1.3e-4 in fp32 arithmetic


def _eval(x):
    lib = _ext.load()
    y = torch.empty_like(x)
    rc = lib.kf_selftest_exp2_poly(x.data_ptr(), y.data_ptr(), x.numel(), _ext.stream_of(x))
    _ext.check(rc, "kf_selftest_exp2_poly")
    torch.cuda.synchronize()
    return y


def test_exp2_poly_relative_error_over_minus125_to_127():
    g = torch.Generator(device="cuda").manual_seed(0)
    grid = torch.linspace(-125.0, 127.0, 4_000_000, device="cuda")
    rnd = torch.rand(2_000_000, device="cuda", generator=g) * 252.0 - 125.0
    # the split's edges: f = +-0.5 exactly and just inside, where rint() switches
    j = torch.arange(-124, 127, device="cuda", dtype=torch.float32)
    edges = torch.cat([j + 0.5, j - 0.5, j + 0.49999997, j - 0.49999997, j])
    x = torch.cat([grid, rnd, edges]).contiguous()
    if x.numel() % 2:
        x = torch.cat([x, x[:1]])
    y = _eval(x)
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref).abs() / ref).max().item()
    print(f"[parity] exp2_poly2 max relative error over [-125, 127]: {rel:.3e}")
    assert torch.isfinite(y).all()
    assert rel <= MAX_REL_ERR


def test_exp2_poly_clamps_arguments_below_minus125():
    x = torch.tensor([-125.0, -125.5, -126.0, -149.0, -1000.0, float("-inf")], device="cuda")
    y = _eval(x)
    floor = 2.0 ** -125
    rel = ((y.double() - floor).abs() / floor).max().item()
    assert (y > 0).all() and torch.isfinite(y).all()
    assert rel <= MAX_REL_ERR
