# SPDX-License-Identifier: Apache-2.0
"""The oracle is pinned to the reference's own outputs (tests/golden, CPU)."""
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_oracle as oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.name for p in GOLDEN.glob("attn_*.npz"))


def _load(name):
    z = np.load(GOLDEN / name)
    return {k: torch.from_numpy(z[k]) for k in z.files}


@pytest.mark.parametrize("name", CASES)
def test_oracle_forward_matches_reference_sdpa(name):
    z = _load(name)
    b, hq, hkv, sq, sk, d, causal, seed = z["meta"].tolist()
    o, lse = oracle.forward(z["q"], z["k"], z["v"], causal=bool(causal))
    torch.testing.assert_close(o, z["o"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(lse, z["lse"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", CASES)
def test_oracle_backward_matches_reference_autograd_and_blockwise(name):
    z = _load(name)
    causal = bool(z["meta"][6].item())
    dq, dk, dv = oracle.backward(z["q"], z["k"], z["v"], z["o"], z["lse"], z["do"], causal=causal)
    for got, ref, bw, tag in ((dq, z["dq"], z["bw_dq"], "dq"), (dk, z["dk"], z["bw_dk"], "dk"),
                              (dv, z["dv"], z["bw_dv"], "dv")):
        torch.testing.assert_close(got, ref, rtol=2e-4, atol=2e-5, msg=f"{name} {tag} vs autograd")
        torch.testing.assert_close(got, bw, rtol=2e-4, atol=2e-5, msg=f"{name} {tag} vs blockwise")


def test_oracle_on_cpu_plumbing_config():
    """B2 Hq8 Hkv2 S512 D64 fp32 causal fwd O+LSE and bwd."""
    z = np.load(GOLDEN / "cfg1_plumbing.npz")
    torch.manual_seed(2024)
    q = torch.randn(2, 8, 512, 64)
    k = torch.randn(2, 2, 512, 64)
    v = torch.randn(2, 2, 512, 64)
    do = torch.randn(2, 8, 512, 64)
    sums = [float(t.double().sum()) for t in (q, k, v, do)]
    np.testing.assert_allclose(sums, z["input_sums"], rtol=0, atol=1e-6,
                               err_msg="torch CPU RNG drifted; regenerate the fixture")
    o, lse, dq, dk, dv = oracle.forward_backward(q, k, v, do, causal=True)
    for n, t in (("o", o), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)):
        flat = t.double().flatten()
        np.testing.assert_allclose([float(flat.sum()), float(flat.abs().sum())], z[f"{n}_sum"],
                                   rtol=1e-4, atol=1e-3, err_msg=n)
        sample = flat[:: max(1, flat.numel() // 256)][:256].float().numpy()
        np.testing.assert_allclose(sample, z[f"{n}_sample"], rtol=1e-4, atol=1e-4, err_msg=n)


def test_oracle_split_merge_equals_full_attention():
    z = _load("attn_decode_like.npz")
    q, k, v = z["q"], z["k"], z["v"]
    scale = 1.0 / math.sqrt(q.shape[-1])
    bounds = [(0, 10), (10, 10), (10, 33), (33, 48)]   # includes an empty split
    po, pl = oracle.split_partials(q, k, v, scale=scale, bounds=bounds)
    o, lse = oracle.merge_partials(po, pl)
    torch.testing.assert_close(o, z["o"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(lse, z["lse"], rtol=1e-5, atol=1e-5)


def test_oracle_merge_all_empty_row():
    po = torch.randn(3, 2, 4)
    pl = torch.full((3, 2), float("-inf"))
    o, lse = oracle.merge_partials(po, pl)
    assert torch.equal(o, torch.zeros(2, 4)) and torch.isinf(lse).all()


def test_oracle_append_matches_reference_cache_sequence():
    z = _load("cache_sequence.npz")
    cache = torch.zeros(2, 2, 12, 8)
    cache = oracle.append(cache, z["k_chunks"], 0)
    torch.testing.assert_close(cache[:, :, :8], z["kview"], rtol=0, atol=0)
    o, _ = oracle.forward(z["q"], z["kview"], z["vview"], causal=False)
    torch.testing.assert_close(o, z["attend"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("causal", [False, True])
def test_chunked_oracle_equals_the_full_one(causal):
    """forward_backward_chunked (used at the 16384-token length) computes the
    same fp32 results as forward_backward, chunk by chunk."""
    g = torch.Generator().manual_seed(9)
    q = torch.randn(2, 4, 70, 24, generator=g)
    k = torch.randn(2, 2, 90, 24, generator=g)
    v = torch.randn(2, 2, 90, 24, generator=g)
    do = torch.randn(2, 4, 70, 24, generator=g)
    full = oracle.forward_backward(q, k, v, do, causal=causal)
    chunked = oracle.forward_backward_chunked(q, k, v, do, causal=causal, chunk=16)
    for a, b in zip(full, chunked):
        torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5)
