# SPDX-License-Identifier: Apache-2.0
"""CPU API tests: the reference's tests/test_api.py, test_attention.py and
test_backward_formula.py semantics, run against kotflash_b200."""
import math

import pytest
import torch
import torch.nn.functional as F

import kotflash_b200 as kf
from kotflash_b200 import attention
from kotflash_b200.attention import _blockwise_backward, _sdpa, _sdpa_expanded


def test_public_surface_matches_reference():
    for name in ("attention", "triton_available", "triton_turing_supported"):
        assert hasattr(kf, name)
    assert isinstance(kf.triton_available(), bool)
    if not torch.cuda.is_available():
        assert kf.triton_turing_supported() is False


def test_sdpa_matches_torch_mha():
    torch.manual_seed(0)
    q = torch.randn(2, 4, 7, 32)
    k = torch.randn(2, 4, 9, 32)
    v = torch.randn_like(k)
    torch.testing.assert_close(attention(q, k, v, backend="sdpa"), F.scaled_dot_product_attention(q, k, v))


@pytest.mark.parametrize("causal", [False, True])
def test_sdpa_matches_torch_gqa_with_unequal_sequence_lengths(causal):
    torch.manual_seed(1)
    q = torch.randn(2, 8, 6, 32)
    k = torch.randn(2, 2, 9, 32)
    v = torch.randn_like(k)
    expected = F.scaled_dot_product_attention(
        q, k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1), is_causal=causal)
    torch.testing.assert_close(attention(q, k, v, causal=causal, backend="sdpa"), expected)


def test_auto_on_cpu_uses_sdpa():
    torch.manual_seed(2)
    q = torch.randn(1, 4, 5, 16)
    k = torch.randn(1, 2, 7, 16)
    v = torch.randn_like(k)
    torch.testing.assert_close(attention(q, k, v), attention(q, k, v, backend="sdpa"))


@pytest.mark.parametrize("expanded", [False, True])
def test_default_scale_preserves_pytorch_sdpa_dispatch(monkeypatch, expanded):
    q = torch.randn(1, 4, 5, 16)
    k = torch.randn(1, 1, 7, 16)
    v = torch.randn_like(k)
    observed = {}

    def fake_sdpa(query, key, value, **kwargs):
        observed["kwargs"] = kwargs
        observed["key_shape"] = tuple(key.shape)
        return torch.zeros_like(query)

    monkeypatch.setattr(F, "scaled_dot_product_attention", fake_sdpa)
    (_sdpa_expanded if expanded else _sdpa)(q, k, v, causal=False, scale=1.0 / math.sqrt(16))
    assert "scale" not in observed["kwargs"]
    assert observed["key_shape"][1] == (4 if expanded else 1)


def test_custom_scale_matches_explicit_q_scaling():
    torch.manual_seed(2)
    q = torch.randn(1, 2, 5, 16)
    k = torch.randn(1, 2, 7, 16)
    v = torch.randn_like(k)
    expected = F.scaled_dot_product_attention(q * (0.125 * math.sqrt(16)), k, v)
    torch.testing.assert_close(attention(q, k, v, scale=0.125, backend="sdpa"), expected)


@pytest.mark.parametrize("bad_scale", [float("nan"), float("inf"), float("-inf")])
def test_rejects_nonfinite_scale(bad_scale):
    q = torch.randn(1, 1, 2, 16)
    with pytest.raises(ValueError, match="finite"):
        attention(q, q, q, scale=bad_scale, backend="sdpa")


def test_rejects_non_numeric_scale_and_bad_backend_and_causal():
    q = torch.randn(1, 1, 2, 16)
    with pytest.raises(TypeError, match="finite real number"):
        attention(q, q, q, scale="x", backend="sdpa")
    with pytest.raises(ValueError, match="backend must be one of"):
        attention(q, q, q, backend="cuda")
    with pytest.raises(TypeError, match="causal must be a bool"):
        attention(q, q, q, causal=1)


@pytest.mark.parametrize(
    "qs,ks,vs,msg",
    [
        ((2, 3, 5, 8), (2, 2, 7, 8), (2, 2, 7, 8), "divisible"),
        ((2, 4, 5), (2, 2, 7, 8), (2, 2, 7, 8), "layout"),
        ((0, 4, 5, 8), (0, 2, 7, 8), (0, 2, 7, 8), "Batch dimension"),
        ((2, 4, 5, 8), (1, 2, 7, 8), (1, 2, 7, 8), "Batch dimensions must match"),
        ((2, 4, 5, 8), (2, 2, 7, 8), (2, 2, 6, 8), "K and V shapes"),
        ((2, 4, 5, 8), (2, 2, 7, 4), (2, 2, 7, 4), "head dimensions must match"),
        ((2, 4, 0, 8), (2, 2, 7, 8), (2, 2, 7, 8), "Sequence dimensions"),
        ((2, 4, 5, 0), (2, 2, 7, 0), (2, 2, 7, 0), "Head dimension must be non-zero"),
    ],
)
def test_rejects_invalid_layouts(qs, ks, vs, msg):
    with pytest.raises(ValueError, match=msg):
        attention(torch.randn(*qs), torch.randn(*ks), torch.randn(*vs))


def test_rejects_dtype_mismatch_and_non_tensors():
    q = torch.randn(1, 2, 3, 8)
    with pytest.raises(ValueError, match="dtypes must match"):
        attention(q, q.half(), q.half())
    with pytest.raises(TypeError):
        attention(q, 1, q)


def test_triton_backend_without_sm100_raises():
    q = torch.randn(1, 2, 3, 16)
    with pytest.raises(RuntimeError, match="sm_100"):
        attention(q, q, q, backend="triton")


def test_blockwise_backward_matches_autograd_mha_and_gqa():
    torch.manual_seed(3)
    for hq, hkv in [(2, 2), (4, 2)]:
        q = torch.randn(1, hq, 5, 16, requires_grad=True)
        k = torch.randn(1, hkv, 7, 16, requires_grad=True)
        v = torch.randn_like(k, requires_grad=True)
        scale = 1.0 / math.sqrt(16)
        ek, ev = k.repeat_interleave(hq // hkv, 1), v.repeat_interleave(hq // hkv, 1)
        lse = torch.logsumexp(torch.matmul(q, ek.transpose(-2, -1)) * scale, dim=-1)
        out = F.scaled_dot_product_attention(q, ek, ev)
        grad_out = torch.randn_like(out)
        ref = torch.autograd.grad(out, (q, k, v), grad_out)
        got = _blockwise_backward(q.detach(), k.detach(), v.detach(), out.detach(), lse.detach(),
                                  grad_out, causal=False, scale=scale, q_block=3, kv_block=2)
        for a, e in zip(got, ref):
            torch.testing.assert_close(a, e, rtol=2e-4, atol=2e-5)


@pytest.mark.parametrize(("hq", "hkv", "sq", "sk", "causal"),
                         [(2, 1, 7, 5, True), (4, 2, 5, 9, False), (2, 2, 9, 5, True)])
def test_batched_blockwise_backward_matches_autograd(hq, hkv, sq, sk, causal):
    torch.manual_seed(19)
    q = torch.randn(2, hq, sq, 16, requires_grad=True)
    k = torch.randn(2, hkv, sk, 16, requires_grad=True)
    v = torch.randn(2, hkv, sk, 16, requires_grad=True)
    ek, ev = k.repeat_interleave(hq // hkv, 1), v.repeat_interleave(hq // hkv, 1)
    scale = 1.0 / math.sqrt(16)
    scores = torch.matmul(q, ek.transpose(-2, -1)) * scale
    if causal:
        scores = scores.masked_fill(torch.arange(sk)[None, :] > torch.arange(sq)[:, None], float("-inf"))
    lse = torch.logsumexp(scores, dim=-1)
    out = F.scaled_dot_product_attention(q, ek, ev, is_causal=causal)
    grad_out = torch.randn_like(out)
    expected = torch.autograd.grad(out, (q, k, v), grad_out)
    actual = _blockwise_backward(q.detach(), k.detach(), v.detach(), out.detach(), lse.detach(),
                                 grad_out, causal=causal, scale=scale, q_block=3, kv_block=2)
    for a, e in zip(actual, expected):
        torch.testing.assert_close(a, e, rtol=3e-4, atol=3e-5)
