# SPDX-License-Identifier: Apache-2.0
"""Seeded randomized parity sweep (GPU): forward + backward and split-KV decode
over shapes the fixed tests do not pin (every head_dim step of 8, ragged and
tiny sequence lengths, GQA/MQA ratios, both masks and dtypes), against the
fp32 oracle with the 2e-2 tolerance."""
import random

import pytest
import torch

from kotflash_b200 import attention
from kotflash_b200.attention import _decode_forward
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def _cases(seed, n, decode):
    rng = random.Random(seed)
    out = []
    for i in range(n):
        hkv = rng.choice([1, 2, 3])
        group = rng.choice([1, 2, 4, 5])
        d = rng.choice(range(16, 129, 8))
        dtype = rng.choice([torch.float16, torch.bfloat16])
        if decode:
            sq = rng.randint(1, 16)
            sk = rng.choice([1, 7, 63, 64, 65, 200, 1000, 1537, 4099])
            causal = False
        else:
            causal = rng.random() < 0.5
            sq = rng.choice([1, 17, 64, 127, 128, 129, 300])
            sk = sq if causal and rng.random() < 0.7 else rng.choice([1, 50, 128, 200, 257, 400])
        out.append((rng.randint(1, 2), hkv * group, hkv, sq, sk, d, causal, dtype, seed * 1000 + i))
    return out


def _rand(shape, dtype, g, scale=1.0):
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype)


@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,causal,dtype,seed", _cases(11, 24, decode=False))
def test_fuzz_forward_backward(b, hq, hkv, sq, sk, d, causal, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = _rand((b, hq, sq, d), dtype, g, d ** -0.5).requires_grad_(True)
    k = _rand((b, hkv, sk, d), dtype, g).requires_grad_(True)
    v = _rand((b, hkv, sk, d), dtype, g).requires_grad_(True)
    do = _rand((b, hq, sq, d), dtype, g)
    out = attention(q, k, v, causal=causal, backend="triton")
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do)
    eo, _, edq, edk, edv = oracle.forward_backward(q.detach(), k.detach(), v.detach(), do, causal=causal)
    name = f"fuzz {b},{hq},{hkv},{sq},{sk},{d},{causal},{dtype}"
    check_close(out, eo, name=name + " O")
    check_close(dq, edq, name=name + " dQ")
    check_close(dk, edk, name=name + " dK")
    check_close(dv, edv, name=name + " dV")


@pytest.mark.parametrize("b,hq,hkv,sq,sk,d,causal,dtype,seed", _cases(23, 30, decode=True))
def test_fuzz_decode(b, hq, hkv, sq, sk, d, causal, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = _rand((b, hq, sq, d), dtype, g)
    k = _rand((b, hkv, sk, d), dtype, g)
    v = _rand((b, hkv, sk, d), dtype, g)
    scale = d ** -0.5
    with torch.no_grad():
        o, lse = _decode_forward(q, k, v, scale=scale, want_lse=True)
    eo, el = oracle.forward(q, k, v, causal=False, scale=scale)
    name = f"fuzz decode {b},{hq},{hkv},{sq},{sk},{d},{dtype}"
    check_close(o, eo, name=name + " O")
    check_close(lse, el, name=name + " LSE")
