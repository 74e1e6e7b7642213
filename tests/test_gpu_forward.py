# SPDX-License-Identifier: Apache-2.0
"""K1 tcgen05 forward (O and LSE) vs the fp32 oracle (GPU)."""
import pytest
import torch

from kotflash_b200 import attention
from kotflash_b200.attention import attention_forward
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype)


@pytest.mark.parametrize("head_dim", [32, 64, 72, 96, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_forward_reference_shapes(head_dim, causal, dtype):
    # reference tests/test_triton.py:19-32: B1 Hq8 Hkv2 Sq129 Sk161
    q = _rand((1, 8, 129, head_dim), dtype, 11)
    k = _rand((1, 2, 161, head_dim), dtype, 12)
    v = _rand((1, 2, 161, head_dim), dtype, 13)
    out, lse = attention_forward(q, k, v, causal=causal, scale=head_dim ** -0.5)
    eo, el = oracle.forward(q, k, v, causal=causal)
    check_close(out, eo, name=f"fwd O D{head_dim} causal={causal} {dtype}")
    check_close(lse, el, name=f"fwd LSE D{head_dim} causal={causal} {dtype}")


@pytest.mark.parametrize(
    "b,hq,hkv,sq,sk,d,causal",
    [
        (2, 4, 4, 300, 300, 64, True),      # MHA: tile pairs are two row blocks
        (1, 3, 1, 257, 513, 128, True),     # MQA, odd group, unequal lengths
        (1, 8, 2, 700, 130, 64, True),      # causal with Sq > Sk
        (2, 8, 2, 1, 777, 128, True),       # single causal query row
        (1, 4, 2, 1000, 1000, 16, False),   # smallest head dim
        (1, 4, 2, 200, 1100, 48, False),
        (1, 4, 1, 256, 384, 80, True),
        (1, 2, 2, 130, 77, 20, True),       # head dim not a multiple of 8 (padded)
        (2, 16, 4, 1024, 1024, 128, True),
        (1, 16, 4, 2048, 2048, 96, False),
        (2, 40, 40, 300, 300, 64, True),   # 160 items > 148 CTAs: persistent CTAs run several,
        (2, 40, 40, 300, 300, 64, False),  # single-tile items (odd row-block count) among them
        (2, 80, 80, 300, 300, 64, True),   # 320 items, 160 single-tile ones first in the item order:
        (2, 80, 80, 300, 300, 64, False),  # without one item per CTA, CTAs would meet one before a pair
    ],
)
def test_forward_shapes(b, hq, hkv, sq, sk, d, causal):
    q = _rand((b, hq, sq, d), torch.bfloat16, 1)
    k = _rand((b, hkv, sk, d), torch.bfloat16, 2)
    v = _rand((b, hkv, sk, d), torch.bfloat16, 3)
    out, lse = attention_forward(q, k, v, causal=causal, scale=d ** -0.5)
    eo, el = oracle.forward(q, k, v, causal=causal)
    check_close(out, eo, name=f"fwd O {b},{hq},{hkv},{sq},{sk},{d},{causal}")
    check_close(lse, el, name=f"fwd LSE {b},{hq},{hkv},{sq},{sk},{d},{causal}")


def test_forward_strided_inputs_and_custom_scale():
    # [B, S, H, D] storage viewed as [B, H, S, D] (TMA-legal strides, no copy)
    q = _rand((2, 333, 8, 64), torch.float16, 4).transpose(1, 2)
    k = _rand((2, 400, 2, 64), torch.float16, 5).transpose(1, 2)
    v = _rand((2, 400, 2, 64), torch.float16, 6).transpose(1, 2)
    out = attention(q, k, v, causal=True, scale=0.3, backend="triton")
    eo, _ = oracle.forward(q, k, v, causal=True, scale=0.3)
    check_close(out, eo, name="fwd strided scale=0.3")


def test_forward_large_logits_rescale_path():
    # growing logits along the key axis force repeated running-max updates
    q = _rand((1, 2, 256, 64), torch.bfloat16, 7, scale=4.0)
    k = (_rand((1, 1, 1024, 64), torch.float32, 8) *
         torch.linspace(0.1, 3.0, 1024, device="cuda")[None, None, :, None]).to(torch.bfloat16)
    v = _rand((1, 1, 1024, 64), torch.bfloat16, 9)
    out, lse = attention_forward(q, k, v, causal=False, scale=0.125)
    eo, el = oracle.forward(q, k, v, causal=False, scale=0.125)
    check_close(out, eo, name="fwd rescale O")
    check_close(lse, el, name="fwd rescale LSE")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_forward_prefill_config_full_size(dtype):
    """BASELINE cfg2 forward at full size: B4 Hq32 Hkv8 S4096 D128 causal,
    q scaled by 1/sqrt(D).  Checked per batch against the oracle run on GPU."""
    b, hq, hkv, s, d = 4, 32, 8, 4096, 128
    q = _rand((b, hq, s, d), dtype, 21, scale=d ** -0.5)
    k = _rand((b, hkv, s, d), dtype, 22)
    v = _rand((b, hkv, s, d), dtype, 23)
    out, lse = attention_forward(q, k, v, causal=True, scale=d ** -0.5)
    for i in range(b):
        eo, el = oracle.forward(q[i:i + 1], k[i:i + 1], v[i:i + 1], causal=True)
        check_close(out[i:i + 1], eo, name=f"cfg2 fwd O batch {i}")
        check_close(lse[i:i + 1], el, name=f"cfg2 fwd LSE batch {i}")
