# SPDX-License-Identifier: Apache-2.0
"""K2 tcgen05 backward (dQ, dK, dV) vs the fp32 oracle (GPU)."""
import pytest
import torch

from kotflash_b200 import attention
from kotflash_b200.attention import attention_backward, attention_forward
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype)


def _run(b, hq, hkv, sq, sk, d, causal, dtype, seed=12, q_scale=1.0):
    q = _rand((b, hq, sq, d), dtype, seed, q_scale).requires_grad_(True)
    k = _rand((b, hkv, sk, d), dtype, seed + 1).requires_grad_(True)
    v = _rand((b, hkv, sk, d), dtype, seed + 2).requires_grad_(True)
    do = _rand((b, hq, sq, d), dtype, seed + 3)
    out = attention(q, k, v, causal=causal, backend="triton")
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do)
    eo, _lse, edq, edk, edv = oracle.forward_backward(q.detach(), k.detach(), v.detach(), do,
                                                       causal=causal)
    tag = f"{b},{hq},{hkv},{sq},{sk},{d},{causal},{dtype}"
    check_close(out, eo, name=f"bwd-path O {tag}")
    check_close(dq, edq, name=f"dQ {tag}")
    check_close(dk, edk, name=f"dK {tag}")
    check_close(dv, edv, name=f"dV {tag}")


@pytest.mark.parametrize(
    ("hq", "hkv", "sq", "sk", "head_dim", "causal"),
    [   # reference tests/test_triton.py:160-173
        (4, 4, 64, 80, 32, False),
        (8, 2, 64, 80, 64, True),
        (8, 1, 80, 64, 32, True),
        (8, 2, 48, 64, 72, False),
        (4, 4, 48, 64, 96, True),
        (8, 1, 64, 48, 128, False),
        (8, 2, 1024, 1024, 64, True),
        (4, 1, 1024, 768, 32, False),
        (4, 2, 2048, 2048, 32, True),
        (8, 2, 1, 1024, 64, False),
    ],
)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_backward_reference_shapes(hq, hkv, sq, sk, head_dim, causal, dtype):
    _run(1, hq, hkv, sq, sk, head_dim, causal, dtype)


@pytest.mark.parametrize(
    "b,hq,hkv,sq,sk,d,causal",
    [
        (2, 4, 2, 200, 333, 128, True),     # Sk > Sq causal: trailing key blocks get zero grads
        (1, 2, 2, 129, 1, 64, False),       # single key
        (1, 4, 2, 7, 130, 16, True),
        (2, 6, 3, 300, 300, 80, False),
        (1, 2, 1, 77, 91, 20, True),        # head dim not a multiple of 8 (padded)
    ],
)
def test_backward_edge_shapes(b, hq, hkv, sq, sk, d, causal):
    _run(b, hq, hkv, sq, sk, d, causal, torch.bfloat16, seed=3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_backward_prefill_config_full_size(dtype):
    """BASELINE cfg2 fwd+bwd at full size (B4 Hq32 Hkv8 S4096 D128, causal,
    q scaled by 1/sqrt(D)); oracle run per batch on the GPU in fp32."""
    b, hq, hkv, s, d = 4, 32, 8, 4096, 128
    q = _rand((b, hq, s, d), dtype, 21, d ** -0.5)
    k = _rand((b, hkv, s, d), dtype, 22)
    v = _rand((b, hkv, s, d), dtype, 23)
    do = _rand((b, hq, s, d), dtype, 24)
    out, lse = attention_forward(q, k, v, causal=True, scale=d ** -0.5)
    dq, dk, dv = attention_backward(q, k, v, out, lse, do, causal=True, scale=d ** -0.5)
    for i in range(b):
        sl = slice(i, i + 1)
        eo, el, edq, edk, edv = oracle.forward_backward(q[sl], k[sl], v[sl], do[sl], causal=True)
        check_close(dq[sl], edq, name=f"cfg2 dQ batch {i}")
        check_close(dk[sl], edk, name=f"cfg2 dK batch {i}")
        check_close(dv[sl], edv, name=f"cfg2 dV batch {i}")


@pytest.mark.parametrize("d", [72, 96])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_odd_head_dim_config(d, causal):
    """BASELINE cfg5 geometry (B2 Hq16 Hkv4 D72/96 fp16) at S=2048 (oracle cost)."""
    _run(2, 16, 4, 2048, 2048, d, causal, torch.float16, seed=5)


@pytest.mark.parametrize("d", [72, 96])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_odd_head_dim_full_length_unit(d, causal):
    """BASELINE cfg5 at its full length S=16384 (fp16, D72/96), one (batch,
    KV-head) unit: 4 query heads over one KV head, the unit each of the 8
    ranks owns when cfg5 is sharded.  The oracle runs chunked over query rows
    on the GPU in fp32."""
    s = 16384
    q = _rand((1, 4, s, d), torch.float16, 50 + d)
    k = _rand((1, 1, s, d), torch.float16, 51 + d)
    v = _rand((1, 1, s, d), torch.float16, 52 + d)
    do = _rand((1, 4, s, d), torch.float16, 53 + d)
    scale = d ** -0.5
    out, lse = attention_forward(q, k, v, causal=causal, scale=scale)
    dq, dk, dv = attention_backward(q, k, v, out, lse, do, causal=causal, scale=scale)
    eo, el, edq, edk, edv = oracle.forward_backward_chunked(q, k, v, do, causal=causal, scale=scale)
    tag = f"cfg5 S16384 D{d} causal={causal}"
    check_close(out, eo, name=f"{tag} O")
    check_close(lse, el, name=f"{tag} LSE")
    check_close(dq, edq, name=f"{tag} dQ")
    check_close(dk, edk, name=f"{tag} dK")
    check_close(dv, edv, name=f"{tag} dV")


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("b,hq,hkv,s,d", [(1, 4, 1, 4096, 128), (2, 8, 2, 1000, 64), (1, 4, 2, 777, 96)])
def test_backward_query_split_matches_single_cta_per_key_block(b, hq, hkv, s, d, causal):
    """A backward with few key-block CTAs splits each key block's query range
    over several CTAs when the workspace holds the dK/dV accumulators
    (kf_attn_bwd_workspace_bytes_kv) -- causal grids to balance their unequal
    key blocks, non-causal ones to fill the last wave of SMs -- and runs one
    CTA per key block with the smaller kf_attn_bwd_workspace_bytes: both must
    match the oracle (the split path of the reference is
    kotflash/kernels/triton_backward.py:199-332)."""
    from kotflash_b200 import _ext

    lib = _ext.load()
    q = _rand((b, hq, s, d), torch.bfloat16, 61, d ** -0.5)
    k = _rand((b, hkv, s, d), torch.bfloat16, 62)
    v = _rand((b, hkv, s, d), torch.bfloat16, 63)
    do = _rand((b, hq, s, d), torch.bfloat16, 64)
    scale = d ** -0.5
    out, lse = attention_forward(q, k, v, causal=causal, scale=scale)
    results = {}
    for name, ws_bytes in (("split", lib.kf_attn_bwd_workspace_bytes_kv(b, hq, hkv, s, s, d)),
                           ("single", lib.kf_attn_bwd_workspace_bytes(b, hq, s, d))):
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        rc = lib.kf_attn_bwd(_ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(k)), _ext.ref(_ext.t4(v)),
                             _ext.ref(_ext.t4(out)), lse.data_ptr(), _ext.ref(_ext.t4(do)),
                             _ext.ref(_ext.t4(dq)), _ext.ref(_ext.t4(dk)), _ext.ref(_ext.t4(dv)),
                             _ext.KF_BF16, scale, int(causal), ws.data_ptr(), ws.numel(),
                             _ext.status_word(q.device).data_ptr(), _ext.stream_of(q))
        _ext.check(rc, "kf_attn_bwd")
        results[name] = (dq, dk, dv)
    _, _, edq, edk, edv = oracle.forward_backward_chunked(q, k, v, do, causal=causal, scale=scale)
    for name, (dq, dk, dv) in results.items():
        tag = f"{name} {b},{hq},{hkv},{s},{d},causal={causal}"
        check_close(dq, edq, name=f"dQ {tag}")
        check_close(dk, edk, name=f"dK {tag}")
        check_close(dv, edv, name=f"dV {tag}")
