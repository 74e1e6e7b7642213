# SPDX-License-Identifier: Apache-2.0
"""K4 append kernel: bit-exact against index_copy / torch.cat (GPU)."""
import pytest
import torch

from kotflash_b200.cache import PreallocatedKVCache
from kotflash_b200._cuda_append import append_kv_cuda
from oracle import attention_oracle as oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_two_appends_match_cat(dtype):
    # mirrors the reference's tests/test_cuda_append.py:14-34
    torch.manual_seed(37)
    cache = PreallocatedKVCache(2, 2, 64, 32, device="cuda", dtype=dtype)
    past_k = torch.randn(2, 2, 7, 32, device="cuda", dtype=dtype)
    past_v = torch.randn_like(past_k)
    new_k = torch.randn(2, 2, 3, 32, device="cuda", dtype=dtype)
    new_v = torch.randn_like(new_k)
    cache.append(past_k, past_v, backend="cuda")
    cache.append(new_k, new_v, backend="cuda")
    k, v = cache.view()
    assert torch.equal(k, torch.cat((past_k, new_k), dim=2))
    assert torch.equal(v, torch.cat((past_v, new_v), dim=2))
    assert cache.length == 10


@pytest.mark.parametrize("d", [16, 72, 128, 20])
def test_append_strided_sources_and_odd_dims(d):
    torch.manual_seed(5)
    b, h, cap, s = 3, 4, 50, 9
    kc = torch.randn(b, h, cap, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    # non-contiguous sources: [B, S, H, D] storage viewed as [B, H, S, D]
    nk = torch.randn(b, s, h, d, device="cuda", dtype=torch.bfloat16).transpose(1, 2)
    nv = torch.randn(b, s, h, d + 8, device="cuda", dtype=torch.bfloat16)[..., :d].transpose(1, 2)
    ek = oracle.append(kc, nk, 11)
    ev = oracle.append(vc, nv, 11)
    append_kv_cuda(kc, vc, nk, nv, 11)
    torch.cuda.synchronize()
    assert torch.equal(kc, ek) and torch.equal(vc, ev)


def test_append_rejects_overflow_without_writing():
    cache = PreallocatedKVCache(1, 2, 4, 16, device="cuda", dtype=torch.float16)
    cache.append(torch.ones(1, 2, 3, 16, device="cuda", dtype=torch.float16),
                 torch.ones(1, 2, 3, 16, device="cuda", dtype=torch.float16), backend="cuda")
    before = cache.k.clone()
    with pytest.raises(ValueError, match="full"):
        cache.append(torch.zeros(1, 2, 2, 16, device="cuda", dtype=torch.float16),
                     torch.zeros(1, 2, 2, 16, device="cuda", dtype=torch.float16), backend="cuda")
    assert cache.length == 3 and torch.equal(cache.k, before)
    with pytest.raises(ValueError, match="capacity"):
        append_kv_cuda(cache.k, cache.v, torch.zeros(1, 2, 2, 16, device="cuda", dtype=torch.float16),
                       torch.zeros(1, 2, 2, 16, device="cuda", dtype=torch.float16), 3)


def test_kv_cache_loop_config_append_bit_exact():
    """BASELINE cfg4 cache: capacity 32768, B8 Hkv8 D128 bf16; 4096-token prefill
    then 256 single-token appends, bit-exact vs index_copy."""
    torch.manual_seed(4)
    b, hkv, cap, d = 8, 8, 32768, 128
    cache = PreallocatedKVCache(b, hkv, cap, d, device="cuda", dtype=torch.bfloat16)
    pk = torch.randn(b, hkv, 4096, d, device="cuda", dtype=torch.bfloat16)
    pv = torch.randn_like(pk)
    cache.append(pk, pv, backend="cuda")
    ref_k = torch.zeros(b, hkv, 4096 + 256, d, device="cuda", dtype=torch.bfloat16)
    ref_v = torch.zeros_like(ref_k)
    ref_k.index_copy_(2, torch.arange(4096, device="cuda"), pk)
    ref_v.index_copy_(2, torch.arange(4096, device="cuda"), pv)
    for step in range(256):
        nk = torch.randn(b, hkv, 1, d, device="cuda", dtype=torch.bfloat16)
        nv = torch.randn_like(nk)
        cache.append(nk, nv, backend="cuda")
        idx = torch.tensor([4096 + step], device="cuda")
        ref_k.index_copy_(2, idx, nk)
        ref_v.index_copy_(2, idx, nv)
    k, v = cache.view()
    assert cache.length == 4096 + 256
    assert torch.equal(k, ref_k) and torch.equal(v, ref_v)
