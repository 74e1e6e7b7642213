# SPDX-License-Identifier: Apache-2.0
"""CPU cache tests: the reference's tests/test_kv_cache.py and
tests/test_preallocated_cache.py semantics, plus the golden cache sequence."""
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from kotflash_b200.cache import PreallocatedKVCache, append_kv_cache, decode_step

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_append_kv_cache_preserves_order_and_does_not_mutate_inputs():
    k_cache = torch.arange(24, dtype=torch.float32).view(1, 2, 3, 4)
    v_cache = -k_cache
    new_k = torch.full((1, 2, 1, 4), 100.0)
    new_v = torch.full((1, 2, 1, 4), -100.0)
    old_k, old_v = k_cache.clone(), v_cache.clone()
    uk, uv = append_kv_cache(k_cache, v_cache, new_k, new_v)
    torch.testing.assert_close(uk, torch.cat((old_k, new_k), dim=2))
    torch.testing.assert_close(uv, torch.cat((old_v, new_v), dim=2))
    torch.testing.assert_close(k_cache, old_k)
    torch.testing.assert_close(v_cache, old_v)


@pytest.mark.parametrize("bad_field", ["batch", "heads", "dim", "dtype"])
def test_append_kv_cache_rejects_incompatible_new_tensors(bad_field):
    k_cache = torch.zeros(1, 2, 4, 8)
    new_k = torch.zeros(1, 2, 1, 8)
    if bad_field == "batch":
        new_k = torch.zeros(2, 2, 1, 8)
    elif bad_field == "heads":
        new_k = torch.zeros(1, 1, 1, 8)
    elif bad_field == "dim":
        new_k = torch.zeros(1, 2, 1, 16)
    else:
        new_k = new_k.half()
    with pytest.raises(ValueError):
        append_kv_cache(k_cache, torch.zeros_like(k_cache), new_k, torch.zeros_like(new_k))


def test_decode_step_matches_expanded_sdpa_for_one_visible_token():
    torch.manual_seed(7)
    q = torch.randn(1, 4, 1, 16)
    k_cache = torch.randn(1, 2, 5, 16)
    v_cache = torch.randn_like(k_cache)
    k_new, v_new = torch.randn(1, 2, 1, 16), torch.randn(1, 2, 1, 16)
    actual, uk, uv = decode_step(q, k_cache, v_cache, k_new, v_new, backend="sdpa")
    expected = F.scaled_dot_product_attention(q, uk.repeat_interleave(2, 1), uv.repeat_interleave(2, 1))
    torch.testing.assert_close(actual, expected)
    assert uk.shape[2] == 6 and uv.shape[2] == 6


def test_decode_step_rejections():
    cache = torch.randn(1, 2, 4, 16)
    new = torch.randn(1, 2, 1, 16)
    with pytest.raises(ValueError, match="exactly one new query token"):
        decode_step(torch.randn(1, 4, 2, 16), cache, cache, new, new, backend="sdpa")
    with pytest.raises(ValueError, match="divisible"):
        decode_step(torch.randn(1, 3, 1, 16), cache, cache, new, new, backend="sdpa")
    with pytest.raises(ValueError, match="exactly one new K/V token"):
        decode_step(torch.randn(1, 4, 1, 16), cache, cache, torch.randn(1, 2, 2, 16),
                    torch.randn(1, 2, 2, 16), backend="sdpa")
    empty = torch.empty(1, 0, 2, 8)
    with pytest.raises(ValueError, match="non-zero"):
        append_kv_cache(empty, empty, torch.empty(1, 0, 1, 8), torch.empty(1, 0, 1, 8))


def test_preallocated_cache_appends_and_returns_only_populated_prefix():
    cache = PreallocatedKVCache(1, 2, 8, 4, device="cpu", dtype=torch.float32)
    k1 = torch.arange(24, dtype=torch.float32).view(1, 2, 3, 4)
    k2 = torch.full((1, 2, 1, 4), 100.0)
    cache.append(k1, -k1)
    cache.append(k2, -k2)
    assert cache.length == 4
    vk, vv = cache.view()
    torch.testing.assert_close(vk, torch.cat((k1, k2), dim=2))
    torch.testing.assert_close(vv, -torch.cat((k1, k2), dim=2))
    assert vk.untyped_storage().data_ptr() == cache.k.untyped_storage().data_ptr()
    ck, cv = cache.contiguous_view()
    assert ck.is_contiguous() and cv.is_contiguous()
    torch.testing.assert_close(ck, vk)


def test_preallocated_cache_rejects_invalid_append_without_advancing():
    cache = PreallocatedKVCache(1, 2, 3, 4, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError, match="empty"):
        cache.view()
    with pytest.raises(ValueError, match="batch, heads"):
        cache.append(torch.zeros(1, 1, 1, 4), torch.zeros(1, 1, 1, 4))
    with pytest.raises(ValueError, match="dtype"):
        cache.append(torch.zeros(1, 2, 1, 4, dtype=torch.float16), torch.zeros(1, 2, 1, 4, dtype=torch.float16))
    with pytest.raises(ValueError, match="shapes must match"):
        cache.append(torch.zeros(1, 2, 1, 4), torch.zeros(1, 2, 2, 4))
    with pytest.raises(ValueError, match="cannot append an empty"):
        cache.append(torch.zeros(1, 2, 0, 4), torch.zeros(1, 2, 0, 4))
    with pytest.raises(ValueError, match="append backend"):
        cache.append(torch.zeros(1, 2, 1, 4), torch.zeros(1, 2, 1, 4), backend="bogus")
    assert cache.length == 0
    cache.append(torch.zeros(1, 2, 2, 4), torch.zeros(1, 2, 2, 4))
    with pytest.raises(ValueError, match="full"):
        cache.append(torch.zeros(1, 2, 2, 4), torch.zeros(1, 2, 2, 4))
    assert cache.length == 2


@pytest.mark.parametrize("bad", [0, -1, True, 2.0])
def test_preallocated_cache_rejects_bad_dimensions(bad):
    with pytest.raises(ValueError, match="positive integer"):
        PreallocatedKVCache(bad, 2, 4, 4, device="cpu", dtype=torch.float32)


def test_cuda_append_backend_on_cpu_raises():
    cache = PreallocatedKVCache(1, 2, 4, 16, device="cpu", dtype=torch.float16)
    with pytest.raises((RuntimeError, ValueError)):
        cache.append(torch.zeros(1, 2, 1, 16, dtype=torch.float16),
                     torch.zeros(1, 2, 1, 16, dtype=torch.float16), backend="cuda")
    assert cache.length == 0


def test_append_and_attend_validation_and_fused_on_cpu():
    cache = PreallocatedKVCache(1, 2, 8, 16, device="cpu", dtype=torch.float32)
    cache.append(torch.randn(1, 2, 3, 16), torch.randn(1, 2, 3, 16))
    q, nk = torch.randn(1, 4, 1, 16), torch.randn(1, 2, 1, 16)
    with pytest.raises(ValueError, match="attention backend"):
        cache.append_and_attend(q, nk, nk, attention_backend="x")
    with pytest.raises(ValueError, match="append backend"):
        cache.append_and_attend(q, nk, nk, append_backend="x")
    with pytest.raises(ValueError, match="requires attention_backend"):
        cache.append_and_attend(q, nk, nk, append_backend="fused", attention_backend="sdpa")
    with pytest.raises(RuntimeError, match="fused append/decode requires"):
        cache.append_and_attend(q, nk, nk, append_backend="fused")
    assert cache.length == 3


def test_cache_sequence_matches_reference_golden():
    z = np.load(GOLDEN / "cache_sequence.npz")
    t = {k: torch.from_numpy(z[k]) for k in z.files}
    cache = PreallocatedKVCache(2, 2, 12, 8, device="cpu", dtype=torch.float32)
    off = 0
    for n in (3, 1, 4):
        cache.append(t["k_chunks"][:, :, off:off + n], t["v_chunks"][:, :, off:off + n])
        off += n
    kv, vv = cache.view()
    assert torch.equal(kv, t["kview"]) and torch.equal(vv, t["vview"])
    torch.testing.assert_close(cache.attend(t["q"], backend="sdpa"), t["attend"])
    out2 = cache.append_and_attend(t["q2"], t["new_k"], t["new_v"], append_backend="torch",
                                   attention_backend="sdpa")
    torch.testing.assert_close(out2, t["attend2"])
    k2, v2 = cache.view()
    assert torch.equal(k2, t["k_after"]) and torch.equal(v2, t["v_after"])
    assert cache.length == int(t["length"][0])
    dout, uk, uv = decode_step(t["ds_q"], t["ds_k0"], t["ds_v0"], t["ds_nk"], t["ds_nv"], backend="sdpa")
    torch.testing.assert_close(dout, t["ds_out"])
    assert torch.equal(uk, t["ds_uk"]) and torch.equal(uv, t["ds_uv"])
    ck, cv = append_kv_cache(t["ds_k0"], t["ds_v0"], t["ds_nk"], t["ds_nv"])
    assert torch.equal(ck, t["cat_k"]) and torch.equal(cv, t["cat_v"])


@pytest.mark.parametrize("value,kernel", [(None, False), ("1", True), ("0", False), ("", False),
                                          ("true", False), ("yes", False)])
def test_cuda_append_opt_in_follows_the_reference(value, kernel, monkeypatch):
    """KOTFLASH_ENABLE_CUDA_APPEND keeps the reference's meaning
    (kotflash/cache.py:163-168, :248): only "1" lets append(backend="auto")
    use the append kernel, and the same value turns the fused auto route of
    append_and_attend off."""
    from kotflash_b200.cache import cuda_append_opted_in, fused_append_auto_allowed

    if value is None:
        monkeypatch.delenv("KOTFLASH_ENABLE_CUDA_APPEND", raising=False)
    else:
        monkeypatch.setenv("KOTFLASH_ENABLE_CUDA_APPEND", value)
    assert cuda_append_opted_in() is kernel
    assert fused_append_auto_allowed() is (not kernel)
    assert cuda_append_opted_in(env=value) is kernel


def test_auto_append_on_cpu_stays_on_torch_copies_with_the_opt_in(monkeypatch):
    monkeypatch.setenv("KOTFLASH_ENABLE_CUDA_APPEND", "1")
    cache = PreallocatedKVCache(1, 2, 8, 4, device="cpu", dtype=torch.float16)
    k = torch.randn(1, 2, 3, 4).half()
    cache.append(k, -k)  # CPU tensors never reach the kernel
    assert torch.equal(cache.k[:, :, :3], k) and cache.length == 3
