# SPDX-License-Identifier: Apache-2.0
"""K3 split-KV decode (+ K3b merge, + fused append) vs the fp32 oracle (GPU)."""
import math

import pytest
import torch

from kotflash_b200 import attention
from kotflash_b200.attention import _decode_forward
from kotflash_b200.cache import PreallocatedKVCache
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", dtype=torch.float32, generator=g).to(dtype)


@pytest.mark.parametrize("q_seq,kv_seq", [(1, 2048), (4, 1024), (16, 4096)])
def test_split_kv_decode_reference_shapes(q_seq, kv_seq):
    # reference tests/test_triton.py:35-53 (B2 Hq8 Hkv2 D64 fp16)
    q = _rand((2, 8, q_seq, 64), torch.float16, 17)
    k = _rand((2, 2, kv_seq, 64), torch.float16, 18)
    v = _rand((2, 2, kv_seq, 64), torch.float16, 19)
    with torch.no_grad():
        out = attention(q, k, v, causal=False, backend="triton")
    exp, _ = oracle.forward(q, k, v, causal=False)
    check_close(out, exp, name=f"decode Sq{q_seq} Sk{kv_seq}")


@pytest.mark.parametrize("q_seq,kv_seq", [(2, 1537), (8, 8193), (3, 1), (5, 7), (1, 65), (16, 63)])
def test_split_kv_decode_partial_chunks_mqa(q_seq, kv_seq):
    # reference tests/test_triton.py:56-69 plus tiny/ragged key counts
    q = _rand((1, 4, q_seq, 32), torch.float16, 23)
    k = _rand((1, 1, kv_seq, 32), torch.float16, 24)
    v = _rand((1, 1, kv_seq, 32), torch.float16, 25)
    with torch.no_grad():
        out = attention(q, k, v, causal=False, backend="triton")
    exp, _ = oracle.forward(q, k, v, causal=False)
    check_close(out, exp, name=f"decode mqa Sq{q_seq} Sk{kv_seq}")


@pytest.mark.parametrize("sq", [1, 4, 16])
@pytest.mark.parametrize("sk", [1024, 2048, 8192, 32768, 131072])
def test_decode_sweep_config_with_lse(sq, sk):
    """BASELINE cfg3: B2 Hq8 Hkv2 D64 fp16 non-causal, O and merged LSE."""
    q = _rand((2, 8, sq, 64), torch.float16, 100 + sq)
    k = _rand((2, 2, sk, 64), torch.float16, 200)
    v = _rand((2, 2, sk, 64), torch.float16, 201)
    out, lse = _decode_forward(q, k, v, scale=0.125, want_lse=True)
    exp_o, exp_lse = oracle.forward(q, k, v, causal=False, scale=0.125)
    check_close(out, exp_o, name=f"cfg3 O Sq{sq} Sk{sk}")
    check_close(lse, exp_lse, name=f"cfg3 LSE Sq{sq} Sk{sk}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("d", [16, 40, 72, 96, 128])
def test_decode_head_dims_and_dtypes(dtype, d):
    q = _rand((2, 6, 3, d), dtype, 31)
    k = _rand((2, 3, 1500, d), dtype, 32)
    v = _rand((2, 3, 1500, d), dtype, 33)
    with torch.no_grad():
        out = attention(q, k, v, causal=False, backend="triton")
    exp, _ = oracle.forward(q, k, v, causal=False)
    check_close(out, exp, name=f"decode D{d} {dtype}")



@pytest.mark.parametrize("hq,hkv,sq,d,sk", [(8, 2, 5, 96, 3000), (8, 2, 16, 128, 1500), (4, 1, 5, 72, 777),
                                            (32, 2, 16, 64, 2049), (16, 1, 9, 16, 300)])
def test_decode_tensor_core_path(hq, hkv, sq, d, sk):
    """More than 16 packed rows per KV head (tcgen05 decode), incl. head dims that
    pad to two 64-column panels and more than 128 rows (two row blocks)."""
    q = _rand((2, hq, sq, d), torch.bfloat16, 41)
    k = _rand((2, hkv, sk, d), torch.bfloat16, 42)
    v = _rand((2, hkv, sk, d), torch.bfloat16, 43)
    out, lse = _decode_forward(q, k, v, scale=d ** -0.5, want_lse=True)
    exp_o, exp_lse = oracle.forward(q, k, v, causal=False, scale=d ** -0.5)
    check_close(out, exp_o, name=f"tc decode O {hq},{hkv},{sq},{d},{sk}")
    check_close(lse, exp_lse, name=f"tc decode LSE {hq},{hkv},{sq},{d},{sk}")

def test_strided_cache_decode_reads_prefix_in_place():
    # reference tests/test_triton.py:212-240 at the BASELINE cfg4 geometry
    torch.manual_seed(29)
    cache = PreallocatedKVCache(8, 8, 32768, 128, device="cuda", dtype=torch.bfloat16)
    pk = _rand((8, 8, 4096, 128), torch.bfloat16, 40)
    pv = _rand((8, 8, 4096, 128), torch.bfloat16, 41)
    cache.append(pk, pv)
    q = _rand((8, 32, 1, 128), torch.bfloat16, 42)
    with torch.inference_mode():
        out = cache.attend(q, backend="triton")
        kv, vv = cache.view()
        assert not kv.is_contiguous()
    exp, _ = oracle.forward(q, pk, pv, causal=False)
    check_close(out, exp, name="cfg4 strided decode")


@pytest.mark.parametrize("dtype,d,past", [(torch.float16, 64, 2047), (torch.bfloat16, 128, 4096),
                                           (torch.bfloat16, 128, 5)])
def test_fused_append_and_attend(dtype, d, past):
    # reference tests/test_triton.py:265-297
    b, hkv, hq = 2, 2, 8
    cache = PreallocatedKVCache(b, hkv, past + 64, d, device="cuda", dtype=dtype)
    pk = _rand((b, hkv, past, d), dtype, 50)
    pv = _rand((b, hkv, past, d), dtype, 51)
    nk = _rand((b, hkv, 1, d), dtype, 52)
    nv = _rand((b, hkv, 1, d), dtype, 53)
    q = _rand((b, hq, 1, d), dtype, 54)
    cache.append(pk, pv, backend="torch")
    with torch.inference_mode():
        out = cache.append_and_attend(q, nk, nv, append_backend="fused", attention_backend="triton")
    torch.cuda.synchronize()
    assert cache.length == past + 1
    sk, sv = cache.view()
    assert torch.equal(sk[:, :, -1:], nk) and torch.equal(sv[:, :, -1:], nv)
    assert torch.equal(sk[:, :, :past], pk)
    exp, _ = oracle.forward(q, torch.cat((pk, nk), 2), torch.cat((pv, nv), 2), causal=False)
    check_close(out, exp, name=f"fused append D{d} past{past}")


def test_kv_cache_decode_loop_config():
    """BASELINE cfg4 loop (shortened check cadence): append + 1-token attention."""
    b, hkv, hq, d = 8, 8, 32, 128
    cache = PreallocatedKVCache(b, hkv, 32768, d, device="cuda", dtype=torch.bfloat16)
    pk = _rand((b, hkv, 4096, d), torch.bfloat16, 60)
    pv = _rand((b, hkv, 4096, d), torch.bfloat16, 61)
    cache.append(pk, pv)
    for step in range(256):
        nk = _rand((b, hkv, 1, d), torch.bfloat16, 1000 + step)
        nv = _rand((b, hkv, 1, d), torch.bfloat16, 5000 + step)
        q = _rand((b, hq, 1, d), torch.bfloat16, 9000 + step)
        with torch.inference_mode():
            out = cache.append_and_attend(q, nk, nv)
        if step in (0, 127, 255):
            kv, vv = cache.view()
            exp, _ = oracle.forward(q, kv, vv, causal=False)
            check_close(out, exp, name=f"cfg4 step {step}")
    assert cache.length == 4096 + 256


def test_merge_partials_matches_oracle():
    import kotflash_b200._ext as ext

    lib = ext.load()
    torch.manual_seed(3)
    s, rows, d = 5, 37, 64
    po = torch.randn(s, rows, d, device="cuda")
    pl = torch.randn(s, rows, device="cuda") * 3
    pl[1, :5] = float("-inf")      # empty partials
    pl[:, 7] = float("-inf")       # a row with no keys at all
    out = torch.empty(rows, d, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(rows, device="cuda")
    rc = lib.kf_merge_partials(po.data_ptr(), pl.data_ptr(), s, rows, d, out.data_ptr(),
                               lse.data_ptr(), ext.KF_BF16, ext.stream_of(out))
    ext.check(rc, "kf_merge_partials")
    eo, el = oracle.merge_partials(po, pl)
    check_close(out, eo, name="merge O")
    check_close(lse, el, name="merge LSE")
