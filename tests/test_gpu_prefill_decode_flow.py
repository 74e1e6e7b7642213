# SPDX-License-Identifier: Apache-2.0
"""The reference example's GQA prefill + fixed-capacity cache decode flow
(examples/gqa_kv_cache_decode.py:44-84) through the kernels: causal prefill
attention reading the cache's strided prefix view in place (K1), then decode
steps of append + attend (K4 + K3, and the fused K3 append), the decode steps
also captured once in a CUDA graph and replayed.  Checked against the fp32
oracle."""
import pytest
import torch

from kotflash_b200 import attention
from kotflash_b200.cache import PreallocatedKVCache
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", dtype=torch.float32, generator=g).to(dtype)


@pytest.mark.parametrize("b,hq,hkv,d,prefill,steps,dtype", [
    (2, 8, 2, 64, 2047, 4, torch.float16),      # the example's defaults (odd capacity)
    (1, 32, 8, 128, 1000, 3, torch.bfloat16),
])
def test_prefill_through_cache_view_then_decode(b, hq, hkv, d, prefill, steps, dtype):
    cache = PreallocatedKVCache(b, hkv, prefill + steps, d, device="cuda", dtype=dtype)
    qp = _rand((b, hq, prefill, d), dtype, 1)
    kp = _rand((b, hkv, prefill, d), dtype, 2)
    vp = _rand((b, hkv, prefill, d), dtype, 3)
    with torch.inference_mode():
        cache.append(kp, vp)
        pk, pv = cache.view()
        assert not pk.is_contiguous() or steps == 0
        out = attention(qp, pk, pv, causal=True, backend="triton")
    eo, _ = oracle.forward(qp, kp, vp, causal=True)
    check_close(out, eo, name=f"prefill over cache view {b},{hq},{hkv},{d},{prefill}")
    ks, vs = [kp], [vp]
    for step in range(steps):
        q = _rand((b, hq, 1, d), dtype, 100 + step)
        nk = _rand((b, hkv, 1, d), dtype, 200 + step)
        nv = _rand((b, hkv, 1, d), dtype, 300 + step)
        with torch.inference_mode():
            if step % 2 == 0:
                cache.append(nk, nv)
                o = cache.attend(q, backend="triton")
            else:
                o = cache.append_and_attend(q, nk, nv, append_backend="fused", attention_backend="triton")
        ks.append(nk)
        vs.append(nv)
        eo, _ = oracle.forward(q, torch.cat(ks, 2), torch.cat(vs, 2), causal=False)
        check_close(o, eo, name=f"decode step {step}")
    assert cache.length == prefill + steps


def test_decode_steps_replay_in_a_cuda_graph():
    # cfg4 geometry, shortened: 4096-token prefill, 16 fused append+decode steps in one graph
    b, hkv, hq, d, pre, steps = 8, 8, 32, 128, 4096, 16
    cache = PreallocatedKVCache(b, hkv, pre + steps, d, device="cuda", dtype=torch.bfloat16)
    kp = _rand((b, hkv, pre, d), torch.bfloat16, 11)
    vp = _rand((b, hkv, pre, d), torch.bfloat16, 12)
    cache.append(kp, vp)
    qs = _rand((steps, b, hq, 1, d), torch.bfloat16, 13)
    nks = _rand((steps, b, hkv, 1, d), torch.bfloat16, 14)
    nvs = _rand((steps, b, hkv, 1, d), torch.bfloat16, 15)
    outs = torch.empty(steps, b, hq, 1, d, dtype=torch.bfloat16, device="cuda")

    def loop():
        cache.length = pre
        for i in range(steps):
            with torch.inference_mode():
                outs[i].copy_(cache.append_and_attend(qs[i], nks[i], nvs[i]))

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        loop()  # warm-up
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        loop()
    outs.zero_()
    cache.k[:, :, pre:].zero_()
    cache.v[:, :, pre:].zero_()
    g.replay()
    torch.cuda.synchronize()
    k_all = torch.cat((kp, nks.permute(1, 2, 0, 3, 4).reshape(b, hkv, steps, d)), 2)
    v_all = torch.cat((vp, nvs.permute(1, 2, 0, 3, 4).reshape(b, hkv, steps, d)), 2)
    assert torch.equal(cache.k[:, :, pre:pre + steps], k_all[:, :, pre:])
    for i in (0, steps // 2, steps - 1):
        eo, _ = oracle.forward(qs[i], k_all[:, :, :pre + i + 1], v_all[:, :, :pre + i + 1], causal=False)
        check_close(outs[i], eo, name=f"graph decode step {i}")
    del g
