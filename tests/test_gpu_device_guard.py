# SPDX-License-Identifier: Apache-2.0
"""Every C-ABI entry point runs on the GPU that owns its tensors, whatever
device the calling thread has current: the boundary's counterpart of the
reference extension's CUDAGuard (kotflash/csrc/kv_append_cuda.cu:77).
Tensors live on cuda:1 while cuda:0 is current; forward, backward, decode,
fused append + decode and the append kernel are checked against the fp32
oracle (bit-exact for the appends)."""
import pytest
import torch

from kotflash_b200 import _ext, attention
from kotflash_b200._cuda_append import append_kv_cuda
from kotflash_b200.attention import _decode_forward
from kotflash_b200.cache import PreallocatedKVCache
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                       reason="needs two CUDA devices"),
]


def _rand(shape, dtype, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(*shape, device=dev, generator=g).to(dtype)


def test_kernels_follow_the_tensors_device_not_the_current_one():
    dev = torch.device("cuda", 1)
    _ext.clear_device_status(dev)
    with torch.cuda.device(0):
        assert torch.cuda.current_device() == 0
        # forward + backward through the public API with autograd
        q = _rand((2, 8, 300, 64), torch.bfloat16, 1, dev).requires_grad_(True)
        k = _rand((2, 2, 300, 64), torch.bfloat16, 2, dev).requires_grad_(True)
        v = _rand((2, 2, 300, 64), torch.bfloat16, 3, dev).requires_grad_(True)
        do = _rand((2, 8, 300, 64), torch.bfloat16, 4, dev)
        out = attention(q, k, v, causal=True, backend="triton")
        dq, dk, dv = torch.autograd.grad(out, (q, k, v), do)
        eo, _, edq, edk, edv = oracle.forward_backward(q.detach(), k.detach(), v.detach(), do, causal=True)
        for name, got, want in (("O", out, eo), ("dQ", dq, edq), ("dK", dk, edk), ("dV", dv, edv)):
            assert got.device == dev
            check_close(got, want, name=f"cuda:1 {name}")
        assert torch.cuda.current_device() == 0

        # split-KV decode with LSE
        qd = _rand((2, 8, 4, 64), torch.float16, 5, dev)
        kd = _rand((2, 2, 5000, 64), torch.float16, 6, dev)
        vd = _rand((2, 2, 5000, 64), torch.float16, 7, dev)
        o, lse = _decode_forward(qd, kd, vd, scale=0.125, want_lse=True)
        eo, el = oracle.forward(qd, kd, vd, causal=False, scale=0.125)
        check_close(o, eo, name="cuda:1 decode O")
        check_close(lse, el, name="cuda:1 decode LSE")

        # append kernel and fused append + decode through the cache API
        cache = PreallocatedKVCache(1, 2, 256, 64, device=dev, dtype=torch.bfloat16)
        pk = _rand((1, 2, 100, 64), torch.bfloat16, 8, dev)
        pv = _rand((1, 2, 100, 64), torch.bfloat16, 9, dev)
        cache.append(pk, pv, backend="cuda")
        assert torch.equal(cache.k[:, :, :100], pk) and torch.equal(cache.v[:, :, :100], pv)
        qn = _rand((1, 8, 1, 64), torch.bfloat16, 10, dev)
        nk = _rand((1, 2, 1, 64), torch.bfloat16, 11, dev)
        nv = _rand((1, 2, 1, 64), torch.bfloat16, 12, dev)
        with torch.no_grad():
            got = cache.append_and_attend(qn, nk, nv, append_backend="fused")
        assert torch.equal(cache.k[:, :, 100:101], nk) and torch.equal(cache.v[:, :, 100:101], nv)
        kf, vf = cache.view()
        eo, _ = oracle.forward(qn, kf, vf, causal=False)
        check_close(got, eo, name="cuda:1 fused append + decode")

        kc = torch.zeros(1, 2, 64, 64, device=dev, dtype=torch.float16)
        vc = torch.zeros_like(kc)
        sk_ = _rand((1, 2, 5, 64), torch.float16, 13, dev)
        sv_ = _rand((1, 2, 5, 64), torch.float16, 14, dev)
        append_kv_cuda(kc, vc, sk_, sv_, 9)
        assert torch.equal(kc, oracle.append(torch.zeros_like(kc), sk_, 9))
        assert torch.equal(vc, oracle.append(torch.zeros_like(vc), sv_, 9))
        assert torch.cuda.current_device() == 0
    torch.cuda.synchronize(dev)
    assert _ext.read_device_status(dev) == 0
