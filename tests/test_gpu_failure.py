# SPDX-License-Identifier: Apache-2.0
"""Failure detection on the GPU without faulting it: a bounded device wait on a
barrier nothing completes expires, reports KF_DEV_TIMEOUT through the status
word, and the context stays usable for the next attention call."""
import pytest
import torch

from kotflash_b200 import _ext, attention
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def test_expired_device_wait_is_reported_and_context_survives():
    lib = _ext.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.kf_selftest_bounded_wait(status.data_ptr(), 20000, _ext.stream_of(status))  # 20 ms
    _ext.check(rc, "kf_selftest_bounded_wait")
    torch.cuda.synchronize()
    assert int(status.item()) == 1  # KF_DEV_TIMEOUT
    # the context is still healthy: a normal call runs and is correct
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(1, 4, 100, 64, device="cuda", generator=g).bfloat16()
    k = torch.randn(1, 2, 100, 64, device="cuda", generator=g).bfloat16()
    v = torch.randn(1, 2, 100, 64, device="cuda", generator=g).bfloat16()
    out = attention(q, k, v, causal=True, backend="triton")
    eo, _ = oracle.forward(q, k, v, causal=True)
    check_close(out, eo, name="after timeout")


def test_selftest_rejects_bad_arguments():
    lib = _ext.load()
    assert lib.kf_selftest_bounded_wait(None, 10, None) == _ext.KF_ERR_INVALID
