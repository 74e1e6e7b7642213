# SPDX-License-Identifier: Apache-2.0
"""kf_decode_noalloc: the decode entry point for callers that cannot allocate.

Some hosts (a serving runtime that owns every device allocation, or an FFI
embedder with a fixed device-memory budget) give this library no allocator and
no workspace.  kf_decode_noalloc keeps its split partials in a static 8 MiB
device array instead.  This test calls it through the C ABI twice in a row,
on different shapes, and checks each result against the workspace-taking
kf_decode on the same inputs and against the fp32 oracle.  The file is named
to be collected last.
"""
import pytest
import torch

from kotflash_b200 import _ext
from oracle import attention_oracle as oracle
from tests._util import TOL, check_close

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", generator=g).to(dtype)


def _with_workspace(lib, q, k, v, num_splits):
    b, hq, sq, d = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(b, hq, sq, device="cuda", dtype=torch.float32)
    ws_bytes = lib.kf_decode_workspace_bytes(b, hq, sq, d, num_splits)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    rc = lib.kf_decode(_ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(k)), _ext.ref(_ext.t4(v)), None,
                       None, 0, _ext.ref(_ext.t4(out)), lse.data_ptr(), _ext.dtype_code(q.dtype),
                       float(d ** -0.5), num_splits, ws.data_ptr(), ws.numel(), _ext.stream_of(q))
    _ext.check(rc, "kf_decode")
    return out, lse


def _no_alloc(lib, q, k, v, num_splits):
    b, hq, sq, d = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(b, hq, sq, device="cuda", dtype=torch.float32)
    rc = lib.kf_decode_noalloc(_ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(k)), _ext.ref(_ext.t4(v)),
                               None, None, 0, _ext.ref(_ext.t4(out)), lse.data_ptr(),
                               _ext.dtype_code(q.dtype), float(d ** -0.5), num_splits,
                               _ext.stream_of(q))
    _ext.check(rc, "kf_decode_noalloc")
    return out, lse


def test_decode_noalloc_matches_decode_on_two_calls_in_a_row():
    lib = _ext.load()
    cases = [
        # (B, Hq, Hkv, Sq, Sk, D, dtype, seed)
        (2, 8, 2, 16, 32768, 64, torch.float16, 1),
        (8, 32, 8, 1, 4352, 128, torch.bfloat16, 2),
    ]
    for b, hq, hkv, sq, sk, d, dtype, seed in cases:
        q = _rand((b, hq, sq, d), dtype, seed)
        k = _rand((b, hkv, sk, d), dtype, seed + 10)
        v = _rand((b, hkv, sk, d), dtype, seed + 20)
        splits = lib.kf_decode_num_splits(b, hq, hkv, sq, sk, d, _ext.sm_count(0))
        want_o, want_lse = _with_workspace(lib, q, k, v, splits)
        got_o, got_lse = _no_alloc(lib, q, k, v, 0)
        torch.cuda.synchronize()
        check_close(got_o, want_o, name=f"no-alloc O {b},{hq},{hkv},{sq},{sk},{d}", atol=TOL, rtol=TOL)
        check_close(got_lse, want_lse, name=f"no-alloc LSE {b},{hq},{hkv},{sq},{sk},{d}", atol=TOL, rtol=TOL)
        # and against the fp32 oracle directly, not only through kf_decode
        exp_o, exp_lse = oracle.forward(q, k, v, causal=False, scale=d ** -0.5)
        check_close(got_o, exp_o, name=f"no-alloc O vs oracle {b},{hq},{hkv},{sq},{sk},{d}")
        check_close(got_lse, exp_lse, name=f"no-alloc LSE vs oracle {b},{hq},{hkv},{sq},{sk},{d}")


def test_decode_noalloc_rejects_splits_beyond_the_static_scratch():
    lib = _ext.load()
    q = _rand((2, 8, 16, 128), torch.float16, 3)
    k = _rand((2, 2, 65536, 128), torch.float16, 4)
    v = _rand((2, 2, 65536, 128), torch.float16, 5)
    out = torch.empty_like(q)
    # 512 splits x 256 rows x 129 x 4 bytes is about 67 MB > 8 MiB
    rc = lib.kf_decode_noalloc(_ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(k)), _ext.ref(_ext.t4(v)),
                               None, None, 0, _ext.ref(_ext.t4(out)), None,
                               _ext.dtype_code(q.dtype), 0.1, 512, _ext.stream_of(q))
    assert rc == _ext.KF_ERR_WORKSPACE
    assert "static maximum" in _ext.last_error()


def test_decode_noalloc_lowers_the_planned_split_count_to_fit():
    """B2 Hq256 Hkv128 Sq16 D128 Sk1024: the planner asks for 2 splits whose
    partials (2 x 4.2 MB) overflow the 8 MiB array, so the entry point lowers
    the count to what fits (1 split, written straight to O).  Its result must
    equal kf_decode's with that one split bit for bit, on two calls in a row."""
    lib = _ext.load()
    b, hq, hkv, sq, sk, d = 2, 256, 128, 16, 1024, 128
    planned = lib.kf_decode_num_splits(b, hq, hkv, sq, sk, d, _ext.sm_count(0))
    assert planned == 2
    per_split = b * hq * sq * (d + 1) * 4
    assert planned * per_split + 256 > 8 << 20  # the plan does not fit the static array
    q = _rand((b, hq, sq, d), torch.bfloat16, 7)
    k = _rand((b, hkv, sk, d), torch.bfloat16, 8)
    v = _rand((b, hkv, sk, d), torch.bfloat16, 9)
    want_o, want_lse = _with_workspace(lib, q, k, v, 1)
    for _ in range(2):
        got_o, got_lse = _no_alloc(lib, q, k, v, 0)
        torch.cuda.synchronize()
        assert torch.equal(got_o, want_o) and torch.equal(got_lse, want_lse)
