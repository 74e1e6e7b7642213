# SPDX-License-Identifier: Apache-2.0
"""Peer-memory exchange of decode partials (kf_decode_peer_put / _merge /
_exchange, and the fused kf_decode_kv_split_peer[_send]) vs the fp32 oracle.

On one GPU, W ranks are emulated by W mailboxes in this process: all sends
are launched first, then the merges, so every wait is on a counter that
earlier, already finished kernels filled.  The 2-GPU test runs real ranks
(one process per GPU, NVLS off) and skips when fewer GPUs are visible."""
import ctypes
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from kotflash_b200 import _ext
from kotflash_b200 import distributed as kd
from kotflash_b200.attention import _decode_forward
from oracle import attention_oracle as oracle
from tests._util import check_close

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, device="cuda", dtype=torch.float32, generator=g).to(dtype)


class _Mailboxes:
    """W zero-filled, 256-byte aligned mailboxes on this GPU (emulated ranks)."""

    def __init__(self, world, rows, d):
        lib = _ext.load()
        n = lib.kf_peer_mailbox_bytes(world, rows, d)
        assert n > 0
        self.bufs = [torch.zeros(n + 256, dtype=torch.uint8, device="cuda") for _ in range(world)]
        ptrs = [(b.data_ptr() + 255) // 256 * 256 for b in self.bufs]
        self.ptrs = (ctypes.c_void_p * world)(*ptrs)
        self.world, self.rows, self.d = world, rows, d


def _run_round(mb, parts, lses, outs, out_lses, status, dtype):
    lib = _ext.load()
    code = _ext.dtype_code(dtype)
    stream = torch.cuda.current_stream().cuda_stream
    for r in range(mb.world):
        _ext.check(lib.kf_decode_peer_put(parts[r].data_ptr(), lses[r].data_ptr(), mb.rows, mb.d, code,
                                          mb.ptrs, mb.world, r, stream), "kf_decode_peer_put")
    for r in range(mb.world):
        _ext.check(lib.kf_decode_peer_merge(mb.ptrs[r], mb.rows, mb.d, code, mb.world, outs[r].data_ptr(),
                                            out_lses[r].data_ptr(), status.data_ptr(), stream),
                   "kf_decode_peer_merge")


def _expected(parts, lses):
    po = torch.stack([p.float().reshape(-1, p.shape[-1]) for p in parts])
    pl = torch.stack([l.float().reshape(-1) for l in lses])
    return oracle.merge_partials(po, pl)


@pytest.mark.parametrize("world,rows,d,dtype", [
    (2, 16, 64, torch.float16),
    (3, 300, 64, torch.bfloat16),   # several pieces per sender
    (8, 256, 128, torch.float16),
    (4, 5, 8, torch.bfloat16),
    (8, 2048, 128, torch.bfloat16),  # 16 pieces per sender
])
def test_emulated_ranks_merge_matches_oracle(world, rows, d, dtype):
    mb = _Mailboxes(world, rows, d)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [torch.empty(rows, d, dtype=dtype, device="cuda") for _ in range(world)]
    out_lses = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(world)]
    for epoch in range(3):  # both mailbox halves, and back to the first
        parts = [_rand((rows, d), dtype, 100 * epoch + r) for r in range(world)]
        lses = [_rand((rows,), torch.float32, 50 + 100 * epoch + r) * 3.0 for r in range(world)]
        if epoch == 1:
            lses[0][: rows // 2] = float("-inf")  # an empty chunk on one rank
        _run_round(mb, parts, lses, outs, out_lses, status, dtype)
        eo, el = _expected(parts, lses)
        torch.cuda.synchronize()
        assert status.item() == 0
        for r in range(world):
            check_close(outs[r], eo, name=f"peer merge W{world} rank{r} epoch{epoch}", atol=1e-2, rtol=1e-2)
            torch.testing.assert_close(out_lses[r], el.to(out_lses[r].device), rtol=1e-5, atol=1e-5)


def _kv_split_inputs(world, sk, sq=4, dtype=torch.float16):
    # cfg3 shapes (B2 Hq8 Hkv2 D64), the KV sequence split over `world` ranks
    q = _rand((2, 8, sq, 64), dtype, 1)
    k = _rand((2, 2, sk, 64), dtype, 2)
    v = _rand((2, 2, sk, 64), dtype, 3)
    chunks = []
    for r in range(world):
        lo, hi = kd.kv_chunk(sk, world, r)
        chunks.append((k[:, :, lo:hi].contiguous(), v[:, :, lo:hi].contiguous()))
    return q, k, v, chunks


def test_emulated_kv_split_decode_via_put_matches_full_decode():
    world, sk = 4, 5000
    q, k, v, chunks = _kv_split_inputs(world, sk)
    parts, lses = [], []
    for kl, vl in chunks:
        o, lse = _decode_forward(q, kl, vl, scale=0.125, want_lse=True)
        parts.append(o)
        lses.append(lse)
    rows = 2 * 8 * 4
    mb = _Mailboxes(world, rows, 64)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [torch.empty_like(q) for _ in range(world)]
    out_lses = [torch.empty(2, 8, 4, dtype=torch.float32, device="cuda") for _ in range(world)]
    _run_round(mb, parts, lses, outs, out_lses, status, torch.float16)
    eo, el = oracle.forward(q, k, v, causal=False, scale=0.125)
    torch.cuda.synchronize()
    assert status.item() == 0
    for r in range(world):
        check_close(outs[r], eo, name=f"kv-split decode rank{r}")
        check_close(out_lses[r], el, name=f"kv-split lse rank{r}")


@pytest.mark.parametrize("world,sk,sq,dtype", [
    (2, 131072, 1, torch.float16),   # cfg3 long context
    (4, 5000, 4, torch.bfloat16),
    (8, 20000, 16, torch.float16),   # tensor-core decode kernel per rank
    (3, 700, 2, torch.bfloat16),     # one split per rank (partials forced)
])
def test_emulated_fused_kv_split_send_matches_full_decode(world, sk, sq, dtype):
    from kotflash_b200._planning import split_kv_plan

    lib = _ext.load()
    q, k, v, chunks = _kv_split_inputs(world, sk, sq, dtype)
    rows = 2 * 8 * sq
    mb = _Mailboxes(world, rows, 64)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    code = _ext.dtype_code(dtype)
    eo, el = oracle.forward(q, k, v, causal=False, scale=0.125)
    for epoch in range(2):
        keep = []
        for r, (kl, vl) in enumerate(chunks):
            plan = split_kv_plan(sq, kl.shape[2], 64, causal=False, batch=2, q_heads=8, kv_heads=2,
                                 sm_count=_ext.sm_count(0))
            ws = torch.empty(lib.kf_decode_workspace_bytes(2, 8, sq, 64, max(2, plan.num_splits)),
                             dtype=torch.uint8, device="cuda")
            keep.append(ws)
            _ext.check(lib.kf_decode_kv_split_peer_send(
                _ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(kl)), _ext.ref(_ext.t4(vl)), code, 0.125,
                int(plan.num_splits), ws.data_ptr(), int(ws.numel()), mb.ptrs, world, r, stream), "send")
        outs = [torch.empty(rows, 64, dtype=dtype, device="cuda") for _ in range(world)]
        out_lses = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(world)]
        for r in range(world):
            _ext.check(lib.kf_decode_peer_merge(mb.ptrs[r], rows, 64, code, world, outs[r].data_ptr(),
                                                out_lses[r].data_ptr(), status.data_ptr(), stream), "merge")
        torch.cuda.synchronize()
        assert status.item() == 0
        for r in range(world):
            check_close(outs[r].reshape(q.shape), eo, name=f"fused send W{world} Sq{sq} rank{r} epoch{epoch}")
            check_close(out_lses[r].reshape(q.shape[:-1]), el, name=f"fused send lse rank{r}")


def test_emulated_exchange_replays_in_a_cuda_graph():
    world, rows, d, dtype = 2, 64, 64, torch.bfloat16
    mb = _Mailboxes(world, rows, d)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    parts = [torch.zeros(rows, d, dtype=dtype, device="cuda") for _ in range(world)]
    lses = [torch.zeros(rows, dtype=torch.float32, device="cuda") for _ in range(world)]
    outs = [torch.empty(rows, d, dtype=dtype, device="cuda") for _ in range(world)]
    out_lses = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(world)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _run_round(mb, parts, lses, outs, out_lses, status, dtype)  # warm-up, epoch 1
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _run_round(mb, parts, lses, outs, out_lses, status, dtype)
    for it in range(5):  # the epoch advances in device memory on every replay
        for r in range(world):
            parts[r].copy_(_rand((rows, d), dtype, 7 * it + r))
            lses[r].copy_(_rand((rows,), torch.float32, 70 + 7 * it + r))
        g.replay()
        eo, el = _expected(parts, lses)
        torch.cuda.synchronize()
        assert status.item() == 0
        for r in range(world):
            check_close(outs[r], eo, name=f"graph replay {it} rank{r}", atol=1e-2, rtol=1e-2)
    del g


def test_missing_sender_times_out_with_status_and_nan():
    # rank 1 never puts: rank 0's merge waits on a flag that nothing sets, gives up
    # after its bounded wait (about one second), reports KF_DEV_TIMEOUT and writes NaN
    world, rows, d, dtype = 2, 8, 64, torch.float16
    mb = _Mailboxes(world, rows, d)
    lib = _ext.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    part = _rand((rows, d), dtype, 3)
    lse = torch.zeros(rows, dtype=torch.float32, device="cuda")
    out = torch.zeros(rows, d, dtype=dtype, device="cuda")
    out_lse = torch.zeros(rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    code = _ext.dtype_code(dtype)
    _ext.check(lib.kf_decode_peer_put(part.data_ptr(), lse.data_ptr(), rows, d, code, mb.ptrs, world, 0, stream),
               "put")
    _ext.check(lib.kf_decode_peer_merge(mb.ptrs[0], rows, d, code, world, out.data_ptr(), out_lse.data_ptr(),
                                        status.data_ptr(), stream), "merge")
    torch.cuda.synchronize()
    assert status.item() == 1
    assert torch.isnan(out.float()).all() and torch.isnan(out_lse).all()
    # the context stays usable
    x = torch.ones(1024, device="cuda")
    assert float(x.sum()) == 1024.0


def test_one_rank_peer_exchange_is_identity():
    ex = kd.PeerExchange(rows=32, d=64, dtype=torch.float16)
    assert ex.world == 1
    for i in range(3):
        o = _rand((2, 4, 4, 64), torch.float16, 40 + i)
        lse = _rand((2, 4, 4), torch.float32, 50 + i)
        out, out_lse = ex.exchange(o, lse)
        torch.cuda.synchronize()
        torch.testing.assert_close(out, o, rtol=0, atol=0)
        torch.testing.assert_close(out_lse, lse, rtol=1e-6, atol=1e-6)
    assert ex.status() == 0
    ex.close()


def test_one_rank_fused_decode_matches_single_gpu_decode():
    q, k, v, _ = _kv_split_inputs(1, 3000, 16, torch.bfloat16)
    ex = kd.PeerExchange(rows=2 * 8 * 16, d=64, dtype=torch.bfloat16)
    for _ in range(3):
        o, lse = kd.decode_kv_split(q, k, v, scale=0.125, exchange=ex)
        ro, rl = _decode_forward(q, k, v, scale=0.125, want_lse=True)
        torch.cuda.synchronize()
        torch.testing.assert_close(o, ro, rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(lse, rl, rtol=1e-5, atol=1e-5)
    assert ex.status() == 0
    ex.close()


def test_bad_arguments_are_rejected():
    lib = _ext.load()
    assert lib.kf_peer_mailbox_bytes(9, 16, 64) == 0
    assert lib.kf_peer_mailbox_bytes(0, 16, 64) == 0
    mb = _Mailboxes(2, 16, 64)
    x = torch.zeros(16, 64, dtype=torch.float16, device="cuda")
    l = torch.zeros(16, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.kf_decode_peer_put(x.data_ptr(), l.data_ptr(), 16, 60, 0, mb.ptrs, 2, 0, s) == _ext.KF_ERR_INVALID
    assert lib.kf_decode_peer_put(x.data_ptr(), l.data_ptr(), 16, 64, 0, mb.ptrs, 2, 2, s) == _ext.KF_ERR_INVALID
    assert lib.kf_decode_peer_merge(mb.ptrs[0] + 16, 16, 64, 0, 2, x.data_ptr(), None, None, s) == _ext.KF_ERR_INVALID


# ---------------------------------------------------------------------------- real ranks
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _two_gpu_worker(rank, world, port, errors):
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                                timeout=datetime.timedelta(seconds=60))
        sk = 20000
        q = _rand((2, 8, 16, 64), torch.float16, 1)
        k = _rand((2, 2, sk, 64), torch.float16, 2)
        v = _rand((2, 2, sk, 64), torch.float16, 3)
        lo, hi = kd.kv_chunk(sk, world, rank)
        kl, vl = k[:, :, lo:hi].contiguous(), v[:, :, lo:hi].contiguous()
        ex = kd.PeerExchange(rows=2 * 8 * 16, d=64, dtype=torch.float16)
        eo, el = oracle.forward(q, k, v, causal=False, scale=0.125)
        for it in range(3):
            po, pl = kd.decode_kv_split(q, kl, vl, scale=0.125, exchange=ex)
            no, nl = kd.decode_kv_split(q, kl, vl, scale=0.125)
            torch.cuda.synchronize()
            check_close(po, eo, name=f"peer rank{rank} it{it}")
            check_close(pl, el, name=f"peer lse rank{rank} it{it}")
            torch.testing.assert_close(po, no, rtol=1e-3, atol=1e-3)
        assert ex.status() == 0
        dist.barrier()
        ex.close()
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent
        errors.put(f"rank {rank}: {exc!r}")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_peer_exchange_matches_nccl_and_oracle():
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errors.empty():
        errs.append(errors.get())
    assert not alive, "a rank did not finish"
    assert not errs, "; ".join(errs)
    assert all(p.exitcode == 0 for p in procs)
