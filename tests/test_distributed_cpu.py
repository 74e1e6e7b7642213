# SPDX-License-Identifier: Apache-2.0
"""Multi-rank host logic on CPU gloo ranks (world size 2): unit sharding,
KV-sequence split with the packed (O, LSE) all-gather and the merge, and a
rank that dies before the exchange (failure surfaces as an error, no hang)."""
import datetime
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kotflash_b200 import distributed as kd


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _kv_split_worker(rank, world, port, q, k, v, expected_o, expected_lse, errors):
    from oracle import attention_oracle as oracle

    try:
        _init(rank, world, port)
        lo, hi = kd.kv_chunk(k.shape[2], world, rank)
        o, lse = oracle.forward(q, k[:, :, lo:hi], v[:, :, lo:hi], causal=False)
        part_o, part_lse = kd.gather_partials(kd.pack_partial(o, lse))
        assert part_o.shape == (world, q.shape[0] * q.shape[1] * q.shape[2], q.shape[3])
        mo, ml = oracle.merge_partials(part_o, part_lse)
        torch.testing.assert_close(mo.reshape(q.shape), expected_o, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(ml.reshape(q.shape[:-1]), expected_lse, rtol=1e-5, atol=1e-5)
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent
        errors.put(f"rank {rank}: {exc!r}")


def test_kv_split_decode_allgather_merge_two_ranks():
    from oracle import attention_oracle as oracle

    torch.manual_seed(0)
    q = torch.randn(2, 8, 4, 64)
    k = torch.randn(2, 2, 1000, 64)
    v = torch.randn(2, 2, 1000, 64)
    eo, el = oracle.forward(q, k, v, causal=False)
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_kv_split_worker, args=(r, 2, port, q, k, v, eo, el, errors))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert errors.empty(), errors.get()


def _dead_peer_worker(rank, world, port, errors, results):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            os._exit(0)  # leaves before the exchange, between steps
        packed = kd.pack_partial(torch.zeros(1, 2, 1, 8), torch.zeros(1, 2, 1))
        try:
            kd.gather_partials(packed)
            results.put("no error")
        except Exception as exc:  # the collective must fail, not hang
            results.put(f"error: {type(exc).__name__}")
    except Exception as exc:
        errors.put(f"rank {rank}: {exc!r}")


def test_rank_that_dies_before_the_exchange_is_detected():
    ctx = mp.get_context("spawn")
    errors, results = ctx.Queue(), ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, errors, results))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert errors.empty(), errors.get()
    assert results.get(timeout=5).startswith("error")


@pytest.mark.parametrize("batch,kv_heads,world", [(4, 8, 1), (4, 8, 2), (4, 8, 8), (2, 4, 8), (3, 5, 4)])
def test_shard_units_cover_every_unit_once(batch, kv_heads, world):
    seen = []
    for r in range(world):
        mine = kd.shard_units(batch, kv_heads, world, r)
        seen.extend(mine)
        for b, hs, qs in kd.shard_slices(mine, group=4):
            assert qs.start == hs.start * 4 and qs.stop == hs.stop * 4
    assert sorted(seen) == [(b, h) for b in range(batch) for h in range(kv_heads)]
    sizes = [len(kd.shard_units(batch, kv_heads, world, r)) for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_kv_chunks_tile_the_sequence():
    for sk in (1, 64, 1000, 131072):
        for world in (1, 2, 4, 8):
            spans = [kd.kv_chunk(sk, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == sk
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
