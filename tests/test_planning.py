# SPDX-License-Identifier: Apache-2.0
"""CPU planning tests: the reference's split-KV partition invariant
(tests/test_planning.py:66-79) on the B200 planner, its envelope, the int32
guard, and agreement between the Python and C planners."""
import pytest

from kotflash_b200 import _ext
from kotflash_b200._planning import INT32_MAX, cdiv, check_int32_indexing, split_kv_plan


@pytest.mark.parametrize("sq,sk,d,causal", [(17, 4096, 64, False), (1, 4096, 64, True),
                                            (1, 4096, 136, False), (1, 4096, 8, False)])
def test_split_kv_envelope(sq, sk, d, causal):
    assert split_kv_plan(sq, sk, d, causal=causal) is None


def test_split_kv_partitions_without_gaps_or_empty_splits():
    lengths = [1, 2, 63, 64, 65, 1023] + list(range(1024, 3000, 7)) + [4096, 8191, 8192, 16384,
                                                                       20000, 131072, 1 << 20]
    for sk in lengths:
        for b, hq, hkv, sq, d in [(2, 8, 2, 1, 64), (8, 32, 8, 1, 128), (1, 4, 1, 16, 32),
                                  (2, 8, 2, 16, 64)]:
            plan = split_kv_plan(sq, sk, d, causal=False, batch=b, q_heads=hq, kv_heads=hkv)
            assert plan is not None and 1 <= plan.num_splits <= 512
            assert plan.chunk_n % plan.block_n == 0
            covered = 0
            for split in range(plan.num_splits):
                start = split * plan.chunk_n
                end = min(start + plan.chunk_n, sk)
                assert start == covered and start < end
                assert start + plan.blocks_per_split * plan.block_n >= end
                covered = end
            assert covered == sk


def test_split_kv_fills_the_gpu_for_long_contexts():
    plan = split_kv_plan(1, 131072, 64, causal=False, batch=2, q_heads=8, kv_heads=2)
    assert plan.num_splits * 2 * 2 >= 148  # at least one wave of 148 SMs


def test_python_and_c_planners_agree():
    lib = _ext.load()
    for sk in (1, 100, 1024, 4097, 32768, 131072):
        for b, hq, hkv, sq, d in [(2, 8, 2, 1, 64), (8, 32, 8, 1, 128), (2, 8, 2, 16, 64), (1, 3, 1, 5, 96)]:
            plan = split_kv_plan(sq, sk, d, causal=False, batch=b, q_heads=hq, kv_heads=hkv)
            assert lib.kf_decode_num_splits(b, hq, hkv, sq, sk, d, 148) == plan.num_splits


def test_cdiv_and_int32_index_guard():
    assert cdiv(0, 3) == 0 and cdiv(7, 3) == 3
    with pytest.raises(ValueError):
        cdiv(-1, 2)
    check_int32_indexing(q=INT32_MAX)
    with pytest.raises(ValueError, match="32-bit"):
        check_int32_indexing(q=INT32_MAX + 1)
    with pytest.raises(ValueError, match="non-negative"):
        check_int32_indexing(q=-1)
