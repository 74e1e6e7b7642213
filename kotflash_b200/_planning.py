# SPDX-License-Identifier: Apache-2.0
"""Pure-Python launch planning for the B200 kernels (no torch imports).

Replaces the reference's ``kotflash/_planning.py``.  The helpers ``cdiv``,
``SplitKVPlan`` and ``check_int32_indexing`` keep the reference's names and
contracts (``_planning.py:11-46``).  ``split_kv_plan`` keeps the reference's
partition invariant (splits cover ``[0, Sk)`` with no gap and no empty split,
``tests/test_planning.py:66-79``) but is sized for a 148-SM B200 instead of a
40-SM T4: the split count fills about two CTAs per SM, where one CTA works
on one (split, batch, KV head) with every query row of the GQA group packed
together.  The reference's T4 exact-shape routing tables
(``_planning.py:49-76``) have no counterpart here.
"""
from __future__ import annotations

from typing import NamedTuple, Optional

INT32_MAX = 2**31 - 1

# Decode kernel tiling (kotflash_b200/csrc/decode.cu): keys per pipeline tile
# and the minimum number of keys a split should own.
DECODE_BLOCK_N = 64
DECODE_MIN_KEYS_PER_SPLIT = 64  # one K/V tile: a split's latency, not its length, sets short calls
DECODE_MAX_SQ = 16
DECODE_MAX_SPLITS = 512
DEFAULT_SM_COUNT = 148


def cdiv(a: int, b: int) -> int:
    if a < 0 or b <= 0:
        raise ValueError("cdiv expects a >= 0 and b > 0")
    return -(-a // b)


class SplitKVPlan(NamedTuple):
    block_m: int
    block_n: int
    num_splits: int
    chunk_n: int
    blocks_per_split: int


def decode_rows_per_cta(head_dim: int) -> int:
    """Packed query rows one decode CTA holds (fp32 accumulators fit registers)."""
    return 64 if head_dim <= 64 else 32


def split_kv_plan(
    sq: int,
    sk: int,
    d: int,
    *,
    causal: bool,
    batch: int = 1,
    q_heads: int = 1,
    kv_heads: int = 1,
    sm_count: int = DEFAULT_SM_COUNT,
) -> Optional[SplitKVPlan]:
    """Split-KV plan for short-query decode, or None outside the envelope.

    Envelope: non-causal, ``Sq <= 16``, ``16 <= D <= 128``.  Any ``Sk >= 1``.
    ``chunk_n`` is a multiple of the kernel's 64-key tile and the split count
    is recomputed from it, so no split is empty.
    """
    if min(sq, sk, d) <= 0:
        raise ValueError("sq, sk and d must be positive")
    if causal or sq > DECODE_MAX_SQ or d > 128 or d < 16:
        return None
    group = max(1, q_heads // max(1, kv_heads))
    rows = group * sq
    row_blocks = cdiv(rows, decode_rows_per_cta(d))
    units = batch * kv_heads * row_blocks
    target_ctas = 2 * sm_count
    max_by_len = max(1, cdiv(sk, DECODE_MIN_KEYS_PER_SPLIT))
    splits = max(1, min(cdiv(target_ctas, units), max_by_len, DECODE_MAX_SPLITS))
    chunk = cdiv(cdiv(sk, splits), DECODE_BLOCK_N) * DECODE_BLOCK_N
    splits = cdiv(sk, chunk)
    return SplitKVPlan(16, DECODE_BLOCK_N, splits, chunk, chunk // DECODE_BLOCK_N)


def check_int32_indexing(**numels: int) -> None:
    """Reject element counts above signed int32 (reference ``_planning.py:37-46``).

    The B200 kernels index with 64-bit offsets, so this guard is kept only for
    API compatibility; the library itself does not call it.
    """
    for name, n in numels.items():
        if isinstance(n, bool) or not isinstance(n, int) or n < 0:
            raise ValueError(f"{name} must be a non-negative integer element count")
        if n > INT32_MAX:
            raise ValueError(
                f"{name} has {n} elements; 32-bit offsets are limited to {INT32_MAX}"
            )
