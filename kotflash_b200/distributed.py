# SPDX-License-Identifier: Apache-2.0
"""Box-level sharding of the attention hot path (one process per GPU).

The reference is single-GPU; this module adds the two partitions the work
allows:

* prefill / backward: independent (batch, KV-head group) units — a KV head and
  its query heads (``kv_head = q_head // (Hq // Hkv)``, reference
  kotflash/kernels/triton_forward.py:33; dK/dV sum over the same group,
  triton_backward.py:136-137).  Units are split across ranks with no
  communication (``shard_units`` / ``shard_slices``);
* long-context decode: the KV sequence is split into contiguous chunks, each
  rank computes a partial (O, LSE) over its chunk with the split-KV decode
  kernel, one all-gather exchanges the packed partials
  ``[B, Hq, Sq, D + 1]`` (fp32), and every rank merges them with the
  LSE-weighted merge kernel (the same math as the reference's split-KV
  reduce, triton_forward.py:287-349).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _ext
from ._planning import cdiv


def shard_units(batch: int, kv_heads: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """(batch, kv_head) units owned by ``rank``: a contiguous, balanced range."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    units = [(b, h) for b in range(batch) for h in range(kv_heads)]
    per, extra = divmod(len(units), world)
    start = rank * per + min(rank, extra)
    return units[start:start + per + (1 if rank < extra else 0)]


def shard_slices(units: Sequence[Tuple[int, int]], group: int):
    """Group a rank's units into (batch index, kv-head slice, q-head slice) runs."""
    runs = []
    for b, h in units:
        if runs and runs[-1][0] == b and runs[-1][1].stop == h:
            kv = slice(runs[-1][1].start, h + 1)
            runs[-1] = (b, kv, slice(kv.start * group, kv.stop * group))
        else:
            runs.append((b, slice(h, h + 1), slice(h * group, (h + 1) * group)))
    return runs


def kv_chunk(seq_len: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) key range of ``rank`` (64-key aligned, no gaps)."""
    chunk = cdiv(cdiv(seq_len, world), 64) * 64
    start = min(rank * chunk, seq_len)
    return start, min(start + chunk, seq_len)


def pack_partial(o: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    """[B, Hq, Sq, D] partial O + [B, Hq, Sq] LSE -> packed fp32 [B, Hq, Sq, D + 1]."""
    return torch.cat((o.float(), lse.float()[..., None]), dim=-1).contiguous()


def gather_partials(packed: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather the packed partials of every rank; returns ([W, rows, D], [W, rows])."""
    world = dist.get_world_size(group)
    # concatenated along dim 0 (the form both NCCL and gloo accept)
    out = torch.empty((world * packed.shape[0],) + tuple(packed.shape[1:]), dtype=packed.dtype,
                      device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)
    d = packed.shape[-1] - 1
    rows = packed[..., 0].numel()
    flat = out.reshape(world, rows, d + 1)
    return flat[..., :d].contiguous(), flat[..., d].contiguous()


def merge_partials(part_o: torch.Tensor, part_lse: torch.Tensor, out_shape, dtype):
    """LSE-weighted merge on the GPU (``kf_merge_partials``); returns (O, LSE)."""
    lib = _ext.load()
    s, rows, d = part_o.shape
    out = torch.empty(out_shape, dtype=dtype, device=part_o.device)
    lse = torch.empty(out_shape[:-1], dtype=torch.float32, device=part_o.device)
    rc = lib.kf_merge_partials(part_o.data_ptr(), part_lse.data_ptr(), s, rows, d,
                               out.data_ptr(), lse.data_ptr(), _ext.dtype_code(dtype),
                               _ext.stream_of(out))
    _ext.check(rc, "kf_merge_partials")
    return out, lse


def decode_kv_split(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor, *,
                    scale: float, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Decode over a KV sequence split across ranks; every rank returns the full (O, LSE).

    ``k_local``/``v_local`` hold this rank's contiguous key chunk (see
    ``kv_chunk``).  One NCCL all-gather of the packed partials, then the merge.
    """
    from .attention import _decode_forward

    o, lse = _decode_forward(q, k_local, v_local, scale=scale, want_lse=True)
    part_o, part_lse = gather_partials(pack_partial(o, lse), group)
    return merge_partials(part_o, part_lse, tuple(q.shape), q.dtype)
