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
  reduce, triton_forward.py:287-349).  ``PeerExchange`` replaces the
  all-gather + merge over NVLink peer memory: the kernel that merges a
  rank's own splits stores the fp32 result straight into every peer's
  mailbox, and one more kernel merges what arrives in the rank's own.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _ext
from ._planning import cdiv, split_kv_plan


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


class PeerExchange:
    """Mailboxes in every rank's GPU memory, mapped by all ranks of one box.

    ``exchange(o, lse)`` sends this rank's partial ``o`` ([..., D], fp16/bf16)
    and ``lse`` (fp32, natural log) to every rank and returns the LSE merge of
    all ranks' partials (``kf_decode_peer_exchange``).  Every rank must call it
    in the same order with the same shapes; the call count lives in device
    memory, so the call may be captured in a CUDA graph.  A bounded wait
    (about one second) guards every arrival: on expiry the output is NaN and
    ``status()`` reports it.  The exchange is then unusable (the timed-out
    mailbox half is short of rows and a late sender may still write into it):
    after ``status()`` has returned non-zero, ``decode`` and ``exchange``
    raise, and every rank must ``close()`` it and build a new one, which
    starts from zeroed mailboxes.

    Build it after ``init_process_group`` (it all-gathers the CUDA IPC
    handles); with no process group it is a one-rank exchange.  The mailbox
    comes from the caching allocator and needs plain ``cudaMalloc`` memory
    (not ``expandable_segments``).
    """

    HANDLE_BYTES = 64

    def __init__(self, rows: int, d: int, dtype: torch.dtype, device=None, group=None):
        self.lib = _ext.load()
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        if dist.is_available() and dist.is_initialized():
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.rows, self.d, self.dtype = int(rows), int(d), dtype
        self.dtype_code = _ext.dtype_code(dtype)
        nbytes = self.lib.kf_peer_mailbox_bytes(self.world, self.rows, self.d)
        if nbytes == 0:
            raise ValueError(f"PeerExchange: unsupported world={self.world} rows={rows} d={d}")
        self.mailbox = torch.zeros(nbytes + 256, dtype=torch.uint8, device=self.device)
        base = self.mailbox.data_ptr()
        self.local = (base + 255) // 256 * 256
        self.status_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._failed = False
        torch.cuda.synchronize(self.device)  # zeros land before any peer can write
        handle = (ctypes.c_uint8 * self.HANDLE_BYTES)()
        offset = ctypes.c_uint64(0)
        _ext.check(self.lib.kf_ipc_get_handle(ctypes.c_void_p(self.local), handle, ctypes.byref(offset)),
                   "kf_ipc_get_handle")
        mine = (bytes(handle), int(offset.value))
        if self.world > 1:
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        self._opened = []
        ptrs = []
        error = ""
        for r, (h, off) in enumerate(allh):
            if r == self.rank:
                ptrs.append(self.local)
                continue
            hb = (ctypes.c_uint8 * self.HANDLE_BYTES).from_buffer_copy(h)
            p = ctypes.c_void_p()
            if self.lib.kf_ipc_open_handle(hb, ctypes.c_uint64(off), ctypes.byref(p)) != _ext.KF_OK:
                error = f"rank {self.rank} cannot map rank {r}'s mailbox: {_ext.last_error()}"
                break
            self._opened.append((p.value, off))
            ptrs.append(p.value)
        if self.world > 1:
            # every rank learns whether all mappings succeeded (the same collective on all ranks)
            ok = torch.tensor([0 if error else 1], dtype=torch.int32, device=self.device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if int(ok.item()) == 0:
                self.close()
                raise RuntimeError("PeerExchange: " + (error or "a peer could not map the mailboxes"))
        elif error:
            raise RuntimeError("PeerExchange: " + error)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)

    def decode(self, q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor, *,
               scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
        """Split-KV decode of this rank's key chunk fused with the exchange
        (``kf_decode_kv_split_peer``): the split kernel, one kernel that
        merges this rank's splits and stores the fp32 result into every
        mailbox, and the final merge.  Returns the full (O, LSE)."""
        self._check_usable()
        b, hq, sq, d = q.shape
        if q.dtype != self.dtype or d != self.d or b * hq * sq != self.rows:
            raise ValueError("PeerExchange.decode: q does not match the exchange's rows/d/dtype")
        hkv, sk = k_local.shape[1], k_local.shape[2]
        plan = split_kv_plan(sq, sk, d, causal=False, batch=b, q_heads=hq, kv_heads=hkv,
                             sm_count=_ext.sm_count(self.device.index))
        ws = self.lib.kf_decode_workspace_bytes(b, hq, sq, d, max(2, plan.num_splits))
        workspace = torch.empty(ws, dtype=torch.uint8, device=q.device)
        out = torch.empty((b, hq, sq, d), dtype=q.dtype, device=q.device)
        lse = torch.empty((b, hq, sq), dtype=torch.float32, device=q.device)
        rc = self.lib.kf_decode_kv_split_peer(
            _ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(k_local)), _ext.ref(_ext.t4(v_local)),
            _ext.ref(_ext.t4(out)), lse.data_ptr(), self.dtype_code, float(scale), int(plan.num_splits),
            workspace.data_ptr(), int(workspace.numel()), self.ptrs, self.world, self.rank,
            self.status_word.data_ptr(), _ext.stream_of(q))
        _ext.check(rc, "kf_decode_kv_split_peer")
        return out, lse

    def exchange(self, o: torch.Tensor, lse: torch.Tensor, out: torch.Tensor = None,
                 out_lse: torch.Tensor = None) -> Tuple[torch.Tensor, torch.Tensor]:
        self._check_usable()
        if o.dtype != self.dtype or o.shape[-1] != self.d or o[..., 0].numel() != self.rows:
            raise ValueError("PeerExchange.exchange: o does not match the exchange's rows/d/dtype")
        if lse.numel() != self.rows or lse.dtype != torch.float32:
            raise ValueError("PeerExchange.exchange: lse must be fp32 with one value per row")
        o = o.contiguous()
        lse = lse.contiguous()
        if out is None:
            out = torch.empty_like(o)
        if out_lse is None:
            out_lse = torch.empty(lse.shape, dtype=torch.float32, device=o.device)
        rc = self.lib.kf_decode_peer_exchange(o.data_ptr(), lse.data_ptr(), self.rows, self.d,
                                              self.dtype_code, self.ptrs, self.world, self.rank,
                                              out.data_ptr(), out_lse.data_ptr(),
                                              self.status_word.data_ptr(), _ext.stream_of(o))
        _ext.check(rc, "kf_decode_peer_exchange")
        return out, out_lse

    def status(self) -> int:
        """KF_DEV_TIMEOUT (1) once a wait expired, else 0 (synchronises).

        A non-zero answer retires the exchange: later ``decode``/``exchange``
        calls raise until a new ``PeerExchange`` replaces this one."""
        s = int(self.status_word.item())
        if s:
            self._failed = True
        return s

    def _check_usable(self) -> None:
        if self._failed:
            raise RuntimeError("PeerExchange: a peer wait timed out; close() this exchange on every "
                               "rank and build a new one (its mailboxes start zeroed)")

    def close(self) -> None:
        """Unmap the peers' mailboxes (every rank, after its last exchange)."""
        torch.cuda.synchronize(self.device)
        for p, off in self._opened:
            self.lib.kf_ipc_close_handle(ctypes.c_void_p(p), ctypes.c_uint64(off))
        self._opened = []


def decode_kv_split(q: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor, *,
                    scale: float, group=None,
                    exchange: PeerExchange = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Decode over a KV sequence split across ranks; every rank returns the full (O, LSE).

    ``k_local``/``v_local`` hold this rank's contiguous key chunk (see
    ``kv_chunk``).  With ``exchange`` (a ``PeerExchange`` built for
    ``B * Hq * Sq`` rows) the partials cross NVLink through peer memory;
    otherwise one NCCL all-gather of the packed partials, then the merge.
    """
    from .attention import _decode_forward

    if exchange is not None:
        return exchange.decode(q, k_local, v_local, scale=scale)
    o, lse = _decode_forward(q, k_local, v_local, scale=scale, want_lse=True)
    part_o, part_lse = gather_partials(pack_partial(o, lse), group)
    return merge_partials(part_o, part_lse, tuple(q.shape), q.dtype)
