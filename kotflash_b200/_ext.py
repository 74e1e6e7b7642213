# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of the C-ABI library ``libkotflash_b200.so``.

The library is built in-tree by ``python -m kotflash_b200.csrc.build`` (or
``__graft_entry__.build()``) into ``kotflash_b200/_lib/``.  Nothing here falls
back to another implementation: if the library is missing, every GPU entry
point raises ``RuntimeError``.

The entry points mirror the reference's native/launcher boundary:
``append_kv_`` (kotflash/csrc/kv_append.cpp:11-14), ``attention_forward``
(kotflash/kernels/triton_forward.py:372), ``attention_backward``
(kotflash/kernels/triton_backward.py:335) and
``attention_forward_strided_decode`` / ``attention_forward_strided_append``
(kotflash/kernels/triton_decode.py:412, :302).
"""
from __future__ import annotations

import ctypes
import os
import threading
from functools import lru_cache
from pathlib import Path
from typing import Optional, Tuple

import torch

LIB_NAME = "libkotflash_b200.so"
LIB_PATH = Path(__file__).resolve().parent / "_lib" / LIB_NAME

KF_OK = 0
KF_ERR_INVALID = 1
KF_ERR_UNSUPPORTED = 2
KF_ERR_CUDA = 3
KF_ERR_WORKSPACE = 4

KF_F16 = 0
KF_BF16 = 1


class KFTensor4(ctypes.Structure):
    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("size", ctypes.c_int64 * 4),
        ("stride", ctypes.c_int64 * 4),
    ]


_P = ctypes.POINTER
_T4 = _P(KFTensor4)
_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); exactly the declarations of include/kotflash_b200.h
SIGNATURES = {
    "kf_version": (_I, []),
    "kf_last_error": (ctypes.c_char_p, []),
    "kf_append": (_I, [_T4, _T4, _T4, _T4, _I64, _I, _VP]),
    "kf_attn_fwd": (_I, [_T4, _T4, _T4, _T4, _VP, _I, _F, _I, _VP, _VP]),
    "kf_attn_bwd_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64]),
    "kf_attn_bwd_workspace_bytes_kv": (_SZ, [_I64, _I64, _I64, _I64, _I64, _I64]),
    "kf_attn_bwd": (_I, [_T4, _T4, _T4, _T4, _VP, _T4, _T4, _T4, _T4, _I, _F, _I, _VP, _SZ,
                         _VP, _VP]),
    "kf_decode_num_splits": (_I, [_I64, _I64, _I64, _I64, _I64, _I64, _I]),
    "kf_decode_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _I]),
    "kf_decode": (_I, [_T4, _T4, _T4, _T4, _T4, _I64, _T4, _VP, _I, _F, _I, _VP, _SZ, _VP]),
    "kf_merge_partials": (_I, [_VP, _VP, _I, _I64, _I64, _VP, _VP, _I, _VP]),
    "kf_decode_noalloc": (_I, [_T4, _T4, _T4, _T4, _T4, _I64, _T4, _VP, _I, _F, _I, _VP]),
    "kf_selftest_bounded_wait": (_I, [_VP, _I64, _VP]),
    "kf_selftest_exp2_poly": (_I, [_VP, _VP, _I64, _VP]),
    "kf_peer_mailbox_bytes": (_SZ, [_I, _I64, _I64]),
    "kf_ipc_get_handle": (_I, [_VP, _VP, ctypes.POINTER(ctypes.c_uint64)]),
    "kf_ipc_open_handle": (_I, [_VP, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "kf_ipc_close_handle": (_I, [_VP, ctypes.c_uint64]),
    "kf_decode_peer_exchange": (_I, [_VP, _VP, _I64, _I64, _I, _VP, _I, _I, _VP, _VP, _VP, _VP]),
    "kf_decode_peer_put": (_I, [_VP, _VP, _I64, _I64, _I, _VP, _I, _I, _VP]),
    "kf_decode_peer_merge": (_I, [_VP, _I64, _I64, _I, _I, _VP, _VP, _VP, _VP]),
    "kf_decode_kv_split_peer": (_I, [_T4, _T4, _T4, _T4, _VP, _I, _F, _I, _VP, _SZ, _VP, _I, _I, _VP, _VP]),
    "kf_decode_kv_split_peer_send": (_I, [_T4, _T4, _T4, _I, _F, _I, _VP, _SZ, _VP, _I, _I, _VP]),
}

_load_lock = threading.Lock()


@lru_cache(maxsize=1)
def _load_cached() -> ctypes.CDLL:
    if not LIB_PATH.is_file():
        raise RuntimeError(
            f"kotflash_b200 CUDA library not found at {LIB_PATH}; build it with "
            "`python -m kotflash_b200.csrc.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def load() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raises if it is missing."""
    with _load_lock:
        return _load_cached()


def available() -> bool:
    try:
        load()
        return True
    except (RuntimeError, OSError):
        return False


def last_error() -> str:
    msg = load().kf_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc == KF_OK:
        return
    msg = last_error()
    if rc in (KF_ERR_INVALID,):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return KF_F16
    if dtype == torch.bfloat16:
        return KF_BF16
    raise TypeError(f"kotflash_b200 kernels support float16 and bfloat16, got {dtype}")


def t4(t: Optional[torch.Tensor]) -> Optional[KFTensor4]:
    """Describe a 4-D tensor (sizes and element strides) for the C ABI."""
    if t is None:
        return None
    if t.ndim != 4:
        raise ValueError("expected a 4-D tensor")
    d = KFTensor4()
    d.ptr = t.data_ptr()
    for i in range(4):
        d.size[i] = int(t.shape[i])
        d.stride[i] = int(t.stride(i))
    return d


def ref(d: Optional[KFTensor4]):
    return ctypes.byref(d) if d is not None else None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


_status_words = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels set when a bounded wait expires."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = w
    return w


def read_device_status(device: torch.device) -> int:
    """Synchronising read of the device status word (0 = no wait expired)."""
    return int(status_word(device).item())


def clear_device_status(device: torch.device) -> None:
    status_word(device).zero_()


@lru_cache(maxsize=16)
def sm_count(device_index: int) -> int:
    return torch.cuda.get_device_properties(device_index).multi_processor_count


@lru_cache(maxsize=16)
def is_sm100(device_index: int) -> bool:
    return torch.cuda.get_device_capability(device_index) == (10, 0)


def exported_symbols() -> Tuple[str, ...]:
    return tuple(SIGNATURES)
