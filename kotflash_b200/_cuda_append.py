# SPDX-License-Identifier: Apache-2.0
"""One-launch K/V cache append through the prebuilt ``kf_append`` kernel.

Keeps the reference entry point ``append_kv_cuda(k_cache, v_cache, new_k,
new_v, start)`` (``kotflash/_cuda_append.py:31-44``) and its checks, but loads
the in-tree C-ABI library instead of JIT-building a pybind extension, and
accepts fp16 and bf16.
"""
from __future__ import annotations

import torch

from . import _ext


def append_kv_cuda(k_cache, v_cache, new_k, new_v, start: int) -> None:
    """Copy new_k/new_v [B,H,S,D] into the caches at sequence offset ``start``."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required for the KOTFlash append kernel")
    tensors = (k_cache, v_cache, new_k, new_v)
    if any(not t.is_cuda for t in tensors):
        raise ValueError("all cache and source tensors must be CUDA tensors")
    if any(t.dtype not in (torch.float16, torch.bfloat16) for t in tensors):
        raise TypeError("the CUDA append kernel supports FP16 and BF16 only")
    if any(t.dtype != k_cache.dtype for t in tensors):
        raise TypeError("cache and source tensors must share one dtype")
    if any(t.device != k_cache.device for t in tensors):
        raise ValueError("all cache and source tensors must be on the same CUDA device")
    lib = _ext.load()
    rc = lib.kf_append(
        _ext.ref(_ext.t4(k_cache)), _ext.ref(_ext.t4(v_cache)),
        _ext.ref(_ext.t4(new_k)), _ext.ref(_ext.t4(new_v)), int(start),
        _ext.dtype_code(k_cache.dtype), _ext.stream_of(k_cache),
    )
    _ext.check(rc, "kf_append")
