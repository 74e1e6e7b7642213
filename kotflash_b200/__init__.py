# SPDX-License-Identifier: Apache-2.0
"""kotflash_b200: the KOTFlash attention hot path, rebuilt for NVIDIA B200 (sm_100a).

Drop-in for the reference package's public surface (``kotflash/__init__.py``):
``attention``, ``triton_available`` and ``triton_turing_supported``, plus the
cache API in ``kotflash_b200.cache``.  ``import kotflash_b200 as kotflash``.
"""
from __future__ import annotations

from . import _ext
from .attention import attention
from .cache import PreallocatedKVCache, append_kv_cache, decode_step


def triton_available() -> bool:
    """Compat shim: True when the prebuilt sm_100a kernel library loads."""
    return _ext.available()


def triton_turing_supported() -> bool:
    """Compat shim: True when the kernel library loads and device 0 is sm_100."""
    import torch

    if not _ext.available() or not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(0) == (10, 0)


__all__ = [
    "attention",
    "triton_available",
    "triton_turing_supported",
    "PreallocatedKVCache",
    "append_kv_cache",
    "decode_step",
]
__version__ = "1.0.0"
