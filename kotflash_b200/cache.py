# SPDX-License-Identifier: Apache-2.0
"""Caller-managed KV-cache helpers for incremental decoding (B200 edition).

Mirrors ``kotflash/cache.py``: the concat helpers ``append_kv_cache`` and
``decode_step`` (``cache.py:42-88``), and ``PreallocatedKVCache``
(``cache.py:91-290``) with the same constructor, validation messages,
append-before-write guarantees and prefix views.  Appends go through the
vectorised append kernel (``kf_append``) and ``append_and_attend`` can fuse the
one-token append into the split-KV decode launch (``kf_decode``).  No paging
or eviction; not thread-safe.
"""
from __future__ import annotations

import os
from typing import Tuple, Union

import torch

from .attention import attention, strided_decode_supported


def _validate_kv_tensors(k_cache, v_cache, new_k, new_v) -> None:
    tensors = (k_cache, v_cache, new_k, new_v)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        raise TypeError("K/V cache and new K/V values must be torch.Tensor instances")
    if any(t.ndim != 4 for t in tensors):
        raise ValueError("All K/V tensors must use [B, Hkv, S, D] layout")
    if k_cache.shape != v_cache.shape:
        raise ValueError("K and V cache shapes must match")
    if k_cache.shape[0] <= 0 or k_cache.shape[1] <= 0 or k_cache.shape[3] <= 0:
        raise ValueError("K/V cache batch, head count and head dimension must be non-zero")
    if new_k.shape != new_v.shape:
        raise ValueError("New K and V shapes must match")
    if (
        k_cache.shape[0] != new_k.shape[0]
        or k_cache.shape[1] != new_k.shape[1]
        or k_cache.shape[3] != new_k.shape[3]
    ):
        raise ValueError("New K/V batch, head count and head dimension must match the cache")
    if any(t.device != k_cache.device for t in tensors):
        raise ValueError("All K/V tensors must be on the same device")
    if any(t.dtype != k_cache.dtype for t in tensors):
        raise ValueError("All K/V tensors must have the same dtype")
    if new_k.shape[2] == 0:
        raise ValueError("Appended K/V sequence length must be non-zero")


def append_kv_cache(k_cache, v_cache, new_k, new_v) -> Tuple[torch.Tensor, torch.Tensor]:
    """Append [B, Hkv, Snew, D] entries without mutating the old cache (torch.cat)."""
    _validate_kv_tensors(k_cache, v_cache, new_k, new_v)
    return torch.cat((k_cache, new_k), dim=2), torch.cat((v_cache, new_v), dim=2)


def decode_step(q_new, k_cache, v_cache, k_new, v_new, *, backend: str = "auto"):
    """Append one K/V token and attend with one newest query token (ref ``cache.py:57-88``)."""
    _validate_kv_tensors(k_cache, v_cache, k_new, v_new)
    if k_new.shape[2] != 1:
        raise ValueError("decode_step accepts exactly one new K/V token")
    if not isinstance(q_new, torch.Tensor) or q_new.ndim != 4:
        raise ValueError("q_new must use [B, Hq, 1, D] layout")
    if q_new.shape[2] != 1:
        raise ValueError("decode_step accepts exactly one new query token")
    if q_new.shape[0] != k_cache.shape[0] or q_new.shape[-1] != k_cache.shape[-1]:
        raise ValueError("Query batch and head dimension must match the KV cache")
    if q_new.shape[1] <= 0 or q_new.shape[1] % k_cache.shape[1] != 0:
        raise ValueError("Query heads must be non-zero and divisible by the cache KV-head count")
    if q_new.device != k_cache.device or q_new.dtype != k_cache.dtype:
        raise ValueError("Query device and dtype must match the KV cache")
    updated_k = torch.cat((k_cache, k_new), dim=2)
    updated_v = torch.cat((v_cache, v_new), dim=2)
    output = attention(q_new, updated_k, updated_v, causal=False, backend=backend)
    return output, updated_k, updated_v


def _kernel_append_ok(t: torch.Tensor) -> bool:
    from .attention import _kernel_device_ok

    return _kernel_device_ok(t) and t.dtype in (torch.float16, torch.bfloat16)


_APPEND_OPT_IN = "KOTFLASH_ENABLE_CUDA_APPEND"


def cuda_append_opted_in(env=None) -> bool:
    """Whether ``append(backend="auto")`` may use the append kernel.

    Same opt-in as the reference (``kotflash/cache.py:163-168``): only the
    exact value ``"1"`` of ``KOTFLASH_ENABLE_CUDA_APPEND`` selects the kernel;
    unset or any other value keeps the torch copies.  ``env`` overrides the
    process environment (used by tests).
    """
    value = os.environ.get(_APPEND_OPT_IN) if env is None else env
    return value == "1"


def fused_append_auto_allowed(env=None) -> bool:
    """Whether ``append_and_attend(append_backend="auto")`` may fuse the append.

    The reference turns its fused route off when the append-kernel opt-in is
    set (``kotflash/cache.py:248``): the caller then gets the separate append
    kernel followed by attention.
    """
    return not cuda_append_opted_in(env)


class PreallocatedKVCache:
    """Fixed-capacity K/V storage with append-only writes.

    ``view()`` returns storage-backed prefix views (non-contiguous once the
    cache is not full); the decode kernel reads them in place.
    ``contiguous_view()`` copies the populated prefix.  Not thread-safe; no
    paging or eviction.
    """

    def __init__(self, batch: int, kv_heads: int, max_len: int, head_dim: int, *,
                 device: Union[torch.device, str], dtype: torch.dtype) -> None:
        dims = {"batch": batch, "kv_heads": kv_heads, "max_len": max_len, "head_dim": head_dim}
        for name, value in dims.items():
            if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
                raise ValueError(f"{name} must be a positive integer")
        self.k = torch.empty((batch, kv_heads, max_len, head_dim), device=device, dtype=dtype)
        self.v = torch.empty_like(self.k)
        self.max_len = max_len
        self.length = 0

    def _check_new(self, new_k, new_v) -> None:
        if not isinstance(new_k, torch.Tensor) or not isinstance(new_v, torch.Tensor):
            raise TypeError("new_k and new_v must be torch.Tensor instances")
        if new_k.ndim != 4 or new_v.ndim != 4:
            raise ValueError("new K/V must use [B, Hkv, S, D] layout")
        if new_k.shape != new_v.shape:
            raise ValueError("new K and V shapes must match")
        if (new_k.shape[0] != self.k.shape[0] or new_k.shape[1] != self.k.shape[1]
                or new_k.shape[3] != self.k.shape[3]):
            raise ValueError("new K/V batch, heads and head_dim must match the cache")
        if new_k.shape[2] <= 0:
            raise ValueError("cannot append an empty K/V sequence")
        if new_k.device != self.k.device or new_v.device != self.v.device:
            raise ValueError("new K/V must be on the cache device")
        if new_k.dtype != self.k.dtype or new_v.dtype != self.v.dtype:
            raise ValueError("new K/V dtype must match the cache dtype")

    def append(self, new_k: torch.Tensor, new_v: torch.Tensor, *, backend: str = "auto") -> None:
        """Append positions after validation (ref ``cache.py:124-178``).

        backend="torch" uses tensor ``copy_``; backend="cuda" forces the
        append kernel (fp16/bf16 on an sm_100 device); backend="auto" uses the
        kernel for such tensors only when ``KOTFLASH_ENABLE_CUDA_APPEND=1``,
        the reference's opt-in, and the torch copies otherwise.
        """
        self._check_new(new_k, new_v)
        if backend not in {"auto", "torch", "cuda"}:
            raise ValueError("append backend must be one of: auto, torch or cuda")
        end = self.length + new_k.shape[2]
        if end > self.max_len:
            raise ValueError(
                f"KV cache full: {self.length} + {new_k.shape[2]} tokens "
                f"exceeds max_len={self.max_len}"
            )
        use_cuda = backend == "cuda" or (
            backend == "auto" and cuda_append_opted_in() and _kernel_append_ok(self.k)
        )
        if use_cuda:
            from ._cuda_append import append_kv_cuda

            append_kv_cuda(self.k, self.v, new_k, new_v, self.length)
        else:
            # All user-facing validation is complete before either buffer is written.
            self.k[:, :, self.length:end].copy_(new_k)
            self.v[:, :, self.length:end].copy_(new_v)
        self.length = end

    def view(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Storage-backed views of only the populated cache prefix."""
        if self.length == 0:
            raise ValueError("KV cache is empty")
        return self.k[:, :, :self.length, :], self.v[:, :, :self.length, :]

    def contiguous_view(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Contiguous copies of only the populated cache prefix."""
        k, v = self.view()
        return k.contiguous(), v.contiguous()

    def _check_query(self, q_new) -> None:
        if not isinstance(q_new, torch.Tensor) or q_new.ndim != 4 or q_new.shape[2] != 1:
            raise ValueError("q_new must use [B, Hq, 1, D] layout")
        if q_new.shape[0] != self.k.shape[0] or q_new.shape[-1] != self.k.shape[-1]:
            raise ValueError("Query batch and head dimension must match the cache")
        if q_new.shape[1] <= 0 or q_new.shape[1] % self.k.shape[1] != 0:
            raise ValueError("Query heads must be non-zero and divisible by the cache KV-head count")
        if q_new.device != self.k.device or q_new.dtype != self.k.dtype:
            raise ValueError("Query device and dtype must match the cache")

    def append_and_attend(self, q_new, new_k, new_v, *, append_backend: str = "auto",
                          attention_backend: str = "auto") -> torch.Tensor:
        """Append one token and attend without copying the cache prefix.

        append_backend="fused" (and "auto" for inference on fp16/bf16 sm_100
        tensors) writes the new row inside the split-KV decode launch; every
        split substitutes the new row from new_k/new_v, so no CTA reads a row
        another CTA is writing (ref ``triton_decode.py:109-238``).
        Grad-enabled calls use append + attention, and so does "auto" when
        ``KOTFLASH_ENABLE_CUDA_APPEND=1`` asks for the append kernel (as the
        reference routes it, ``kotflash/cache.py:248``).
        """
        if attention_backend not in {"auto", "triton", "sdpa"}:
            raise ValueError("attention backend must be one of: auto, triton or sdpa")
        if append_backend not in {"auto", "torch", "cuda", "fused"}:
            raise ValueError("append backend must be one of: auto, torch, cuda or fused")
        self._check_query(q_new)
        _validate_kv_tensors(self.k, self.v, new_k, new_v)
        if new_k.shape[2] != 1:
            raise ValueError("append_and_attend accepts exactly one new K/V token")
        end = self.length + 1
        if end > self.max_len:
            raise ValueError(f"KV cache full: {self.length} + 1 tokens exceeds max_len={self.max_len}")

        has_grad_inputs = torch.is_grad_enabled() and any(
            t.requires_grad for t in (q_new, new_k, new_v)
        )
        k_full = self.k[:, :, :end, :]
        v_full = self.v[:, :, :end, :]
        fusable = (
            attention_backend in {"auto", "triton"}
            and strided_decode_supported(q_new, k_full, v_full)
            and strided_decode_supported(q_new, new_k, new_v)
        )
        use_fused = append_backend == "fused" or (
            append_backend == "auto" and fusable and not has_grad_inputs
            and fused_append_auto_allowed()
        )
        if use_fused:
            if attention_backend == "sdpa":
                raise ValueError("append_backend='fused' requires attention_backend='auto' or 'triton'")
            if has_grad_inputs:
                raise RuntimeError("append_backend='fused' is inference-only; disable gradients")
            if not fusable:
                raise RuntimeError(
                    "fused append/decode requires fp16/bf16 CUDA tensors on an sm_100 device, "
                    "16 <= head_dim <= 128 with head_dim % 8 == 0"
                )
            from .attention import _decode_forward

            scale = 1.0 / (self.k.shape[-1] ** 0.5)
            out, _ = _decode_forward(q_new, k_full, v_full, scale=scale, want_lse=False,
                                     new_k=new_k, new_v=new_v, past_len=self.length)
            self.length = end
            return out

        self.append(new_k, new_v, backend=append_backend)
        return self.attend(q_new, backend=attention_backend)

    def attend(self, q_new: torch.Tensor, *, backend: str = "auto") -> torch.Tensor:
        """Attend one newest query token to the currently populated cache."""
        self._check_query(q_new)
        k, v = self.view()
        return attention(q_new, k, v, causal=False, backend=backend)
