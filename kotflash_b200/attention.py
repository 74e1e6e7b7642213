# SPDX-License-Identifier: Apache-2.0
"""Public attention API, B200 edition.

Mirrors ``kotflash/attention.py`` of the reference: same signature
(``attention(q, k, v, *, causal=False, scale=None, backend="auto")``,
``attention.py:223-231``), the same validation order and messages
(``_validate``, ``attention.py:21-45``; scale checks ``:252-264``), the same
``backend="sdpa"`` path (``_sdpa``/``_sdpa_kwargs``/``_sdpa_expanded``,
``:48-71,120-135``) and the PyTorch blockwise backward (``:138-201``).

``backend="triton"`` keeps its name for drop-in compatibility but routes to
the hand-written sm_100a CUDA kernels of ``libkotflash_b200.so``:

* short non-causal queries (``Sq <= 16``) without autograd go to the split-KV
  decode kernel, which reads padded KV-cache prefix views in place
  (replaces ``attention_forward_strided_decode``, ``triton_decode.py:412``);
* everything else goes through ``_FusedAttention``: the tcgen05 forward
  (O + LSE) and the fused backward (dQ/dK/dV).

``backend="auto"`` uses the same kernels for CUDA fp16/bf16 tensors on an
sm_100 device and PyTorch SDPA otherwise (CPU tensors, fp32, other GPUs),
as the reference's ``auto`` falls back to SDPA for unprofiled stacks
(``attention.py:303-312``).  On an sm_100 device the CUDA path never falls
back silently: a missing library raises.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from . import _ext
from ._planning import DECODE_MAX_SQ, split_kv_plan


def _validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    if not all(isinstance(x, torch.Tensor) for x in (q, k, v)):
        raise TypeError("q, k and v must be torch.Tensor instances")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("Expected q/k/v in [batch, heads, sequence, head_dim] layout")
    if q.shape[0] == 0:
        raise ValueError("Batch dimension must be non-zero")
    if q.shape[1] == 0 or k.shape[1] == 0:
        raise ValueError("Head dimensions must be non-zero")
    if q.shape[-1] == 0:
        raise ValueError("Head dimension must be non-zero")
    if q.shape[0] != k.shape[0] or q.shape[0] != v.shape[0]:
        raise ValueError("Batch dimensions must match")
    if k.shape != v.shape:
        raise ValueError("K and V shapes must match")
    if q.shape[-1] != k.shape[-1]:
        raise ValueError("Q/K/V head dimensions must match")
    if q.shape[1] % k.shape[1] != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads (GQA/MQA)")
    if q.device != k.device or q.device != v.device:
        raise ValueError("Q/K/V must be on the same device")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("Q/K/V dtypes must match")
    if q.shape[2] == 0 or k.shape[2] == 0:
        raise ValueError("Sequence dimensions must be non-zero")


def _sdpa_kwargs(q, *, causal: bool, scale: Optional[float]):
    """SDPA kwargs that keep PyTorch's default-scale dispatch (ref ``:48-61``)."""
    kwargs = {"attn_mask": None, "dropout_p": 0.0, "is_causal": causal}
    default_scale = 1.0 / math.sqrt(q.shape[-1])
    if scale is not None and not math.isclose(scale, default_scale, rel_tol=0.0, abs_tol=1e-12):
        kwargs["scale"] = scale
    return kwargs


def _sdpa_expanded(q, k, v, *, causal: bool, scale: Optional[float]):
    """SDPA after expanding grouped KV heads (ref ``:64-71``)."""
    if q.shape[1] != k.shape[1]:
        repeat = q.shape[1] // k.shape[1]
        k = k.repeat_interleave(repeat, dim=1)
        v = v.repeat_interleave(repeat, dim=1)
    return F.scaled_dot_product_attention(q, k, v, **_sdpa_kwargs(q, causal=causal, scale=scale))


def _sdpa(q, k, v, *, causal: bool, scale: Optional[float]):
    """Native-GQA SDPA, expanding heads only on old PyTorch (ref ``:120-135``)."""
    kwargs = _sdpa_kwargs(q, causal=causal, scale=scale)
    if q.shape[1] != k.shape[1]:
        try:
            return F.scaled_dot_product_attention(q, k, v, enable_gqa=True, **kwargs)
        except TypeError as exc:
            if "enable_gqa" not in str(exc):
                raise
            repeat = q.shape[1] // k.shape[1]
            k = k.repeat_interleave(repeat, dim=1)
            v = v.repeat_interleave(repeat, dim=1)
    return F.scaled_dot_product_attention(q, k, v, **kwargs)


def _blockwise_backward(
    q, k, v, out, lse, grad_out, *, causal: bool, scale: float,
    q_block: int = 64, kv_block: int = 128,
):
    """Memory-bounded PyTorch backward (ref ``attention.py:138-201``).

    Recomputes score tiles from (q, k, LSE) instead of storing the S x S
    matrix; grouped KV gradients are summed back onto their shared KV head.
    """
    bsz, hq, sq, d = q.shape
    _, hkv, sk, _ = k.shape
    group = hq // hkv
    qf, kf, vf = q.float(), k.float(), v.float()
    of, dof, lsef = out.float(), grad_out.float(), lse.float()
    dq = torch.zeros_like(qf)
    dk = torch.zeros_like(kf)
    dv = torch.zeros_like(vf)
    for qs in range(0, sq, q_block):
        qe = min(qs + q_block, sq)
        qb, dob, lseb = qf[:, :, qs:qe], dof[:, :, qs:qe], lsef[:, :, qs:qe]
        delta = (of[:, :, qs:qe] * dob).sum(dim=-1)
        dq_block = torch.zeros_like(qb)
        qpos = torch.arange(qs, qe, device=q.device)
        for ks in range(0, sk, kv_block):
            ke = min(ks + kv_block, sk)
            kb = kf[:, :, ks:ke].repeat_interleave(group, dim=1)
            vb = vf[:, :, ks:ke].repeat_interleave(group, dim=1)
            scores = torch.matmul(qb, kb.transpose(-2, -1)) * scale
            if causal:
                kpos = torch.arange(ks, ke, device=q.device)
                scores = scores.masked_fill(
                    kpos[None, None, None, :] > qpos[None, None, :, None], float("-inf")
                )
            p = torch.nan_to_num(torch.exp(scores - lseb[..., None]), nan=0.0, posinf=0.0,
                                 neginf=0.0)
            dp = torch.matmul(dob, vb.transpose(-2, -1))
            ds = p * (dp - delta[..., None])
            dq_block.add_(torch.matmul(ds, kb) * scale)
            dk_g = torch.matmul(ds.transpose(-2, -1), qb)
            dv_g = torch.matmul(p.transpose(-2, -1), dob)
            dk[:, :, ks:ke].add_(dk_g.reshape(bsz, hkv, group, ke - ks, d).sum(dim=2) * scale)
            dv[:, :, ks:ke].add_(dv_g.reshape(bsz, hkv, group, ke - ks, d).sum(dim=2))
        dq[:, :, qs:qe] = dq_block
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


# ----------------------------------------------------------------------------
# CUDA path
# ----------------------------------------------------------------------------

def _kernel_device_ok(t: torch.Tensor) -> bool:
    if not t.is_cuda:
        return False
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    return _ext.is_sm100(idx)


def cuda_supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """Whether the sm_100a kernels accept these (already validated) inputs."""
    return (
        _kernel_device_ok(q)
        and q.dtype in (torch.float16, torch.bfloat16)
        and 16 <= q.shape[-1] <= 128
    )


def strided_decode_supported(q, k, v) -> bool:
    """Layout predicate of the split-KV decode kernel.

    Generalises ``strided_decode_supported`` (ref ``triton_decode.py:389-409``):
    any short query (``Sq <= 16``) over K/V views whose last dimension is
    contiguous with 16-byte aligned rows; the prefix may sit inside a larger
    preallocated cache.  fp16 and bf16, ``16 <= D <= 128``, any ``Sk``.
    """
    if not all(isinstance(t, torch.Tensor) for t in (q, k, v)):
        return False
    if q.ndim != 4 or k.ndim != 4 or v.shape != k.shape:
        return False
    if not cuda_supported(q, k, v) or k.dtype != q.dtype or v.dtype != q.dtype:
        return False
    if q.shape[2] > DECODE_MAX_SQ or q.shape[0] != k.shape[0] or q.shape[1] % k.shape[1]:
        return False
    d = q.shape[-1]
    for t in (q, k, v):
        if t.stride(3) != 1 or t.data_ptr() % 16:
            return False
        if any((t.stride(i) * t.element_size()) % 16 for i in range(3) if t.shape[i] > 1):
            return False
    return d % 8 == 0


def _decode_forward(q, k, v, *, scale: float, want_lse: bool, new_k=None, new_v=None,
                    past_len: int = 0):
    """Split-KV decode through ``kf_decode``; returns (O, LSE or None)."""
    lib = _ext.load()
    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    dev = q.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    plan = split_kv_plan(sq, sk, d, causal=False, batch=b, q_heads=hq, kv_heads=hkv,
                         sm_count=_ext.sm_count(idx))
    ws_bytes = lib.kf_decode_workspace_bytes(b, hq, sq, d, plan.num_splits)
    workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    out = torch.empty((b, hq, sq, d), dtype=q.dtype, device=dev)
    lse = torch.empty((b, hq, sq), dtype=torch.float32, device=dev) if want_lse else None
    rc = lib.kf_decode(
        _ext.ref(_ext.t4(q)), _ext.ref(_ext.t4(k)), _ext.ref(_ext.t4(v)),
        _ext.ref(_ext.t4(new_k)), _ext.ref(_ext.t4(new_v)), int(past_len),
        _ext.ref(_ext.t4(out)), lse.data_ptr() if lse is not None else None,
        _ext.dtype_code(q.dtype), float(scale), int(plan.num_splits),
        workspace.data_ptr(), int(workspace.numel()), _ext.stream_of(q),
    )
    _ext.check(rc, "kf_decode")
    return out, lse


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """Return t, or a contiguous copy when its strides are not TMA-legal."""
    ok = t.stride(3) == 1 and t.data_ptr() % 16 == 0 and all(
        (t.stride(i) * t.element_size()) % 16 == 0 for i in range(3) if t.shape[i] > 1
    )
    return t if ok else t.contiguous()


def _pad_head_dim(t: torch.Tensor, d_pad: int) -> torch.Tensor:
    return F.pad(t, (0, d_pad - t.shape[-1])) if t.shape[-1] != d_pad else t


def attention_forward(q, k, v, *, causal: bool, scale: float):
    """Run the sm_100a forward; returns ``(out, lse)`` with LSE in fp32.

    Same contract as the reference launcher ``attention_forward``
    (``triton_forward.py:372-456``).  Head dims that are not a multiple of 8
    are zero-padded (exact: zero columns add nothing to Q.K and produce
    zero output columns that are sliced away).
    """
    lib = _ext.load()
    d = q.shape[-1]
    d_pad = (d + 7) // 8 * 8
    qp, kp, vp = (_tma_ready(_pad_head_dim(t, d_pad)) for t in (q, k, v))
    b, hq, sq, _ = q.shape
    out = torch.empty((b, hq, sq, d_pad), dtype=q.dtype, device=q.device)
    lse = torch.empty((b, hq, sq), dtype=torch.float32, device=q.device)
    rc = lib.kf_attn_fwd(
        _ext.ref(_ext.t4(qp)), _ext.ref(_ext.t4(kp)), _ext.ref(_ext.t4(vp)),
        _ext.ref(_ext.t4(out)), lse.data_ptr(), _ext.dtype_code(q.dtype), float(scale),
        int(bool(causal)), _ext.status_word(q.device).data_ptr(), _ext.stream_of(q),
    )
    _ext.check(rc, "kf_attn_fwd")
    if d_pad != d:
        out = out[..., :d].contiguous()
    return out, lse


def attention_backward(q, k, v, out, lse, grad_out, *, causal: bool, scale: float):
    """Run the sm_100a backward; returns ``(dq, dk, dv)`` in the input dtype.

    Same contract as the reference launcher ``attention_backward``
    (``triton_backward.py:335-421``).
    """
    lib = _ext.load()
    d = q.shape[-1]
    d_pad = (d + 7) // 8 * 8
    qp, kp, vp, op, dop = (
        _tma_ready(_pad_head_dim(t, d_pad)) for t in (q, k, v, out, grad_out)
    )
    b, hq, sq, _ = q.shape
    dq = torch.empty((b, hq, sq, d_pad), dtype=q.dtype, device=q.device)
    dk = torch.empty(kp.shape, dtype=k.dtype, device=q.device)
    dv = torch.empty(vp.shape, dtype=v.dtype, device=q.device)
    ws_bytes = lib.kf_attn_bwd_workspace_bytes_kv(b, hq, kp.shape[1], sq, kp.shape[2], d_pad)
    workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
    lse_c = lse.contiguous()
    rc = lib.kf_attn_bwd(
        _ext.ref(_ext.t4(qp)), _ext.ref(_ext.t4(kp)), _ext.ref(_ext.t4(vp)),
        _ext.ref(_ext.t4(op)), lse_c.data_ptr(), _ext.ref(_ext.t4(dop)),
        _ext.ref(_ext.t4(dq)), _ext.ref(_ext.t4(dk)), _ext.ref(_ext.t4(dv)),
        _ext.dtype_code(q.dtype), float(scale), int(bool(causal)),
        workspace.data_ptr(), int(workspace.numel()),
        _ext.status_word(q.device).data_ptr(), _ext.stream_of(q),
    )
    _ext.check(rc, "kf_attn_bwd")
    if d_pad != d:
        dq, dk, dv = (t[..., :d].contiguous() for t in (dq, dk, dv))
    return dq, dk, dv


class _FusedAttention(torch.autograd.Function):
    """Autograd boundary (replaces ``_TritonAttention``, ref ``attention.py:203-220``)."""

    @staticmethod
    def forward(ctx, q, k, v, causal: bool, scale: float):
        if not causal and q.shape[2] <= DECODE_MAX_SQ and strided_decode_supported(q, k, v):
            out, lse = _decode_forward(q, k, v, scale=scale, want_lse=True)
        else:
            out, lse = attention_forward(q, k, v, causal=causal, scale=scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal = causal
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = attention_backward(
            q, k, v, out, lse, grad_out, causal=ctx.causal, scale=ctx.scale
        )
        return dq, dk, dv, None, None


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = False,
    scale: Optional[float] = None,
    backend: str = "auto",
) -> torch.Tensor:
    """Scaled dot-product attention with MHA, GQA and MQA support.

    Tensors use [batch, heads, sequence, head_dim] layout; Hq must be
    divisible by Hkv.  The causal mask is upper-left aligned (key position
    <= query position), matching PyTorch SDPA.  backend is one of auto,
    triton or sdpa; "triton" names the sm_100a CUDA kernels (fp16/bf16,
    16 <= head_dim <= 128, CUDA device of compute capability 10.0).
    """
    _validate(q, k, v)
    if not isinstance(causal, bool):
        raise TypeError("causal must be a bool")
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    else:
        try:
            scale = float(scale)
        except (TypeError, ValueError) as exc:
            raise TypeError("scale must be a finite real number or None") from exc
        if not math.isfinite(scale):
            raise ValueError("scale must be finite")
    if backend not in {"auto", "triton", "sdpa"}:
        raise ValueError("backend must be one of: auto, triton, sdpa")

    use_kernels = backend == "triton" or (backend == "auto" and cuda_supported(q, k, v))
    if backend == "triton" and not cuda_supported(q, k, v):
        raise RuntimeError(
            "CUDA kernel backend requires an sm_100 (B200) CUDA device, FP16 or BF16 "
            "and 16 <= head_dim <= 128"
        )
    if use_kernels:
        needs_grad = torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v))
        if not needs_grad and not causal and strided_decode_supported(q, k, v):
            out, _ = _decode_forward(q, k, v, scale=float(scale), want_lse=False)
            return out
        return _FusedAttention.apply(q, k, v, causal, float(scale))
    return _sdpa(q, k, v, causal=causal, scale=scale)
