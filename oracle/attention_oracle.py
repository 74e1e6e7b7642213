# SPDX-License-Identifier: Apache-2.0
"""CPU oracle for the KOTFlash attention hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker.  The product path
(``kotflash_b200``) never calls it.

This is a plain fp32 restatement of the reference's own CPU path for each
piece of the hot path, written from the mathematics rather than copied:

* forward O: the ``backend="sdpa"`` route (kotflash/attention.py:120-135),
  i.e. softmax(scale * Q K^T + mask) V with GQA head map
  ``kv_head = q_head // (Hq // Hkv)`` and an upper-left causal mask
  (key j visible to query i iff j <= i, attention.py:232-236);
* LSE: ``logsumexp(scale * Q K^T)`` over visible keys, natural log, as the
  reference tests compute it (tests/test_attention.py:90-91, 109-112);
* backward: the formulas of ``_blockwise_backward`` (attention.py:138-201):
  P = exp(S - LSE), dP = dO V^T, Delta = rowsum(O * dO), dS = P (dP - Delta),
  dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO, with dK/dV summed over
  each KV head's query-head group;
* split-KV partials and their merge: ``_attention_fwd_split_kv`` and
  ``_attention_fwd_split_kv_reduce`` (kotflash/kernels/triton_forward.py:
  196-246, 287-349) — empty split -> (O = 0, LSE = -inf); merge weights
  w_s = exp(lse_s - max) / sum;
* KV append: ``cache[:, :, start:start+S] = new`` (kotflash/cache.py:176-177).

Parity of this restatement is pinned against outputs of the reference package
itself (``tests/golden/make_golden.py`` imports it and records fixtures).
Works on any torch device (tests run it on CUDA for full-size checks).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import torch


def _expand_kv(x: torch.Tensor, hq: int) -> torch.Tensor:
    group = hq // x.shape[1]
    return x.repeat_interleave(group, dim=1)


def _mask(sq: int, sk: int, causal: bool, device) -> Optional[torch.Tensor]:
    if not causal:
        return None
    qpos = torch.arange(sq, device=device)[:, None]
    kpos = torch.arange(sk, device=device)[None, :]
    return kpos > qpos  # True = hidden


def scores(q, k, *, causal: bool, scale: float) -> torch.Tensor:
    """fp32 scale * Q K^T with -inf at hidden (q, k) pairs; [B, Hq, Sq, Sk]."""
    qf = q.float()
    kf = _expand_kv(k.float(), q.shape[1])
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    m = _mask(q.shape[2], k.shape[2], causal, q.device)
    if m is not None:
        s = s.masked_fill(m, float("-inf"))
    return s


def forward(q, k, v, *, causal: bool, scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 (O, LSE) of scaled dot-product attention."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    s = scores(q, k, causal=causal, scale=scale)
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.matmul(p, _expand_kv(v.float(), q.shape[1]))
    return o, lse


def backward(q, k, v, o, lse, do, *, causal: bool, scale: Optional[float] = None):
    """fp32 (dQ, dK, dV) from saved O and LSE."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    group = hq // hkv
    qf, of, dof = q.float(), o.float(), do.float()
    kf = _expand_kv(k.float(), hq)
    vf = _expand_kv(v.float(), hq)
    s = scores(q, k, causal=causal, scale=scale)
    p = torch.nan_to_num(torch.exp(s - lse.float()[..., None]), nan=0.0)
    dp = torch.matmul(dof, vf.transpose(-2, -1))
    delta = (of * dof).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    dq = torch.matmul(ds, kf) * scale
    dk = torch.matmul(ds.transpose(-2, -1), qf) * scale
    dv = torch.matmul(p.transpose(-2, -1), dof)
    dk = dk.reshape(b, hkv, group, sk, d).sum(2)
    dv = dv.reshape(b, hkv, group, sk, d).sum(2)
    return dq, dk, dv


def forward_backward(q, k, v, do, *, causal: bool, scale: Optional[float] = None):
    o, lse = forward(q, k, v, causal=causal, scale=scale)
    dq, dk, dv = backward(q, k, v, o, lse, do, causal=causal, scale=scale)
    return o, lse, dq, dk, dv


def forward_backward_chunked(q, k, v, do, *, causal: bool, scale: Optional[float] = None,
                             chunk: int = 1024):
    """``forward_backward`` computed one query head and ``chunk`` query rows
    at a time, so memory stays O(chunk x Sk) at long sequence lengths (the
    16384-token training config).  Same formulas, fp32; returns
    (O, LSE, dQ, dK, dV)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    group = hq // hkv
    dev = q.device
    o = torch.empty(b, hq, sq, d, device=dev)
    lse = torch.empty(b, hq, sq, device=dev)
    dq = torch.empty(b, hq, sq, d, device=dev)
    dk = torch.zeros(b, hkv, sk, d, device=dev)
    dv = torch.zeros(b, hkv, sk, d, device=dev)
    kpos = torch.arange(sk, device=dev)[None, :]
    for bi in range(b):
        for h in range(hq):
            g = h // group
            kh, vh = k[bi, g].float(), v[bi, g].float()
            for r0 in range(0, sq, chunk):
                r1 = min(sq, r0 + chunk)
                qc, dc = q[bi, h, r0:r1].float(), do[bi, h, r0:r1].float()
                s = torch.matmul(qc, kh.t()) * scale
                if causal:
                    s = s.masked_fill(kpos > torch.arange(r0, r1, device=dev)[:, None], float("-inf"))
                l = torch.logsumexp(s, dim=-1)
                p = torch.nan_to_num(torch.exp(s - l[:, None]), nan=0.0)
                oc = torch.matmul(p, vh)
                ds = p * (torch.matmul(dc, vh.t()) - (oc * dc).sum(-1, keepdim=True))
                o[bi, h, r0:r1] = oc
                lse[bi, h, r0:r1] = l
                dq[bi, h, r0:r1] = torch.matmul(ds, kh) * scale
                dk[bi, g] += torch.matmul(ds.t(), qc) * scale
                dv[bi, g] += torch.matmul(p.t(), dc)
    return o, lse, dq, dk, dv


def split_partials(q, k, v, *, scale: float, bounds: Sequence[Tuple[int, int]]):
    """Per-split (O normalised, LSE) over key ranges ``bounds`` (non-causal)."""
    outs, lses = [], []
    for start, end in bounds:
        if end <= start:
            shape = q.shape[:-1]
            outs.append(torch.zeros(*shape, q.shape[-1], device=q.device))
            lses.append(torch.full(shape, float("-inf"), device=q.device))
            continue
        o, l = forward(q, k[:, :, start:end], v[:, :, start:end], causal=False, scale=scale)
        outs.append(o)
        lses.append(l)
    return torch.stack(outs), torch.stack(lses)


def merge_partials(part_o: torch.Tensor, part_lse: torch.Tensor):
    """LSE-weighted merge over dim 0; all-empty rows give (0, -inf)."""
    mx = part_lse.max(dim=0).values
    safe = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    w = torch.exp(part_lse - safe[None])
    w = torch.where(torch.isfinite(part_lse), w, torch.zeros_like(w))
    den = w.sum(0)
    o = (w[..., None] * part_o).sum(0) / torch.clamp(den, min=1e-30)[..., None]
    o = torch.where((den > 0)[..., None], o, torch.zeros_like(o))
    lse = torch.where(den > 0, safe + torch.log(torch.clamp(den, min=1e-30)),
                      torch.full_like(den, float("-inf")))
    return o, lse


def append(cache: torch.Tensor, new: torch.Tensor, start: int) -> torch.Tensor:
    """Return a copy of ``cache`` with ``new`` written at sequence offset ``start``."""
    out = cache.clone()
    out[:, :, start:start + new.shape[2]] = new
    return out


def attention_flops(b: int, hq: int, sq: int, sk: int, d: int, causal: bool) -> Tuple[int, int]:
    """(forward FLOPs, backward FLOPs) counting only visible (q, k) pairs."""
    if causal:
        pairs = sum(min(i + 1, sk) for i in range(sq)) if sq <= 65536 else None
    else:
        pairs = sq * sk
    fwd = 4 * b * hq * d * pairs
    return fwd, int(2.5 * fwd)


def sdpa_reference_route(q, k, v, do, *, causal: bool):
    """The reference's ``backend="sdpa"`` route with autograd, as a timed CPU baseline.

    Restates ``_sdpa`` (kotflash/attention.py:120-135): PyTorch SDPA with
    native GQA (``enable_gqa=True``) and the default scale left implicit, then
    autograd for dQ/dK/dV.  Returns (O, dQ, dK, dV).
    """
    import torch.nn.functional as F

    q = q.detach().requires_grad_(True)
    k = k.detach().requires_grad_(True)
    v = v.detach().requires_grad_(True)
    kwargs = {"attn_mask": None, "dropout_p": 0.0, "is_causal": causal}
    if q.shape[1] != k.shape[1]:
        kwargs["enable_gqa"] = True
    o = F.scaled_dot_product_attention(q, k, v, **kwargs)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do)
    return o.detach(), dq, dk, dv
