# SPDX-License-Identifier: Apache-2.0
"""Regenerate tests/golden/*.npz from the reference package itself.

    python tests/golden/make_golden.py --reference /path/to/KOTFlash

Imports the reference ``kotflash`` package (its CPU ``backend="sdpa"`` route,
``_blockwise_backward`` and the cache helpers) and records its outputs on
seeded inputs.  The fixtures pin the oracle in ``oracle/`` to the reference's
own behaviour; the GPU box never runs this script (it has no reference tree).

Recorded per attention case: inputs q, k, v, dO; O from
``attention(..., backend="sdpa")``; LSE as the reference tests compute it
(``torch.logsumexp`` over scaled, upper-left-causal-masked scores,
tests/test_attention.py:90-91); dQ/dK/dV by autograd through the reference
route; and the reference ``_blockwise_backward`` gradients.  The larger CPU
plumbing config is recorded as checksums plus a strided
sample, with a checksum of its seeded inputs to detect RNG drift.
"""
from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CASES = [
    # name, B, Hq, Hkv, Sq, Sk, D, causal, seed
    ("mha_noncausal", 2, 4, 4, 7, 9, 32, False, 0),
    ("gqa_causal", 1, 8, 2, 13, 17, 16, True, 1),
    ("gqa_noncausal_unequal", 2, 8, 2, 6, 9, 32, False, 2),
    ("mqa_causal_q_longer", 2, 2, 1, 9, 5, 16, True, 3),
    ("gqa_causal_long", 1, 4, 2, 40, 40, 24, True, 4),
    ("decode_like", 2, 8, 2, 1, 48, 64, False, 5),
]


def _lse(q, k, causal, scale):
    group = q.shape[1] // k.shape[1]
    kk = k.repeat_interleave(group, dim=1)
    s = torch.matmul(q, kk.transpose(-2, -1)) * scale
    if causal:
        mask = torch.arange(k.shape[2])[None, :] > torch.arange(q.shape[2])[:, None]
        s = s.masked_fill(mask, float("-inf"))
    return torch.logsumexp(s, dim=-1)


def attention_case(kf, name, b, hq, hkv, sq, sk, d, causal, seed):
    from kotflash.attention import _blockwise_backward

    torch.manual_seed(seed)
    q = torch.randn(b, hq, sq, d)
    k = torch.randn(b, hkv, sk, d)
    v = torch.randn(b, hkv, sk, d)
    do = torch.randn(b, hq, sq, d)
    scale = 1.0 / math.sqrt(d)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = kf.attention(qg, kg, vg, causal=causal, backend="sdpa")
    dq, dk, dv = torch.autograd.grad(o, (qg, kg, vg), do)
    lse = _lse(q, k, causal, scale)
    bq, bk, bv = _blockwise_backward(q, k, v, o.detach(), lse, do, causal=causal, scale=scale,
                                     q_block=5, kv_block=7)
    arrays = {"q": q, "k": k, "v": v, "do": do, "o": o.detach(), "lse": lse,
              "dq": dq, "dk": dk, "dv": dv, "bw_dq": bq, "bw_dk": bk, "bw_dv": bv}
    meta = np.array([b, hq, hkv, sq, sk, d, int(causal), seed], dtype=np.int64)
    np.savez_compressed(HERE / f"attn_{name}.npz", meta=meta,
                        **{n: t.detach().numpy().astype(np.float32) for n, t in arrays.items()})


def plumbing_config(kf):
    """B2 Hq8 Hkv2 S512 D64 fp32 causal, fwd O+LSE and bwd."""
    torch.manual_seed(2024)
    b, hq, hkv, s, d = 2, 8, 2, 512, 64
    q = torch.randn(b, hq, s, d)
    k = torch.randn(b, hkv, s, d)
    v = torch.randn(b, hkv, s, d)
    do = torch.randn(b, hq, s, d)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = kf.attention(qg, kg, vg, causal=True, backend="sdpa")
    dq, dk, dv = torch.autograd.grad(o, (qg, kg, vg), do)
    lse = _lse(q, k, True, 1.0 / math.sqrt(d))
    out = {"input_sums": np.array([float(t.double().sum()) for t in (q, k, v, do)])}
    for n, t in (("o", o.detach()), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv)):
        flat = t.detach().double().flatten()
        out[f"{n}_sum"] = np.array([float(flat.sum()), float(flat.abs().sum())])
        out[f"{n}_sample"] = flat[:: max(1, flat.numel() // 256)][:256].numpy().astype(np.float32)
    np.savez_compressed(HERE / "cfg1_plumbing.npz", **out)


def cache_case():
    from kotflash.cache import PreallocatedKVCache, append_kv_cache, decode_step

    torch.manual_seed(7)
    cache = PreallocatedKVCache(2, 2, 12, 8, device="cpu", dtype=torch.float32)
    chunks = [torch.randn(2, 2, n, 8) for n in (3, 1, 4)]
    vchunks = [torch.randn(2, 2, n, 8) for n in (3, 1, 4)]
    for kc, vc in zip(chunks, vchunks):
        cache.append(kc, vc)
    kview, vview = cache.view()
    q = torch.randn(2, 4, 1, 8)
    att = cache.attend(q, backend="sdpa")
    nk, nv = torch.randn(2, 2, 1, 8), torch.randn(2, 2, 1, 8)
    q2 = torch.randn(2, 4, 1, 8)
    att2 = cache.append_and_attend(q2, nk, nv, append_backend="torch", attention_backend="sdpa")
    k2, v2 = cache.view()
    dk0, dv0 = torch.randn(1, 2, 5, 8), torch.randn(1, 2, 5, 8)
    dnk, dnv, dq = torch.randn(1, 2, 1, 8), torch.randn(1, 2, 1, 8), torch.randn(1, 4, 1, 8)
    dout, uk, uv = decode_step(dq, dk0, dv0, dnk, dnv, backend="sdpa")
    cat_k, cat_v = append_kv_cache(dk0, dv0, dnk, dnv)
    np.savez_compressed(
        HERE / "cache_sequence.npz",
        k_chunks=np.concatenate([c.numpy() for c in chunks], axis=2),
        v_chunks=np.concatenate([c.numpy() for c in vchunks], axis=2),
        kview=kview.numpy(), vview=vview.numpy(), q=q.numpy(), attend=att.numpy(),
        new_k=nk.numpy(), new_v=nv.numpy(), q2=q2.numpy(), attend2=att2.numpy(),
        k_after=k2.numpy(), v_after=v2.numpy(), length=np.array([cache.length]),
        ds_k0=dk0.numpy(), ds_v0=dv0.numpy(), ds_nk=dnk.numpy(), ds_nv=dnv.numpy(),
        ds_q=dq.numpy(), ds_out=dout.numpy(), ds_uk=uk.numpy(), ds_uv=uv.numpy(),
        cat_k=cat_k.numpy(), cat_v=cat_v.numpy(),
    )


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args(argv)
    sys.path.insert(0, args.reference)
    import kotflash as kf

    assert Path(kf.__file__).resolve().is_relative_to(Path(args.reference).resolve())
    torch.set_num_threads(1)
    for case in CASES:
        attention_case(kf, *case)
    plumbing_config(kf)
    cache_case()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
