#!/usr/bin/env python3
# SPDX-License-Identifier: Apache-2.0
"""Benchmark of the KOTFlash attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (BASELINE.json metric "attn fwd+bwd TFLOP/s & %peak"): one step is
one causal forward + backward of the GQA prefill config B=4, Hq=32, Hkv=8,
Sq=Sk=4096, D=128, bf16, q scaled by 1/sqrt(D), through the public
``kotflash_b200.attention`` API with autograd.  The job is sharded by
(batch x KV-head group) units with no communication: every rank owns the
32 units of one full config (global batch 4*N), so the scaling is weak.
FLOPs count only visible (q, k) pairs: fwd 4*B*Hq*D*P, bwd 2.5x fwd.

Output: detail lines first (``{"detail": ...}``: the decode sweep, the
odd-head-dim runs, the GPU comparators, the decoder-block step, the LM
training A/B on a synthetic token stream), then the
headline JSON line LAST, which also carries compact summaries:
  * ``parity``: max |err| of O, LSE, dQ, dK, dV against a chunked fp32
    reference computed on the GPU (cfg2 bf16 and fp16 batch 0, cfg5 one unit
    at S=16384 for D72/96 causal and not, cfg3 Sq 1/16 at Sk=131072) and the
    bit-exactness of the cache appends (cfg4), tolerance atol=rtol=2e-2;
  * ``fp16``: the fp16 variant of the prefill config;
  * ``cfg5``: the odd-head-dim training config (B2 Hq16 Hkv4 S16384 D72/96
    fp16) sharded by (batch x KV head) units over the ranks (strong scaling);
  * ``decode``: split-KV decode (B2 Hq8 Hkv2 D64 fp16) Sq=1 points, the
    Sq=4/16 points at Sk=32768/131072, and the KV-cache loop (capacity
    32768, B8 Hq32 Hkv8 D128 bf16, 256 fused append+decode steps in one CUDA
    graph);
  * ``decode_multi_gpu`` (N > 1): Sk=131072 split across ranks, NVLink
    peer-memory exchange and NCCL all-gather, with max_err against an fp32
    reference over the full sequence;
  * ``e2e``: the step through the public API with host inputs and outputs,
    and ``copy_bound``, the same copies alone with all ranks copying at once;
  * ``cpu_baseline``: the reference's CPU route (PyTorch SDPA + autograd,
    restated in oracle/) on one (batch, KV-head) unit on the host cores.

``--impl reference`` runs only that CPU route on the full config (rank 0;
other ranks exit at once, no process group).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG = dict(B=4, Hq=32, Hkv=8, S=4096, D=128)
METRIC = "attn fwd+bwd TFLOP/s"
L2_BYTES = 126 * 1024 * 1024


def causal_pairs(sq: int, sk: int) -> int:
    n = min(sq, sk)
    return n * (n + 1) // 2 + max(0, sq - sk) * sk


def fwd_flops(b, hq, sq, sk, d, causal=True) -> float:
    pairs = causal_pairs(sq, sk) if causal else sq * sk
    return 4.0 * b * hq * d * pairs


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            j = json.loads(p.read_text())
            return {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]),
                    "bf16_tflops_sustained": float(j.get("bf16_tflops_sustained", j["bf16_tflops"])),
                    "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s, pw in zip(sm, power) if pw > 300.0] or sm
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# --------------------------------------------------------------------------- dist
def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- prefill fwd+bwd
def make_prefill_inputs(dtype, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    b, hq, hkv, s, d = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["S"], CFG["D"]
    q = (torch.randn(b, hq, s, d, device=device, generator=g) * d ** -0.5).to(dtype)
    k = torch.randn(b, hkv, s, d, device=device, generator=g).to(dtype)
    v = torch.randn(b, hkv, s, d, device=device, generator=g).to(dtype)
    do = torch.randn(b, hq, s, d, device=device, generator=g).to(dtype)
    return q, k, v, do


def prefill_step(q, k, v, do, ev=None):
    from kotflash_b200 import attention

    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    if ev is not None:
        ev[0].record()
    out = attention(q, k, v, causal=True, backend="triton")
    if ev is not None:
        ev[1].record()
    grads = torch.autograd.grad(out, (q, k, v), do)
    if ev is not None:
        ev[2].record()
    return out, grads


def bench_prefill(args, world, rank, local, dtype):
    q, k, v, do = make_prefill_inputs(dtype, 1234 + rank, "cuda")
    for _ in range(args.warmup):
        prefill_step(q, k, v, do)
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if not args.no_clocks else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    for i in range(args.steps):
        prefill_step(q, k, v, do, evs[i])
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    total_ms = max_over_ranks(start.elapsed_time(end), world)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    return total_ms / args.steps, fwd_ms, bwd_ms, clocks


def bench_prefill_e2e(args, world, rank, dtype):
    """Same step with host (pinned) inputs copied in and all outputs copied out.

    Steps are software-pipelined the way a training loop feeding the GPU from
    host memory would run them: step i's inputs are copied in on an H2D stream
    while step i-1 computes, and step i-1's O/dQ/dK/dV are copied out on a D2H
    stream while step i computes (PCIe moves both directions at once).  Device
    inputs are double-buffered.  Every step's copies lie inside the timed
    region: the clock stops after the last step's outputs have reached host
    memory.
    """
    hosts = [tuple(t.cpu().pin_memory() for t in make_prefill_inputs(dtype, 99 + rank + 7 * j, "cuda"))
             for j in range(2)]
    outs_h = [tuple(torch.empty_like(t).pin_memory() for t in (hosts[j][0], hosts[j][0], hosts[j][1], hosts[j][2]))
              for j in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in hosts[0])
    d2h = sum(t.numel() * t.element_size() for t in outs_h[0])
    dev = [tuple(torch.empty_like(t, device="cuda") for t in hosts[j]) for j in range(2)]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    for j in range(2):
        in_free[j].record(comp)
        out_done[j].record(s_out)

    def copy_in(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(in_free[j])
            for d, h in zip(dev[j], hosts[j]):
                d.copy_(h, non_blocking=True)
            in_ready[j].record(s_in)

    def compute_and_copy_out(i):
        j = i % 2
        comp.wait_event(in_ready[j])
        q, k, v, do = dev[j]
        out, (dq, dk, dv) = prefill_step(q.detach(), k.detach(), v.detach(), do)
        in_free[j].record(comp)
        ready = torch.cuda.Event()
        ready.record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ready)
            for h, d in zip(outs_h[j], (out.detach(), dq, dk, dv)):
                d.record_stream(s_out)
                h.copy_(d, non_blocking=True)
            out_done[j].record(s_out)

    def run(n):
        s_in.wait_stream(comp)  # the first copy starts after the clock does
        copy_in(0)
        for i in range(n):
            if i + 1 < n:
                copy_in(i + 1)
            compute_and_copy_out(i)
        comp.wait_stream(s_out)

    run(max(2, args.warmup))
    torch.cuda.synchronize()
    # the same K steps as the device-resident leg: the pipeline fill (first
    # copy in) and drain (last copy out) lie in the timed region and amortise
    # over K, as they would over a training run
    steps = max(4, args.steps)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(comp)
    run(steps)
    end.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world) / steps

    # The bound on that number: the same copies with no compute, both
    # directions at once, every rank copying at the same time (the host's
    # memory and PCIe fabric are shared by the ranks).
    outs_d = [tuple(torch.empty_like(h, device="cuda") for h in outs_h[j]) for j in range(2)]

    def copies(n):
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        for i in range(n):
            j = i % 2
            with torch.cuda.stream(s_in):
                for d, h in zip(dev[j], hosts[j]):
                    d.copy_(h, non_blocking=True)
            with torch.cuda.stream(s_out):
                for h, d in zip(outs_h[j], outs_d[j]):
                    h.copy_(d, non_blocking=True)
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)

    copies(2)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start.record(comp)
    copies(steps)
    end.record(comp)
    torch.cuda.synchronize()
    barrier(world)
    copy_ms = max_over_ranks(start.elapsed_time(end), world) / steps
    return ms, h2d, d2h, copy_ms


# --------------------------------------------------------------------------- parity
PARITY_TOL = 2e-2  # atol = rtol, BASELINE north star (fp16/bf16 vs an fp32 reference)


def fp32_attention_reference(q, k, v, do=None, *, causal, scale, chunk=1024):
    """Plain fp32 attention on the GPU, one query head and ``chunk`` query rows
    at a time: (O, LSE) and, with ``do``, (dQ, dK, dV) by the standard
    formulas (P = exp(S - LSE), dS = P (dO V^T - rowsum(O dO)), dQ = scale dS K,
    dK = scale dS^T Q, dV = P^T dO, summed over each KV head's query heads).
    The checker for the parity block; nothing here is timed."""
    b, hq, sq, d = q.shape
    hkv, sk = k.shape[1], k.shape[2]
    group = hq // hkv
    dev = q.device
    o = torch.empty(b, hq, sq, d, device=dev)
    lse = torch.empty(b, hq, sq, device=dev)
    grads = do is not None
    if grads:
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
                qc = q[bi, h, r0:r1].float()
                s = (qc @ kh.t()) * scale
                if causal:
                    s = s.masked_fill(kpos > torch.arange(r0, r1, device=dev)[:, None], float("-inf"))
                l = torch.logsumexp(s, dim=-1)
                p = torch.nan_to_num(torch.exp(s - l[:, None]), nan=0.0)
                oc = p @ vh
                o[bi, h, r0:r1] = oc
                lse[bi, h, r0:r1] = l
                if grads:
                    dc = do[bi, h, r0:r1].float()
                    ds = p * (dc @ vh.t() - (oc * dc).sum(-1, keepdim=True))
                    dq[bi, h, r0:r1] = (ds @ kh) * scale
                    dk[bi, g] += (ds.t() @ qc) * scale
                    dv[bi, g] += p.t() @ dc
    return (o, lse, dq, dk, dv) if grads else (o, lse)


def max_err(got, want):
    """(max |got - want|, max |got - want| / (atol + rtol |want|)) over finite entries."""
    a, e = got.float(), want.float()
    fin = torch.isfinite(e)
    if not bool(torch.equal(torch.isfinite(a), fin)):
        return float("inf"), float("inf")
    diff = (a - e).abs()[fin]
    if diff.numel() == 0:
        return 0.0, 0.0
    return diff.max().item(), (diff / (PARITY_TOL + PARITY_TOL * e.abs()[fin])).max().item()


def _sig(x):
    return float(f"{x:.3g}")


def bench_parity():
    """Max errors of the CUDA path against the fp32 reference at the BASELINE
    configs, in the driver-kept record.  Returns {case: [errors]} plus the
    worst error/tolerance ratio."""
    from kotflash_b200.attention import _decode_forward, attention_backward, attention_forward

    out = {"tol": PARITY_TOL, "fields": "O,LSE,dQ,dK,dV"}
    worst = 0.0

    def record(name, pairs):
        nonlocal worst
        errs = []
        for got, want in pairs:
            e, r = max_err(got, want)
            errs.append(_sig(e))
            worst = max(worst, r)
        out[name] = errs

    # cfg2 at full size, both dtypes; the reference on batch 0 (32 heads)
    for dt, name in ((torch.bfloat16, "cfg2_bf16"), (torch.float16, "cfg2_fp16")):
        q, k, v, do = make_prefill_inputs(dt, 555, "cuda")
        d = CFG["D"]
        o, lse = attention_forward(q, k, v, causal=True, scale=d ** -0.5)
        dq, dk, dv = attention_backward(q, k, v, o, lse, do, causal=True, scale=d ** -0.5)
        ref = fp32_attention_reference(q[:1], k[:1], v[:1], do[:1], causal=True, scale=d ** -0.5)
        record(name, zip((o[:1], lse[:1], dq[:1], dk[:1], dv[:1]), ref))
        del q, k, v, do, o, lse, dq, dk, dv, ref
        torch.cuda.empty_cache()
    # cfg5: one (batch, KV-head) unit at the full 16384 length
    s = 16384
    for d in (72, 96):
        g = torch.Generator(device="cuda").manual_seed(700 + d)
        q = torch.randn(1, 4, s, d, device="cuda", generator=g).half()
        k = torch.randn(1, 1, s, d, device="cuda", generator=g).half()
        v = torch.randn(1, 1, s, d, device="cuda", generator=g).half()
        do = torch.randn(1, 4, s, d, device="cuda", generator=g).half()
        for causal in (False, True):
            o, lse = attention_forward(q, k, v, causal=causal, scale=d ** -0.5)
            dq, dk, dv = attention_backward(q, k, v, o, lse, do, causal=causal, scale=d ** -0.5)
            ref = fp32_attention_reference(q, k, v, do, causal=causal, scale=d ** -0.5)
            record(f"cfg5_d{d}_{'causal' if causal else 'full'}", zip((o, lse, dq, dk, dv), ref))
        del q, k, v, do
        torch.cuda.empty_cache()
    # cfg3 at the longest visible length
    g = torch.Generator(device="cuda").manual_seed(808)
    k = torch.randn(2, 2, 131072, 64, device="cuda", generator=g).half()
    v = torch.randn(2, 2, 131072, 64, device="cuda", generator=g).half()
    for sq in (1, 16):
        q = torch.randn(2, 8, sq, 64, device="cuda", generator=g).half()
        o, lse = _decode_forward(q, k, v, scale=0.125, want_lse=True)
        ref = fp32_attention_reference(q, k, v, causal=False, scale=0.125)
        record(f"cfg3_sq{sq}_sk131072", zip((o, lse), ref))
    del k, v
    torch.cuda.empty_cache()
    out["worst_err_over_tol"] = _sig(worst)
    out["pass"] = worst <= 1.0
    return out


# --------------------------------------------------------------------------- decode
def _graph_time(fn, reps, replays=5):
    """Capture ``reps`` calls of fn(i) in one CUDA graph; mean ms per call over replays."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(min(reps, 3)):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(replays):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / reps)
    del g
    return min(times)


def bench_decode_sweep(peaks):
    from kotflash_b200.attention import _decode_forward

    res = []
    for sq in (1, 4, 16):
        for sk in (1024, 2048, 8192, 32768, 131072):
            kv_bytes = 2 * 2 * 2 * sk * 64 * 2
            copies = max(1, min(256, math.ceil(3 * L2_BYTES / kv_bytes)))
            g = torch.Generator(device="cuda").manual_seed(sk + sq)
            ks = torch.randn(copies, 2, 2, sk, 64, device="cuda", generator=g, dtype=torch.float32).half()
            vs = torch.randn(copies, 2, 2, sk, 64, device="cuda", generator=g, dtype=torch.float32).half()
            qs = torch.randn(copies, 2, 8, sq, 64, device="cuda", generator=g).half()
            reps = max(copies, 8)
            ms = _graph_time(lambda i: _decode_forward(qs[i % copies], ks[i % copies], vs[i % copies],
                                                       scale=0.125, want_lse=False), reps)
            alg = 1024 * sk + 4096 * sq + 64 * sq  # K+V read, Q read + O write (+LSE)
            gbs = alg / (ms * 1e-3) / 1e9
            res.append({"sq": sq, "sk": sk, "us_per_call": round(ms * 1e3, 2),
                        "us_per_token": round(ms * 1e3 / sq, 3), "hbm_gbs": round(gbs, 1),
                        "hbm_frac": round(gbs / peaks["hbm_gbs"], 3)})
            del ks, vs, qs
            torch.cuda.empty_cache()
    return res


def bench_cache_loop(peaks):
    from kotflash_b200.cache import PreallocatedKVCache

    b, hkv, hq, d, cap, pre, steps = 8, 8, 32, 128, 32768, 4096, 256
    cache = PreallocatedKVCache(b, hkv, cap, d, device="cuda", dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(7)
    pk = torch.randn(b, hkv, pre, d, device="cuda", generator=g).bfloat16()
    pv = torch.randn(b, hkv, pre, d, device="cuda", generator=g).bfloat16()
    # prefill append bandwidth (K4), timed as graph replays of the same append
    ms_app = _graph_time(lambda i: _append_at(cache, pk, pv, 0), 8)
    app_bytes = 2 * 2 * pk.numel() * 2  # read new K,V + write cache K,V
    torch.cuda.synchronize()
    prefill_exact = bool(torch.equal(cache.k[:, :, :pre], pk) and torch.equal(cache.v[:, :, :pre], pv))
    cache.length = pre
    # prefill attention reading the cache's strided prefix view in place (K1), the
    # reference example's prefill -> decode handoff (examples/gqa_kv_cache_decode.py:58-65)
    from kotflash_b200 import attention

    q_pre = (torch.randn(b, hq, pre, d, device="cuda", generator=g) * d ** -0.5).bfloat16()

    def prefill(_i):
        with torch.inference_mode():
            ck, cv = cache.view()
            attention(q_pre, ck, cv, causal=True, backend="triton")

    ms_pre = _graph_time(prefill, 3, replays=3)
    f_pre = fwd_flops(b, hq, pre, pre, d, True)
    del q_pre
    nk = torch.randn(steps, b, hkv, 1, d, device="cuda", generator=g).bfloat16()
    nv = torch.randn(steps, b, hkv, 1, d, device="cuda", generator=g).bfloat16()
    qq = torch.randn(steps, b, hq, 1, d, device="cuda", generator=g).bfloat16()
    base = cache.length

    def one(i):
        cache.length = base + (i % steps)
        with torch.inference_mode():
            cache.append_and_attend(qq[i % steps], nk[i % steps], nv[i % steps])

    ms = _graph_time(one, steps, replays=3)
    cache.length = base + steps
    torch.cuda.synchronize()
    # every replay wrote step i's row at base + i with the fused append (K3)
    loop_exact = bool(torch.equal(cache.k[:, :, base:base + steps], nk[:, :, :, 0].permute(1, 2, 0, 3))
                      and torch.equal(cache.v[:, :, base:base + steps], nv[:, :, :, 0].permute(1, 2, 0, 3)))
    mean_len = base + (steps + 1) / 2
    step_bytes = 2 * b * hkv * mean_len * d * 2 + 2 * b * hq * d * 2 + 2 * b * hkv * d * 2
    gbs = step_bytes / (ms * 1e-3) / 1e9
    return {
        "prefill_append": {"tokens": pre, "us": round(ms_app * 1e3, 2),
                           "hbm_gbs": round(app_bytes / (ms_app * 1e-3) / 1e9, 1),
                           "hbm_frac": round(app_bytes / (ms_app * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)},
        "prefill_attention": {"tokens": pre, "ms": round(ms_pre, 4),
                              "tflops": round(f_pre / ms_pre / 1e9, 1),
                              "frac": round(f_pre / ms_pre / 1e9 / peaks["bf16_tflops"], 3),
                              "note": "causal K1 forward over the strided cache view (capacity 32768), no copy"},
        "steps": steps, "us_per_step": round(ms * 1e3, 2), "us_per_token": round(ms * 1e3, 2),
        "loop_ms": round(ms * steps, 3), "hbm_gbs": round(gbs, 1),
        "hbm_frac": round(gbs / peaks["hbm_gbs"], 3),
        "note": "fused append+decode, 256 steps in one CUDA graph; working set 134-143 MB (> L2)",
        "append_bit_exact": {"prefill_append_kernel": prefill_exact, "fused_append_256_steps": loop_exact},
    }


def _append_at(cache, k, v, start):
    from kotflash_b200._cuda_append import append_kv_cuda

    append_kv_cuda(cache.k, cache.v, k, v, start)


def bench_odd_head_dim(peaks, world, rank, iters=3):
    """B2 Hq16 Hkv4 S16384 fp16, D in {72, 96}, causal
    and not, fwd+bwd.  The job's 8 (batch, KV-head) units are sharded over the
    ranks with no communication (1 unit per rank at N=8: strong scaling);
    every rank builds the same seeded full inputs and takes its units.  Time
    = max over ranks of the CUDA-event time of the rank's units, mean of
    ``iters`` runs after one warm-up."""
    from kotflash_b200 import distributed as kd
    from kotflash_b200.attention import attention_backward, attention_forward

    b, hq, hkv, s = 2, 16, 4, 16384
    group = hq // hkv
    units = kd.shard_units(b, hkv, world, rank)
    runs = kd.shard_slices(units, group)
    res = []
    for d in (72, 96):
        g = torch.Generator(device="cuda").manual_seed(d)
        full = [torch.randn(b, h, s, d, device="cuda", generator=g).half() for h in (hq, hkv, hkv, hq)]
        parts = [tuple(t[bi:bi + 1, sl].contiguous() for t, sl in zip(full, (qs, kvs, kvs, qs)))
                 for bi, kvs, qs in runs]
        del full
        torch.cuda.empty_cache()
        for causal in (False, True):
            scale = d ** -0.5

            def once(ev=None):
                for q, k, v, do in parts:
                    if ev is not None:
                        ev[0].record()
                    out, lse = attention_forward(q, k, v, causal=causal, scale=scale)
                    if ev is not None:
                        ev[1].record()
                    attention_backward(q, k, v, out, lse, do, causal=causal, scale=scale)
                    if ev is not None:
                        ev[2].record()

            once()
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(iters)]
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier(world)
            torch.cuda.synchronize()
            start.record()
            for i in range(iters):
                once(evs[i])
            end.record()
            torch.cuda.synchronize()
            barrier(world)
            ms = max_over_ranks(start.elapsed_time(end) / iters, world)
            f = fwd_flops(b, hq, s, s, d, causal)
            tf = 3.5 * f / (ms * 1e-3) / 1e12
            line = {"d": d, "causal": causal, "ms": round(ms, 3), "fwd_bwd_tflops": round(tf, 1),
                    "per_rank_frac": round(tf / world / peaks["bf16_tflops"], 3),
                    "units_per_rank": len(units)}
            if len(parts) == 1:  # forward/backward split of this rank's one run
                line["fwd_ms"] = round(statistics.mean(e[0].elapsed_time(e[1]) for e in evs), 3)
                line["bwd_ms"] = round(statistics.mean(e[1].elapsed_time(e[2]) for e in evs), 3)
            res.append(line)
        del parts
        torch.cuda.empty_cache()
    return res


def bench_decode_multi_gpu(world, rank):
    """cfg3 at Sk=131072 with the KV sequence split across ranks.

    Each rank's sequence (split-KV decode of its chunk, then the exchange of
    partials and the LSE merge) is captured in a CUDA graph and replayed; the
    compute-only part is captured separately so compute and exchange are
    reported apart.  Two exchanges: NVLink peer memory (``PeerExchange``, two
    kernels) and the NCCL route (pack, all-gather, merge).  Max over ranks of
    device time per call.  Correctness: every rank also holds the full K/V
    and compares both routes' (O, LSE) with an fp32 reference over the whole
    sequence; ``max_err`` is the max over ranks."""
    from kotflash_b200 import distributed as kd
    from kotflash_b200.attention import _decode_forward

    out = []
    sk = 131072
    for sq in (1, 16):
        lo, hi = kd.kv_chunk(sk, world, rank)
        g = torch.Generator(device="cuda").manual_seed(5)
        k_full = torch.randn(2, 2, sk, 64, device="cuda", generator=g).half()
        v_full = torch.randn(2, 2, sk, 64, device="cuda", generator=g).half()
        q = torch.randn(2, 8, sq, 64, device="cuda", generator=g).half()
        kl, vl = k_full[:, :, lo:hi].contiguous(), v_full[:, :, lo:hi].contiguous()
        ref_o, ref_lse = fp32_attention_reference(q, k_full, v_full, causal=False, scale=0.125)
        del k_full, v_full
        try:
            ex = kd.PeerExchange(rows=q[..., 0].numel(), d=64, dtype=q.dtype)
        except RuntimeError as exc:  # raised on every rank alike
            ex, peer_error = None, str(exc).splitlines()[0][:200]

        def nccl(_i):
            kd.decode_kv_split(q, kl, vl, scale=0.125)

        def peer(_i):
            kd.decode_kv_split(q, kl, vl, scale=0.125, exchange=ex)

        def local(_i):
            _decode_forward(q, kl, vl, scale=0.125, want_lse=True)

        barrier(world)
        o_n, l_n = kd.decode_kv_split(q, kl, vl, scale=0.125)
        err_n = max(max_err(o_n, ref_o)[0], max_err(l_n, ref_lse)[0])
        if ex is not None:
            o_p, l_p = kd.decode_kv_split(q, kl, vl, scale=0.125, exchange=ex)
            err_p = max(max_err(o_p, ref_o)[0], max_err(l_p, ref_lse)[0])
        barrier(world)
        t_n = _graph_time(nccl, 8, replays=5)
        if ex is not None:
            barrier(world)
            t_p = _graph_time(peer, 32, replays=5)
        barrier(world)
        t_c = _graph_time(local, 8, replays=5)
        n = max_over_ranks(t_n, world)
        c = max_over_ranks(t_c, world)
        err_n = max_over_ranks(err_n, world)
        if ex is not None:
            pp = max_over_ranks(t_p, world)
            err_p = max_over_ranks(err_p, world)
            timeouts = max_over_ranks(float(ex.status()), world)
            barrier(world)
            ex.close()
            peer_line = {"exchange_merge_us": round((pp - c) * 1e3, 2), "total_us": round(pp * 1e3, 2),
                         "us_per_token": round(pp * 1e3 / sq, 3), "timeouts": int(timeouts),
                         "max_err": _sig(err_p)}
        else:
            peer_line = {"unavailable": peer_error}
        out.append({"sq": sq, "sk": sk, "ranks": world, "keys_per_rank": hi - lo,
                    "compute_us": round(c * 1e3, 2),
                    "peer": peer_line,
                    "nccl": {"exchange_merge_us": round((n - c) * 1e3, 2), "total_us": round(n * 1e3, 2),
                             "us_per_token": round(n * 1e3 / sq, 3), "max_err": _sig(err_n)},
                    "max_err_tol": PARITY_TOL,
                    "timing": "CUDA-graph replay, max over ranks"})
        torch.cuda.synchronize()
    return out


# --------------------------------------------------------------------------- decoder block
class DecoderBlock(torch.nn.Module):
    """Pre-norm GQA decoder block (LayerNorm, Q/K/V/O projections, SiLU-gated
    MLP of width 4x) with fp32 parameters whose attention runs in 16-bit: the
    block of the reference's decoder-block benchmark
    (benchmarks/benchmark_decoder_block.py:34-103), kept structurally alike so
    the step times compare."""

    def __init__(self, q_heads, kv_heads, head_dim, mlp_ratio=4):
        super().__init__()
        nn = torch.nn
        hidden = q_heads * head_dim
        self.hq, self.hkv, self.d = q_heads, kv_heads, head_dim
        self.norm1, self.norm2 = nn.LayerNorm(hidden), nn.LayerNorm(hidden)
        self.wq = nn.Linear(hidden, hidden, bias=False)
        self.wk = nn.Linear(hidden, kv_heads * head_dim, bias=False)
        self.wv = nn.Linear(hidden, kv_heads * head_dim, bias=False)
        self.wo = nn.Linear(hidden, hidden, bias=False)
        self.w_gate = nn.Linear(hidden, mlp_ratio * hidden, bias=False)
        self.w_up = nn.Linear(hidden, mlp_ratio * hidden, bias=False)
        self.w_down = nn.Linear(mlp_ratio * hidden, hidden, bias=False)

    def forward(self, x, backend, attn_dtype=torch.float16):
        import torch.nn.functional as F
        from kotflash_b200 import attention

        b, s, h = x.shape
        y = self.norm1(x)
        q = self.wq(y).view(b, s, self.hq, self.d).transpose(1, 2).to(attn_dtype)
        k = self.wk(y).view(b, s, self.hkv, self.d).transpose(1, 2).to(attn_dtype)
        v = self.wv(y).view(b, s, self.hkv, self.d).transpose(1, 2).to(attn_dtype)
        if backend == "kotflash_b200":
            a = attention(q, k, v, causal=True, backend="triton")
        elif backend == "sdpa_gqa":
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        else:  # "sdpa_expanded_kv"
            g = self.hq // self.hkv
            a = F.scaled_dot_product_attention(q, k.repeat_interleave(g, 1), v.repeat_interleave(g, 1),
                                               is_causal=True)
        x = x + self.wo(a.transpose(1, 2).reshape(b, s, h).to(x.dtype))
        y = self.norm2(x)
        return x + self.w_down(F.silu(self.w_gate(y)) * self.w_up(y))


def decoder_block_step(model, opt, x, target, backend, attn_dtype=torch.float16):
    import torch.nn.functional as F

    opt.zero_grad(set_to_none=True)
    loss = F.mse_loss(model(x, backend, attn_dtype), target)
    loss.backward()
    opt.step()
    return loss.detach()


def bench_decoder_block(batch=2, seq=4096, q_heads=32, kv_heads=8, head_dim=128, warmup=3, iters=5,
                        bf16_block=False):
    """Training step (forward, backward, AdamW) of the decoder block per
    attention backend, same initial weights and inputs; tokens/s from the
    median CUDA-event step time.  Default: fp32 projections (no TF32), fp16
    attention, as the reference benchmark runs it; there the fp32
    projections take nearly all of the step.  ``bf16_block``: the whole block
    (parameters, projections, attention) in bf16, so the attention's share
    of the step shows."""
    torch.manual_seed(1234)
    hidden = q_heads * head_dim
    pdt = torch.bfloat16 if bf16_block else torch.float32
    adt = torch.bfloat16 if bf16_block else torch.float16
    x = torch.randn(batch, seq, hidden, device="cuda").to(pdt)
    target = torch.randn_like(x)
    init = {k: v.detach().clone() for k, v in DecoderBlock(q_heads, kv_heads, head_dim).state_dict().items()}
    out = {"shape": {"batch": batch, "seq": seq, "q_heads": q_heads, "kv_heads": kv_heads, "head_dim": head_dim,
                     "hidden": hidden},
           "precision": ("bf16 parameters, projections and attention, AdamW" if bf16_block else
                         "fp32 parameters and projections (TF32 off), fp16 attention, AdamW")}
    for backend in ("kotflash_b200", "sdpa_gqa", "sdpa_expanded_kv"):
        try:
            model = DecoderBlock(q_heads, kv_heads, head_dim).cuda()
            model.load_state_dict(init)
            model = model.to(pdt)
            opt = torch.optim.AdamW(model.parameters(), lr=1e-4)
            for _ in range(warmup):
                decoder_block_step(model, opt, x, target, backend, adt)
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
            loss = None
            for a, e in evs:
                a.record()
                loss = decoder_block_step(model, opt, x, target, backend, adt)
                e.record()
            torch.cuda.synchronize()
            ms = statistics.median(a.elapsed_time(e) for a, e in evs)
            out[backend] = {"step_ms": round(ms, 3), "tokens_per_s": round(batch * seq * 1e3 / ms, 1),
                            "last_loss": round(float(loss), 6),
                            "params_finite": all(bool(torch.isfinite(p).all()) for p in model.parameters())}
            del model, opt
        except Exception as exc:
            out[backend] = {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}"}
        torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------------- LM training A/B
GPT2_VOCAB = 50257  # vocabulary size of the tokenizer the reference's LM benchmark uses ("gpt2")


def synthetic_story_tokens(n, vocab=GPT2_VOCAB, seed=0):
    """Seeded stand-in for a tokenized story corpus (the reference's LM A/B
    streams TinyStories, which is not available offline): ``n`` token ids in
    ``[0, vocab)`` with a Zipf-like unigram law (p(r) ~ (r + 10)^-1.1 over a
    seeded ranking of the ids), a learnable bigram structure (with
    probability 0.6 a token is followed by its fixed successor under a seeded
    permutation) and an end-of-story id (``vocab - 1``) closing stories of
    geometric length (mean 200 tokens).  Only the statistics are modelled;
    no text of any corpus is involved."""
    rng = np.random.default_rng(seed)
    body = vocab - 1
    p = 1.0 / (np.arange(body) + 10.0) ** 1.1
    p /= p.sum()
    ids_by_rank = rng.permutation(body)
    draws = ids_by_rank[rng.choice(body, size=n, p=p)]
    successor = rng.permutation(body)
    follow = rng.random(n) < 0.6
    story_end = rng.random(n) < 1.0 / 200.0
    out = np.empty(n, dtype=np.int64)
    prev = -1
    for i in range(n):
        if story_end[i]:
            tok = body
        elif prev >= 0 and prev != body and follow[i]:
            tok = successor[prev]
        else:
            tok = draws[i]
        out[i] = tok
        prev = tok
    return torch.from_numpy(out)


class StoryLM(torch.nn.Module):
    """Next-token LM of the reference's LM training A/B
    (benchmarks/benchmark_tinystories_training.py:90-125): token and learned
    position embeddings, ``layers`` pre-norm GQA decoder blocks with a SiLU-gated
    MLP (the ``DecoderBlock`` above), a final LayerNorm and an output head tied
    to the token embedding; N(0, 0.02) initialisation."""

    def __init__(self, vocab, max_seq, layers=2, q_heads=8, kv_heads=2, head_dim=64, mlp_ratio=4):
        super().__init__()
        nn = torch.nn
        hidden = q_heads * head_dim
        self.tok = nn.Embedding(vocab, hidden)
        self.pos = nn.Embedding(max_seq, hidden)
        self.blocks = nn.ModuleList(DecoderBlock(q_heads, kv_heads, head_dim, mlp_ratio) for _ in range(layers))
        self.norm = nn.LayerNorm(hidden)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)

    def forward(self, ids, backend):
        import torch.nn.functional as F

        x = self.tok(ids) + self.pos(torch.arange(ids.shape[1], device=ids.device))[None]
        for blk in self.blocks:
            x = blk(x, backend)
        return F.linear(self.norm(x), self.tok.weight)


def bench_story_lm_ab(seq=4096, batch=1, steps=100, warmup=5, lr=3e-4, weight_decay=0.01, seed=1337):
    """LM training A/B of the reference's TinyStories benchmark on a synthetic
    token stream of the same vocabulary: identical initial weights and
    paired batches for both attention routes, fp32 master weights with fp16
    autocast and a gradient scaler, AdamW, backend order shuffled per step;
    CUDA-event step times (forward, cross-entropy, backward, optimizer) and
    the evaluation loss on a held-out window before and after training.
    Routes: this library (``backend="triton"``) and PyTorch SDPA on K/V
    expanded to the query heads (the reference benchmark's baseline)."""
    import random

    import torch.nn.functional as F

    n_train = (warmup + steps) * batch * seq + 1
    stream = synthetic_story_tokens(n_train + batch * seq + 1, seed=seed)
    train, held = stream[:n_train], stream[n_train:]
    windows = train.unfold(0, batch * seq + 1, batch * seq)
    order = torch.randperm(windows.shape[0], generator=torch.Generator().manual_seed(seed))
    windows = windows[order].cuda()
    xs = windows[:, :-1].reshape(-1, batch, seq)
    ys = windows[:, 1:].reshape(-1, batch, seq)
    ex = held[:-1].reshape(batch, seq).cuda()
    ey = held[1:].reshape(batch, seq).cuda()

    torch.manual_seed(seed)
    init = StoryLM(GPT2_VOCAB, seq).state_dict()
    routes = {"kotflash_b200": "kotflash_b200", "sdpa_expanded": "sdpa_expanded_kv"}
    models, opts, scalers = {}, {}, {}
    for name in routes:
        m = StoryLM(GPT2_VOCAB, seq).cuda()
        m.load_state_dict(init)
        models[name] = m
        opts[name] = torch.optim.AdamW(m.parameters(), lr=lr, weight_decay=weight_decay)
        scalers[name] = torch.amp.GradScaler("cuda")

    def loss_of(name, x, y):
        with torch.autocast("cuda", dtype=torch.float16):
            logits = models[name](x, routes[name])
            return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), y.reshape(-1))

    def evaluate(name):
        models[name].eval()
        with torch.no_grad():
            v = float(loss_of(name, ex, ey).float())
        models[name].train()
        return v

    def step(name, x, y):
        opts[name].zero_grad(set_to_none=True)
        loss = loss_of(name, x, y)
        scalers[name].scale(loss).backward()
        scalers[name].step(opts[name])
        scalers[name].update()
        return loss.detach()

    initial = {name: evaluate(name) for name in routes}
    rng = random.Random(seed + 1)
    for i in range(warmup):
        names = list(routes)
        rng.shuffle(names)
        for name in names:
            step(name, xs[i], ys[i])
    torch.cuda.synchronize()
    events = {name: [] for name in routes}
    last = {}
    for i in range(warmup, warmup + steps):
        names = list(routes)
        rng.shuffle(names)
        for name in names:
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            last[name] = step(name, xs[i], ys[i])
            e.record()
            events[name].append((a, e))
    torch.cuda.synchronize()
    out = {"shape": {"batch": batch, "seq": seq, "layers": 2, "q_heads": 8, "kv_heads": 2, "head_dim": 64,
                     "hidden": 512, "vocab": GPT2_VOCAB,
                     "parameters": sum(p.numel() for p in models["kotflash_b200"].parameters())},
           "data": "synthetic token stream (Zipf unigrams, seeded bigram successors, end-of-story id): "
                   "stand-in for TinyStories, which needs a download",
           "precision": "fp32 master weights, fp16 autocast, GradScaler; fp16 attention; AdamW",
           "steps": steps, "warmup": warmup}
    for name in routes:
        times = [a.elapsed_time(e) for a, e in events[name]]
        finite = bool(torch.isfinite(last[name]).all()) and all(
            bool(torch.isfinite(p).all()) for p in models[name].parameters())
        out[name] = {"median_step_ms": round(statistics.median(times), 3),
                     "tokens_per_s": round(steps * batch * seq * 1e3 / sum(times), 1),
                     "initial_eval_loss": round(initial[name], 5), "final_eval_loss": round(evaluate(name), 5),
                     "last_train_loss": round(float(last[name].float()), 5), "finite": finite}
    a, b = out["kotflash_b200"], out["sdpa_expanded"]
    out["initial_eval_loss_abs_delta"] = round(abs(a["initial_eval_loss"] - b["initial_eval_loss"]), 6)
    out["final_eval_loss_abs_delta"] = round(abs(a["final_eval_loss"] - b["final_eval_loss"]), 6)
    out["speedup_vs_sdpa_expanded"] = round(b["median_step_ms"] / a["median_step_ms"], 3)
    del models, opts
    torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------------- GPU comparator
def bench_sdpa_comparators(dtype):
    """PyTorch SDPA's own GPU backends (cuDNN, flash, memory-efficient) on this
    B200 at the prefill config (fwd+bwd, causal, GQA through ``enable_gqa``)
    and at the cfg3 decode point (Sq=1, Sk=131072): a reference point beside
    the roofline, since the reference's own Triton route cannot run on sm_100.
    CUDA events, warm-up first; a backend that rejects the inputs is reported
    with its error."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    backends = {"cudnn": SDPBackend.CUDNN_ATTENTION, "flash": SDPBackend.FLASH_ATTENTION,
                "efficient": SDPBackend.EFFICIENT_ATTENTION}
    b, hq, s, d = CFG["B"], CFG["Hq"], CFG["S"], CFG["D"]
    f_fwd = fwd_flops(b, hq, s, s, d, True)
    out = {"prefill": {}, "decode_sq1_sk131072": {}}
    q, k, v, do = make_prefill_inputs(dtype, 4321, "cuda")
    for name, be in backends.items():
        try:
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))

            def step():
                with sdpa_kernel([be]):
                    o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=True)
                return o, torch.autograd.grad(o, (qq, kk, vv), do)

            for _ in range(3):
                step()
            torch.cuda.synchronize()
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(5)]
            for e in evs:
                e[0].record()
                with sdpa_kernel([be]):
                    o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=True)
                e[1].record()
                torch.autograd.grad(o, (qq, kk, vv), do)
                e[2].record()
            torch.cuda.synchronize()
            fwd = statistics.median(e[0].elapsed_time(e[1]) for e in evs)
            tot = statistics.median(e[0].elapsed_time(e[2]) for e in evs)
            out["prefill"][name] = {"fwd_ms": round(fwd, 4), "fwd_bwd_ms": round(tot, 4),
                                    "fwd_tflops": round(f_fwd / fwd / 1e9, 1),
                                    "fwd_bwd_tflops": round(3.5 * f_fwd / tot / 1e9, 1)}
        except Exception as exc:  # backend not available for these inputs
            out["prefill"][name] = {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}"}
        torch.cuda.empty_cache()
    del q, k, v, do
    sk, copies = 131072, 2
    g = torch.Generator(device="cuda").manual_seed(77)
    ks = torch.randn(copies, 2, 2, sk, 64, device="cuda", generator=g).half()
    vs = torch.randn(copies, 2, 2, sk, 64, device="cuda", generator=g).half()
    qs = torch.randn(copies, 2, 8, 1, 64, device="cuda", generator=g).half()
    alg = 1024 * sk + 4096 + 64
    for name, be in backends.items():
        try:
            def call(i):
                with sdpa_kernel([be]):
                    F.scaled_dot_product_attention(qs[i % copies], ks[i % copies], vs[i % copies], enable_gqa=True)

            for i in range(3):
                call(i)
            torch.cuda.synchronize()
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for i in range(20):
                call(i)
            e.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(e) / 20
            out["decode_sq1_sk131072"][name] = {"us_per_call": round(ms * 1e3, 2),
                                                "hbm_gbs": round(alg / (ms * 1e-3) / 1e9, 1),
                                                "timing": "eager launches, 2 rotating K/V sets (268 MB)"}
        except Exception as exc:
            out["decode_sq1_sk131072"][name] = {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}"}
    del ks, vs, qs
    torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------------- CPU baseline
def use_all_host_cores() -> int:
    """Let the CPU baseline use every core this process may run on (torchrun sets
    OMP_NUM_THREADS=1 for its workers; rank 0 runs the CPU legs alone)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def cpu_unit_sample(dtype_name: str, budget_s: float = 12.0, min_runs: int = 1):
    """Time the reference CPU route on (batch, KV-head) units of the prefill config.

    One unit = one KV head with its Hq/Hkv query heads at S=4096, D=128,
    causal.  Runs units until ``budget_s`` of CPU time is spent; returns
    (TFLOP/s, seconds per unit, dtype used, units run, threads)."""
    from oracle import attention_oracle as oracle

    g = torch.Generator().manual_seed(0)
    group = CFG["Hq"] // CFG["Hkv"]
    s, d = CFG["S"], CFG["D"]
    dt = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    try:
        q = (torch.randn(1, group, s, d, generator=g) * d ** -0.5).to(dt)
        k = torch.randn(1, 1, s, d, generator=g).to(dt)
        v = torch.randn(1, 1, s, d, generator=g).to(dt)
        do = torch.randn(1, group, s, d, generator=g).to(dt)
        oracle.sdpa_reference_route(q[:, :, :256], k[:, :, :256], v[:, :, :256], do[:, :, :256], causal=True)
    except RuntimeError:
        dt = torch.float32
        q, k, v, do = (t.float() for t in (q, k, v, do))
    times = []
    t_start = time.perf_counter()
    while len(times) < min_runs or (time.perf_counter() - t_start) < budget_s:
        t0 = time.perf_counter()
        oracle.sdpa_reference_route(q, k, v, do, causal=True)
        times.append(time.perf_counter() - t0)
        if len(times) >= 50:
            break
    per_unit = statistics.median(times)
    unit_flops = 3.5 * fwd_flops(1, group, s, s, d, True)
    return unit_flops / per_unit / 1e12, per_unit, ("bf16" if dt == torch.bfloat16 else "fp32"), len(times), torch.get_num_threads()


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU route on the host cores, rank 0 only.

    At N=1 every step is the full prefill config (B4 Hq32 Hkv8 S4096 D128
    bf16, causal, forward + autograd backward through PyTorch SDPA with native
    GQA, as ``backend="sdpa"`` runs it).  At N>1 the job (global batch 4N) is
    far beyond a bounded CPU run, so each step is one (batch, KV-head) unit of
    it and ``ms_per_step`` is that unit's measured time.  Throughput in
    TFLOP/s counts the same visible-pair FLOPs as the GPU arm."""
    if rank != 0:
        return 0
    use_all_host_cores()
    from oracle import attention_oracle as oracle

    g = torch.Generator().manual_seed(0)
    b, hq, hkv, s, d = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["S"], CFG["D"]
    group = hq // hkv
    full = world == 1
    shape_q = (b, hq, s, d) if full else (1, group, s, d)
    shape_k = (b, hkv, s, d) if full else (1, 1, s, d)
    q = (torch.randn(*shape_q, generator=g) * d ** -0.5).bfloat16()
    k = torch.randn(*shape_k, generator=g).bfloat16()
    v = torch.randn(*shape_k, generator=g).bfloat16()
    do = torch.randn(*shape_q, generator=g).bfloat16()
    dtn = "bf16"
    try:
        oracle.sdpa_reference_route(q[:1, :group, :256], k[:1, :1, :256], v[:1, :1, :256], do[:1, :group, :256],
                                    causal=True)
    except RuntimeError:
        q, k, v, do = (t.float() for t in (q, k, v, do))
        dtn = "fp32"
    for _ in range(args.warmup):
        oracle.sdpa_reference_route(q, k, v, do, causal=True)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.sdpa_reference_route(q, k, v, do, causal=True)
        times.append(time.perf_counter() - t0)
    per_step = statistics.median(times)
    step_flops = 3.5 * fwd_flops(shape_q[0], shape_q[1], s, s, d, True)
    tflops = step_flops / per_step / 1e12
    sample = ("the full config per step" if full else
              f"1 (batch, kv-head) unit of the job's {b * hkv * world} per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tflops, 4), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per_step * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtn, "data": "synthetic",
        "config": {"workload": "GQA causal prefill fwd+bwd B4 Hq32 Hkv8 S4096 D128 per rank "
                               "(BASELINE configs[1])",
                   "global_batch": 4 * world, "seq_len": s, "head_dim": d,
                   "parallelism": "host CPU cores (rank 0 only)", "sample": sample},
        "cpu_baseline": {"value": round(tflops, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": f"{sample} ({dtn}): reference backend='sdpa' route "
                                                   "(PyTorch SDPA, native GQA) + autograd"},
        "e2e": {"value": round(tflops, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_decode_case(args, world, rank):
    """One decode shape, plain launches (no graph): for profiling and quick timing."""
    from kotflash_b200.attention import _decode_forward

    sq, sk = (int(x) for x in args.decode_case.split(","))
    g = torch.Generator(device="cuda").manual_seed(sk + sq)
    k = torch.randn(2, 2, sk, 64, device="cuda", generator=g).half()
    v = torch.randn(2, 2, sk, 64, device="cuda", generator=g).half()
    q = torch.randn(2, 8, sq, 64, device="cuda", generator=g).half()
    for _ in range(args.warmup):
        _decode_forward(q, k, v, scale=0.125, want_lse=False)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        _decode_forward(q, k, v, scale=0.125, want_lse=False)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    if rank == 0:
        alg = 1024 * sk + 4096 * sq + 64 * sq
        print(json.dumps({"decode_case": [sq, sk], "us_per_call": round(ms * 1e3, 2),
                          "hbm_gbs": round(alg / (ms * 1e-3) / 1e9, 1),
                          "note": "plain launches incl. host overhead; inputs L2-warm when < 126 MB"}))
    return 0


# --------------------------------------------------------------------------- main
def guarded(fn, *args, **kwargs):
    """Run an optional sub-benchmark; an exception becomes {"error": ...} in
    the line instead of ending the run (the headline is already measured).
    Every rank runs the same code, so a failure in a collective sub-benchmark
    is met by every rank alike."""
    try:
        return fn(*args, **kwargs)
    except Exception as exc:  # noqa: BLE001 - reported in the JSON line
        print(f"{getattr(fn, '__name__', fn)} failed: {type(exc).__name__}: {exc}", file=sys.stderr, flush=True)
        return {"error": f"{type(exc).__name__}: {str(exc).splitlines()[0][:200] if str(exc) else ''}"}


def detail(name, payload):
    """A detail line (no "metric" key): printed before the headline line."""
    print(json.dumps({"detail": name, "data": payload}), flush=True)


def bench_fp16_prefill(args, world, peaks):
    """The fp16 variant of the prefill config (same step, same timing rules)."""
    ns = argparse.Namespace(steps=args.steps, warmup=args.warmup, no_clocks=True)
    ms, fwd_ms, bwd_ms, _ = bench_prefill(ns, world, 0, 0, torch.float16)
    b, hq, s, d = CFG["B"], CFG["Hq"], CFG["S"], CFG["D"]
    f = fwd_flops(b, hq, s, s, d, True)
    tf = world * 3.5 * f / (ms * 1e-3) / 1e12
    return {"value": round(tf, 1), "ms_per_step": round(ms, 4),
            "frac": round(tf / world / peaks["bf16_tflops"], 4),
            "fwd_tflops": round(f / (fwd_ms * 1e-3) / 1e12, 1),
            "bwd_tflops": round(2.5 * f / (bwd_ms * 1e-3) / 1e12, 1)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode sub-benchmarks")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity block")
    ap.add_argument("--no-comparators", action="store_true",
                    help="skip timing PyTorch SDPA's own GPU backends and the decoder block")
    ap.add_argument("--only-prefill", action="store_true",
                    help="time only the headline prefill step (no fp16, cfg5, parity, decode, e2e, CPU or "
                         "comparator legs): the short command the ncu captures in profiles/ use")
    ap.add_argument("--only-odd-head-dim", action="store_true",
                    help="time only the odd-head-dim training config (BASELINE configs[4], sharded over "
                         "the ranks) and print its detail line: the command the cfg5 ncu captures use")
    ap.add_argument("--decode-case", default=None, metavar="SQ,SK",
                    help="time only the split-KV decode config (B2 Hq8 Hkv2 D64 fp16) at one "
                         "(Sq, Sk) with --warmup/--steps plain launches; prints one JSON line")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    if args.only_prefill:
        args.no_decode = args.no_cpu = args.no_e2e = args.no_parity = args.no_comparators = True

    if args.impl == "reference":
        # CPU only: no process group, no GPU; ranks other than 0 exit at once
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)

    world, rank, local = init_dist(args)
    from kotflash_b200 import _ext

    _ext.load()  # fail loudly when the kernel library is missing
    if args.decode_case:
        return run_decode_case(args, world, rank)
    if args.only_odd_head_dim:
        res = bench_odd_head_dim(load_peaks(), world, rank)
        if rank == 0:
            detail("odd_head_dim_training", res)
        if world > 1:
            import torch.distributed as dist

            barrier(world)
            dist.destroy_process_group()
        return 0
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    peaks = load_peaks()
    ms_step, fwd_ms, bwd_ms, clocks = bench_prefill(args, world, rank, local, dtype)
    b, hq, s, d = CFG["B"], CFG["Hq"], CFG["S"], CFG["D"]
    f_fwd = fwd_flops(b, hq, s, s, d, True)
    f_bwd = 2.5 * f_fwd
    per_rank = f_fwd + f_bwd
    value = world * per_rank / (ms_step * 1e-3) / 1e12

    e2e = None
    if not args.no_e2e:
        e2e_ms, h2d, d2h, copy_ms = bench_prefill_e2e(args, world, rank, dtype)
        e2e = {"value": round(world * per_rank / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "ms_per_step": round(e2e_ms, 3),
               "copy_bound": {"ms_per_step": round(copy_ms, 3),
                              "tflops": round(world * per_rank / (copy_ms * 1e-3) / 1e12, 2),
                              "agg_gbs": round(world * (h2d + d2h) / (copy_ms * 1e-3) / 1e9, 1),
                              "frac": round(copy_ms / e2e_ms, 3),
                              "note": "the copies alone, all ranks at once"}}

    peak = peaks["bf16_tflops"]
    bwd_achieved = f_bwd / (bwd_ms * 1e-3) / 1e12
    fwd_achieved = f_fwd / (fwd_ms * 1e-3) / 1e12
    traffic = load_traffic() or {}
    roofline = {
        "bound": "tensor", "kernel": "kf_attn_bwd (prep + main + finish launches)",
        "achieved": round(bwd_achieved, 1), "peak": peak, "unit": "TFLOP/s",
        "frac": round(bwd_achieved / peak, 4),
        "traffic": traffic.get("bwd_main_bytes_per_launch"),
        "traffic_source": "ncu, one launch: profiles/traffic.json",
        "peak_source": f"{peaks['source']} (burst bf16 cuBLAS)",
        "forward": {"kernel": "kf_attn_fwd", "achieved": round(fwd_achieved, 1),
                    "frac": round(fwd_achieved / peak, 4),
                    "traffic": traffic.get("fwd_bytes_per_launch")},
        "step_frac": round(value / world / peak, 4),
    }

    fp16 = None if args.only_prefill else guarded(bench_fp16_prefill, args, world, peaks)
    odd = [] if args.only_prefill else guarded(bench_odd_head_dim, peaks, world, rank)
    parity = guarded(bench_parity) if (rank == 0 and not args.no_parity) else None

    decode = None
    multi = None
    if not args.no_decode:
        if world > 1:
            multi = guarded(bench_decode_multi_gpu, world, rank)
        elif rank == 0:
            decode = {"sweep": guarded(bench_decode_sweep, peaks), "kv_cache_loop": guarded(bench_cache_loop, peaks)}
    comparators = (guarded(bench_sdpa_comparators, dtype)
                   if (rank == 0 and world == 1 and not args.no_comparators) else None)
    block = ({"fp32_projections": guarded(bench_decoder_block),
              "bf16_block": guarded(bench_decoder_block, bf16_block=True)}
             if (rank == 0 and world == 1 and not args.no_comparators) else None)
    lm_ab = (guarded(bench_story_lm_ab) if (rank == 0 and world == 1 and not args.no_comparators) else None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        use_all_host_cores()
        tflops, per_unit, dtn, runs, threads = cpu_unit_sample(args.dtype)
        cpu = {"value": round(tflops, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{runs} x 1 (batch, kv-head) unit of 32 ({dtn}), backend='sdpa' + autograd, "
                         f"{per_unit:.2f} s/unit"}

    if rank == 0:
        if decode is not None:
            detail("decode_sweep", decode["sweep"])
        if odd and not isinstance(odd, dict):
            detail("odd_head_dim_training", odd)
        if comparators is not None:
            detail("gpu_comparators", comparators)
        if block is not None:
            detail("decoder_block_training_step", block)
        if lm_ab is not None:
            detail("lm_training_ab", lm_ab)
        if parity is not None and not parity.get("pass", False):
            print("parity check FAILED: " + json.dumps(parity), file=sys.stderr, flush=True)
        dec = None
        if decode is not None:
            dec = {}
            sweep, loop = decode["sweep"], decode["kv_cache_loop"]
            if isinstance(sweep, dict):
                dec["sweep"] = sweep
            else:
                keep = [r for r in sweep if r["sq"] == 1 or r["sk"] >= 32768]
                dec["cols"] = "sq,sk,us_per_call,us_per_token,hbm_frac"
                dec["rows"] = [[r["sq"], r["sk"], r["us_per_call"], r["us_per_token"], r["hbm_frac"]] for r in keep]
            dec["kv_cache_loop"] = loop if "error" in loop else {
                "us_per_token": loop["us_per_token"], "hbm_frac": loop["hbm_frac"],
                "prefill_append_hbm_frac": loop["prefill_append"]["hbm_frac"],
                "append_bit_exact": loop["append_bit_exact"]}
        if isinstance(odd, dict):
            cfg5 = odd
        else:
            cfg5 = None if not odd else {
                "cols": "d,causal,ms,fwd_bwd_tflops,per_rank_frac",
                "rows": [[r["d"], int(r["causal"]), r["ms"], r["fwd_bwd_tflops"], r["per_rank_frac"]] for r in odd],
                "units_per_rank": odd[0]["units_per_rank"], "scaling": "strong (8 units over the ranks)"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": args.dtype, "data": "synthetic",
            "config": {"workload": "GQA causal prefill fwd+bwd B4 Hq32 Hkv8 S4096 D128 per rank "
                                   "(BASELINE configs[1])",
                       "global_batch": 4 * world, "seq_len": s, "head_dim": d,
                       "parallelism": f"(batch x kv-head) units, {world} rank(s), no collective",
                       "l2": "inputs larger than L2 (q/dO 134 MB each)"},
            "frac_of_peak": round(value / world / peak, 4),
            "roofline": roofline, "clocks": clocks,
            "gpu_launches": 4 * args.steps,  # per step: forward, backward prep, main, finish
            "e2e": e2e, "cpu_baseline": cpu,
            # extras: the end of the line is what a 1500-character tail keeps
            "decode_multi_gpu": multi, "cfg5": cfg5, "fp16": fp16,
            "fwd": {"tflops": round(fwd_achieved, 1), "frac": round(fwd_achieved / peak, 4),
                    "bwd_tflops": round(bwd_achieved, 1), "bwd_frac": round(bwd_achieved / peak, 4)},
            "decode": dec, "parity": parity,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
