# SPDX-License-Identifier: Apache-2.0
"""The decoder-block training step (the reference's
benchmarks/benchmark_decoder_block.py consumer of fwd+bwd): from the same
initial weights, a few AdamW steps with the kernels and with PyTorch SDPA give
the same losses and finite parameters."""
import pytest
import torch

import bench

pytestmark = pytest.mark.gpu


def test_decoder_block_steps_match_sdpa():
    torch.manual_seed(5)
    hq, hkv, d = 8, 2, 64
    x = torch.randn(2, 256, hq * d, device="cuda")
    target = torch.randn_like(x)
    init = {k: v.detach().clone() for k, v in bench.DecoderBlock(hq, hkv, d).state_dict().items()}
    losses = {}
    for backend in ("kotflash_b200", "sdpa_expanded_kv"):
        model = bench.DecoderBlock(hq, hkv, d).cuda()
        model.load_state_dict(init)
        opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
        losses[backend] = [float(bench.decoder_block_step(model, opt, x, target, backend)) for _ in range(4)]
        assert all(bool(torch.isfinite(p).all()) for p in model.parameters())
    print("[parity] decoder block losses", losses)
    for a, b in zip(losses["kotflash_b200"], losses["sdpa_expanded_kv"]):
        assert abs(a - b) <= 2e-3 * abs(b) + 1e-4
