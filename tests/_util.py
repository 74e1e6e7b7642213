# SPDX-License-Identifier: Apache-2.0
"""Shared test helpers: tolerance checks that print the measured max error."""
import torch

TOL = 2e-2  # atol = rtol for fp16/bf16 outputs, LSE and gradients vs the fp32 oracle

# (name, max abs error, worst error / tolerance) of every check in this process;
# conftest prints a summary line at the end of the run
RECORDS = []


def check_close(actual, expected, *, name="", atol=TOL, rtol=TOL):
    a = actual.float()
    e = expected.float().to(a.device)
    finite = torch.isfinite(e)
    assert torch.equal(torch.isfinite(a), finite), f"{name}: non-finite pattern differs"
    diff = (a - e).abs()[finite]
    max_err = diff.max().item() if diff.numel() else 0.0
    bound = (atol + rtol * e.abs())[finite]
    worst = (diff - bound).max().item() if diff.numel() else -1.0
    ratio = (diff / bound).max().item() if diff.numel() else 0.0
    RECORDS.append((name, max_err, ratio))
    print(f"[parity] {name}: max_abs_err={max_err:.3e}")
    assert worst <= 0, f"{name}: max abs error {max_err:.3e} exceeds atol={atol} rtol={rtol}"
    return max_err


def sm100():
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
