# SPDX-License-Identifier: Apache-2.0
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")


def pytest_collection_modifyitems(config, items):
    import torch

    has_gpu = torch.cuda.is_available()
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords and not has_gpu:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """One line with the largest measured error of the run's oracle checks."""
    try:
        from tests._util import RECORDS
    except ImportError:
        return
    if not RECORDS:
        return
    name, err, _ = max(RECORDS, key=lambda r: r[1])
    rname, rerr, ratio = max(RECORDS, key=lambda r: r[2])
    terminalreporter.write_line(
        f"[parity] {len(RECORDS)} checks vs the fp32 oracle (atol=rtol=2e-2): largest max_abs_err "
        f"{err:.3e} ({name}); closest to tolerance {ratio:.2f} of it ({rname}, {rerr:.3e})")


@pytest.fixture(autouse=True)
def _device_wait_status(request):
    """GPU tests must finish with no expired device-side wait."""
    if "gpu" not in request.keywords:
        yield
        return
    import torch

    from kotflash_b200 import _ext

    dev = torch.device("cuda", 0)
    _ext.clear_device_status(dev)
    yield
    torch.cuda.synchronize()
    assert _ext.read_device_status(dev) == 0, "a device-side bounded wait expired"
