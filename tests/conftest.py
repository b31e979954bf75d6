import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built library")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Print the parity figures the scan tests recorded (errors are norm-wise
    relative: max|a - ref| / max|ref|)."""
    try:
        from helpers import PARITY_TABLE
    except ImportError:
        return
    if not PARITY_TABLE:
        return
    tr = terminalreporter
    tr.section("scan parity: norm-wise relative errors")
    tr.write_line("%-44s %-8s %-5s %10s %10s %10s  %s" % (
        "case", "output", "type", "vs fp32ref", "vs fp64", "ref vs 64", "verdict"))
    worst = {}
    for case, out, dt, e32, e64, r64, verdict in PARITY_TABLE:
        tr.write_line("%-44s %-8s %-5s %10.2e %10.2e %10.2e  %s" % (
            case[:44], out, dt, e32, e64, r64, verdict))
        if dt == "fp32" and out != "y":
            kind = "wide" if case.startswith("wide_") else "bench"
            key = (kind, "vs fp64" if kind == "wide" else "vs fp32ref")
            worst[key] = max(worst.get(key, 0.0), e64 if kind == "wide" else e32)
    for (kind, basis), v in sorted(worst.items()):
        tr.write_line("max fp32 gradient error, %s cases, %s: %.2e" % (kind, basis, v))
