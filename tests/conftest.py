import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "deepseek-v4-flash_b200"))
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def pytest_terminal_summary(terminalreporter):
    """List the comparisons whose elements passed only by the one-ulp allowance."""
    try:
        from helpers import ULP_ONLY_LOG
    except ImportError:
        return
    tr = terminalreporter
    tr.section("elements within 1 bf16 ulp but beyond 2e-2 * RMS")
    if not ULP_ONLY_LOG:
        tr.write_line("none")
    for what, n, total in ULP_ONLY_LOG:
        tr.write_line(f"{what}: {n} of {total}")
