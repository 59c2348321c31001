import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


_PARITY_LINES = []


import pytest  # noqa: E402


@pytest.fixture
def parity_report(request):
    """Record a one-line parity figure (errors, excused selections) that the
    session summary prints, so the measured margins appear in the log of a
    quiet run."""
    return lambda msg: _PARITY_LINES.append(f"{request.node.nodeid}: {msg}")


def pytest_terminal_summary(terminalreporter):
    if _PARITY_LINES:
        terminalreporter.write_sep("-", "parity figures")
        for line in _PARITY_LINES:
            terminalreporter.write_line(line)
