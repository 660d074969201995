"""Shared pytest setup.

Markers: ``gpu`` tests need a CUDA device (run with ``-m gpu`` on a B200);
everything else runs on CPU. The parity oracle (oracle/) is test
infrastructure; it is built here on first use.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def ms():
    import torch

    import musapy_b200 as ms

    if torch.cuda.is_available():
        # musapy has no implicit device (DeviceNotConfiguredError until one is set)
        ms.set_default_device("cuda:0")
    return ms


# Full-size parity tests report how many output elements they compared with
# the oracle; the counts are printed in pytest's terminal summary (also
# under -q), one line per check.
_COMPARED: list = []


@pytest.fixture
def compared(request):
    def note(what: str, n: int) -> None:
        _COMPARED.append((request.node.name, what, int(n)))
    return note


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not _COMPARED:
        return
    terminalreporter.write_sep("-", "full-size parity: elements compared with the oracle")
    for test, what, n in _COMPARED:
        terminalreporter.write_line(f"{test}: {what}: {n:,} elements")
