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
