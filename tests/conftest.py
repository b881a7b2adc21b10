"""Test configuration: the ``gpu`` marker, deterministic seeds and the in-tree package on the path."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")
    config.addinivalue_line("markers", "slow: long-running test")
    # the e3nn stand-in goes in before any test can import the reference package: a reference
    # module imported without it would record e3nn as missing for the rest of the process
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    if tests_dir not in sys.path:
        sys.path.insert(0, tests_dir)
    from ref_oracle import _stub_e3nn
    _stub_e3nn()


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _seed():
    import torch
    torch.manual_seed(0)
    yield
