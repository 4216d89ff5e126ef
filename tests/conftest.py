"""Shared test setup.

* ``gpu`` marks tests that need a B200 (run with ``-m gpu``); everything else runs
  on CPU (``-m "not gpu"``).  GPU tests are skipped only when no CUDA device is
  visible at all; on a GPU box a missing native library is a failure, not a skip.
* The repository root (for ``oracle``) and ``ferrite-tpu_b200`` (for the
  ``ferrite`` package) are put on ``sys.path``.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "ferrite-tpu_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: large parity case")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def rng():
    return np.random.default_rng(0)


def pytest_report_header(config):
    dev = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    return f"ferrite-b200 device={dev} torch={torch.__version__}"
