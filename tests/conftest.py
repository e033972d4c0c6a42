"""pytest setup: import paths, the `gpu` marker, checked mode for the CUDA kernels."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "sparse-memory-lm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

# every kernel call in the tests synchronises and checks the device status word (out-of-range rows)
os.environ.setdefault("SMLM_B200_CHECK", "1")

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
