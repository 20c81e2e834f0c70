"""Test configuration: the ``gpu`` marker, import paths and shared helpers.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on the
CPU.  The package lives in ``flashinfer-competition-codebase_b200/`` (not an
importable name), so that directory and the repository root (for ``oracle``)
go on ``sys.path`` here.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "flashinfer-competition-codebase_b200")
for p in (PKG_ROOT, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def gdn_lib():
    """The built C-ABI library (built here if missing; needs nvcc)."""
    from gdn_b200 import build, _lib

    build.build()
    return _lib.load()
