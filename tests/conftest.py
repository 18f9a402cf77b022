"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a B200; the driver runs them with
  ``-m gpu`` on the GPU box and everything else with ``-m "not gpu"`` here);
* puts the package directory (``fast-cuda-cross-attention_b200``) and ``oracle`` on
  ``sys.path`` so tests import ``xattn``, ``cuda_wrappers`` and ``xattn_oracle``;
* skips ``gpu`` tests when no CUDA device is visible instead of failing them.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "fast-cuda-cross-attention_b200")
ORACLE = os.path.join(REPO, "oracle")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _cuda_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
