"""Shared pytest setup: the ``gpu`` marker and torch seeding, as the reference's conftest does.

Tests marked ``gpu`` need a CUDA device and are skipped without one; everything else runs on
CPU. The repository root is put on ``sys.path`` so ``oracle`` and ``vinfer_b200`` import from
the checkout.
"""

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip_gpu = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip_gpu)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
