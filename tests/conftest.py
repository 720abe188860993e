"""Shared pytest setup.

Markers: ``gpu`` — needs a CUDA (sm_100) device; everything else runs on CPU.
The repo root is put on sys.path so tests import ``luma_b200`` (the product)
and ``oracle`` (the test-only reference restatement) from the tree.
"""

import os
import random
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")


def seed_all(seed: int = 42):
    random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


@pytest.fixture(autouse=True)
def _seed():
    seed_all(42)
