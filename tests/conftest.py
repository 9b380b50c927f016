"""Shared fixtures. GPU tests are marked `gpu` (run with -m gpu on a B200);
everything else runs on CPU."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))
GOLDEN = Path(__file__).resolve().parent / "golden"

# the reference's kernel-test shapes (tests/test_kernels.py:12-13 of lowbit)
SHAPES = [(1, 1, 1), (1, 64, 128), (3, 5, 127), (7, 33, 129), (5, 37, 300),
          (17, 70, 1000), (2, 16, 4096 + 32)]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN / "golden.npz"))


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def case(g, i, tag):
    """Inputs and reference outputs of golden shape i for an int4 tag (sym/asym/smax)."""
    p = f"s{i}_"
    return dict(x=g[p + "x"], w=g[p + "w"], qw=g[p + f"{tag}_qw"], scales=g[p + f"{tag}_scales"],
                zeros=g.get(p + f"{tag}_zeros"))
