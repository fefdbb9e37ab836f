import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "s1-infer_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libs1kv.so")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def s1kv():
    """The product binding.  On a GPU run the library must exist: a missing
    build is a failure, not a skip."""
    import s1kv as S
    S.lib()
    return S


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "gpu test without a CUDA device"
    torch.cuda.set_device(0)
    return torch


def seeded(seed):
    return np.random.default_rng(seed)


def shuffled_free_list(max_blocks, seed):
    """A seeded permutation of 0..max_blocks-1 (free list bottom .. top)."""
    return np.random.default_rng(seed).permutation(max_blocks).astype(np.int32)
