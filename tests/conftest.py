"""Shared pytest setup: import paths, the ``gpu`` marker and golden fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / 'tests' / 'golden'
for p in (REPO, REPO / 'musc-gpu_b200'):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA B200 (sm_100) device and the built library')


def golden(name: str) -> dict:
    with np.load(GOLDEN / f'{name}.npz') as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope='session')
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('GPU test collected without a CUDA device (run with -m "not gpu" on CPU)')
    cap = torch.cuda.get_device_capability(0)
    assert cap == (10, 0), f'expected a B200 (sm_100), found sm_{cap[0]}{cap[1]}'
    return torch.device('cuda:0')
