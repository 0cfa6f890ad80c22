"""Shared test set-up: import paths, the `gpu` marker, golden-fixture loading."""
import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, 'colabfold-legacy-kernels_b200', 'src'))
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, 'tests', 'golden')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (sm_100) and the built CUDA library')


def golden(pattern):
    """Sorted (name, arrays) pairs of the fixtures matching pattern."""
    out = []
    for path in sorted(glob.glob(os.path.join(GOLDEN, pattern))):
        with np.load(path) as z:
            out.append((os.path.basename(path)[:-4], {k: z[k] for k in z.files}))
    return out


@pytest.fixture(scope='session')
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('a gpu-marked test ran without a CUDA device')
    return torch.device('cuda:0')
