import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, 'tests', 'golden')
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA B200 (sm_100a) device')


def load_golden(name):
    with np.load(os.path.join(GOLDEN, f'{name}.npz')) as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope='session')
def golden():
    return load_golden


@pytest.fixture(scope='session')
def pkg():
    """The product package (directory name is not a Python identifier)."""
    return importlib.import_module('qwen3-dspark_b200')
