"""Shared fixtures. GPU tests carry @pytest.mark.gpu; `-m "not gpu"` runs on CPU only."""
import importlib.util
import sys
from functools import lru_cache
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / 'golden'
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def _load_oracle():
    spec = importlib.util.spec_from_file_location('mica_oracle', ROOT / 'oracle' / 'mica_oracle.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


ORACLE = _load_oracle()


def _load_oracle_c():
    spec = importlib.util.spec_from_file_location('mica_oracle_c', ROOT / 'oracle' / 'oracle_c.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


ORACLE_C = _load_oracle_c()


@lru_cache(maxsize=None)
def golden(name):
    return np.load(GOLDEN / f'{name}.npz')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (sm_100a) GPU')


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if cuda_ok():
        return
    skip = pytest.mark.skip(reason='needs a B200 GPU')
    for item in items:
        if 'gpu' in item.keywords:
            item.add_marker(skip)
