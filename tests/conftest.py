"""Shared test setup: markers, import helpers for the package (hyphenated directory) and the oracle."""
import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / 'tests' / 'golden'
if str(GOLDEN) not in sys.path:
    sys.path.insert(0, str(GOLDEN))

PKG = 'hybrid-latent-attention_b200'


def pkg(module=None):
    """Import the package or one of its modules by name (the directory name has hyphens)."""
    return importlib.import_module(PKG if module is None else f'{PKG}.{module}')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a) and libhla_s6.so')


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason='no CUDA device')
    for item in items:
        if 'gpu' in item.keywords:
            item.add_marker(skip)
