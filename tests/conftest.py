import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / 'qwen38-sparse-attn_b200'
for p in (str(ROOT), str(PKG), str(ROOT / 'tests')):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')
    config.addinivalue_line('markers', 'slow: long-running CPU test')


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason='no CUDA device')
    for it in items:
        if 'gpu' in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope='session')
def golden():
    import numpy as np
    return dict(np.load(ROOT / 'tests' / 'golden' / 'golden.npz'))


def unpack_mask(g, key):
    import numpy as np
    shape = tuple(int(s) for s in g[key + '_shape'])
    return np.unpackbits(g[key], axis=-1, count=shape[-1]).astype(bool).reshape(shape)
