import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / 'tests' / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200 / sm_100a) and the built libspeckv.so')


@pytest.fixture(scope='session')
def golden():
    import numpy as np

    def load(name):
        with np.load(GOLDEN / f'{name}.npz') as f:
            return {k: f[k] for k in f.files}
    return load
