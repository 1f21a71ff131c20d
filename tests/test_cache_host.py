"""Host bookkeeping of the product cache on CPU, with the oracle standing in for the kernels.

The cache's growth decisions, views, counters and lifetimes are host logic; here
the product's ``_ops`` kernel front end is replaced by tests/cpu_ops.py (oracle
row moves on CPU tensors) and results are compared with the reference's
recorded behaviour. test_cache_gpu.py runs the same scenarios on the CUDA path.
"""
import pytest

import analysis_spec_b200.opd_static_cache as cache_mod
from tests import cache_scenarios, cpu_ops


@pytest.fixture(autouse=True)
def oracle_ops(monkeypatch):
    monkeypatch.setattr(cache_mod, '_ops', cpu_ops)


@pytest.mark.parametrize('scenario', cache_scenarios.SCENARIOS_WITH_GOLDEN, ids=lambda f: f.__name__)
def test_reference_scenarios_with_golden(golden, scenario):
    scenario(golden, 'cpu')


@pytest.mark.parametrize('scenario', cache_scenarios.SCENARIOS, ids=lambda f: f.__name__)
def test_reference_scenarios(scenario):
    scenario('cpu')


def test_product_kernels_refuse_cpu_tensors(monkeypatch):
    import torch
    from analysis_spec_b200 import _ops
    monkeypatch.undo()
    with pytest.raises(RuntimeError, match='need CUDA tensors'):
        _ops.append_rows([torch.zeros(1, 1, 4, 2)], [torch.zeros(1, 1, 4, 2)], [torch.zeros(1, 1, 1, 2)],
                         [torch.zeros(1, 1, 1, 2)], 0)
    with pytest.raises(RuntimeError, match='need CUDA tensors'):
        cache_mod.OPDStaticCache(8).update(torch.zeros(1, 1, 1, 2), torch.zeros(1, 1, 1, 2), 0)
