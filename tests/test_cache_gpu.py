"""The product cache on CUDA: the reference's hot-path scenarios through libspeckv."""
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200.opd_static_cache import OPDStaticCache
from tests import cache_scenarios

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.parametrize('scenario', cache_scenarios.SCENARIOS_WITH_GOLDEN, ids=lambda f: f.__name__)
def test_reference_scenarios_with_golden(golden, scenario):
    scenario(golden, 'cuda')


@pytest.mark.parametrize('scenario', cache_scenarios.SCENARIOS, ids=lambda f: f.__name__)
def test_reference_scenarios(scenario):
    scenario('cuda')


@pytest.mark.parametrize('batch', [16, 32, 64])
def test_remap_race_free_for_permutations_with_duplicates(batch):
    # Race stress of tests/test_opd_memory_revision.py:74-91 in the reference.
    gen = torch.Generator(device='cuda').manual_seed(batch)
    c = OPDStaticCache(256, batch_capacity=batch)
    k = torch.randn(batch, 3, 517, 37, device='cuda', dtype=torch.bfloat16, generator=gen)
    v = torch.randn(batch, 3, 517, 37, device='cuda', dtype=torch.bfloat16, generator=gen)
    c.update(k, v, 0)
    ptr = c.layers[0].key_pool.data_ptr()
    for _ in range(5):
        ids = torch.randperm(batch, device='cuda', generator=gen)
        ids[-4:] = ids[:4]
        k, v = k.index_select(0, ids), v.index_select(0, ids)
        c.batch_select_indices(ids)
        assert torch.equal(c[0][0], k) and torch.equal(c[0][1], v)
        assert c.layers[0].key_pool.data_ptr() == ptr
    stats = c.statistics()
    assert stats['full_kv_reallocations'] == 0
    assert stats['kv_compaction_workspace_bytes'] <= 2 * stats['kv_cache_bytes']


def test_repeat_interleave_over_all_layers_in_one_call():
    gen = torch.Generator(device='cuda').manual_seed(1)
    layers = [torch.randn(8, 2, 300, 128, device='cuda', dtype=torch.bfloat16, generator=gen) for _ in range(5)]
    c = OPDStaticCache(256, batch_capacity=64)
    for l, x in enumerate(layers):
        c.update(x, x * 2, l)
    c.batch_repeat_interleave(8)
    for l, x in enumerate(layers):
        assert torch.equal(c[l][0], x.repeat_interleave(8, 0))
        assert torch.equal(c[l][1], (x * 2).repeat_interleave(8, 0))
    assert c.kv_rows_moved == 0
