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


def _fused_pair(monkeypatch, layers=2, batch=3, heads=2, past=10):
    """A fuse_append cache and a plain one holding the same prefix; on CPU the rows a fused
    update leaves pending are stored by whichever cache operation comes next."""
    import torch
    monkeypatch.setattr(cache_mod.StaticAppendLayer, '_fusable',
                        lambda self, k, v: self.owner is not None and self.owner.fuse_append)
    torch.manual_seed(0)
    fused = cache_mod.OPDStaticCache(16, batch_capacity=batch, chunk_size=16, fuse_append=True)
    plain = cache_mod.OPDStaticCache(16, batch_capacity=batch, chunk_size=16)
    for l in range(layers):
        k, v = torch.randn(batch, heads, past, 8).bfloat16(), torch.randn(batch, heads, past, 8).bfloat16()
        fused.update(k, v, l)
        plain.update(k, v, l)
    return fused, plain


def _same(fused, plain):
    import torch
    assert [l.length for l in fused.layers] == [l.length for l in plain.layers]
    assert [l.batch_size for l in fused.layers] == [l.batch_size for l in plain.layers]
    for a, b in zip(fused.layers, plain.layers):
        assert a._pending is None
        assert torch.equal(a.keys.view(torch.int16), b.keys.view(torch.int16))
        assert torch.equal(a.values.view(torch.int16), b.values.view(torch.int16))


def _new_rows(layers=2, batch=3, heads=2, rows=4):
    import torch
    return [(torch.randn(batch, heads, rows, 8).bfloat16(), torch.randn(batch, heads, rows, 8).bfloat16())
            for _ in range(layers)]


@pytest.mark.parametrize('then', ['read', 'update', 'crop', 'select', 'repeat', 'swap_remove', 'commit',
                                  'update_layers', 'grow'])
def test_fused_append_rows_are_stored_before_the_next_operation(monkeypatch, then):
    """OPDStaticCache(fuse_append=True): an update returns views with its rows still pending
    (left to the verify attention); every other cache operation stores them first, so the
    cache ends as a plain cache given the same calls."""
    import torch
    fused, plain = _fused_pair(monkeypatch)
    rows = _new_rows()
    for c in (fused, plain):
        for l, (k, v) in enumerate(rows):
            keys, values = c.update(k, v, l)
            assert keys.shape[-2] == 14
    assert all(l._pending is not None for l in fused.layers)
    # only the views update returned carry the pending rows
    assert getattr(fused.layers[0]._view(fused.layers[0].key_pool), '_speckv_pending', None) is None
    more = _new_rows(rows=3)
    big = _new_rows(rows=5)
    for c in (fused, plain):
        if then == 'read':
            _ = [(l.keys, l.values) for l in c.layers]
        elif then == 'update':
            for l, (k, v) in enumerate(more):
                c.update(k, v, l)
        elif then == 'crop':
            c.crop(12)
        elif then == 'select':
            c.batch_select_indices(torch.tensor([2, 0]))
        elif then == 'repeat':
            c.batch_repeat_interleave(2)
        elif then == 'swap_remove':
            c.swap_remove(2, torch.tensor([2]), torch.tensor([0]))
        elif then == 'commit':
            chosen = torch.tensor([[10, 12, 13], [10, 11, 13], [10, 13, 12]])
            c.commit_accepted(chosen, 10, 1)
        elif then == 'update_layers':
            c.update_layers([k for k, _ in more], [v for _, v in more])
        elif then == 'grow':  # an append past the capacity copies the history into new pools
            for l, (k, v) in enumerate(big):
                c.update(k, v, l)
    fused.flush()  # rows a final fused update left pending (update / grow) are stored now
    _same(fused, plain)


def test_fused_append_pending_rows_are_dropped_by_reset(monkeypatch):
    fused, plain = _fused_pair(monkeypatch)
    for l, (k, v) in enumerate(_new_rows()):
        fused.update(k, v, l)
    fused.begin_rollout(3, 3)
    assert all(l._pending is None and l.length == 0 for l in fused.layers)


def test_verify_attention_takes_the_fused_kernel_only_for_matching_pending_rows(monkeypatch):
    """tree_verify_attention's choice for views of a fuse_append cache (kernels stubbed): pending
    rows that are exactly the query's tree rows go to speckv_tree_attention_bits_append (and are
    then no longer pending); any other shape stores them first and runs the bits kernel."""
    import torch
    from types import SimpleNamespace
    from analysis_spec_b200 import tree_attention
    calls = []
    stub = SimpleNamespace(
        tree_attention_bits_append=lambda q, kp, vp, past, k, v, bits, first, scale, out=None: calls.append(
            ('fused', past, k.shape[-2])) or torch.zeros(q.shape[0], q.shape[2], q.shape[1], q.shape[3]),
        tree_attention_bits=lambda q, k, v, bits, first, scale, row_table=None: calls.append(
            ('bits', k.shape[-2])) or torch.zeros(q.shape[0], q.shape[2], q.shape[1], q.shape[3]))
    monkeypatch.setattr(tree_attention, '_ops', stub)
    fused, _ = _fused_pair(monkeypatch)
    rows = _new_rows(rows=4)
    module = SimpleNamespace(is_causal=True, training=False)
    vis = SimpleNamespace(bits=None, first_col=None, past=10, rows=4)
    for l, (k, v) in enumerate(rows):
        keys, values = fused.update(k, v, l)
        q = torch.zeros(3, 4, 4, 8).bfloat16()
        tree_attention.tree_verify_attention(module, q, keys, values, vis)
        assert fused.layers[l]._pending is None
    assert calls == [('fused', 10, 4), ('fused', 10, 4)]
    calls.clear()
    keys, values = fused.update(*_new_rows(rows=4)[0], 0)  # pending again at position 14
    q = torch.zeros(3, 4, 2, 8).bfloat16()  # 2 query rows for 4 pending rows: not the fused case
    tree_attention.tree_verify_attention(module, q, keys, values, SimpleNamespace(bits=None, first_col=None,
                                                                                  past=16, rows=2))
    assert calls == [('bits', 18)] and fused.layers[0]._pending is None
