"""Cache scenarios of the reference's hot-path tests, parametrised by device.

Run on CPU by test_cache_host.py (oracle row moves standing in for the kernels)
and on CUDA by test_cache_gpu.py (the product kernels). Expected values come
from the reference's own code (tests/golden/*.npz); the scenarios follow the
reference's tests/test_opd_memory_revision.py:13-72,
tests/test_opd_last_three.py:15-56 and tests/test_opd_final_optimization.py:14-35.
"""
import weakref

import numpy as np
import pytest
import torch

from analysis_spec_b200.opd_static_cache import OPDStaticCache, persistent_cache, swap_remove_plan

STAT_KEYS = ('pool_allocations', 'full_kv_reallocations', 'full_history_copies', 'full_history_copy_bytes',
             'row_compactions', 'row_compaction_bytes', 'kv_cache_bytes', 'kv_rows_moved', 'kv_history_copy_bytes')


def stats_vec(c):
    s = c.statistics()
    return np.array([s[k] for k in STAT_KEYS], dtype=np.int64)


def to(device, x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device)


def idx(device, values):
    return torch.tensor(np.asarray(values).tolist(), dtype=torch.long, device=device)


def growth_repeat_select_crop(golden, device):
    g = golden('kv_sequence')
    full, suffix = g['full'], g['suffix']
    c = OPDStaticCache(8, batch_capacity=8, chunk_size=8)
    step = 0
    for i, (start, end) in enumerate(g['bounds']):
        k, v = c.update(to(device, full[..., start:end, :]), to(device, full[..., start:end, :] + 1), 0)
        assert torch.equal(k, to(device, full[..., :end, :])) and torch.equal(v, to(device, full[..., :end, :] + 1))
        assert (c.layers[0].capacity, c.layers[0].batch_capacity) == tuple(g['caps'][i])
        assert np.array_equal(stats_vec(c), g['stats'][step])
        step += 1
    ptr = c[0][0].untyped_storage().data_ptr()
    c.batch_repeat_interleave(4)
    assert np.array_equal(stats_vec(c), g['stats'][step])
    step += 1
    for n in range(3):
        c.batch_select_indices(idx(device, g[f'select{n}']))
        assert torch.equal(c[0][0], to(device, g[f'after{n}']))
        assert c[0][0].untyped_storage().data_ptr() == ptr
        assert np.array_equal(stats_vec(c), g['stats'][step])
        step += 1
    c.crop(13)
    c.update(to(device, suffix), to(device, suffix + 1), 0)
    assert np.array_equal(stats_vec(c), g['stats'][step])
    assert torch.equal(c[0][0], to(device, g['final_k'])) and torch.equal(c[0][1], to(device, g['final_v']))
    assert c.get_seq_length() == int(g['final_len'])


def swap_remove_counters(golden, device):
    g = golden('swap_remove')
    for n in range(int(g['count'])):
        finished = g[f'finished{n}'].tolist()
        k = g[f'k{n}']
        b = len(finished)
        c = OPDStaticCache(256, batch_capacity=b)
        c.update(to(device, k), to(device, k + 1), 0)
        keep, sources, destinations = swap_remove_plan(finished)
        assert keep == g[f'keep{n}'].tolist()
        assert np.array_equal(stats_vec(c), g[f'stats_before{n}'])
        ptr = c.layers[0].key_pool.data_ptr()
        c.swap_remove(len(keep), idx(device, sources), idx(device, destinations))
        assert torch.equal(c[0][0], to(device, g[f'out_k{n}']))
        assert torch.equal(c[0][1], to(device, g[f'out_k{n}'] + 1))
        assert c.layers[0].key_pool.data_ptr() == ptr
        assert np.array_equal(stats_vec(c), g[f'stats_after{n}'])
        assert set(sources).isdisjoint(destinations) and all(s >= len(keep) for s in sources)


def persistent_pools(golden, device):
    g = golden('persistent')
    model = type('Model', (), {})()
    pointers = []
    c = None
    for iteration, row in enumerate(g['rows']):
        b, length = int(row[0]), int(row[1])
        c = persistent_cache(model, '_opd_target_kv_pool', b, 4, device, torch.float32)
        assert c.get_seq_length() == 0 and not c
        k = torch.full((b, 2, length, 7), float(iteration + 1), device=device)
        c.update(k, k + 10, 0)
        c.batch_repeat_interleave(4)
        assert torch.equal(c[0][0], k.repeat_interleave(4, 0))
        assert [c.layers[0].capacity, c.layers[0].batch_capacity] == row[2:4].tolist()
        assert np.array_equal(stats_vec(c), row[4:])
        pointers.append(c.layers[0].key_pool.data_ptr())
        c.end_rollout()
        assert c.get_seq_length() == 0 and c[0][0].shape[0] == 0
    assert len(set(pointers)) == 1
    c.end_rollout(max_retained_tokens=256)
    assert bool(g['released']) and not c.layers and not c._scratch


def append_crop_repeat_select(golden, device):
    g = golden('append_crop_repeat')
    c = OPDStaticCache(64)
    parts = [g['p0'], g['p1'], g['p2']]
    ptr = None
    for n, x in enumerate(parts):
        k, _ = c.update(to(device, x), to(device, x + 1), 0)
        ptr = k.untyped_storage().data_ptr() if ptr is None else ptr
        assert k.untyped_storage().data_ptr() == ptr
        assert torch.equal(k, to(device, np.concatenate(parts[:n + 1], axis=2)))
    c.crop(6)
    c.batch_repeat_interleave(2)
    assert torch.equal(c[0][0], to(device, g['repeated']))
    c.batch_select_indices(idx(device, [1, 3]))
    assert torch.equal(c[0][0], to(device, g['selected_k'])) and torch.equal(c[0][1], to(device, g['selected_v']))
    assert np.array_equal(stats_vec(c), g['stats'])
    c.crop(0)
    one = torch.ones(2, 3, 1, 4, device=device)
    c.update(one, one, 0)
    assert c.get_seq_length() == 1


def pools_freed_without_cycle(device):
    c = OPDStaticCache(8)
    x = torch.zeros(2, 3, 4, 5, device=device)
    c.update(x, x, 0)
    cache_ref, pool_ref = weakref.ref(c), weakref.ref(c.layers[0].key_pool)
    del c
    assert cache_ref() is None and pool_ref() is None


def reference_error_messages(device):
    with pytest.raises(ValueError, match='positive KV capacity'):
        OPDStaticCache(0)
    c = OPDStaticCache(8)
    z = torch.zeros(2, 1, 3, 4, device=device)
    c.update(z, z, 0)
    with pytest.raises(ValueError, match='KV batch differs'):
        w = torch.zeros(3, 1, 1, 4, device=device)
        c.update(w, w, 0)
    with pytest.raises(RuntimeError, match='external KV replacement'):
        c.layers[0].keys = torch.zeros(2, 1, 3, 4, device=device)
    with pytest.raises(ValueError, match='positive repeats'):
        c.batch_repeat_interleave(0)


def batched_layers_equal_per_layer(device):
    rng = np.random.RandomState(5)
    layers, b, h, d = 3, 4, 2, 6
    prefix = [rng.randn(b, h, 9, d).astype(np.float32) for _ in range(layers)]
    tree = [rng.randn(b, h, 5, d).astype(np.float32) for _ in range(layers)]
    c = OPDStaticCache(16, batch_capacity=b)
    for l in range(layers):
        c.update(to(device, prefix[l]), to(device, prefix[l] * 2), l)
    views = c.update_layers([to(device, x) for x in tree], [to(device, x * 2) for x in tree])
    for l in range(layers):
        assert torch.equal(views[l][0], to(device, np.concatenate([prefix[l], tree[l]], 2)))
    chosen_np = np.array([[9, 10, 12], [9, 11, 13], [9, 10, 11], [9, 13, 13]])
    c.commit_accepted(idx(device, chosen_np), 9, 1)
    assert c.get_seq_length() == 12
    for l in range(layers):
        full = np.concatenate([prefix[l], tree[l]], 2)
        gathered = np.take_along_axis(full, np.broadcast_to(chosen_np[:, None, :, None], (b, h, 3, d)), 2)
        expect = np.concatenate([full[:, :, :9], gathered], 2)
        assert torch.equal(c[l][0], to(device, expect))
        assert torch.equal(c[l][1], to(device, expect * 2))
    c.batch_select_indices(idx(device, [3, 3, 0]))
    assert c.kv_rows_moved == 3 and c[0][0].shape[0] == 3
    c.swap_remove(2, idx(device, [2]), idx(device, [1]))
    assert c.kv_rows_moved == 4 and c[2][0].shape[0] == 2


def deferred_update_layers(device):
    """update_layers(deferred=True) writes nothing and keeps the length until the returned
    callable runs, then equals the immediate form."""
    rng = np.random.RandomState(6)
    layers, b, h, d = 2, 3, 2, 4
    prefix = [rng.randn(b, h, 7, d).astype(np.float32) for _ in range(layers)]
    tree = [rng.randn(b, h, 4, d).astype(np.float32) for _ in range(layers)]
    c = OPDStaticCache(16, batch_capacity=b)
    for l in range(layers):
        c.update(to(device, prefix[l]), to(device, prefix[l] * 2), l)
    launch = c.update_layers([to(device, x) for x in tree], [to(device, x * 2) for x in tree], deferred=True)
    assert c.get_seq_length() == 7  # pools may have grown, but no row is written yet
    before = [l.key_pool.clone() for l in c.layers]
    views = launch()
    assert all(not torch.equal(p[:, :, 7:11], l.key_pool[:, :, 7:11]) for p, l in zip(before, c.layers))
    assert c.get_seq_length() == 11
    for l in range(layers):
        assert torch.equal(views[l][0], to(device, np.concatenate([prefix[l], tree[l]], 2)))
        assert torch.equal(views[l][1], to(device, np.concatenate([prefix[l], tree[l]], 2) * 2))


SCENARIOS_WITH_GOLDEN = (growth_repeat_select_crop, swap_remove_counters, persistent_pools, append_crop_repeat_select)
SCENARIOS = (pools_freed_without_cycle, reference_error_messages, batched_layers_equal_per_layer,
             deferred_update_layers)
