"""The previous round's compaction folded into the next round's append (speckv_append_commit_rows).

OPDStaticCache.update_layers(keys, values, commit=(chosen, past, extension, width)) must leave
every pool byte as the two steps it replaces: the accepted-suffix compaction of every layer
(compact_suffix_inplace, helper/opd_scheduling.py:35-58, here commit_accepted) followed by the
append of the next round's rows (StaticAppendLayer.update, helper/opd_static_cache.py:99-109).
Checked for a growing cache (the next rows land after the committed ones) and for a cache
cropped back below past + width (the new rows overwrite the compacted ones), for the fused
kernel and for shapes past its register stage (two launches), and for the positions-only
commit of a round whose compaction is folded.
"""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200.opd_static_cache import OPDStaticCache

pytestmark = pytest.mark.gpu


def accepted(rng, batch, past, rows, width):
    """Cache positions of accepted paths: slot 0 the root, then increasing tree rows."""
    chosen = np.empty((batch, width), dtype=np.int64)
    for b in range(batch):
        n = rng.randint(1, width + 1)
        idx = np.sort(rng.choice(np.arange(1, rows), size=n - 1, replace=False)) if n > 1 else np.array([], int)
        picks = np.concatenate([[0], idx, np.arange(n, width)])  # padding slots: the identity
        chosen[b] = past + picks[:width]
    return torch.from_numpy(chosen).cuda()


def make(layers, batch, heads, past, seed, capacity=1024):
    gen = torch.Generator(device='cuda').manual_seed(seed)
    cache = OPDStaticCache(capacity, batch_capacity=batch)
    prefix = [(0.5 * torch.randn(batch, heads, past, 128, device='cuda', generator=gen)).bfloat16()
              for _ in range(2 * layers)]
    cache.update_layers(prefix[:layers], prefix[layers:])
    return cache, gen


def new_rows(gen, layers, batch, heads, rows):
    ks = [(0.5 * torch.randn(batch, rows, heads * 128, device='cuda', generator=gen)).bfloat16()
          .view(batch, rows, heads, 128).transpose(1, 2) for _ in range(layers)]
    vs = [(0.5 * torch.randn(batch, rows, heads * 128, device='cuda', generator=gen)).bfloat16()
          .view(batch, rows, heads, 128).transpose(1, 2) for _ in range(layers)]
    return ks, vs


@pytest.mark.parametrize('grow', [True, False])
@pytest.mark.parametrize('rows2', [17, 61, 300])
def test_folded_commit_equals_compaction_then_append(grow, rows2):
    layers, batch, heads, past, rows, width = 3, 8, 2, 300, 61, 7
    rng = np.random.RandomState(rows2 + grow)
    out = []
    for fold in (False, True):
        cache, gen = make(layers, batch, heads, past, seed=5)
        k1, v1 = new_rows(gen, layers, batch, heads, rows)
        cache.update_layers(k1, v1)  # round 1's tree rows at [past, past + rows)
        chosen = accepted(np.random.RandomState(rows2 + grow), batch, past, rows, width)
        ext = 1
        k2, v2 = new_rows(gen, layers, batch, heads, rows2)
        if fold:
            cache.crop(past + width if grow else past)
            cache.update_layers(k2, v2, commit=(chosen, past, ext, width))
        else:
            cache.commit_accepted(chosen, past, ext)  # compacts, crops to past + width
            if not grow:
                cache.crop(past)
            cache.update_layers(k2, v2)
        torch.cuda.synchronize()
        out.append([(l.key_pool.clone(), l.value_pool.clone(), l.length) for l in cache.layers])
    for (k0, v0, n0), (k1, v1, n1) in zip(*out):
        assert n0 == n1
        assert torch.equal(k0[:, :, :n0].view(torch.int16), k1[:, :, :n1].view(torch.int16))
        assert torch.equal(v0[:, :, :n0].view(torch.int16), v1[:, :, :n1].view(torch.int16))
    assert _ops.device_error() is None
    del rng


def test_positions_only_commit_leaves_the_pools():
    """compact=False: positions and padding are updated from the device packet, K/V untouched."""
    layers, batch, heads, past = 2, 4, 2, 40
    cache, gen = make(layers, batch, heads, past, seed=9, capacity=256)
    k1, v1 = new_rows(gen, layers, batch, heads, 9)
    cache.update_layers(k1, v1)
    before = [l.key_pool.clone() for l in cache.layers]
    width = 4
    chosen = accepted(np.random.RandomState(2), batch, past, 9, width)
    packet = torch.zeros(batch, width + 4, dtype=torch.long, device='cuda')
    packet[:, 0] = torch.tensor([1, 4, 2, 3])
    packet[:, 2] = torch.tensor([1, 1, 2, 3])
    newly = torch.zeros(batch, width, dtype=torch.bool, device='cuda')
    newly[0, 1:] = True
    positions = torch.zeros(batch, width, dtype=torch.long, device='cuda')
    past_positions = torch.full((batch,), past - 1, dtype=torch.long, device='cuda')
    cache.commit_scheduled(chosen, past, packet, newly_padded=newly, positions=positions,
                           past_positions=past_positions, compact=False)
    torch.cuda.synchronize()
    for l, k in zip(cache.layers, before):
        assert torch.equal(l.key_pool.view(torch.int16), k.view(torch.int16))
    expect = torch.cumsum(~newly, 1) + (past - 1)
    assert torch.equal(positions, expect)
    assert torch.equal(past_positions, expect[:, -1])
    assert _ops.device_error() is None
