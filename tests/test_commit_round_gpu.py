"""Device-scheduled commit of a verify round (speckv_commit_round through
schedule_commit) against the host-scheduled commit and the CPU oracle: pools,
positions and padding bit-exact, including rounds where sequences finish."""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops, tree_kernels
from analysis_spec_b200.opd_scheduling import schedule, schedule_commit
from analysis_spec_b200.opd_static_cache import OPDStaticCache
from analysis_spec_b200.tree_verification import PackedTree, trace_verified_path
from oracle import oracle
from tests.test_tree_gpu import cu, random_packed_tree

pytestmark = pytest.mark.gpu


def _round_inputs(seed, batch, rows, depth, topk, past, layers, heads, dim, eos_rate):
    rng = np.random.RandomState(seed)
    vocab, eos = 5, 4
    parents, tokens = random_packed_tree(rng, batch, rows, depth, topk, vocab)
    samples = rng.randint(0, vocab, size=(batch, rows))
    if eos_rate == 0:
        samples[samples == eos] = 0
        tokens[tokens == eos] = 0
    contexts = rng.randint(-1, 50, size=(batch, rows))
    prefix = [rng.randn(batch, heads, past + rows, dim).astype(np.float32) for _ in range(2 * layers)]
    past_pos = rng.randint(0, 3000, size=batch).astype(np.int64)
    owners = rng.permutation(batch + 5)[:batch].astype(np.int64)
    return parents, tokens, contexts, samples, eos, prefix, past_pos, owners


def _cache(prefix, layers, past, rows, dtype):
    cache = OPDStaticCache(past + rows + 16, batch_capacity=prefix[0].shape[0])
    for l in range(layers):
        k = torch.from_numpy(prefix[2 * l]).cuda().to(dtype)
        v = torch.from_numpy(prefix[2 * l + 1]).cuda().to(dtype)
        cache.update(k[:, :, :past], v[:, :, :past], l)
    cache.update_layers([torch.from_numpy(prefix[2 * l][:, :, past:]).cuda().to(dtype) for l in range(layers)],
                        [torch.from_numpy(prefix[2 * l + 1][:, :, past:]).cuda().to(dtype) for l in range(layers)])
    return cache


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('batch,rows,depth,topk,past,eos_rate', [(64, 61, 6, 10, 300, 0), (64, 61, 6, 10, 300, 1),
                                                                 (5, 17, 4, 4, 40, 1), (33, 30, 9, 3, 7, 0)])
def test_schedule_commit_matches_host_commit_and_oracle(dtype, batch, rows, depth, topk, past, eos_rate):
    layers, heads, dim = 3, 2, 128
    parents, tokens, contexts, samples, eos, prefix, past_pos, owners = _round_inputs(
        batch + rows + past, batch, rows, depth, topk, past, layers, heads, dim, eos_rate)
    tree = PackedTree(cu(parents), cu(tokens), cu(contexts), depth)
    width_cap = depth + 1
    pad_cols = past + width_cap + 8

    # oracle round
    ot, oi, oc, ol = oracle.trace_path(parents, tokens, contexts, samples, eos, width_cap)
    _, o_idx, o_mask, _, o_packet, o_width = oracle.pad_schedule(ot, oi, ol, past, eos)
    live = o_packet[:, 1] == 0
    o_ext = int(o_packet[live, 2].min()) if live.any() else o_width
    o_pools = [p.copy() if dtype == torch.float32 else
               torch.from_numpy(p).to(dtype).view(torch.int16).numpy().copy() for p in prefix]
    for l in range(layers):
        bad = oracle.compact_suffix(o_pools[2 * l], o_pools[2 * l + 1], batch, past + rows, o_idx, past, o_ext)
        assert bad == 0
    o_rows = np.zeros((batch + 5, pad_cols), dtype=bool)
    o_live = np.zeros((batch, pad_cols), dtype=bool)
    o_pos, o_past = oracle.position_update(o_mask, past, past_pos, pad_rows=o_rows, owners=owners, pad_live=o_live)

    results = []
    for device_commit in (False, True):
        cache = _cache(prefix, layers, past, rows, dtype)
        path = trace_verified_path(tree, cu(samples), eos)
        positions = torch.full((batch, width_cap), -7, device='cuda', dtype=torch.long)
        pp = cu(past_pos)
        g_rows = torch.zeros(batch + 5, pad_cols, device='cuda', dtype=torch.bool)
        g_live = torch.zeros(batch, pad_cols, device='cuda', dtype=torch.bool)
        if device_commit:
            out = schedule_commit(path, past, eos, None, None, cache, positions, pp, pad_rows=g_rows,
                                  owners=cu(owners), pad_live=g_live, kernels=tree_kernels)
        else:
            out = schedule(path, past, eos, None, None, tree_kernels)
            r = out[0]
            ext = min([row[2] for row in r if row[1] == 0], default=out[5])
            cache.commit_accepted(out[2], past, ext)
            _ops.position_update(out[3], past, positions[:, :out[5]], pp, pad_rows=g_rows, owners=cu(owners),
                                 pad_live=g_live)
        torch.cuda.synchronize()
        assert _ops.device_error() is None
        width = out[5]
        assert width == o_width and out[0] == oracle.schedule_rows(o_packet)
        assert cache.get_seq_length() == past + width
        assert np.array_equal(positions[:, :width].cpu().numpy(), o_pos)
        assert np.array_equal(pp.cpu().numpy(), o_past)
        assert np.array_equal(g_rows.cpu().numpy(), o_rows) and np.array_equal(g_live.cpu().numpy(), o_live)
        pools = []
        for l in range(layers):
            for pool in (cache.layers[l].key_pool, cache.layers[l].value_pool):
                x = pool[:batch, :, :past + rows]
                x = x.view(torch.int16) if dtype == torch.bfloat16 else x
                pools.append(x.cpu().numpy())
        for got, exp in zip(pools, o_pools):
            assert np.array_equal(got[:, :, :past + width], exp[:, :, :past + width])
        results.append(pools)
    for a, b in zip(*results):
        assert np.array_equal(a, b)


def test_commit_round_positions_only_and_all_finished():
    batch, width, past = 9, 5, 20
    packet = torch.zeros(batch, 3 + width, device='cuda', dtype=torch.long)
    packet[:, 0] = torch.arange(batch, device='cuda') % width + 1
    packet[:, 1] = 1  # every sequence finished: extension = width, nothing to move
    rng = np.random.RandomState(0)
    newly = rng.rand(batch, width) < 0.5
    past_pos = rng.randint(0, 100, size=batch)
    exp_pos, exp_past = oracle.position_update(newly, past, past_pos)
    positions = torch.empty(batch, width, device='cuda', dtype=torch.long)
    pp = cu(past_pos.astype(np.int64))
    _ops.commit_round([], [], batch, 0, None, past, packet, newly_padded=cu(newly), positions=positions,
                      past_positions=pp)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    assert np.array_equal(positions.cpu().numpy(), exp_pos) and np.array_equal(pp.cpu().numpy(), exp_past)


def test_commit_round_rejects_packet_wider_than_schedule():
    batch, heads, dim, past, rows, width = 4, 2, 64, 10, 6, 4
    pools = [torch.randn(batch, heads, 32, dim, device='cuda') for _ in range(2)]
    before = [p.clone() for p in pools]
    packet = torch.zeros(batch, 3 + width, device='cuda', dtype=torch.long)
    packet[:, 0] = 2
    packet[1, 0] = width + 1  # longer than the schedule's columns
    chosen = torch.full((batch, width), past, device='cuda', dtype=torch.long)
    _ops.commit_round([pools[0]], [pools[1]], batch, past + rows, chosen, past, packet)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('scheduling packet', width + 1)
    assert all(torch.equal(a, b) for a, b in zip(pools, before))
