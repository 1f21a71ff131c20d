"""Rollout-history pools (ContiguousRolloutHistory, helper/opd_history.py:10-67) and the
accepted-feature gather fused with their append (helper/opd_generate.py:567-579).

Fixture tests/golden/history.npz: the reference class run on CPU through three verify
rounds (repeated initial copy, two capacity grows, rows finishing between rounds,
finalize), written by tests/golden/make_golden.py. Everything is compared bit for bit.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

FIELDS = ('generated_ids', 'features', 'input_ids')


def replay_oracle(g):
    hist = oracle.RolloutHistory({k: g[f'init_{k}'] for k in FIELDS}, int(g['repeats']), int(g['max_length']))
    gathered, caps = [], []
    for n in range(int(g['rounds'])):
        feats = oracle.gather_positions(g[f'r{n}_tree'], g[f'r{n}_index'])
        gathered.append(feats)
        tok = g[f'r{n}_next_token']
        hist.append(g[f'r{n}_owners'], {'generated_ids': tok, 'features': feats, 'input_ids': tok})
        for row in g[f'r{n}_finish']:
            hist.mark_finished(int(row))
        caps.append([hist.capacities[k] for k in FIELDS])
    return hist.finalize(), gathered, caps


def check_final(final, g):
    for name in FIELDS:
        assert [len(r[name]) for r in final] == g[f'final_{name}_lengths'].tolist()
        got = np.concatenate([np.asarray(r[name]) for r in final])
        assert np.array_equal(got.view(np.uint8), g[f'final_{name}'].view(np.uint8)), name


def test_oracle_history_matches_reference(golden):
    g = golden('history')
    final, gathered, caps = replay_oracle(g)
    for n in range(int(g['rounds'])):
        assert np.array_equal(gathered[n], g[f'r{n}_gathered'])
        assert caps[n] == g[f'r{n}_capacities'].tolist()
    check_final(final, g)


def test_history_host_validation():
    from analysis_spec_b200.opd_history import ContiguousRolloutHistory
    with pytest.raises(ValueError, match='positive'):
        ContiguousRolloutHistory({'generated_ids': torch.zeros(2, 3, dtype=torch.long)}, repeats=0, max_length=4)
    with pytest.raises(ValueError, match='batch sizes'):
        ContiguousRolloutHistory({'a': torch.zeros(2, 3), 'b': torch.zeros(3, 3)}, max_length=4)
    with pytest.raises(RuntimeError, match='CUDA'):
        ContiguousRolloutHistory({'generated_ids': torch.zeros(2, 3, dtype=torch.long)}, max_length=4)


def gpu_initial(g):
    return {k: torch.from_numpy(g[f'init_{k}']).cuda() for k in FIELDS}


@pytest.mark.gpu
@pytest.mark.parametrize('fused', [False, True])
def test_history_matches_reference(golden, fused):
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_history import ContiguousRolloutHistory
    g = golden('history')
    hist = ContiguousRolloutHistory(gpu_initial(g), repeats=int(g['repeats']), max_length=int(g['max_length']))
    for n in range(int(g['rounds'])):
        residual = g[f'r{n}_residual'].tolist()
        owners = torch.from_numpy(g[f'r{n}_owners']).cuda()
        tree = torch.from_numpy(g[f'r{n}_tree']).cuda()
        index = torch.from_numpy(g[f'r{n}_index']).cuda()
        tok = torch.from_numpy(g[f'r{n}_next_token']).cuda()
        if fused:
            feats = hist.append_accepted(residual, tok, tree, index, owners=owners)
        else:
            feats = tree.gather(dim=1, index=index.unsqueeze(-1).expand(len(residual), -1, tree.shape[-1]))
            hist.append(residual, {'generated_ids': tok, 'features': feats, 'input_ids': tok}, owners=owners)
        assert np.array_equal(feats.cpu().numpy().view(np.uint16), g[f'r{n}_gathered'].view(np.uint16))
        for row in g[f'r{n}_finish']:
            hist.mark_finished(int(row))
        assert [hist.capacities[k] for k in FIELDS] == g[f'r{n}_capacities'].tolist()
    final = hist.finalize()
    check_final([{k: v.cpu().numpy() for k, v in r.items()} for r in final], g)
    assert hist.buffers == {}
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.gpu
def test_history_rollout_scale_vs_oracle():
    """Qwen2.5-3B-like rounds: 64 live rows of 128 responses, 2048-wide bf16 features (as
    16-bit words), 61-row trees, accepted widths up to 7, rows finishing each round."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_history import ContiguousRolloutHistory
    rng = np.random.RandomState(5)
    batch, repeats, dim, tree_rows = 64, 2, 2048, 61
    init = {'generated_ids': rng.randint(0, 150000, size=(batch, 300)),
            'features': rng.randint(-30000, 30000, size=(batch, 300, dim)).astype(np.int16),
            'input_ids': rng.randint(0, 150000, size=(batch, 300))}
    hist = ContiguousRolloutHistory({k: torch.from_numpy(v).cuda() for k, v in init.items()}, repeats=repeats,
                                    max_length=320)
    ref = oracle.RolloutHistory(init, repeats, 320)
    live = list(range(batch * repeats))
    for rnd in range(5):
        rows = len(live)
        width = 7
        tree = rng.randint(-30000, 30000, size=(rows, tree_rows, dim)).astype(np.int16)
        index = np.stack([np.sort(rng.choice(tree_rows, width, replace=False)) for _ in range(rows)])
        tok = rng.randint(0, 150000, size=(rows, width))
        feats = hist.append_accepted(live, torch.from_numpy(tok).cuda(), torch.from_numpy(tree).cuda(),
                                     torch.from_numpy(index).cuda())
        expect = oracle.gather_positions(tree, index)
        ref.append(live, {'generated_ids': tok, 'features': expect, 'input_ids': tok})
        assert np.array_equal(feats.cpu().numpy(), expect)
        for row in rng.choice(live, size=rows // 4, replace=False):
            hist.mark_finished(int(row))
            ref.mark_finished(int(row))
            live.remove(int(row))
    final = hist.finalize()
    expect = ref.finalize()
    for got, want in zip(final, expect):
        for name in FIELDS:
            assert np.array_equal(got[name].cpu().numpy(), want[name]), name
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.gpu
def test_history_bad_owner_and_position_report_device_error():
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_history import ContiguousRolloutHistory
    assert _ops.device_error() is None
    hist = ContiguousRolloutHistory({'generated_ids': torch.zeros(2, 1, dtype=torch.long, device='cuda')},
                                    max_length=8)
    hist.append([0, 1], {'generated_ids': torch.ones(2, 2, dtype=torch.long, device='cuda')},
                owners=torch.tensor([0, 7], device='cuda'))
    torch.cuda.synchronize()
    assert _ops.device_error() == ('history index', 7)
    assert hist.buffers['generated_ids'][0, 1:3].tolist() == [1, 1]  # the valid row still lands
    tree = torch.zeros(2, 4, 3, dtype=torch.float16, device='cuda')
    hist.append_accepted([0, 1], torch.ones(2, 1, dtype=torch.long, device='cuda'), tree,
                         torch.tensor([[1], [9]], device='cuda'))
    torch.cuda.synchronize()
    assert _ops.device_error() == ('history index', 9)
