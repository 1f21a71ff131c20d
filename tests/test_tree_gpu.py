"""Tree kernels (pack / trace / pad / schedule packet / mask / positions) vs the reference's
golden vectors and the CPU oracle, exact."""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200 import tree_kernels
from analysis_spec_b200.opd_scheduling import compact_suffix_inplace, schedule
from analysis_spec_b200.tree_verification import PackedTree, VerifiedPath, pack_tree, trace_verified_path
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def cu(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize('case', range(4))
@pytest.mark.parametrize('plugin', [None, tree_kernels])
def test_golden_tree_pipeline(golden, case, plugin):
    g = golden('trees')
    c = f'c{case}_'
    eos = int(g['eos'])
    depth = int(g[c + 'depth'])
    past = int(g[c + 'past'])
    tree = pack_tree(cu(g[c + 'full_parents']), cu(g[c + 'full_contexts']), cu(g[c + 'chosen']),
                     cu(g[c + 'full_tokens']), depth)
    assert np.array_equal(tree.parents.cpu().numpy(), g[c + 'parents'])
    assert np.array_equal(tree.tokens.cpu().numpy(), g[c + 'tokens'])
    assert np.array_equal(tree.feedback_contexts.cpu().numpy(), g[c + 'contexts'])
    path = trace_verified_path(tree, cu(g[c + 'samples']), eos, kernels=plugin)
    assert np.array_equal(path.tokens.cpu().numpy(), g[c + 'triton_path_tokens'])
    assert np.array_equal(path.packed_indices.cpu().numpy(), g[c + 'triton_path_indices'])
    assert np.array_equal(path.feedback_contexts.cpu().numpy(), g[c + 'triton_path_contexts'])
    assert np.array_equal(path.lengths.cpu().numpy(), g[c + 'triton_path_lengths'])
    batch = path.tokens.shape[0]
    ws = [torch.empty(batch, depth + 1, device='cuda', dtype=torch.bool if i == 2 else torch.long) for i in range(3)]
    ws.append(torch.empty(batch, 1, device='cuda', dtype=torch.long))
    packet = torch.full((batch, depth + 5), -7, device='cuda', dtype=torch.long)
    rows, tok, idx, msk, last, width = schedule(path, past, eos, ws, packet, plugin)
    assert width == int(g[c + 'width'])
    expect_rows = g[c + 'packet'].tolist() if plugin is not None else \
        [[x for x in r if x != -9] for r in g[c + 'rows_torch'].tolist()]
    assert rows == expect_rows
    assert np.array_equal(tok.cpu().numpy(), g[c + 'pad_tokens'])
    assert np.array_equal(idx.cpu().numpy(), g[c + 'pad_indices'])
    assert np.array_equal(msk.cpu().numpy(), g[c + 'pad_mask'])
    assert np.array_equal(last.cpu().numpy(), g[c + 'pad_last'])
    padded = path.padded_gpu(past, width, eos, kernels=plugin)
    for a, e in zip(padded, ('pad_tokens', 'pad_indices', 'pad_mask', 'pad_last')):
        assert np.array_equal(a.cpu().numpy(), g[c + e])
    rows_n = tree.parents.shape[1]
    key, value = cu(g[c + 'key']), cu(g[c + 'value'])
    ka, va = compact_suffix_inplace(key[:, :, :past + rows_n], value[:, :, :past + rows_n], idx, past,
                                    int(g[c + 'extension']), object())
    assert np.array_equal(key.cpu().numpy(), g[c + 'key_out']) and np.array_equal(value.cpu().numpy(),
                                                                                  g[c + 'value_out'])
    assert ka.shape[2] == past + width and ka.untyped_storage().data_ptr() == key.untyped_storage().data_ptr()
    for dtype, name in ((torch.float32, 'visible'), (torch.bfloat16, 'visible_bf16')):
        m = tree.attention_mask(past, dtype, kernels=plugin)
        assert np.array_equal((m == 0).cpu().numpy()[:, 0], g[c + name])
        assert bool(((m == 0) | (m == torch.finfo(dtype).min)).all())
    m = tree.attention_mask(past, torch.float32, cu(g[c + 'pad']), kernels=plugin)
    assert np.array_equal((m == 0).cpu().numpy()[:, 0], g[c + 'visible_padded'])


def test_schedule_known_answer(golden):
    g = golden('schedule_kat')
    path = VerifiedPath(cu(g['tokens']), cu(g['indices']), cu(g['indices']), cu(g['lengths']))
    ws = [torch.empty(3, 4, device='cuda', dtype=torch.bool if i == 2 else torch.long) for i in range(3)]
    ws.append(torch.empty(3, 1, device='cuda', dtype=torch.long))
    packet = torch.empty(3, 7, device='cuda', dtype=torch.long)
    rows, t, i, m, last, width = schedule(path, 5, 16, ws, packet, tree_kernels)
    assert width == 3 and [r[0] for r in rows] == [3, 1, 2]
    assert np.array_equal(np.array(rows), g['triton_rows'][:, :7])
    for a, e in zip((t, i, m, last), ('triton_tokens', 'triton_indices', 'triton_mask', 'triton_last')):
        assert np.array_equal(a.cpu().numpy(), g[e])
    key, value = cu(g['key']), cu(g['value'])
    a, b = compact_suffix_inplace(key, value, i, 5, int(g['extension']), object())
    assert np.array_equal(a.cpu().numpy(), g['key_out']) and np.array_equal(b.cpu().numpy(), g['value_out'])


def test_packet_snapshot_column_sync_and_async():
    # tests/test_opd_profiles.py:224-236 of the reference: snapshot column of the packet.
    from types import SimpleNamespace
    path = VerifiedPath(cu(np.array([[4, 5]])), cu(np.array([[0, 1]])), cu(np.array([[0, 1]])), cu(np.array([2])))
    ws = [torch.empty(1, 2, device='cuda', dtype=torch.bool if i == 2 else torch.long) for i in range(3)]
    ws.append(torch.empty(1, 1, device='cuda', dtype=torch.long))
    packet = torch.empty(1, 6, device='cuda', dtype=torch.long)
    s = SimpleNamespace(host_sync_count=0, active_count=torch.tensor([9], device='cuda'),
                        dispatch_snapshot=torch.tensor([3], device='cuda'))
    for async_mode, expected in ((False, 9), (True, 3)):
        s.async_updates = async_mode
        schedule(path, 0, 99, ws, packet, tree_kernels, s)
        assert s.host_active_count == expected
    assert s.host_sync_count == 2


def random_packed_tree(rng, batch, rows, depth, topk, vocab):
    parents = np.full((batch, rows), -1, dtype=np.int64)
    for b in range(batch):
        dep = [0]
        kids = [0]
        for r in range(1, rows):
            cands = [p for p in range(r) if dep[p] < depth and kids[p] < topk]
            p = cands[rng.randint(len(cands))]
            parents[b, r] = p
            dep.append(dep[p] + 1)
            kids.append(0)
            kids[p] += 1
    tokens = rng.randint(0, vocab, size=(batch, rows))
    tokens[:, 0] = -1
    return parents, tokens


@pytest.mark.parametrize('batch,rows,depth,topk,past', [(64, 61, 6, 10, 2048), (256, 61, 6, 10, 700),
                                                       (3, 200, 12, 3, 5)])
def test_random_trees_vs_oracle(batch, rows, depth, topk, past):
    rng = np.random.RandomState(batch + rows)
    vocab, eos = 6, 5
    parents, tokens = random_packed_tree(rng, batch, rows, depth, topk, vocab)
    contexts = rng.randint(-1, 50, size=(batch, rows))
    samples = rng.randint(0, vocab, size=(batch, rows))
    tree = PackedTree(cu(parents), cu(tokens), cu(contexts), depth)
    path = trace_verified_path(tree, cu(samples), eos)
    ot, oi, oc, ol = oracle.trace_path(parents, tokens, contexts, samples, eos, depth + 1)
    for a, e in zip((path.tokens, path.packed_indices, path.feedback_contexts, path.lengths), (ot, oi, oc, ol)):
        assert np.array_equal(a.cpu().numpy(), e)
    rows_h, tok, idx, msk, last, width = schedule(path, past, eos, None, None, tree_kernels)
    et, ei, em, el, ep, ew = oracle.pad_schedule(ot, oi, ol, past, eos)
    assert width == ew and rows_h == ep.tolist()
    for a, e in zip((tok, idx, msk, last), (et, ei, em, el)):
        assert np.array_equal(a.cpu().numpy(), e)
    pad = rng.rand(batch, past + rows) < 0.3
    pad[:, past:] = False
    for dtype, name in ((torch.bfloat16, 'bfloat16'), (torch.float16, 'float16'), (torch.float32, 'float32')):
        m = tree.attention_mask(past, dtype, cu(pad))
        vis = oracle.tree_visible(parents, past, depth + 1, pad=pad)
        assert np.array_equal((m == 0).cpu().numpy()[:, 0], vis)
        assert bool(((m == 0) | (m == torch.finfo(dtype).min)).all())


def test_position_update_vs_oracle():
    rng = np.random.RandomState(4)
    batch, width, past = 37, 7, 300
    newly = rng.rand(batch, width) < 0.4
    past_pos = rng.randint(0, 1000, size=batch)
    owners = rng.permutation(64)[:batch]
    pad_rows = np.zeros((64, 400), dtype=bool)
    pad_live = np.zeros((batch, 400), dtype=bool)
    exp_pos, exp_past = oracle.position_update(newly, past, past_pos, pad_rows=pad_rows, owners=owners,
                                               pad_live=pad_live)
    g_rows, g_live = cu(np.zeros((64, 400), dtype=bool)), cu(np.zeros((batch, 400), dtype=bool))
    positions = torch.empty(batch, width, device='cuda', dtype=torch.long)
    pp = cu(past_pos.astype(np.int64))
    _ops.position_update(cu(newly), past, positions, pp, pad_rows=g_rows, owners=cu(owners.astype(np.int64)),
                         pad_live=g_live)
    assert np.array_equal(positions.cpu().numpy(), exp_pos) and np.array_equal(pp.cpu().numpy(), exp_past)
    assert np.array_equal(g_rows.cpu().numpy(), pad_rows) and np.array_equal(g_live.cpu().numpy(), pad_live)


def test_pack_tree_reports_unclosed_parent():
    full_parents = cu(np.array([[-1, 0, 1, 2]]))
    chosen = cu(np.array([[0, 2]]))  # node 2's parent (1) is not chosen
    tree = pack_tree(full_parents, full_parents.clone(), chosen, full_parents.clone(), 3)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('tree parent index', 2)
    assert tree.parents.cpu().tolist() == [[-1, 0, -1]]
