"""Generates the golden fixtures of tests/golden/ by running the REFERENCE's own code.

Run from the repository root with the reference checkout available:

    python tests/golden/make_golden.py /path/to/analysis_spec

(the path of the reference checkout is required).

The reference's torch (CPU) branch and its Triton kernels (executed on CPU
tensors by the Triton interpreter, TRITON_INTERPRET=1) produce the expected
outputs; inputs are seeded numpy draws. The fixtures pin the CPU oracle
(tests/test_oracle_golden.py) and the CUDA kernels (tests/test_*_gpu.py); the
tests themselves never read the reference.

Scenarios follow the reference's hot-path tests (tests/test_opd_memory_revision.py:43-72,
tests/test_opd_last_three.py:15-56, tests/test_opd_final_optimization.py:14-35,
tests/test_opd_revision.py:73-98) with inputs of our own, plus random draft
trees shaped like the 16-node and 60-node trees of the benchmark configurations.
"""
import os
import sys
from pathlib import Path
from types import SimpleNamespace

os.environ['TRITON_INTERPRET'] = '1'  # must precede the first triton import

import numpy as np  # noqa: E402
import torch  # noqa: E402

if len(sys.argv) < 2:
    sys.exit('usage: python tests/golden/make_golden.py /path/to/analysis_spec (the reference checkout)')
REF = Path(sys.argv[1]).resolve()
sys.path.insert(0, str(REF))
OUT = Path(__file__).resolve().parent

from helper import opd_kv_kernels as ref_kv  # noqa: E402
from helper import tree_kernels as ref_tk  # noqa: E402
from helper.opd_scheduling import compact_suffix_inplace, schedule  # noqa: E402
from helper.opd_static_cache import OPDStaticCache, persistent_cache, swap_remove_plan  # noqa: E402
from helper.tree_verification import pack_tree, trace_verified_path  # noqa: E402

STAT_KEYS = ('pool_allocations', 'full_kv_reallocations', 'full_history_copies', 'full_history_copy_bytes',
             'row_compactions', 'row_compaction_bytes', 'kv_cache_bytes', 'kv_rows_moved', 'kv_history_copy_bytes')


def stats_vec(cache):
    s = cache.statistics()
    return np.array([s[k] for k in STAT_KEYS], dtype=np.int64)


def save(name, **arrays):
    np.savez_compressed(OUT / f'{name}.npz', **{k: np.asarray(v) for k, v in arrays.items()})
    print('wrote', name, sum(np.asarray(v).nbytes for v in arrays.values()), 'bytes')


def t(x, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(x)) if dtype is None else torch.from_numpy(np.ascontiguousarray(x)).to(dtype)


# ---------------------------------------------------------------------------
def kv_sequence():
    """Append with geometric growth, repeat, duplicate-index select, crop, append (CPU branch)."""
    rng = np.random.RandomState(11)
    full = rng.randn(2, 3, 39, 5).astype(np.float32)
    suffix = rng.randn(2, 3, 6, 5).astype(np.float32)
    c = OPDStaticCache(8, batch_capacity=8, chunk_size=8)
    caps, stats = [], []
    bounds = [(0, 5), (5, 8), (8, 9), (9, 17), (17, 39)]
    for start, end in bounds:
        c.update(t(full[..., start:end, :]), t(full[..., start:end, :] + 1), 0)
        caps.append((c.layers[0].capacity, c.layers[0].batch_capacity))
        stats.append(stats_vec(c))
    c.batch_repeat_interleave(4)
    stats.append(stats_vec(c))
    selects = [[7, 0, 4, 2, 6], [4, 0, 0, 3], [3, 1]]
    after = []
    for ids in selects:
        c.batch_select_indices(torch.tensor(ids))
        after.append(c[0][0].numpy().copy())
        stats.append(stats_vec(c))
        caps.append((c.layers[0].capacity, c.layers[0].batch_capacity))
    c.crop(13)
    c.update(t(suffix), t(suffix + 1), 0)
    stats.append(stats_vec(c))
    save('kv_sequence', full=full, suffix=suffix, bounds=np.array(bounds), caps=np.array(caps),
         stats=np.stack(stats), select0=np.array(selects[0]), select1=np.array(selects[1]),
         select2=np.array(selects[2]), after0=after[0], after1=after[1], after2=after[2],
         final_k=c[0][0].numpy(), final_v=c[0][1].numpy(), final_len=c.get_seq_length())


def remap_move_triton():
    """remap_rows / move_tail_rows of the reference's Triton kernels (interpreted on CPU)."""
    rng = np.random.RandomState(12)
    k = rng.randn(6, 3, 21, 7).astype(np.float32)
    v = rng.randn(6, 3, 21, 7).astype(np.float32)
    idx = np.array([5, 0, 5, 2, 2, 1])
    kt, vt = t(k.copy()), t(v.copy())
    ref_kv.remap_rows(kt, vt, torch.tensor(idx), 17, torch.empty(1 << 14))
    k2, v2 = kt.numpy().copy(), vt.numpy().copy()
    src, dst = np.array([5, 4]), np.array([0, 2])
    ref_kv.move_tail_rows(kt, vt, torch.tensor(src), torch.tensor(dst), 19)
    save('remap_move', k=k, v=v, idx=idx, remap_len=17, k_remap=k2, v_remap=v2, src=src, dst=dst, move_len=19,
         k_move=kt.numpy(), v_move=vt.numpy())


def swap_remove_cases():
    patterns = [[0, 0, 0, 1], [1, 0, 0, 0], [0, 1, 1, 0, 0, 1, 0], [1, 0, 1, 0, 1, 0], [1, 1, 1]]
    out = {}
    rng = np.random.RandomState(13)
    for n, finished in enumerate(patterns):
        b = len(finished)
        k = rng.randn(b, 3, 37, 7).astype(np.float32)
        c = OPDStaticCache(256, batch_capacity=b)
        c.update(t(k), t(k + 1), 0)
        keep, sources, destinations = swap_remove_plan(finished)
        old = stats_vec(c)
        c.swap_remove(len(keep), torch.tensor(sources, dtype=torch.long), torch.tensor(destinations, dtype=torch.long))
        out[f'finished{n}'] = np.array(finished)
        out[f'k{n}'] = k
        out[f'keep{n}'] = np.array(keep, dtype=np.int64)
        out[f'sources{n}'] = np.array(sources, dtype=np.int64)
        out[f'destinations{n}'] = np.array(destinations, dtype=np.int64)
        out[f'out_k{n}'] = c[0][0].numpy()
        out[f'stats_before{n}'] = old
        out[f'stats_after{n}'] = stats_vec(c)
    save('swap_remove', count=len(patterns), **out)


def persistent_rollouts():
    model = SimpleNamespace()
    rows = []
    for iteration, (b, length) in enumerate(((2, 601), (1, 17), (2, 300), (2, 550))):
        c = persistent_cache(model, '_opd_target_kv_pool', b, 4, 'cpu', torch.float32)
        k = torch.full((b, 2, length, 7), float(iteration + 1))
        c.update(k, k + 10, 0)
        c.batch_repeat_interleave(4)
        rows.append(np.concatenate([[b, length, c.layers[0].capacity, c.layers[0].batch_capacity], stats_vec(c)]))
        c.end_rollout()
    c.end_rollout(max_retained_tokens=256)
    save('persistent', rows=np.stack(rows), released=int(not c.layers and not c._scratch))


def final_optimization():
    rng = np.random.RandomState(14)
    parts = [rng.randn(2, 3, n, 4).astype(np.float32) for n in (5, 3, 7)]
    c = OPDStaticCache(64)
    for x in parts:
        c.update(t(x), t(x + 1), 0)
    c.crop(6)
    c.batch_repeat_interleave(2)
    rep = c[0][0].numpy().copy()
    c.batch_select_indices(torch.tensor([1, 3]))
    sel_k, sel_v = c[0][0].numpy().copy(), c[0][1].numpy().copy()
    save('append_crop_repeat', p0=parts[0], p1=parts[1], p2=parts[2], repeated=rep, selected_k=sel_k,
         selected_v=sel_v, stats=stats_vec(c))


# ---------------------------------------------------------------------------
def schedule_kat():
    """Known-answer schedule packet + in-place suffix (tests/test_opd_revision.py:73-98 inputs)."""
    tokens = np.array([[4, 5, 6, -1], [7, -1, -1, -1], [8, 9, -1, -1]])
    indices = np.array([[0, 1, 4, -1], [0, -1, -1, -1], [0, 3, -1, -1]])
    lengths = np.array([3, 1, 2])
    from helper.tree_verification import VerifiedPath
    path = VerifiedPath(t(tokens), t(indices), t(indices.copy()), t(lengths))
    res = {}
    for tag, kernels in (('triton', ref_tk), ('torch', None)):
        ws = [torch.empty(3, 4, dtype=torch.bool if i == 2 else torch.long) for i in range(3)] + \
             [torch.empty(3, 1, dtype=torch.long)]
        packet = torch.full((3, 8), -7, dtype=torch.long)
        rows, tk, ik, mk, last, width = schedule(path, 5, 16, ws, packet, kernels)
        res[f'{tag}_rows'] = np.array([r + [-9] * (7 - len(r)) for r in rows])
        res[f'{tag}_tokens'] = tk.numpy()
        res[f'{tag}_indices'] = ik.numpy()
        res[f'{tag}_mask'] = mk.numpy()
        res[f'{tag}_last'] = last.numpy()
        res[f'{tag}_width'] = width
    rng = np.random.RandomState(15)
    key = rng.randn(3, 2, 12, 8).astype(np.float32)
    value = rng.randn(3, 2, 12, 8).astype(np.float32)
    kt, vt = t(key.copy()), t(value.copy())
    ext = min(r[2] for r in rows)
    a, b = compact_suffix_inplace(kt, vt, t(res['torch_indices']), 5, ext, SimpleNamespace())
    save('schedule_kat', tokens=tokens, indices=indices, lengths=lengths, past=5, eos=16, key=key, value=value,
         extension=ext, key_out=a.numpy(), value_out=b.numpy(), **res)


def random_tree(rng, nodes, depth, topk, vocab):
    parents, depths = [], []
    children = {-1: 0}
    for i in range(nodes):
        cands = [j for j in range(i) if depths[j] < depth and children.get(j, 0) < topk]
        if children[-1] < topk:
            cands.append(-1)
        p = cands[rng.randint(len(cands))]
        parents.append(p)
        depths.append(1 if p < 0 else depths[p] + 1)
        children[p] = children.get(p, 0) + 1
    tokens = rng.randint(0, vocab, size=nodes)
    return np.array(parents), tokens


def closed_subset(rng, parents, count):
    chosen = set()
    while len(chosen) < count:
        for i, p in enumerate(parents):
            if len(chosen) >= count:
                break
            if i not in chosen and (p < 0 or p in chosen) and rng.rand() < 0.6:
                chosen.add(i)
    return np.array(sorted(chosen))


def sampled_for(rng, parents, tokens, eos, vocab, depth):
    """Target samples whose greedy walk accepts a random-length root-to-leaf prefix."""
    rows = len(parents)
    samples = rng.randint(0, vocab, size=rows)
    kids = {r: [c for c in range(1, rows) if parents[c] == r] for r in range(rows)}
    want = 1 + min(depth, rng.geometric(0.3) - 1)
    node, steps = 0, 1
    while steps < want and kids[node]:
        child = kids[node][rng.randint(len(kids[node]))]
        samples[node] = tokens[child]
        node = child
        steps += 1
    samples[node] = eos if rng.rand() < 0.15 else vocab + 1 + rng.randint(5)
    return samples


def tree_cases():
    out = {}
    specs = [  # (batch, nodes_full, packed, depth, topk, vocab, past, heads, dim)
        (4, 24, 16, 4, 4, 9, 37, 2, 8),
        (4, 16, 16, 4, 4, 50, 120, 2, 8),
        (64, 80, 60, 6, 10, 40, 21, 2, 4),
        (7, 12, 5, 3, 2, 3, 3, 1, 2),
    ]
    rng = np.random.RandomState(16)
    eos = 1000
    for n, (batch, nodes, packed, depth, topk, vocab, past, heads, dim) in enumerate(specs):
        fp, ft, fc, ch = [], [], [], []
        for _ in range(batch):
            parents, tokens = random_tree(rng, nodes, depth, topk, vocab)
            tokens = np.where(rng.rand(nodes) < 0.05, eos, tokens)
            fp.append(parents)
            ft.append(tokens)
            fc.append(rng.randint(-1, 30, size=nodes))
            ch.append(closed_subset(rng, parents, packed))
        fp, ft, fc, ch = map(np.stack, (fp, ft, fc, ch))
        tree = pack_tree(t(fp), t(fc), t(ch), t(ft), depth)
        samples = np.stack([sampled_for(rng, tree.parents[b].numpy(), tree.tokens[b].numpy(), eos, vocab, depth)
                            for b in range(batch)])
        path_t = trace_verified_path(tree, t(samples), eos, kernels=None)
        path_k = trace_verified_path(tree, t(samples), eos, kernels=ref_tk)
        ws = [torch.empty(batch, depth + 1, dtype=torch.bool if i == 2 else torch.long) for i in range(3)] + \
             [torch.empty(batch, 1, dtype=torch.long)]
        packet = torch.full((batch, depth + 5), -7, dtype=torch.long)
        rows, tok, idx, msk, last, width = schedule(path_k, past, eos, ws, packet, ref_tk)
        rows_t, tok_t, idx_t, msk_t, last_t, width_t = schedule(path_t, past, eos, None, None, None)
        assert width == width_t and torch.equal(tok, tok_t) and torch.equal(idx, idx_t)
        rows_p = [r for r in rows if r[1] == 0]
        ext = min(r[2] for r in rows_p) if rows_p else width
        rtree = tree.parents.shape[1]
        length = past + rtree
        key = rng.randn(batch, heads, length + 3, dim).astype(np.float32)
        value = rng.randn(batch, heads, length + 3, dim).astype(np.float32)
        kt, vt = t(key.copy()), t(value.copy())
        ka, va = compact_suffix_inplace(kt[:, :, :length], vt[:, :, :length], idx, past, ext, SimpleNamespace())
        pad = rng.rand(batch, length) < 0.1
        pad[:, past:] = False
        m32 = tree.attention_mask(past, torch.float32, kernels=ref_tk)
        m32_torch = tree.attention_mask(past, torch.float32, kernels=None)
        mbf = tree.attention_mask(past, torch.bfloat16, kernels=ref_tk)
        m32p = m32.clone().masked_fill_(t(pad)[:, None, None, :], torch.finfo(torch.float32).min)
        assert torch.equal(m32, m32_torch)
        lowest = torch.finfo(torch.float32).min
        assert bool(((m32 == 0) | (m32 == lowest)).all())
        out[f'c{n}_full_parents'] = fp
        out[f'c{n}_full_tokens'] = ft
        out[f'c{n}_full_contexts'] = fc
        out[f'c{n}_chosen'] = ch
        out[f'c{n}_depth'] = depth
        out[f'c{n}_parents'] = tree.parents.numpy()
        out[f'c{n}_tokens'] = tree.tokens.numpy()
        out[f'c{n}_contexts'] = tree.feedback_contexts.numpy()
        out[f'c{n}_samples'] = samples
        for tag, p in (('torch', path_t), ('triton', path_k)):
            out[f'c{n}_{tag}_path_tokens'] = p.tokens.numpy()
            out[f'c{n}_{tag}_path_indices'] = p.packed_indices.numpy()
            out[f'c{n}_{tag}_path_contexts'] = p.feedback_contexts.numpy()
            out[f'c{n}_{tag}_path_lengths'] = p.lengths.numpy()
        out[f'c{n}_past'] = past
        out[f'c{n}_packet'] = np.array(rows)
        out[f'c{n}_rows_torch'] = np.array([r + [-9] * (3 + depth + 1 - len(r)) for r in rows_t])
        out[f'c{n}_pad_tokens'] = tok.numpy()
        out[f'c{n}_pad_indices'] = idx.numpy()
        out[f'c{n}_pad_mask'] = msk.numpy()
        out[f'c{n}_pad_last'] = last.numpy()
        out[f'c{n}_width'] = width
        out[f'c{n}_extension'] = ext
        out[f'c{n}_key'] = key
        out[f'c{n}_value'] = value
        out[f'c{n}_key_out'] = kt.numpy()
        out[f'c{n}_value_out'] = vt.numpy()
        out[f'c{n}_visible'] = (m32 == 0).numpy()[:, 0]
        out[f'c{n}_visible_bf16'] = (mbf == 0).numpy()[:, 0]
        out[f'c{n}_pad'] = pad
        out[f'c{n}_visible_padded'] = (m32p == 0).numpy()[:, 0]
    save('trees', count=len(specs), eos=eos, **out)


def attention_cases():
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    out = {}
    specs = [(2, 16, 2, 13, 37, 128), (3, 4, 2, 9, 23, 8), (2, 8, 8, 5, 70, 64)]
    rng = np.random.RandomState(17)
    for n, (batch, hq, hkv, rows, past, dim) in enumerate(specs):
        def bf(x):
            return torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16).float().numpy()
        q = bf(0.5 * rng.randn(batch, hq, rows, dim))
        k = bf(0.5 * rng.randn(batch, hkv, past + rows, dim))
        v = bf(0.5 * rng.randn(batch, hkv, past + rows, dim))
        parents = np.full((batch, rows), -1)
        for b in range(batch):
            for r in range(1, rows):
                parents[b, r] = rng.randint(0, r)
        from helper.tree_verification import PackedTree
        tree = PackedTree(t(parents), t(parents.copy()), t(parents.copy()), rows)
        mask = tree.attention_mask(past, torch.float32, kernels=None)
        pad = rng.rand(batch, past + rows) < 0.2
        pad[:, past:] = False
        mask.masked_fill_(t(pad)[:, None, None, :], torch.finfo(torch.float32).min)
        module = SimpleNamespace(num_key_value_groups=hq // hkv, is_causal=True, training=False)
        o, _ = sdpa_attention_forward(module, t(q), t(k), t(v), mask, dropout=0.0, scaling=dim ** -0.5)
        out[f'a{n}_q'] = q
        out[f'a{n}_k'] = k
        out[f'a{n}_v'] = v
        out[f'a{n}_parents'] = parents
        out[f'a{n}_pad'] = pad
        out[f'a{n}_past'] = past
        out[f'a{n}_mask'] = mask.numpy()
        out[f'a{n}_out'] = o.numpy()
    save('attention', count=len(specs), **out)


def draft_mask_cases():
    """Draft-model masks: AttentionWorkspace.causal on CPU (torch branch) and the Triton kernel
    helper/opd_attention_kernels.causal_mask (interpreted on CPU tensors); the expansion mask
    by the reference's op sequence helper/opd_generate.py:143-162 on CPU tensors."""
    from helper.opd_attention import AttentionWorkspace
    from helper.opd_attention_kernels import causal_mask
    rng = np.random.RandomState(23)
    out = {}
    specs = [(3, 5, 17, torch.float32, True), (2, 10, 40, torch.bfloat16, False), (4, 1, 9, torch.float16, True),
             (2, 7, 300, torch.bfloat16, True)]
    for n, (batch, query, past, dtype, with_pad) in enumerate(specs):
        cols = past + query
        pad = torch.from_numpy(rng.rand(batch, cols + 3) < 0.2) if with_pad else None
        ws = AttentionWorkspace('cpu')
        ref = ws.causal('m', past, query, batch, dtype, pad).clone()
        tri = torch.empty(batch, 1, query, cols, dtype=dtype)
        causal_mask(tri, past, pad)
        assert torch.equal(ref, tri), 'torch and Triton branches disagree'
        out[f'c{n}_shape'] = np.array([batch, query, past])
        out[f'c{n}_dtype'] = str(dtype).split('.')[-1]
        out[f'c{n}_pad'] = pad.numpy() if pad is not None else np.zeros((0, 0), dtype=bool)
        out[f'c{n}_visible'] = (ref.float() == 0).numpy()[:, 0]
    especs = [(3, 4, 30, 12, torch.float32, 'bool'), (2, 10, 64, 20, torch.bfloat16, 'pairs'),
              (4, 3, 12, 9, torch.float16, None), (2, 6, 200, 150, torch.bfloat16, 'bool')]
    for n, (batch, k, cols, init, dtype, pad_kind) in enumerate(especs):
        seen = torch.from_numpy(rng.randint(init, cols, size=(batch, k, 1)).astype(np.int64))
        mask = torch.empty(batch, 1, k, cols, dtype=dtype)
        lowest = torch.finfo(dtype).min
        mask.zero_()
        mask[..., init:] = lowest
        mask.scatter_(dim=-1, index=seen.unsqueeze(1), value=0.)
        pad = pairs = None
        if pad_kind == 'bool':
            pad = torch.from_numpy(rng.rand(batch, cols + 5) < 0.15)
            mask.masked_fill_(pad[:, None, None, :mask.shape[-1]], lowest)
        elif pad_kind == 'pairs':
            pairs = torch.from_numpy(np.array([[b, c] for b in range(batch) for c in rng.choice(cols, 4, replace=False)],
                                              dtype=np.int64))
            mask[pairs[:, 0], 0, :, pairs[:, 1]] = lowest
        out[f'e{n}_shape'] = np.array([batch, k, cols, init])
        out[f'e{n}_dtype'] = str(dtype).split('.')[-1]
        out[f'e{n}_seen'] = seen.numpy()
        out[f'e{n}_pad'] = pad.numpy() if pad is not None else np.zeros((0, 0), dtype=bool)
        out[f'e{n}_pairs'] = pairs.numpy() if pairs is not None else np.zeros((0, 2), dtype=np.int64)
        out[f'e{n}_visible'] = (mask.float() == 0).numpy()[:, 0]
    save('draft_masks', causal_count=len(specs), expansion_count=len(especs), **out)


def history_cases():
    """ContiguousRolloutHistory (helper/opd_history.py:10-67) on CPU through a rollout:
    repeated initial copy, three verify rounds whose chunks follow helper/opd_generate.py:567-579
    (accepted features gathered from the tree hidden states at chosen_index - past, then appended
    with generated_ids / input_ids to the owner rows), two capacity grows, rows finishing between
    rounds, finalize."""
    from helper.opd_history import ContiguousRolloutHistory
    rng = np.random.RandomState(31)
    batch, repeats, dim, tree_rows = 3, 2, 8, 10
    init_len = 4
    initial = {'generated_ids': torch.from_numpy(rng.randint(0, 1000, size=(batch, init_len))),
               'features': torch.from_numpy(rng.randn(batch, init_len, dim).astype(np.float16)),
               'input_ids': torch.from_numpy(rng.randint(0, 1000, size=(batch, init_len)))}
    hist = ContiguousRolloutHistory(initial, repeats=repeats, max_length=6)
    out = {f'init_{k}': v.numpy() for k, v in initial.items()}
    rounds = [(list(range(6)), [5, 4, 3, 2, 1, 0], 3, [2]), ([0, 1, 3, 4, 5], [1, 0, 3, 5, 4], 2, [0, 4]),
              ([1, 3, 5], [3, 1, 5], 4, [])]
    for n, (residual, owners, width, finish) in enumerate(rounds):
        rows = len(residual)
        tree = torch.from_numpy(rng.randn(rows, tree_rows, dim).astype(np.float16))
        index = torch.from_numpy(np.stack([np.sort(rng.choice(tree_rows, width, replace=False))
                                           for _ in range(rows)]).astype(np.int64))
        next_token = torch.from_numpy(rng.randint(0, 1000, size=(rows, width)))
        gathered = tree.gather(dim=1, index=index.unsqueeze(-1).expand(rows, -1, dim))
        hist.append(residual, {'generated_ids': next_token, 'features': gathered, 'input_ids': next_token},
                    owners=torch.tensor(owners))
        for row in finish:
            hist.mark_finished(row)
        out.update({f'r{n}_residual': np.array(residual), f'r{n}_owners': np.array(owners), f'r{n}_tree': tree.numpy(),
                    f'r{n}_index': index.numpy(), f'r{n}_next_token': next_token.numpy(),
                    f'r{n}_gathered': gathered.numpy(), f'r{n}_finish': np.array(finish, dtype=np.int64),
                    f'r{n}_capacities': np.array([hist.capacities[k] for k in ('generated_ids', 'features',
                                                                                  'input_ids')])})
    final = hist.finalize()
    for name in ('generated_ids', 'features', 'input_ids'):
        out[f'final_{name}_lengths'] = np.array([len(r[name]) for r in final])
        out[f'final_{name}'] = np.concatenate([r[name].numpy() for r in final])
    save('history', rounds=len(rounds), repeats=repeats, max_length=6, **out)


if __name__ == '__main__':
    torch.manual_seed(0)
    kv_sequence()
    remap_move_triton()
    swap_remove_cases()
    persistent_rollouts()
    final_optimization()
    schedule_kat()
    tree_cases()
    attention_cases()
    draft_mask_cases()
    history_cases()
