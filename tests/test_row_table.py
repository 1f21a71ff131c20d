"""Row-table caches (OPDStaticCache(..., row_table=True)): sequence b lives in pool row
table[b], so releasing finished sequences and admitting new ones rewrite the table instead
of moving whole histories (the reference's swap_remove moves them,
helper/opd_static_cache.py:157-174, 228-230). The logical view -- pool[table[b]] for each
live sequence b -- must equal, bit for bit, what the reference's row moves produce, which
the CPU oracle restates (oracle.move_rows / compact_suffix / append)."""
import numpy as np
import pytest
import torch

from analysis_spec_b200.opd_static_cache import release_rows, swap_remove_plan
from oracle import oracle


def test_release_rows_matches_swap_remove_host_side():
    """The table after a release names, for every surviving sequence, the row the reference's
    swap_remove would have moved it into, and stays a permutation of the pool rows."""
    rng = np.random.RandomState(3)
    rows = list(rng.permutation(20))
    for _ in range(6):
        batch = int(rng.randint(4, 17))
        finished = [bool(x) for x in rng.rand(batch) < 0.3]
        keep, sources, dests = swap_remove_plan(finished)
        new = release_rows(rows, len(keep), sources, dests)
        assert sorted(new) == sorted(rows)
        assert new[:len(keep)] == [rows[k] for k in keep]
        rows = new
    with pytest.raises(ValueError):
        release_rows(list(range(6)), 4, [1], [0])  # a source below the new batch


def logical(pool, table, batch, length):
    return pool[torch.tensor(table[:batch], device=pool.device)][:, :, :length]


def as_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy()


@pytest.mark.gpu
@pytest.mark.parametrize('layers,batch,heads,rounds', [(3, 16, 8, 4), (2, 9, 2, 3)])
def test_row_table_rollout_bit_exact(layers, batch, heads, rounds):
    """Verify rounds with release and admission through the table: logical views bit-exact
    against the oracle's physical moves, no history row moved."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_static_cache import OPDStaticCache
    from tests.test_kv_gpu import path_like_chosen
    rng = np.random.RandomState(layers * 10 + batch)
    gen = torch.Generator(device='cuda').manual_seed(batch)
    dim, rows, width, prefix = 128, 61, 7, 300
    dt = torch.bfloat16
    cache = OPDStaticCache(1024, batch_capacity=batch, row_table=True)

    def rnd(*shape):
        return (0.5 * torch.randn(*shape, device='cuda', generator=gen)).to(dt)

    prefill = [(rnd(batch, heads, prefix, dim), rnd(batch, heads, prefix, dim)) for _ in range(layers)]
    for l, (k, v) in enumerate(prefill):
        cache.update(k, v, l)
    cap = cache.layers[0].capacity
    opools = []
    for k, v in prefill:
        kp = np.zeros((batch, heads, cap, dim), dtype=np.int16)
        vp = np.zeros_like(kp)
        oracle.append(kp, vp, as_bits(k), as_bits(v), 0)
        opools.append((kp, vp))
    live = batch
    for rnd_i in range(rounds):
        past = cache.get_seq_length()
        tree = [(rnd(live, heads, rows, dim), rnd(live, heads, rows, dim)) for _ in range(layers)]
        cache.update_layers([t[0] for t in tree], [t[1] for t in tree])
        for (kp, vp), (tk, tv) in zip(opools, tree):
            oracle.append(kp, vp, as_bits(tk), as_bits(tv), past)
        chosen = path_like_chosen(rng, live, past, rows, width)
        cache.commit_accepted(torch.from_numpy(chosen).cuda(), past, 1)
        for kp, vp in opools:
            assert oracle.compact_suffix(kp, vp, live, past + rows, chosen, past, 1) == 0
        length = past + width
        finished = [False] * live
        for i in rng.choice(live, size=max(1, live // 4), replace=False):
            finished[i] = True
        keep, sources, dests = swap_remove_plan(finished)
        new_batch = len(keep)
        cache.swap_remove(new_batch, sources, dests)
        for kp, vp in opools:
            assert oracle.move_rows(kp, vp, np.array(sources, dtype=np.int64), np.array(dests, dtype=np.int64),
                                    length) == 0
        admitted = live - new_batch
        fresh = []
        for _ in range(layers):
            k = torch.zeros(admitted, heads, length, dim, device='cuda', dtype=dt)
            v = torch.zeros_like(k)
            for j in range(admitted):
                n = int(rng.randint(16, length + 1))
                k[j, :, length - n:] = rnd(heads, n, dim)
                v[j, :, length - n:] = rnd(heads, n, dim)
            fresh.append((k, v))
        cache.admit([f[0] for f in fresh], [f[1] for f in fresh])
        for (kp, vp), (fk, fv) in zip(opools, fresh):
            kp[new_batch:live, :, :length] = as_bits(fk)
            vp[new_batch:live, :, :length] = as_bits(fv)
        torch.cuda.synchronize()
        assert _ops.device_error() is None
        table = cache.row_table
        assert sorted(cache._rows) == list(range(len(cache._rows)))
        for l, (kp, vp) in enumerate(opools):
            layer = cache.layers[l]
            assert np.array_equal(as_bits(logical(layer.key_pool, table, live, length)), kp[:live, :, :length])
            assert np.array_equal(as_bits(logical(layer.value_pool, table, live, length)), vp[:live, :, :length])
    assert cache.kv_rows_moved == 0
    assert table != list(range(live))  # sequences really live in other rows


@pytest.mark.gpu
def test_row_table_attention_and_device_commit_match_logical_order():
    """The bits attention and the device-scheduled commit through a scrambled table give what
    the table-free path gives on the same sequences laid out in logical order."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.tree_attention import tree_verify_attention
    from analysis_spec_b200.tree_verification import PackedTree
    rng = np.random.RandomState(8)
    gen = torch.Generator(device='cuda').manual_seed(8)
    batch, pool_rows, hq, hkv, rows, past, dim = 6, 11, 16, 2, 13, 400, 128
    dt = torch.bfloat16
    cap = 512
    kpool = (0.5 * torch.randn(pool_rows, hkv, cap, dim, device='cuda', generator=gen)).to(dt)
    vpool = (0.5 * torch.randn(pool_rows, hkv, cap, dim, device='cuda', generator=gen)).to(dt)
    table = torch.from_numpy(rng.permutation(pool_rows)[:batch].astype(np.int64)).cuda()
    klog, vlog = kpool[table].clone(), vpool[table].clone()
    q = (0.5 * torch.randn(batch, hq, rows, dim, device='cuda', generator=gen)).to(dt)
    parents = np.full((batch, rows), -1, dtype=np.int64)
    for b in range(batch):
        for r in range(1, rows):
            parents[b, r] = rng.randint(max(0, r - 4), r)
    pad = np.zeros((batch, past + rows), dtype=bool)
    for b in range(batch):
        pad[b, :rng.randint(0, 200)] = True
    tree = PackedTree(*(torch.from_numpy(parents).cuda() for _ in range(3)), rows)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())

    class M:
        num_key_value_groups, is_causal, training = hq // hkv, True, False

    kview = kpool[:, :, :past + rows]
    vview = vpool[:, :, :past + rows]
    kview._speckv_rows = vview._speckv_rows = table
    out, _ = tree_verify_attention(M(), q, kview, vview, vis, scaling=dim ** -0.5)
    ref, _ = tree_verify_attention(M(), q, klog[:, :, :past + rows], vlog[:, :, :past + rows], vis,
                                   scaling=dim ** -0.5)
    assert torch.equal(out, ref)
    # device-scheduled commit: packet rows [width, eos, extension]
    width = 5
    chosen = torch.from_numpy(np.stack([np.sort(rng.choice(np.arange(past, past + rows), width, replace=False))
                                        for _ in range(batch)])).cuda()
    packet = torch.zeros(batch, width + 4, dtype=torch.long, device='cuda')
    packet[:, 0] = width
    packet[:, 2] = 1
    _ops.commit_round([kpool], [vpool], batch, past + rows, chosen, past, packet, row_table=table)
    _ops.commit_round([klog], [vlog], batch, past + rows, chosen, past, packet)
    torch.cuda.synchronize()
    assert torch.equal(kpool[table][:, :, :past + width], klog[:, :, :past + width])
    assert torch.equal(vpool[table][:, :, :past + width], vlog[:, :, :past + width])
    assert _ops.device_error() is None
    # a table entry outside the pools is reported, the sequence skipped
    bad = table.clone()
    bad[2] = pool_rows + 3
    _ops.commit_round([kpool], [vpool], batch, past + rows, chosen, past, packet, row_table=bad)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('row table', pool_rows + 3)


@pytest.mark.gpu
def test_row_table_survives_pool_release_and_larger_rollout():
    """end_rollout that drops the pools also drops the table; a later, larger rollout starts
    from a fresh identity table."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_static_cache import OPDStaticCache
    cache = OPDStaticCache(256, batch_capacity=4, row_table=True)
    k = torch.randn(4, 2, 8, 128, device='cuda').to(torch.bfloat16)
    cache.update(k, k, 0)
    cache.swap_remove(2, [3], [0])
    assert cache.row_table == [3, 1]
    cache.end_rollout(max_retained_tokens=1)
    big = torch.randn(9, 2, 8, 128, device='cuda').to(torch.bfloat16)
    cache.begin_rollout(9, 9)
    keys, _ = cache.update(big, big, 0)
    assert cache.row_table == list(range(9))
    assert torch.equal(keys[torch.tensor(cache.row_table, device='cuda')], big)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
