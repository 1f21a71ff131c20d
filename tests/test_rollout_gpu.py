"""Several verify rounds of a rollout with finishing and admitted sequences (the Qwen2.5-14B
configuration's pattern at reduced size: 8 KV heads x 128, bf16, a quarter of the live rows
finishing each round): append, commit, swap-remove release and admission through
OPDStaticCache, mirrored on the CPU oracle, pools bit-exact after every round.

Release follows OPDStaticCache.swap_remove / swap_remove_plan
(helper/opd_static_cache.py:157-174, 228-230, 247-254); admission has no reference
implementation (rollouts there start full), so the oracle restates it as a plain copy of
the fresh left-padded prefixes into the released rows."""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200.opd_static_cache import OPDStaticCache, swap_remove_plan
from oracle import oracle
from tests.cpu_ops import _np
from tests.test_kv_gpu import path_like_chosen

pytestmark = pytest.mark.gpu


def as_bits(t):
    return _np(t.detach().cpu().contiguous()).copy()


@pytest.mark.parametrize('layers,batch,heads,rounds', [(3, 16, 8, 4), (2, 9, 4, 3)])
def test_rollout_release_and_admission_bit_exact(layers, batch, heads, rounds):
    rng = np.random.RandomState(layers * 100 + batch)
    gen = torch.Generator(device='cuda').manual_seed(batch)
    dim, rows, width, prefix = 128, 61, 7, 300
    dt = torch.bfloat16
    cache = OPDStaticCache(1024, batch_capacity=batch)

    def rnd(*shape):
        return (0.5 * torch.randn(*shape, device='cuda', generator=gen)).to(dt)

    prefill = [(rnd(batch, heads, prefix, dim), rnd(batch, heads, prefix, dim)) for _ in range(layers)]
    for l, (k, v) in enumerate(prefill):
        cache.update(k, v, l)
    cap = cache.layers[0].capacity
    # oracle pools, same capacity as the cache's, bf16 as raw 16-bit words
    opools = []
    for k, v in prefill:
        kp = np.zeros((batch, heads, cap, dim), dtype=np.int16)
        vp = np.zeros_like(kp)
        oracle.append(kp, vp, as_bits(k), as_bits(v), 0)
        opools.append((kp, vp))
    live = batch
    moved = 0
    for rnd_i in range(rounds):
        past = cache.get_seq_length()
        # append the tree rows of every layer
        tree = [(rnd(live, heads, rows, dim), rnd(live, heads, rows, dim)) for _ in range(layers)]
        cache.update_layers([t[0] for t in tree], [t[1] for t in tree])
        for (kp, vp), (tk, tv) in zip(opools, tree):
            oracle.append(kp, vp, as_bits(tk), as_bits(tv), past)
        # commit accepted paths
        chosen = path_like_chosen(rng, live, past, rows, width)
        cache.commit_accepted(torch.from_numpy(chosen).cuda(), past, 1)
        for kp, vp in opools:
            assert oracle.compact_suffix(kp, vp, live, past + rows, chosen, past, 1) == 0
        length = past + width
        assert cache.get_seq_length() == length
        # a quarter of the live rows finish: release by swap-remove
        finished = [False] * live
        for i in rng.choice(live, size=max(1, live // 4), replace=False):
            finished[i] = True
        keep, sources, dests = swap_remove_plan(finished)
        new_batch = len(keep)
        moved += len(sources)
        cache.swap_remove(new_batch, torch.tensor(sources, device='cuda', dtype=torch.long),
                          torch.tensor(dests, device='cuda', dtype=torch.long))
        for kp, vp in opools:
            assert oracle.move_rows(kp, vp, np.array(sources, dtype=np.int64), np.array(dests, dtype=np.int64),
                                    length) == 0
        # admit as many new sequences with fresh prefixes, left-padded to the shared length
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
        assert cache.layers[0].batch_size == live
        torch.cuda.synchronize()
        assert _ops.device_error() is None
        for l, (kp, vp) in enumerate(opools):
            keys, values = cache[l]
            assert np.array_equal(as_bits(keys), kp[:live, :, :length]), (rnd_i, l)
            assert np.array_equal(as_bits(values), vp[:live, :, :length]), (rnd_i, l)
    assert cache.kv_rows_moved == moved
