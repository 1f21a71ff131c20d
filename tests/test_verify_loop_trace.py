"""The recorded trace of the reference's verify loop (tests/golden/make_verify_loop_trace.py) is
complete and agrees with the reference's own result: the counters recomputed from the recorded
packets equal the ones the loop returned, and the recorded history equals its tokens."""
from tests.verify_loop_replay import host_totals, load_trace


def test_trace_covers_the_loop_and_matches_the_reference_result():
    z, meta = load_trace()
    fns = {c['fn'] for c in meta['calls']}
    for fn in ('opd_static_cache.persistent_cache', 'OPDStaticCache.update', 'OPDStaticCache.crop',
               'OPDStaticCache.batch_repeat_interleave', 'OPDStaticCache.swap_remove', 'OPDStaticCache.statistics',
               'opd_static_cache.swap_remove_plan', 'opd_scheduling.schedule', 'opd_scheduling.compact_suffix_inplace',
               'tree_verification.pack_tree', 'tree_verification.trace_verified_path', 'PackedTree.attention_mask',
               'ContiguousRolloutHistory.append', 'ContiguousRolloutHistory.mark_finished',
               'ContiguousRolloutHistory.finalize', 'AttentionWorkspace.causal', 'attention'):
        assert fn in fns, fn
    res = meta['result']
    for k, v in host_totals(meta).items():
        assert res[k] == v, k
    # the finished rows' histories end with the end-of-sequence token; the others do not
    eos = meta['eos']
    fin = [c for c in meta['calls'] if c['fn'] == 'ContiguousRolloutHistory.finalize'][0]
    generated = [z[row['dict'][0][1]['tensor']].ravel().tolist() for row in fin['out']['list']]
    assert [g[-1] == eos for g in generated] == [t[-1] == eos for t in res['generated_token_ids']]
    for g, t in zip(generated, res['generated_token_ids']):
        it = iter(g)
        assert all(tok in it for tok in t)  # the result is the history with the padding removed
