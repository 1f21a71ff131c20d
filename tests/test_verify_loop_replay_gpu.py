"""The reference's own verify loop (helper/opd_generate.py:461-677, opd_reflex, greedy), replayed
call by call through this package on the GPU: every cache, packet, mask, path and history result
equals the reference's bit for bit, the attention outputs are within the stated tolerance, and the
acceptance counters the loop accumulates (opd_generate.py:551-555) come out identical."""
import pytest
import torch

from analysis_spec_b200 import _ops
from tests.verify_loop_replay import host_totals, replay

pytestmark = pytest.mark.gpu


def test_reference_verify_loop_replays_through_the_drop_in():
    r, meta = replay()
    assert _ops.device_error() is None
    # the counters of the loop, from this package's packets
    acc = dec = draft = 0
    for rows in r.schedules:
        for row in rows:
            acc += row[0]
            dec += 1
            draft += max(row[0] - 1, 0)
    res = meta['result']
    assert (acc, dec, draft) == (res['total_acc_length'], res['total_decoded_token_num'],
                                 res['total_accepted_draft_tokens'])
    assert host_totals(meta)['total_proposed_draft_tokens'] == res['total_proposed_draft_tokens']
    # the target cache's statistics equal the reference's opd_target_* figures (the
    # compaction-scratch figure aside: no scratch here)
    stats = r.statistics['cache0']
    for k, v in stats.items():
        if k != 'kv_compaction_workspace_bytes':
            assert res[f'opd_target_{k}'] == v, k
    assert r.attention and all(m <= 2e-2 for _, m, _ in r.attention)
    torch.cuda.synchronize()


def test_reference_verify_loop_replays_with_the_append_fused_into_the_attention():
    """The same loop with the caches' fuse_append on: each target layer's update is left to the
    verify attention after it (speckv_tree_attention_bits_append), the draft cache's rows are
    stored when the draft side first reads them. Caches, packets, counters and statistics stay
    identical to the reference's, attention within the tolerance."""
    from analysis_spec_b200 import _lib
    _lib.profile.reset()
    _lib.profile.enabled = True
    try:
        r, meta = replay(fused=True)
    finally:
        _lib.profile.enabled = False
    assert _ops.device_error() is None
    assert not r.deferred and all(l._pending is None for o in r.objects.values() if hasattr(o, 'fuse_append')
                                  for l in o.layers)
    fused = len(_lib.profile.events.get('speckv_tree_attention_bits_append', []))
    assert fused > 0, _lib.profile.events.keys()
    acc = dec = draft = 0
    for rows in r.schedules:
        for row in rows:
            acc += row[0]
            dec += 1
            draft += max(row[0] - 1, 0)
    res = meta['result']
    assert (acc, dec, draft) == (res['total_acc_length'], res['total_decoded_token_num'],
                                 res['total_accepted_draft_tokens'])
    stats = r.statistics['cache0']
    for k, v in stats.items():
        if k != 'kv_compaction_workspace_bytes':
            assert res[f'opd_target_{k}'] == v, k
    assert r.attention and all(m <= 2e-2 for _, m, _ in r.attention)
    torch.cuda.synchronize()
