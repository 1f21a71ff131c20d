"""Sequence-sharded ranks on CPU (gloo, world size 2): the per-round acceptance
counter reduction and what a surviving rank sees when its peer fails.

The counter fields follow helper/opd_generate.py:551-555 (accepted / proposed
draft tokens, accepted-length sum and count) plus finished rows.
"""
import os
import socket
import traceback

import pytest
import torch.multiprocessing as mp

from analysis_spec_b200.counters import FIELDS, AcceptanceCounters, round_increments


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rounds(rank, n=5):
    """Seeded host packets `[length, eos?, ext, ...]` of `n` rounds for one rank's 3 sequences."""
    import numpy as np
    rng = np.random.RandomState(rank)
    out = []
    for _ in range(n):
        out.append([[int(rng.randint(1, 8)), int(rng.rand() < 0.2), 0] for _ in range(3)])
    return out


def _worker(rank, world, port, mode, queue):
    import datetime

    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    try:
        dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        counters = AcceptanceCounters('cpu')
        for i, rows in enumerate(_rounds(rank)):
            if mode == 'fail' and rank == 1 and i == 2:
                raise RuntimeError('rank 1 lost its sequences')
            counters.add_round(round_increments(rows, proposed_per_row=60))
        queue.put((rank, 'ok', counters.finish()))
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, which checks who failed and how
        queue.put((rank, 'error', f'{type(exc).__name__}: {exc}\n{traceback.format_exc(limit=2)}'))


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=timeout)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


def test_round_increments_match_reference_counters():
    rows = [[4, 0, 2], [1, 1, 0], [7, 0, 5]]
    inc = dict(zip(FIELDS, round_increments(rows, proposed_per_row=60)))
    assert inc == {'accepted_draft': 3 + 0 + 6, 'proposed_draft': 180, 'accepted_length': 12,
                   'verified_rows': 3, 'finished_rows': 1}


def test_single_process_totals():
    counters = AcceptanceCounters('cpu')
    expect = [0] * len(FIELDS)
    for rows in _rounds(0):
        inc = round_increments(rows, 60)
        counters.add_round(inc)
        expect = [a + b for a, b in zip(expect, inc)]
    assert counters.finish() == dict(zip(FIELDS, expect))


def test_two_ranks_reduce_counters():
    results = _run('ok')
    expect = [0] * len(FIELDS)
    for rank in range(2):
        for rows in _rounds(rank):
            expect = [a + b for a, b in zip(expect, round_increments(rows, 60))]
    for rank in range(2):
        status, payload = results[rank]
        assert status == 'ok', payload
        assert payload == dict(zip(FIELDS, expect))


@pytest.mark.timeout(120)
def test_failed_rank_surfaces_on_survivor():
    results = _run('fail')
    assert results[1][0] == 'error' and 'lost its sequences' in results[1][1]
    status, payload = results[0]
    assert status == 'error', 'the surviving rank finished as if its peer had reduced'
