"""Acceptance counters computed on the device from the schedule packet.

The increments helper/opd_generate.py:551-555 adds on the host after each
verification (accepted draft tokens, proposed draft tokens, accepted-length sum
and row count, finished rows) must equal, round after round, those one kernel
derives from the device packet; AcceptanceCounters accumulates them on a side
stream without a host round trip.
"""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200.counters import FIELDS, AcceptanceCounters, round_increments

pytestmark = pytest.mark.gpu


def packet_rows(rng, batch, width):
    lengths = rng.randint(0, width + 1, size=batch)
    eos = rng.rand(batch) < 0.2
    rows = np.zeros((batch, width + 4), dtype=np.int64)
    rows[:, 0], rows[:, 1], rows[:, 2] = lengths, eos, rng.randint(0, 3, size=batch)
    rows[:, 3:] = rng.randint(-1, 50, size=(batch, width + 1))
    return rows


@pytest.mark.parametrize('batch', [0, 1, 7, 64, 300, 1000])
def test_counts_match_host_increments(batch):
    rng = np.random.RandomState(batch)
    rows = packet_rows(rng, batch, 7)
    packet = torch.from_numpy(rows).cuda()
    counts = torch.full((5,), -1, dtype=torch.long, device='cuda')
    _ops.acceptance_counts(packet, batch, 60, counts)
    assert counts.tolist() == round_increments(rows.tolist(), 60)


def test_strided_packet_and_accumulation_over_rounds():
    rng = np.random.RandomState(3)
    counters = AcceptanceCounters('cuda')
    expect = [0] * len(FIELDS)
    wide = torch.zeros(64, 20, dtype=torch.long, device='cuda')  # packet view with a wider row stride
    for _ in range(7):
        rows = packet_rows(rng, 64, 7)
        wide[:, :rows.shape[1]] = torch.from_numpy(rows).cuda()
        counters.add_device_round(wide[:, :rows.shape[1]], 64, 60)
        expect = [a + b for a, b in zip(expect, round_increments(rows.tolist(), 60))]
    assert counters.finish() == dict(zip(FIELDS, expect))
