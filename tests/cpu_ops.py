"""Oracle-backed stand-in for analysis_spec_b200._ops, for host-logic tests on CPU.

The product's kernel front end (_ops) refuses CPU tensors. To test the cache's
host bookkeeping (growth decisions, counters, views, lifetimes) without a GPU,
tests monkeypatch the cache module's ``_ops`` with this module, whose row
movement runs the CPU oracle on CPU tensors. Never used outside tests/.
"""
import numpy as np
import torch

from oracle import oracle


def _np(t):
    """Writable numpy view sharing memory with a CPU tensor (bf16/f16 as raw 16-bit words)."""
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy()
    return t.numpy()


def append_rows(key_pools, value_pools, key_srcs, value_srcs, length, launch=True, row_table=None, commit=None):
    assert row_table is None, 'the CPU stand-ins cover caches without a row table'
    def go():
        if commit is not None:  # the folded compaction first (its own bounds: the pool capacity)
            chosen, past, extension, width = commit
            compact_suffix(key_pools, value_pools, key_srcs[0].shape[0], key_pools[0].shape[2],
                           chosen[:, :width], past, extension, width)
        for kp, vp, ks, vs in zip(key_pools, value_pools, key_srcs, value_srcs):
            oracle.append(_np(kp), _np(vp), _np(ks), _np(vs), length)
    if launch:
        go()
        return None
    return go


def compact_suffix(key_pools, value_pools, batch, length, chosen, past, extension, width, row_table=None):
    assert row_table is None, 'the CPU stand-ins cover caches without a row table'
    for kp, vp in zip(key_pools, value_pools):
        bad = oracle.compact_suffix(_np(kp), _np(vp), batch, length, chosen.numpy(), past, extension)
        assert bad == 0


def remap_scratch_elements(new_batch, heads, dim, length, element_size):
    return 0


def remap_rows(key_pools, value_pools, indices, length, scratch=None):
    for kp, vp in zip(key_pools, value_pools):
        assert oracle.remap_rows(_np(kp), _np(vp), indices.numpy(), length) == 0


def move_rows(key_pools, value_pools, sources, destinations, length):
    for kp, vp in zip(key_pools, value_pools):
        assert oracle.move_rows(_np(kp), _np(vp), sources.numpy(), destinations.numpy(), length) == 0
