"""KV row remap and tail-to-hole row moves on whole pools.

Drop-in for ``helper/opd_kv_kernels.py`` (``remap_rows`` :34-40,
``move_tail_rows`` :56-58). ``keys`` / ``values`` are full pools
``(batch_capacity, heads, capacity, head_dim)``; rows are moved over the live
prefix ``[0, length)``.

The reference gathers into a scratch and scatters back with two flat,
per-element Triton launches. Here one sm_100a launch stages every batch row of
a tile of positions in shared memory (so arbitrary permutations and duplicate
indices are read before any write) and moves 16-byte vectors; the caller's
scratch is only touched when one position of all rows does not fit on chip.
"""
from . import _ops


def remap_rows(keys, values, indices, length, scratch):
    """pool[:n] = pool[indices] over [0, length) for K and V (n = indices.numel())."""
    _ops.remap_rows([keys], [values], indices, length, scratch)


def move_tail_rows(keys, values, sources, destinations, length):
    """pool[destinations[j]] = pool[sources[j]] over [0, length); sources and destinations disjoint."""
    _ops.move_rows([keys], [values], sources, destinations, length)


def remap_rows_layers(key_pools, value_pools, indices, length, scratch=None):
    """remap_rows over every layer's pools in one launch."""
    _ops.remap_rows(list(key_pools), list(value_pools), indices, length, scratch)


def move_tail_rows_layers(key_pools, value_pools, sources, destinations, length):
    """move_tail_rows over every layer's pools in one launch."""
    _ops.move_rows(list(key_pools), list(value_pools), sources, destinations, length)
