"""The C-ABI library loads and exports every entry point include/speckv.h declares.

No compute calls here (this runs without a GPU); only host-only entry points
(version, scratch sizing, argument validation that fails before any CUDA call)
are exercised.
"""
import ctypes
import re
from pathlib import Path

import pytest

from analysis_spec_b200 import _lib
from analysis_spec_b200.build import build

HEADER = Path(__file__).resolve().parents[1] / 'include' / 'speckv.h'


def declared():
    text = re.sub(r'/\*.*?\*/', '', HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(speckv_\w+)\s*\(', text)))


@pytest.fixture(scope='module')
def lib():
    build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 15
    bound_elsewhere = {'speckv_last_error', 'speckv_remap_scratch_bytes', 'speckv_plan_release'}
    bound_elsewhere |= {name + '_prepare' for name in _lib.PREPARED}
    for name in names:
        assert hasattr(lib, name), name
        if name not in bound_elsewhere:
            assert name in _lib.SIGNATURES, f'{name} has no ctypes signature'


def test_host_only_entry_points(lib):
    assert lib.speckv_version() == 100
    # one position of 64 bf16 rows of 128 dims fits on chip: no scratch
    assert lib.speckv_remap_scratch_bytes(64, 2, 128, 2048, 2) == 0
    # 1000 rows of 256 fp32 dims (1 MB per position) need the two-phase scratch
    assert lib.speckv_remap_scratch_bytes(1000, 2, 256, 10, 4) == 2 * 1000 * 2 * 10 * 256 * 4


def test_argument_errors_are_reported_without_a_launch(lib):
    nul = (ctypes.c_void_p * 1)(None)
    strides = _lib.i64_array([0, 0, 0])
    with pytest.raises(_lib.SpecKVError, match='layers=0'):
        _lib.call('speckv_append_rows', nul, nul, nul, nul, 0, 1, 1, 1, 8, 8, 0, strides, strides, 2, None, 0, None)
    with pytest.raises(_lib.SpecKVError, match='null pool'):
        _lib.call('speckv_move_rows', nul, nul, 1, None, None, 1, 1, 1, 8, 8, 4, 2, None)
    pools = (ctypes.c_void_p * 1)(16)  # never dereferenced: the row-table check comes first
    table = (ctypes.c_int64 * 1)(0)
    with pytest.raises(_lib.SpecKVError, match="row table needs the pools' row count"):
        _lib.call('speckv_append_rows', pools, pools, pools, pools, 1, 1, 1, 1, 8, 8, 0, strides, strides, 2,
                  ctypes.cast(table, ctypes.c_void_p), 0, None)
    with pytest.raises(_lib.SpecKVError, match='pool rows for'):
        _lib.call('speckv_compact_suffix', pools, pools, 1, 4, 1, 8, 8, 8, None, 0, 0, 0, 0, 1, 2, None, 2, None)
    with pytest.raises(_lib.SpecKVError, match='invalid committed path width'):
        _lib.call('speckv_pad_verified_path', None, 0, 0, None, 0, 0, None, 1, 4, 9, 0, 0, None, None, None, 0, 0,
                  None, 0, None)
    with pytest.raises(_lib.SpecKVError, match='not a multiple'):
        _lib.call('speckv_tree_attention', None, strides, None, strides, None, strides, None, 0, None, 1, 3, 2, 1, 1,
                  8, 1.0, 1, None)


def test_prepared_launch_host_side(lib):
    """Preparation validates like the one-call entry (no launch on error); an empty
    append prepares a plan whose launch does nothing, so it runs without a GPU."""
    nul = (ctypes.c_void_p * 1)(None)
    strides = _lib.i64_array([0, 0, 0])
    with pytest.raises(_lib.SpecKVError, match='layers=0'):
        _lib.prepare('speckv_append_rows', nul, nul, nul, nul, 0, 1, 1, 1, 8, 8, 0, strides, strides, 2, None, 0,
                     None)
    pools = (ctypes.c_void_p * 1)(16)  # never dereferenced: batch 0 moves nothing
    plan = _lib.prepare('speckv_append_rows', pools, pools, pools, pools, 1, 0, 1, 1, 8, 8, 0, strides, strides, 2,
                        None, 0, None)
    assert plan.handle
    plan()
    plan()  # a plan can be launched again
    del plan


def test_static_remap_refuses_sizes_that_would_overflow(lib):
    """Sizes whose byte products overflow 64 bits are refused before any CUDA call."""
    pools = (ctypes.c_void_p * 1)(16)  # never dereferenced: the size checks come first
    idx = ctypes.c_void_p(16)
    with pytest.raises(_lib.SpecKVError, match='2\\^31 or more'):
        _lib.call('speckv_remap_rows_static', pools, pools, 1, idx, 1 << 31, 1 << 31, 2, 128, 8, 8, 2, None)
    # each size below 2^31, but 2 * rows * heads * row bytes is about 2^84
    with pytest.raises(_lib.SpecKVError, match='static scratch'):
        _lib.call('speckv_remap_rows_static', pools, pools, 1, idx, 1 << 30, 1 << 30, 1 << 30, 1 << 20, 8, 8, 8,
                  None)


def test_attention_counters_and_hook_arguments(lib):
    tc, cc = ctypes.c_int64(-1), ctypes.c_int64(-1)
    _lib.call('speckv_attention_launches', ctypes.byref(tc), ctypes.byref(cc))
    assert tc.value >= 0 and cc.value >= 0
    with pytest.raises(_lib.SpecKVError, match='0 / 1 switch'):
        _lib.call('speckv_attention_test_hooks', -1, 0)
    with pytest.raises(_lib.SpecKVError, match='0 / 1 switch'):
        _lib.call('speckv_attention_test_hooks', 0, 2)


def test_fused_append_attention_refuses_before_any_launch(lib):
    """speckv_tree_attention_bits_append checks sizes on the host: rows beyond the pools'
    capacity, visibility rows too short for past + rows columns, another head dim, a tree
    wider than one 128-key tile. The pointers are never dereferenced."""
    s = _lib.i64_array([0, 0, 0])
    p = 16

    def call(past, capacity, rows, dim, row_words):
        _lib.call('speckv_tree_attention_bits_append', p, s, p, s, p, s, past, capacity, p, s, p, s, p, row_words,
                  None, p, 1, 16, 2, rows, dim, 1.0, _lib.BF16, None)
    with pytest.raises(_lib.SpecKVError, match='exceed'):
        call(100, 120, 61, 128, 8)
    with pytest.raises(_lib.SpecKVError, match='row_words'):
        call(300, 400, 61, 128, 4)
    with pytest.raises(_lib.SpecKVError, match='head dim 128'):
        call(10, 400, 61, 64, 4)
    with pytest.raises(_lib.SpecKVError, match='128-key tile'):
        call(10, 400, 129, 128, 8)
