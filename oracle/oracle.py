"""CPU oracle of the static-KV-cache / tree-verify path (TEST INFRASTRUCTURE ONLY).

Restates the reference's algorithms (nhatminz/analysis_spec) on the CPU so the
CUDA product can be checked against them; only tests, the smoke check and the
CPU-baseline leg of bench.py use it. The product never imports this module.

Pinned: the restatement is checked against golden vectors produced by running
the reference's own code (tests/golden/make_golden.py, fixtures in
tests/golden/*.npz) in tests/test_oracle_golden.py.

KV row movement is in C (speckv_oracle.c, OpenMP over host cores); tree ops are
numpy; attention is a float32 numpy restatement of
softmax(q k^T * scale + mask) v with GQA head sharing.

Reference code followed (file:line within the reference project):
  append / compact / remap / move   see speckv_oracle.c
  trace_path           helper/tree_verification.py:286-322, helper/tree_kernels.py:68-95
  pad_verified_path    helper/tree_verification.py:237-268 (budget clamped at 0)
  pad_schedule         helper/tree_kernels.py:7-41 (packet layout), helper/opd_scheduling.py:5-32
  tree_mask            helper/tree_kernels.py:139-155, helper/tree_verification.py:19-42,
                       padding masked_fill helper/opd_generate.py:483-484
  pack_tree            helper/tree_verification.py:200-227
  swap_remove_plan     helper/opd_static_cache.py:247-254
  position_update      helper/opd_generate.py:556-558, 644-650
  attention            transformers integrations/sdpa_attention.py:40-104 (repeat_kv + SDPA)
  causal_visible       helper/opd_attention.py:31-43, helper/opd_attention_kernels.py:7-22
  expansion_visible    helper/opd_generate.py:143-162
  RolloutHistory       helper/opd_history.py:10-67
  gather_positions     helper/opd_generate.py:567-571 (accepted-feature gather)
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / 'liboracle_speckv.so'
SRC = HERE / 'speckv_oracle.c'

_lib = None


def build(force=False):
    """Compiles speckv_oracle.c with gcc + OpenMP next to this file."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix('.so.tmp')
    cc = '/usr/bin/gcc' if Path('/usr/bin/gcc').exists() else 'gcc'
    base = [cc, '-O3', '-shared', '-fPIC', '-o', str(tmp), str(SRC)]
    if subprocess.run(base[:2] + ['-fopenmp'] + base[2:], capture_output=True).returncode != 0:
        subprocess.run(base, check=True)  # single-threaded build when OpenMP is unavailable
    os.replace(tmp, LIB)
    return LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        lib.oracle_append.argtypes = [p, p, p, p, i64, i64, i64, i64, i64, i64, p, p, i32]
        lib.oracle_append.restype = None
        lib.oracle_compact_suffix.argtypes = [p, p, i64, i64, i64, i64, i64, p, i64, i64, i64, i64, i64, i32]
        lib.oracle_compact_suffix.restype = i64
        lib.oracle_remap_rows.argtypes = [p, p, p, i64, i64, i64, i64, i64, i64, i32]
        lib.oracle_remap_rows.restype = i64
        lib.oracle_move_rows.argtypes = [p, p, p, p, i64, i64, i64, i64, i64, i64, i32]
        lib.oracle_move_rows.restype = i64
        lib.oracle_set_threads.argtypes = [ctypes.c_int]
        lib.oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def set_threads(n):
    _load().oracle_set_threads(int(n))


def max_threads():
    return _load().oracle_max_threads()


def _addr(a):
    return a.ctypes.data


def _pool_check(pool):
    assert pool.flags.c_contiguous and pool.ndim == 4, 'pools are contiguous (bcap, heads, cap, dim) arrays'


# ---------------------------------------------------------------------------
# KV row movement (C)
# ---------------------------------------------------------------------------
def append(kpool, vpool, ksrc, vsrc, length):
    """pool[:B, :, length:length+q] = src (src (B, H, q, D), any element strides)."""
    _pool_check(kpool)
    b, h, q, d = ksrc.shape
    es = kpool.itemsize
    ks = [s // es for s in ksrc.strides[:3]]
    vs = [s // es for s in vsrc.strides[:3]]
    _load().oracle_append(_addr(kpool), _addr(vpool), _addr(ksrc), _addr(vsrc), b, h, q, d, kpool.shape[2], length,
                          (ctypes.c_int64 * 3)(*ks), (ctypes.c_int64 * 3)(*vs), es)


def compact_suffix(kpool, vpool, batch, length, chosen, past, extension):
    """In-place accepted-suffix compaction of one layer; returns #out-of-range entries."""
    _pool_check(kpool)
    chosen = np.ascontiguousarray(chosen, dtype=np.int64)
    width = chosen.shape[1]
    return _load().oracle_compact_suffix(_addr(kpool), _addr(vpool), batch, kpool.shape[1], kpool.shape[3],
                                         kpool.shape[2], length, _addr(chosen), chosen.shape[1], 1, past, extension,
                                         width, kpool.itemsize)


def remap_rows(kpool, vpool, indices, length):
    _pool_check(kpool)
    indices = np.ascontiguousarray(indices, dtype=np.int64)
    return _load().oracle_remap_rows(_addr(kpool), _addr(vpool), _addr(indices), indices.size, kpool.shape[0],
                                     kpool.shape[1], kpool.shape[3], kpool.shape[2], length, kpool.itemsize)


def move_rows(kpool, vpool, sources, destinations, length):
    _pool_check(kpool)
    sources = np.ascontiguousarray(sources, dtype=np.int64)
    destinations = np.ascontiguousarray(destinations, dtype=np.int64)
    return _load().oracle_move_rows(_addr(kpool), _addr(vpool), _addr(sources), _addr(destinations), sources.size,
                                    kpool.shape[0], kpool.shape[1], kpool.shape[3], kpool.shape[2], length,
                                    kpool.itemsize)


# ---------------------------------------------------------------------------
# tree ops (numpy)
# ---------------------------------------------------------------------------
def trace_path(parents, tokens, contexts, samples, eos, width):
    """Greedy acceptance walk -> (tokens, indices, contexts, lengths), outputs (B, width)."""
    parents, tokens, contexts, samples = (np.asarray(x, dtype=np.int64) for x in (parents, tokens, contexts, samples))
    batch, rows = samples.shape
    out = [np.full((batch, width), -1, dtype=np.int64) for _ in range(3)]
    lengths = np.zeros(batch, dtype=np.int64)
    cur = np.zeros(batch, dtype=np.int64)
    live = np.ones(batch, dtype=bool)
    seq = np.arange(batch)
    cand = np.arange(rows)[None, :]
    for depth in range(width):
        tok = samples[seq, cur]
        out[0][:, depth] = np.where(live, tok, -1)
        out[1][:, depth] = np.where(live, cur, -1)
        out[2][:, depth] = np.where(live, contexts[seq, cur], -1)
        lengths += live
        going = live & (tok != eos)
        match = (parents == cur[:, None]) & (tokens == tok[:, None]) & (cand > 0) & going[:, None]
        found = np.where(match, cand, rows).min(axis=1)
        live = going & (found < rows)
        cur = np.minimum(found, rows - 1)
    return out[0], out[1], out[2], lengths


def _padded(tokens, indices, lengths, width, past, eos):
    tokens = np.asarray(tokens, dtype=np.int64)
    indices = np.asarray(indices, dtype=np.int64)
    lengths = np.asarray(lengths, dtype=np.int64)
    capacity = tokens.shape[1]
    slots = np.arange(capacity)[None, :]
    valid = slots < lengths[:, None]
    budget = np.maximum(width - lengths, 0)[:, None]
    dest = slots + np.minimum(np.maximum(indices - slots, 0), budget)
    positions = np.arange(width)[None, :, None]
    hit = (positions == dest[:, None, :]) & valid[:, None, :]
    accepted = hit.any(-1)
    source = hit.argmax(-1)
    out_tokens = np.where(accepted, np.take_along_axis(tokens, source, 1), eos)
    out_indices = np.where(accepted, np.take_along_axis(indices, source, 1) + past, np.arange(width)[None, :] + past)
    last = np.where(valid, dest, -1).max(axis=1)
    return out_tokens, out_indices, ~accepted, last[:, None]


def pad_verified_path(tokens, indices, lengths, width, past, eos):
    """Gap-first padded layout -> (tokens, indices, mask, last (B, 1))."""
    return _padded(tokens, indices, lengths, width, past, eos)


def pad_schedule(tokens, indices, lengths, past, eos, snapshot=None):
    """Padded layout at width = max(lengths) plus the (B, capacity + 3 [+1]) host packet."""
    tokens = np.asarray(tokens, dtype=np.int64)
    lengths = np.asarray(lengths, dtype=np.int64)
    batch, capacity = tokens.shape
    width = int(min(max(lengths.max(initial=0), 0), capacity))
    out_tokens, out_indices, mask, last = _padded(tokens, indices, lengths, width, past, eos)
    packet = np.full((batch, capacity + 3 + (snapshot is not None)), -1, dtype=np.int64)
    packet[:, 0] = lengths
    tail = tokens[np.arange(batch), np.maximum(lengths - 1, 0)]
    packet[:, 1] = ((tail == eos) & (lengths > 0)).astype(np.int64)
    moved = out_indices != (np.arange(width)[None, :] + past)
    packet[:, 2] = np.where(moved.any(1), moved.argmax(1), width)
    packet[:, 3:3 + width] = np.where(mask, out_indices, -1)
    if snapshot is not None:
        packet[:, capacity + 3] = snapshot
    return out_tokens, out_indices, mask, last, packet, width


def schedule_rows(packet, with_plugin=True):
    """Host rows the scheduler hands back: full packet rows (plugin) or trimmed to 3 + width."""
    rows = [list(map(int, r)) for r in packet]
    width = max(r[0] for r in rows)
    return rows if with_plugin else [r[:3 + width] for r in rows]


def tree_visible(parents, past, steps, pad=None):
    """Visibility (B, R, past + R) of the additive tree mask (True = 0, False = dtype min)."""
    parents = np.asarray(parents, dtype=np.int64)
    batch, rows = parents.shape
    cols = past + rows
    vis = np.zeros((batch, rows, cols), dtype=bool)
    vis[:, :, :past + 1] = True
    cur = np.broadcast_to(np.arange(rows)[None, :], (batch, rows)).copy()
    seq = np.arange(batch)[:, None]
    rr = np.arange(rows)[None, :]
    for _ in range(steps):
        ok = cur >= 0
        col = np.where(ok, past + cur, 0)
        vis[np.broadcast_to(seq, cur.shape)[ok], np.broadcast_to(rr, cur.shape)[ok], col[ok]] = True
        cur = parents[seq, np.maximum(cur, 0)]
    if pad is not None:
        pad = np.asarray(pad, dtype=bool)[:, :cols]
        vis &= ~pad[:, None, :]
    return vis


def additive_mask(visible, dtype_name='float32'):
    """Float32 mask values (0 / lowest of dtype) for a visibility array."""
    lowest = {'float32': np.finfo(np.float32).min, 'bfloat16': -3.3895313892515355e38,
              'float16': -65504.0}[dtype_name]
    return np.where(visible, np.float32(0), np.float32(lowest)).astype(np.float32)[:, None]


def pack_tree(full_parents, full_contexts, chosen, all_tokens):
    """(parents, tokens, contexts) (B, P + 1) and parent-closedness (B, P) bool."""
    full_parents, full_contexts, chosen, all_tokens = (np.asarray(x, dtype=np.int64) for x in
                                                       (full_parents, full_contexts, chosen, all_tokens))
    batch, n = full_parents.shape
    p = chosen.shape[1]
    inverse = np.full((batch, n + 1), -1, dtype=np.int64)
    inverse[:, 0] = 0
    np.put_along_axis(inverse, chosen + 1, np.broadcast_to(np.arange(1, p + 1), (batch, p)), 1)
    parents = np.take_along_axis(inverse, np.take_along_axis(full_parents, chosen, 1) + 1, 1)
    closed = (parents >= 0) & (parents < np.arange(1, p + 1)[None, :])
    out_parents = np.concatenate([np.full((batch, 1), -1), parents], 1)
    out_tokens = np.concatenate([np.full((batch, 1), -1), np.take_along_axis(all_tokens, chosen, 1)], 1)
    out_contexts = np.concatenate([np.zeros((batch, 1), dtype=np.int64),
                                   np.take_along_axis(full_contexts, chosen, 1)], 1)
    return out_parents, out_tokens, out_contexts, closed


def swap_remove_plan(finished):
    """Holes below the new batch filled from live tail rows taken from the end."""
    n = len(finished)
    new_batch = n - int(sum(bool(x) for x in finished))
    holes = [i for i in range(new_batch) if finished[i]]
    tail = [i for i in reversed(range(new_batch, n)) if not finished[i]]
    keep = list(range(new_batch))
    for hole, src in zip(holes, tail):
        keep[hole] = src
    return keep, tail, holes


def position_update(newly_padded, past, past_positions, pad_rows=None, owners=None, pad_live=None):
    """Returns (positions (B, W), new past positions); writes padding columns in place."""
    newly_padded = np.asarray(newly_padded, dtype=bool)
    width = newly_padded.shape[1]
    if pad_rows is not None:
        pad_rows[np.asarray(owners)[:, None], past + np.arange(width)[None, :]] = newly_padded
    if pad_live is not None:
        pad_live[:, past:past + width] = newly_padded
    positions = np.cumsum(~newly_padded, axis=1).astype(np.int64) + np.asarray(past_positions, dtype=np.int64)[:, None]
    return positions, positions[:, -1].copy()


# ---------------------------------------------------------------------------
# attention (float32)
# ---------------------------------------------------------------------------
def attention(q, k, v, mask, scale):
    """q (B, Hq, R, D), k/v (B, Hkv, L, D), mask (B, 1, R, L) additive or None -> (B, R, Hq, D) float32."""
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    batch, hq, rows, dim = q.shape
    group = hq // k.shape[1]
    out = np.empty((batch, rows, hq, dim), dtype=np.float32)
    for b in range(batch):
        kk = np.repeat(k[b], group, axis=0)  # (Hq, L, D)
        vv = np.repeat(v[b], group, axis=0)
        s = np.matmul(q[b], kk.transpose(0, 2, 1)) * np.float32(scale)
        if mask is not None:
            s = s + np.asarray(mask[b], dtype=np.float32)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = np.matmul(p, vv).transpose(1, 0, 2)
    return out


def causal_visible(batch, query, past, columns, pad=None):
    """Visibility (batch, query, columns) of the draft causal mask: c <= past + r, not padding."""
    vis = np.arange(columns)[None, None, :] <= past + np.arange(query)[None, :, None]
    vis = np.broadcast_to(vis, (batch, query, columns)).copy()
    if pad is not None:
        vis &= ~np.asarray(pad, dtype=bool)[:, None, :columns]
    return vis


def expansion_visible(batch, query, columns, init_length, seen, pad=None, pad_pairs=None):
    """Visibility (batch, query, columns) of a draft expansion step: columns below init_length
    and the row's own column seen[b, r]; padding (bool (batch, >= columns) and / or (n, 2)
    pairs (b, column)) off last."""
    vis = np.zeros((batch, query, columns), dtype=bool)
    vis[:, :, :init_length] = True
    seen = np.asarray(seen, dtype=np.int64).reshape(batch, -1)[:, :query]
    b_idx = np.arange(batch)[:, None].repeat(query, 1)
    r_idx = np.arange(query)[None, :].repeat(batch, 0)
    vis[b_idx, r_idx, seen] = True
    if pad is not None:
        vis &= ~np.asarray(pad, dtype=bool)[:, None, :columns]
    if pad_pairs is not None:
        for b, c in np.asarray(pad_pairs, dtype=np.int64).reshape(-1, 2):
            vis[b, :, c] = False
    return vis


# ---------------------------------------------------------------------------
# rollout history
# ---------------------------------------------------------------------------
def gather_positions(tree, index):
    """out[b, w] = tree[b, index[b, w]] for a (B, T, ...) array and (B, W) positions."""
    tree = np.asarray(tree)
    index = np.asarray(index, dtype=np.int64)
    return tree[np.arange(tree.shape[0])[:, None], index]


class RolloutHistory:
    """Contiguous per-response pools: rows = batch x repeats, capacity max(length, max_length),
    grown to max(end, 2 x capacity) on overflow; append writes chunk row i at the pool row
    owners[i] from the field's current length; finalize returns each row's prefix of the
    lengths recorded when the row finished (or at the end)."""

    def __init__(self, initial, repeats, max_length):
        sizes = {a.shape[0] for a in initial.values()}
        assert len(sizes) == 1 and repeats >= 1 and max_length >= 1
        self.rows = sizes.pop() * repeats
        self.pools, self.lengths, self.capacities, self.finished = {}, {}, {}, {}
        for name, a in initial.items():
            a = np.asarray(a)
            cap = max(a.shape[1], int(max_length))
            pool = np.zeros((self.rows, cap) + a.shape[2:], dtype=a.dtype)
            pool[:, :a.shape[1]] = np.repeat(a, repeats, axis=0)
            self.pools[name], self.lengths[name], self.capacities[name] = pool, a.shape[1], cap

    def append(self, owners, chunks):
        owners = np.asarray(owners, dtype=np.int64)
        for name, chunk in chunks.items():
            chunk = np.asarray(chunk)
            pool = self.pools[name]
            start = self.lengths[name]
            end = start + chunk.shape[1]
            if end > pool.shape[1]:
                cap = max(end, 2 * pool.shape[1])
                grown = np.zeros((self.rows, cap) + pool.shape[2:], dtype=pool.dtype)
                grown[:, :start] = pool[:, :start]
                self.pools[name] = pool = grown
                self.capacities[name] = cap
            pool[owners, start:end] = chunk
            self.lengths[name] = end

    def mark_finished(self, row):
        assert row not in self.finished
        self.finished[row] = dict(self.lengths)

    def finalize(self):
        for row in range(self.rows):
            if row not in self.finished:
                self.mark_finished(row)
        return [{name: pool[row, :self.finished[row][name]].copy() for name, pool in self.pools.items()}
                for row in range(self.rows)]
