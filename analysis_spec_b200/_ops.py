"""Torch-tensor front end of the C ABI: shape/stride/device checks, then one
libspeckv call on the current CUDA stream of the tensors' device.

Every function here requires CUDA tensors and raises otherwise; there is no
CPU path in the product. The library launches on the current GPU, so every
entry point here first makes the GPU of its first CUDA tensor argument current
(for the duration of the call); the C side refuses operands of another GPU.
"""
import collections
import functools

import torch

from . import _lib


def _first_device(values):
    """Index of the GPU holding the first CUDA tensor among `values` (tensors or lists of them)."""
    for v in values:
        if isinstance(v, torch.Tensor):
            if v.is_cuda:
                return v.device.index
        elif isinstance(v, (list, tuple)) and v and isinstance(v[0], torch.Tensor) and v[0].is_cuda:
            return v[0].device.index
    return None


def _on_device(fn):
    """Runs `fn` with the GPU of its first CUDA tensor argument current."""
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        dev = _first_device(args)
        if dev is None:
            dev = _first_device(kwargs.values())
        if dev is None or dev == torch.cuda.current_device():
            return fn(*args, **kwargs)
        with torch.cuda.device(dev):
            return fn(*args, **kwargs)
    return wrapper

_DTYPE_CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}

# Prepared append launches of recent calls, keyed by everything the prepared launch holds
# (device, stream, sizes, strides and every operand's address): a verify loop appends the
# same projection buffers into the same pools at the same length round after round, and a
# plan found here skips the packing and the per-pointer device checks of the preparation
# (validated when it was prepared, for operands at these addresses on this device).
_APPEND_PLANS = collections.OrderedDict()
_APPEND_PLANS_MAX = 8


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError('analysis_spec_b200 kernels need CUDA tensors; got a tensor on '
                               f'{t.device} (the product has no CPU path)')


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _pool_geometry(pool):
    if pool.dim() != 4 or pool.stride(3) != 1 or pool.stride(2) != pool.shape[3] or \
            (pool.shape[1] > 1 and pool.stride(1) != pool.shape[2] * pool.shape[3]) or \
            (pool.shape[0] > 1 and pool.stride(0) != pool.shape[1] * pool.shape[2] * pool.shape[3]):
        raise ValueError('KV pools must be contiguous (batch_capacity, heads, capacity, dim) tensors')
    return pool.shape


def _chunks(n):
    for start in range(0, n, _lib.MAX_LAYERS):
        yield start, min(n, start + _lib.MAX_LAYERS)


def _row_table(fn, row_table, batch, pool_rows):
    """(pointer, pool rows) of an optional logical -> physical row table."""
    if row_table is None:
        return None, 0
    _require_cuda(row_table)
    if row_table.dtype != torch.long or not row_table.is_contiguous() or row_table.numel() < batch:
        raise ValueError(f'{fn}: row table must be a contiguous int64 tensor with an entry per sequence')
    return row_table.data_ptr(), pool_rows


@_on_device
def append_rows(key_pools, value_pools, key_srcs, value_srcs, length, launch=True, row_table=None, commit=None):
    """pool[l][:B, :, length:length+q] = src[l] for every layer l (one launch per 64 layers);
    with `row_table` sequence b goes to pool row row_table[b].

    ``commit = (chosen, past, extension, width)`` folds the previous round's accepted-suffix
    compaction (rows chosen[:, extension:width] to past + extension .. past + width) into the
    same launch (speckv_append_commit_rows; without a row table). With ``launch=False`` the
    arguments are validated and marshalled now and a callable that issues the launches is
    returned, so the host work can run while the GPU is still busy with earlier launches."""
    k0, v0 = key_srcs[0], value_srcs[0]
    _require_cuda(key_pools[0], k0)
    bcap, heads, capacity, dim = _pool_geometry(key_pools[0])
    batch, h, rows, d = k0.shape
    if h != heads or d != dim or tuple(v0.shape) != tuple(k0.shape):
        raise ValueError('appended K/V shape does not match the pool')
    if batch > bcap and row_table is None:
        raise ValueError('appended batch exceeds pool batch capacity')
    table, table_rows = _row_table('append_rows', row_table, batch, bcap)
    if k0.stride(3) != 1 or v0.stride(3) != 1:
        raise ValueError('appended K/V need unit stride on head_dim')
    for srcs, first in ((key_srcs, k0), (value_srcs, v0)):
        for t in srcs:
            if t.shape != first.shape or t.stride() != first.stride() or t.dtype != key_pools[0].dtype:
                raise ValueError('every layer must append K/V of one shape, stride and the pool dtype')
    ks =_lib.i64_array(k0.stride()[:3])
    vs = _lib.i64_array(v0.stride()[:3])
    es = key_pools[0].element_size()
    stream = _stream(k0)
    if commit is not None:
        chosen, past, extension, width = commit
        if row_table is not None:
            raise ValueError('the fused append + compaction takes no row table')
        nvec = dim * es // 16
        if (width - extension) * nvec > 256 or -(-rows * nvec // 128) > 32 or len(key_pools) > 64:
            # outside the fused kernel's register stage: the compaction, then the append
            append = append_rows(key_pools, value_pools, key_srcs, value_srcs, length, launch=False)

            def both():
                if width > extension:
                    compact_suffix(key_pools, value_pools, batch, capacity, chosen, past, extension, width)
                append()
            return both() if launch else both
        if width > extension:
            _require_cuda(chosen)
            if chosen.dtype != torch.long or chosen.dim() != 2 or chosen.shape[0] < batch or chosen.shape[1] < width:
                raise ValueError('chosen indices must be a (batch, >= width) int64 tensor')
        cptr, csb, csw = (_ptr(chosen), chosen.stride(0), chosen.stride(1)) if width > extension else (None, 0, 0)
        calls = [(_lib.ptr_array([p.data_ptr() for p in key_pools]), _lib.ptr_array([p.data_ptr() for p in value_pools]),
                  _lib.ptr_array([s.data_ptr() for s in key_srcs]), _lib.ptr_array([s.data_ptr() for s in value_srcs]),
                  len(key_pools), batch, heads, rows, dim, capacity, length, ks, vs, es, cptr, csb, csw, int(past),
                  int(extension), int(width), stream)]
        return _issue('speckv_append_commit_rows', calls, launch)
    if not launch:
        key = (k0.device.index, stream, batch, heads, rows, dim, capacity, bcap, tuple(key_pools[0].stride()), length,
               tuple(k0.stride()), tuple(v0.stride()), es, table, table_rows,
               tuple(p.data_ptr() for p in key_pools), tuple(p.data_ptr() for p in value_pools),
               tuple(t.data_ptr() for t in key_srcs), tuple(t.data_ptr() for t in value_srcs))
        go = _APPEND_PLANS.get(key)
        if go is not None:
            _APPEND_PLANS.move_to_end(key)
            return go
    calls = [(_lib.ptr_array([p.data_ptr() for p in key_pools[a:b]]),
              _lib.ptr_array([p.data_ptr() for p in value_pools[a:b]]),
              _lib.ptr_array([s.data_ptr() for s in key_srcs[a:b]]),
              _lib.ptr_array([s.data_ptr() for s in value_srcs[a:b]]),
              b - a, batch, heads, rows, dim, capacity, length, ks, vs, es, table, table_rows, stream)
             for a, b in _chunks(len(key_pools))]
    go = _issue('speckv_append_rows', calls, launch)
    if not launch:
        _APPEND_PLANS[key] = go
        if len(_APPEND_PLANS) > _APPEND_PLANS_MAX:
            _APPEND_PLANS.popitem(last=False)
    return go


def _issue(name, calls, launch):
    """Issues the entry-point calls now, or prepares them (speckv_<name>_prepare: all
    host-side checks and packing done here) and returns a callable whose only host
    work is one kernel launch per call."""
    if launch:
        for args in calls:
            _lib.call(name, *args)
        return None
    plans = [_lib.prepare(name, *args) for args in calls]

    def go():
        for plan in plans:
            plan()
    return go


@_on_device
def compact_suffix(key_pools, value_pools, batch, length, chosen, past, extension, width, row_table=None):
    """Accepted-suffix compaction of every layer (one launch per 64 layers); with `row_table`
    sequence b is pool row row_table[b]."""
    _require_cuda(key_pools[0], chosen)
    _, heads, capacity, dim = _pool_geometry(key_pools[0])
    if chosen.dtype != torch.long or chosen.dim() != 2:
        raise ValueError('chosen indices must be a (batch, width) int64 tensor')
    if chosen.shape[0] < batch or chosen.shape[1] < width or (batch > key_pools[0].shape[0] and row_table is None):
        raise ValueError('chosen indices do not cover the live batch / width')
    table, table_rows = _row_table('compact_suffix', row_table, batch, key_pools[0].shape[0])
    es = key_pools[0].element_size()
    for a, b in _chunks(len(key_pools)):
        _lib.call('speckv_compact_suffix', _lib.ptr_array([p.data_ptr() for p in key_pools[a:b]]),
                  _lib.ptr_array([p.data_ptr() for p in value_pools[a:b]]), b - a, batch, heads, dim,
                  capacity, length, chosen.data_ptr(), chosen.stride(0), chosen.stride(1), past, extension, width,
                  es, table, table_rows, _stream(chosen))


@_on_device
def commit_round(key_pools, value_pools, batch, length, chosen, past, packet, newly_padded=None, positions=None,
                 past_positions=None, pad_rows=None, owners=None, pad_live=None, launch=True, row_table=None):
    """Compaction of every layer + position/padding update of one verify round in one launch,
    with width and extension taken from the device packet (no host round trip).

    `chosen` / `newly_padded` / `positions` are full-width (batch, max_width) schedule outputs.
    Pass no pools to update positions only, no `positions` to compact only. With
    ``launch=False`` returns a callable that issues the prepared launch (see append_rows);
    with `row_table` sequence b is pool row row_table[b].
    """
    key_pools = list(key_pools or [])
    _require_cuda(packet, chosen, newly_padded, positions, past_positions, pad_rows, owners, pad_live,
                  *(key_pools[:1]))
    if packet.dtype != torch.long or packet.dim() != 2 or packet.stride(1) != 1 or packet.shape[1] < 3 or \
            packet.shape[0] < batch:
        raise ValueError('packet must be a (batch, >= 3) int64 tensor with unit column stride')
    widths = []
    if key_pools:
        if chosen is None or chosen.dtype != torch.long or chosen.dim() != 2 or chosen.shape[0] < batch:
            raise ValueError('chosen indices must be a (batch, width) int64 tensor')
        widths.append(chosen.shape[1])
    if positions is not None:
        if newly_padded is None or past_positions is None:
            raise ValueError('the position update needs newly_padded and past_positions')
        if newly_padded.stride(1) != 1 or positions.stride(1) != 1 or positions.dtype != torch.long or \
                past_positions.dtype != torch.long or not past_positions.is_contiguous():
            raise ValueError('newly_padded / positions need unit column stride; positions must be int64')
        if newly_padded.shape[0] < batch or positions.shape[0] < batch or past_positions.shape[0] < batch:
            raise ValueError('position operands do not cover the batch')
        widths.append(min(newly_padded.shape[1], positions.shape[1]))
        if owners is not None:
            owners = _contig_long('owners', owners)
    if not widths:
        return _issue('speckv_commit_round', [], launch)
    max_width = min(widths)
    pos_args = (_ptr(pad_rows), 0 if pad_rows is None else pad_rows.stride(0),
                0 if pad_rows is None else pad_rows.shape[0], _ptr(owners), _ptr(pad_live),
                0 if pad_live is None else pad_live.stride(0), _ptr(newly_padded),
                0 if newly_padded is None else newly_padded.stride(0), _ptr(positions),
                0 if positions is None else positions.stride(0), _ptr(past_positions))
    no_pos = (None, 0, 0, None, None, 0, None, 0, None, 0, None)
    stream = _stream(packet)
    if not key_pools:
        return _issue('speckv_commit_round', [(None, None, 0, batch, 1, 1, 1, 0, 1, None, 0, 0, past,
                                               packet.data_ptr(), packet.stride(0), max_width, *pos_args, None, 0,
                                               stream)],
                      launch)
    _, heads, capacity, dim = _pool_geometry(key_pools[0])
    table, table_rows = _row_table('commit_round', row_table, batch, key_pools[0].shape[0])
    es = key_pools[0].element_size()
    calls = [(_lib.ptr_array([p.data_ptr() for p in key_pools[a:b]]),
              _lib.ptr_array([p.data_ptr() for p in value_pools[a:b]]), b - a, batch, heads, dim, capacity,
              length, es, chosen.data_ptr(), chosen.stride(0), chosen.stride(1), past, packet.data_ptr(),
              packet.stride(0), max_width, *(pos_args if a == 0 else no_pos), table, table_rows, stream)
             for a, b in _chunks(len(key_pools))]
    return _issue('speckv_commit_round', calls, launch)


def remap_scratch_elements(new_batch, heads, dim, length, element_size):
    """Elements of pool dtype the remap needs as scratch (0 for the single on-chip pass)."""
    nbytes = _lib.load().speckv_remap_scratch_bytes(new_batch, heads, dim, length, element_size)
    return (nbytes + element_size - 1) // element_size


@_on_device
def remap_rows(key_pools, value_pools, indices, length, scratch=None):
    """pool[:n] = pool[indices] over [0, length) for every layer."""
    _require_cuda(key_pools[0], indices)
    bcap, heads, capacity, dim = _pool_geometry(key_pools[0])
    if indices.dtype != torch.long or not indices.is_contiguous():
        indices = indices.to(torch.long).contiguous()
    es = key_pools[0].element_size()
    scratch_bytes = 0 if scratch is None else scratch.numel() * scratch.element_size()
    for a, b in _chunks(len(key_pools)):
        _lib.call('speckv_remap_rows', _lib.ptr_array([p.data_ptr() for p in key_pools[a:b]]),
                  _lib.ptr_array([p.data_ptr() for p in value_pools[a:b]]), b - a, indices.data_ptr(),
                  indices.numel(), bcap, heads, dim, capacity, length, _ptr(scratch), scratch_bytes, es,
                  _stream(indices))


@_on_device
def remap_rows_static(key_pools, value_pools, indices, length):
    """remap_rows without scratch from the caller: uses the library's fixed device array
    (for callers that cannot allocate; concurrent calls on one device must be serialised)."""
    _require_cuda(key_pools[0], indices)
    bcap, heads, capacity, dim = _pool_geometry(key_pools[0])
    if indices.dtype != torch.long or not indices.is_contiguous():
        raise ValueError('indices must be a contiguous int64 tensor')
    es = key_pools[0].element_size()
    for a, b in _chunks(len(key_pools)):
        _lib.call('speckv_remap_rows_static', _lib.ptr_array([p.data_ptr() for p in key_pools[a:b]]),
                  _lib.ptr_array([p.data_ptr() for p in value_pools[a:b]]), b - a, indices.data_ptr(),
                  indices.numel(), bcap, heads, dim, capacity, length, es, _stream(indices))


@_on_device
def move_rows(key_pools, value_pools, sources, destinations, length):
    """pool[destinations[j]] = pool[sources[j]] over [0, length) for every layer."""
    _require_cuda(key_pools[0], sources, destinations)
    bcap, heads, capacity, dim = _pool_geometry(key_pools[0])
    sources = sources.to(torch.long).contiguous()
    destinations = destinations.to(torch.long).contiguous()
    if sources.numel() != destinations.numel():
        raise ValueError('sources and destinations differ in length')
    es = key_pools[0].element_size()
    for a, b in _chunks(len(key_pools)):
        _lib.call('speckv_move_rows', _lib.ptr_array([p.data_ptr() for p in key_pools[a:b]]),
                  _lib.ptr_array([p.data_ptr() for p in value_pools[a:b]]), b - a, sources.data_ptr(),
                  destinations.data_ptr(), sources.numel(), bcap, heads, dim, capacity, length, es,
                  _stream(sources))


def _contig_long(name, t):
    if t.dtype != torch.long:
        raise ValueError(f'{name} must be int64')
    return t if t.is_contiguous() else t.contiguous()


@_on_device
def pack_tree(full_parents, full_contexts, all_tokens, chosen, out_parents, out_tokens, out_contexts):
    _require_cuda(full_parents, full_contexts, all_tokens, chosen, out_parents, out_tokens, out_contexts)
    batch, full_count = full_parents.shape
    packed = chosen.shape[1]
    full_parents, full_contexts, all_tokens, chosen = (_contig_long(n, t) for n, t in (
        ('full_parents', full_parents), ('full_contexts', full_contexts), ('all_tokens', all_tokens),
        ('chosen', chosen)))
    if all_tokens.shape[1] != full_count or full_contexts.shape[1] != full_count:
        raise ValueError('full tree tensors differ in node count')
    for t in (out_parents, out_tokens, out_contexts):
        if t.shape != (batch, packed + 1) or t.stride() != out_parents.stride() or t.stride(1) != 1:
            raise ValueError('packed outputs must be (batch, packed + 1) with unit column stride')
    _lib.call('speckv_pack_tree', full_parents.data_ptr(), full_contexts.data_ptr(), all_tokens.data_ptr(),
              chosen.data_ptr(), batch, full_count, packed, out_parents.data_ptr(), out_tokens.data_ptr(),
              out_contexts.data_ptr(), out_parents.stride(0), _stream(chosen))


@_on_device
def trace_path(parents, tokens, contexts, samples, eos, out_tokens, out_indices, out_contexts, lengths):
    _require_cuda(parents, tokens, contexts, samples, out_tokens, out_indices, out_contexts, lengths)
    batch, rows = samples.shape
    parents, tokens, contexts, samples = (_contig_long(n, t) for n, t in
                                          (('parents', parents), ('tokens', tokens), ('contexts', contexts),
                                           ('samples', samples)))
    if out_tokens.stride() != out_indices.stride() or out_tokens.stride() != out_contexts.stride():
        raise ValueError('trace outputs must share strides')
    if lengths.stride(0) != 1 and lengths.numel() > 1:
        raise ValueError('lengths must be contiguous')
    _lib.call('speckv_trace_path', parents.data_ptr(), tokens.data_ptr(), contexts.data_ptr(), samples.data_ptr(),
              batch, rows, int(eos), out_tokens.data_ptr(), out_indices.data_ptr(), out_contexts.data_ptr(),
              out_tokens.stride(0), out_tokens.stride(1), out_tokens.shape[1], lengths.data_ptr(),
              _stream(samples))


def _check_pad_outputs(tokens, indices, mask):
    if tokens.stride() != indices.stride() or tokens.stride() != mask.stride():
        raise ValueError('padded outputs must share strides')
    if tokens.dtype != torch.long or indices.dtype != torch.long or mask.dtype != torch.bool:
        raise ValueError('padded outputs must be int64, int64, bool')


@_on_device
def pad_verified_path(path_tokens, path_indices, lengths, width, past, eos, tokens, indices, mask, last):
    _require_cuda(path_tokens, path_indices, lengths, tokens, indices, mask, last)
    _check_pad_outputs(tokens, indices, mask)
    batch, capacity = path_tokens.shape
    lengths = _contig_long('lengths', lengths)
    _lib.call('speckv_pad_verified_path', path_tokens.data_ptr(), path_tokens.stride(0), path_tokens.stride(1),
              path_indices.data_ptr(), path_indices.stride(0), path_indices.stride(1), lengths.data_ptr(), batch,
              capacity, int(width), int(past), int(eos), tokens.data_ptr(), indices.data_ptr(), mask.data_ptr(),
              tokens.stride(0), tokens.stride(1), last.data_ptr(), last.stride(0), _stream(path_tokens))


@_on_device
def pad_schedule(path_tokens, path_indices, lengths, past, eos, tokens, indices, mask, last, packet,
                 snapshot=None):
    _require_cuda(path_tokens, path_indices, lengths, tokens, indices, mask, last, packet, snapshot)
    _check_pad_outputs(tokens, indices, mask)
    batch, capacity = path_tokens.shape
    lengths = _contig_long('lengths', lengths)
    if packet.shape[1] < capacity + 3:
        raise ValueError('packet too narrow for the path capacity')
    if snapshot is not None:
        # The snapshot lands in column capacity + 3, just past a (b, capacity + 3)
        # slice of the caller's (b, capacity + 4) packet: check the storage holds it.
        last_elem = packet.storage_offset() + (batch - 1) * packet.stride(0) + (capacity + 3) * packet.stride(1)
        if last_elem >= packet.untyped_storage().nbytes() // packet.element_size():
            raise ValueError('packet storage has no snapshot column')
    _lib.call('speckv_pad_schedule', path_tokens.data_ptr(), path_tokens.stride(0), path_tokens.stride(1),
              path_indices.data_ptr(), path_indices.stride(0), path_indices.stride(1), lengths.data_ptr(), batch,
              capacity, int(past), int(eos), tokens.data_ptr(), indices.data_ptr(), mask.data_ptr(),
              tokens.stride(0), tokens.stride(1), last.data_ptr(), last.stride(0), packet.data_ptr(),
              packet.stride(0), packet.stride(1), _ptr(snapshot), _stream(path_tokens))


@_on_device
def tree_mask(parents, past, steps, mask, pad=None):
    """Dense additive ancestor mask (batch, 1, rows, past + rows); `pad` (batch, >= cols) bool forces columns off."""
    _require_cuda(parents, mask, pad)
    batch, rows = parents.shape
    parents = _contig_long('parents', parents)
    if not mask.is_contiguous() or tuple(mask.shape) != (batch, 1, rows, past + rows):
        raise ValueError('mask must be a contiguous (batch, 1, rows, past + rows) tensor')
    if mask.dtype not in _DTYPE_CODE:
        raise ValueError(f'unsupported mask dtype {mask.dtype}')
    pad_stride = 0
    if pad is not None:
        if pad.dtype != torch.bool or pad.stride(-1) != 1 or pad.shape[-1] < past + rows:
            raise ValueError('pad must be a bool (batch, columns) tensor covering past + rows columns')
        pad_stride = pad.stride(0)
    _lib.call('speckv_tree_mask', parents.data_ptr(), batch, rows, int(past), int(steps), mask.data_ptr(),
              _DTYPE_CODE[mask.dtype], _ptr(pad), pad_stride, _stream(parents))
    torch.autograd.graph.increment_version(mask)


@_on_device
def position_update(newly_padded, past, positions, past_positions, pad_rows=None, owners=None, pad_live=None):
    _require_cuda(newly_padded, positions, past_positions, pad_rows, owners, pad_live)
    batch, width = newly_padded.shape
    if newly_padded.stride(1) != 1 or positions.stride(1) != 1:
        raise ValueError('newly_padded / positions need unit column stride')
    if past_positions.dtype != torch.long or positions.dtype != torch.long or not past_positions.is_contiguous():
        raise ValueError('positions must be contiguous int64')
    if owners is not None:
        owners = _contig_long('owners', owners)
    _lib.call('speckv_position_update', _ptr(pad_rows), 0 if pad_rows is None else pad_rows.stride(0),
              0 if pad_rows is None else pad_rows.shape[0], _ptr(owners), _ptr(pad_live),
              0 if pad_live is None else pad_live.stride(0), newly_padded.data_ptr(), newly_padded.stride(0), batch,
              int(past), width, positions.data_ptr(), positions.stride(0), past_positions.data_ptr(),
              _stream(newly_padded))


@_on_device
def tree_attention(query, key, value, mask, scale, out=None):
    """GQA attention (batch, Hq, R, D) x (batch, Hkv, L, D) -> (batch, R, Hq, D) with an additive mask."""
    _require_cuda(query, key, value, mask)
    batch, q_heads, rows, dim = query.shape
    kv_heads, kv_len = key.shape[1], key.shape[2]
    if query.dtype not in _DTYPE_CODE or key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError('query/key/value must share a float dtype')
    if query.stride(3) != 1 or key.stride(3) != 1 or value.stride(3) != 1:
        raise ValueError('query/key/value need unit stride on head_dim')
    if tuple(value.shape) != tuple(key.shape) or key.shape[0] != batch or key.shape[3] != dim:
        raise ValueError('key/value shapes do not match the query')
    mask_code = 0
    if mask is not None:
        if mask.dim() != 4 or mask.shape[1] != 1 or mask.shape[0] != batch or mask.shape[2] != rows or \
                mask.shape[3] != kv_len:
            mask = mask.expand(batch, 1, rows, kv_len)
        if mask.dtype == torch.bool:
            mask = torch.zeros((), dtype=query.dtype, device=mask.device).masked_fill(
                ~mask, torch.finfo(query.dtype).min).expand(batch, 1, rows, kv_len)
        mask = mask.contiguous()
        mask_code = _DTYPE_CODE[mask.dtype]
    if out is None:
        out = torch.empty((batch, rows, q_heads, dim), device=query.device, dtype=query.dtype)
    _lib.call('speckv_tree_attention', query.data_ptr(), _lib.i64_array(query.stride()[:3]), key.data_ptr(),
              _lib.i64_array(key.stride()[:3]), value.data_ptr(), _lib.i64_array(value.stride()[:3]), _ptr(mask),
              mask_code, out.data_ptr(), batch, q_heads, kv_heads, rows, kv_len, dim, float(scale),
              _DTYPE_CODE[query.dtype], _stream(query))
    return out


def visibility_words(cols):
    """32-bit words per tree row of the visibility bitmap (whole 128-column tiles)."""
    return 4 * (-(-cols // 128))


@_on_device
def tree_mask_bits(parents, past, steps, bits, first_col, pad=None):
    """Bit-packed tree visibility (batch, rows, words) int32 + first visible column per sequence."""
    _require_cuda(parents, bits, first_col, pad)
    batch, rows = parents.shape
    parents = _contig_long('parents', parents)
    if bits.dtype != torch.int32 or not bits.is_contiguous() or bits.shape[:2] != (batch, rows):
        raise ValueError('bits must be a contiguous (batch, rows, words) int32 tensor')
    if first_col.dtype != torch.int32 or first_col.numel() < batch:
        raise ValueError('first_col must be an int32 tensor of batch entries')
    pad_stride = 0
    if pad is not None:
        if pad.dtype != torch.bool or pad.stride(-1) != 1 or pad.shape[-1] < past + rows:
            raise ValueError('pad must be a bool (batch, columns) tensor covering past + rows columns')
        pad_stride = pad.stride(0)
    _lib.call('speckv_tree_mask_bits', parents.data_ptr(), batch, rows, int(past), int(steps), _ptr(pad), pad_stride,
              bits.data_ptr(), bits.shape[2], first_col.data_ptr(), _stream(parents))


def _check_qkv(query, key, value, any_kv_rows=False):
    if query.dtype not in _DTYPE_CODE or key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError('query/key/value must share a float dtype')
    if query.stride(3) != 1 or key.stride(3) != 1 or value.stride(3) != 1:
        raise ValueError('query/key/value need unit stride on head_dim')
    if tuple(value.shape) != tuple(key.shape) or key.shape[3] != query.shape[3] or \
            (key.shape[0] != query.shape[0] and not any_kv_rows):
        raise ValueError('key/value shapes do not match the query')


@_on_device
def tree_attention_bits(query, key, value, bits, first_col, scale, out=None, row_table=None):
    """GQA attention with visibility from tree_mask_bits (no dense mask read). With `row_table`
    the K/V of sequence b are key[row_table[b]] / value[row_table[b]] (key / value then hold
    every pool row)."""
    _require_cuda(query, key, value, bits, first_col, row_table)
    _check_qkv(query, key, value, any_kv_rows=row_table is not None)
    table, kv_batch = _row_table('tree_attention_bits', row_table, query.shape[0], key.shape[0])
    batch, q_heads, rows, dim = query.shape
    kv_heads, kv_len = key.shape[1], key.shape[2]
    if bits.dtype != torch.int32 or not bits.is_contiguous() or bits.shape[:2] != (batch, rows):
        raise ValueError('bits must be a contiguous (batch, rows, words) int32 tensor')
    if out is None:
        out = torch.empty((batch, rows, q_heads, dim), device=query.device, dtype=query.dtype)
    _lib.call('speckv_tree_attention_bits', query.data_ptr(), _lib.i64_array(query.stride()[:3]), key.data_ptr(),
              _lib.i64_array(key.stride()[:3]), value.data_ptr(), _lib.i64_array(value.stride()[:3]),
              bits.data_ptr(), bits.shape[2], _ptr(first_col), out.data_ptr(), batch, q_heads, kv_heads, rows,
              kv_len, dim, float(scale), _DTYPE_CODE[query.dtype], table, kv_batch, _stream(query))
    return out


@_on_device
def tree_attention_bits_append(query, key_pool, value_pool, past, key_states, value_states, bits, first_col, scale,
                               out=None):
    """The round's append fused into the verify attention of one layer
    (speckv_tree_attention_bits_append): key_states / value_states ((batch, kv_heads, rows, dim)
    views, e.g. the projection output) are stored into key_pool / value_pool ((batch, kv_heads,
    capacity, dim)) at position `past`, and the attention runs over the past + rows positions
    with the new rows read straight from key_states / value_states. Same pools as
    append_rows([key_pool], [value_pool], [key_states], [value_states], past) followed by
    tree_attention_bits over key_pool[:, :, :past + rows]; returns the output."""
    _require_cuda(query, key_pool, value_pool, key_states, value_states, bits, first_col)
    _check_qkv(query, key_states, value_states)
    if key_pool.dtype != query.dtype or value_pool.dtype != query.dtype or key_pool.stride(3) != 1 or \
            value_pool.stride(3) != 1 or tuple(key_pool.shape) != tuple(value_pool.shape) or \
            key_pool.shape[0] != query.shape[0] or key_pool.shape[1] != key_states.shape[1] or \
            key_pool.shape[3] != query.shape[3]:
        raise ValueError('key/value pools must be (batch, kv_heads, capacity, head_dim) views of the query dtype')
    batch, q_heads, rows, dim = query.shape
    kv_heads, capacity = key_pool.shape[1], key_pool.shape[2]
    if key_states.shape[2] != rows:
        raise ValueError('one new key/value row per query row required')
    if bits.dtype != torch.int32 or not bits.is_contiguous() or bits.shape[:2] != (batch, rows):
        raise ValueError('bits must be a contiguous (batch, rows, words) int32 tensor')
    if out is None:
        out = torch.empty((batch, rows, q_heads, dim), device=query.device, dtype=query.dtype)
    _lib.call('speckv_tree_attention_bits_append', query.data_ptr(), _lib.i64_array(query.stride()[:3]),
              key_pool.data_ptr(), _lib.i64_array(key_pool.stride()[:3]), value_pool.data_ptr(),
              _lib.i64_array(value_pool.stride()[:3]), int(past), capacity, key_states.data_ptr(),
              _lib.i64_array(key_states.stride()[:3]), value_states.data_ptr(), _lib.i64_array(value_states.stride()[:3]),
              bits.data_ptr(), bits.shape[2], _ptr(first_col), out.data_ptr(), batch, q_heads, kv_heads, rows, dim,
              float(scale), _DTYPE_CODE[query.dtype], _stream(query))
    return out


def device_error(device=None):
    """Reads and clears the library's device error word; returns (kind, value) or None."""
    import ctypes
    word = ctypes.c_uint64(0)
    dev = torch.device('cuda', torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.call('speckv_device_error', ctypes.byref(word), torch.cuda.current_stream(dev).cuda_stream)
    if word.value == 0:
        return None
    kind = word.value >> 48
    value = word.value & 0xFFFFFFFFFFFF
    if value >> 47:
        value -= 1 << 48
    return _lib.DEVICE_ERROR_KINDS.get(kind, str(kind)), value


def _mask_operands(fn, mask, pad):
    if not mask.is_contiguous() or mask.dim() != 4 or mask.shape[1] != 1:
        raise ValueError(f'{fn}: mask must be a contiguous (batch, 1, query, columns) tensor')
    if mask.dtype not in _DTYPE_CODE:
        raise ValueError(f'{fn}: unsupported mask dtype {mask.dtype}')
    if pad is None:
        return 0, 0
    if pad.dtype != torch.bool or pad.dim() != 2 or pad.shape[0] < mask.shape[0] or pad.shape[1] < mask.shape[3]:
        raise ValueError(f'{fn}: padding must be a bool (batch, >= columns) tensor')
    return pad.stride(0), pad.stride(1)


def _bits_operands(fn, mask, bits, first_col):
    if bits is None:
        return 0
    batch, _, query, columns = mask.shape
    if bits.dtype != torch.int32 or not bits.is_contiguous() or tuple(bits.shape[:2]) != (batch, query) or \
            bits.shape[2] < visibility_words(columns):
        raise ValueError(f'{fn}: bits must be a contiguous (batch, query, >= 4 * ceil(columns / 128)) int32 tensor')
    if first_col is None or first_col.dtype != torch.int32 or first_col.numel() < batch:
        raise ValueError(f'{fn}: first_col must be an int32 tensor of batch entries')
    return bits.shape[2]


@_on_device
def causal_mask(mask, past, pad=None, bits=None, first_col=None):
    """mask[b, 0, r, c] = 0 if c <= past + r and not pad[b, c] else finfo(dtype).min (one launch);
    with `bits` / `first_col` the same visibility bit-packed for tree_attention_bits."""
    _require_cuda(mask, pad, bits, first_col)
    ps0, ps1 = _mask_operands('causal_mask', mask, pad)
    words = _bits_operands('causal_mask', mask, bits, first_col)
    batch, _, query, columns = mask.shape
    _lib.call('speckv_causal_mask', mask.data_ptr(), _DTYPE_CODE[mask.dtype], batch, query, int(past), columns,
              _ptr(pad), ps0, ps1, _ptr(bits), words, _ptr(first_col), _stream(mask))
    torch.autograd.graph.increment_version(mask)


@_on_device
def expansion_mask(mask, init_length, seen, pad=None, bits=None, first_col=None):
    """mask[b, 0, r, c] = 0 if (c < init_length or c == seen[b, r, 0]) and not pad[b, c], else
    finfo(dtype).min; `seen` (batch, query[, 1]) int64 (one launch)."""
    _require_cuda(mask, seen, pad, bits, first_col)
    ps0, ps1 = _mask_operands('expansion_mask', mask, pad)
    words = _bits_operands('expansion_mask', mask, bits, first_col)
    batch, _, query, columns = mask.shape
    if seen.dtype != torch.long or seen.shape[0] < batch or seen.shape[1] < query:
        raise ValueError('expansion_mask: seen must be an int64 (batch, query[, 1]) tensor')
    _lib.call('speckv_expansion_mask', mask.data_ptr(), _DTYPE_CODE[mask.dtype], batch, query, columns,
              int(init_length), seen.data_ptr(), seen.stride(0), seen.stride(1), _ptr(pad), ps0, ps1, _ptr(bits),
              words, _ptr(first_col), _stream(mask))
    torch.autograd.graph.increment_version(mask)


def _position_layout(fn, t):
    """(row stride, position stride) in bytes and bytes per position of a (rows, positions,
    *element) tensor whose element dims are contiguous."""
    es = t.element_size()
    expect = 1
    for size, stride in zip(reversed(t.shape[2:]), reversed(t.stride()[2:])):
        if size != 1 and stride != expect:
            raise ValueError(f'{fn}: element dims of a history tensor must be contiguous')
        expect *= size
    return t.stride(0) * es, t.stride(1) * es, expect * es


def _history_layout_key(fields, n, pool_rows):
    key = [n, pool_rows]
    for pool, src, index, gathered, start, width in fields:
        key.append((0 if pool is None else pool.data_ptr(), None if pool is None else (pool.shape, pool.stride()),
                    src.dtype, src.shape, src.stride(), None if index is None else (index.dtype, index.shape, index.stride()),
                    None if gathered is None else (gathered.dtype, gathered.shape, gathered.is_contiguous()), width))
    return tuple(key)


@_on_device
def history_append(fields, owners, pool_rows, n, src_rows=None, cache=None):
    """One launch over up to four history fields. Each field is a tuple
    (pool, src, index, gathered, start, width): pool (pool_rows, capacity, *elem) or None;
    src (rows, positions, *elem); index int64 (n, width) source positions or None (w);
    gathered contiguous (n, width, *elem) or None. owners int64 (n,) pool rows;
    src_rows int64 (n,) source rows or None (i). `cache` (a dict the caller keeps) holds the
    packed argument arrays of each layout seen (pools, shapes, strides, widths): a later call
    with the same layout only refreshes the source, index, output pointers and starts."""
    if not 1 <= len(fields) <= 4:
        raise ValueError('history_append: 1..4 fields')
    _require_cuda(owners, src_rows)
    for t in (owners, src_rows):
        if t is not None and (t.dtype != torch.long or not t.is_contiguous() or t.numel() < n):
            raise ValueError('history_append: owners / src_rows must be contiguous int64 with n entries')
    key = None
    if cache is not None:
        key = _history_layout_key(fields, n, pool_rows)
        packed = cache.get(key)
        if packed is not None:
            args, srcs, idx, gath, starts = packed
            for f, (pool, src, index, gathered, start, width) in enumerate(fields):
                if not src.is_cuda or (index is not None and not index.is_cuda) or \
                        (gathered is not None and not gathered.is_cuda):
                    raise RuntimeError('analysis_spec_b200 kernels need CUDA tensors (the product has no CPU path)')
                srcs[f] = src.data_ptr()
                idx[f] = _ptr(index)
                gath[f] = _ptr(gathered)
                starts[f] = int(start)
            _lib.call('speckv_history_append', *args, _ptr(owners), _ptr(src_rows), int(n), int(pool_rows),
                      _stream(fields[0][1]))
            return
    pools, pstr, srcs, sstr, idx, istr, gath, rbytes, spos, starts, widths, caps = ([] for _ in range(12))
    for pool, src, index, gathered, start, width in fields:
        _require_cuda(pool, src, index, gathered)
        sr, sp, rb = _position_layout('history_append', src)
        if pool is not None:
            if pool.dtype != src.dtype or tuple(pool.shape[2:]) != tuple(src.shape[2:]):
                raise ValueError('history_append: pool and source element shape / dtype differ')
            pr, pp, _ = _position_layout('history_append', pool)
        else:
            pr = pp = 0
        if index is not None and (index.dtype != torch.long or index.dim() != 2 or index.shape[0] < n or
                                  index.shape[1] < width):
            raise ValueError('history_append: index must be an int64 (n, width) tensor')
        if gathered is not None and (not gathered.is_contiguous() or gathered.dtype != src.dtype or
                                     gathered.numel() * gathered.element_size() < n * width * rb):
            raise ValueError('history_append: gathered must be a contiguous (n, width, *element) tensor')
        pools.append(_ptr(pool))
        pstr += [pr, pp]
        srcs.append(src.data_ptr())
        sstr += [sr, sp]
        idx.append(_ptr(index))
        istr += list(index.stride()) if index is not None else [0, 0]
        gath.append(_ptr(gathered))
        rbytes.append(rb)
        spos.append(src.shape[1])
        starts.append(int(start))
        widths.append(int(width))
        caps.append(pool.shape[1] if pool is not None else 0)
    srcs, idx, gath, starts = (_lib.ptr_array(srcs), _lib.ptr_array(idx), _lib.ptr_array(gath),
                               _lib.i64_array(starts))
    args = (len(fields), _lib.ptr_array(pools), _lib.i64_array(pstr), srcs, _lib.i64_array(sstr), idx,
            _lib.i64_array(istr), gath, _lib.i64_array(rbytes), _lib.i64_array(spos), starts, _lib.i64_array(widths),
            _lib.i64_array(caps))
    if cache is not None:
        if len(cache) >= 16:
            cache.clear()
        cache[key] = (args, srcs, idx, gath, starts)
    _lib.call('speckv_history_append', *args, _ptr(owners), _ptr(src_rows), int(n), int(pool_rows),
              _stream(fields[0][1]))


@_on_device
def history_pack(dst, pool, offsets, rows, max_length):
    """dst (total, *elem) contiguous <- the used prefix of each pool row; offsets int64 (rows + 1,)."""
    _require_cuda(dst, pool, offsets)
    pr, pp, rb = _position_layout('history_pack', pool)
    if not dst.is_contiguous() or dst.dtype != pool.dtype:
        raise ValueError('history_pack: dst must be contiguous with the pool dtype')
    if offsets.dtype != torch.long or not offsets.is_contiguous() or offsets.numel() < rows + 1:
        raise ValueError('history_pack: offsets must be contiguous int64 with rows + 1 entries')
    _lib.call('speckv_history_pack', dst.data_ptr(), pool.data_ptr(), pr, pp, rb, offsets.data_ptr(), int(rows),
              int(max_length), _stream(pool))


def set_attention_ctas(ctas):
    """Caps the persistent attention grid of this process at `ctas` CTAs (0: one per SM)."""
    _lib.call('speckv_attention_set_ctas', int(ctas))


def set_attention_chunks(on):
    """Turns key-range chunks of long sequences in the visibility-bits attention on or off for
    this process (off by default): for batches of ragged long sequences."""
    _lib.call('speckv_attention_set_chunks', 1 if on else 0)


@_on_device
def acceptance_counts(packet, batch, proposed_per_row, counts):
    """counts[:5] = the round's acceptance-counter increments from the packet rows (device)."""
    _require_cuda(packet, counts)
    if counts.dtype != torch.long or not counts.is_contiguous() or counts.numel() < 5:
        raise ValueError('acceptance_counts: counts must be a contiguous int64 tensor of 5 entries')
    if batch == 0:  # nothing to read (an empty packet may carry any strides)
        _lib.call('speckv_acceptance_counts', None, 2, 0, int(proposed_per_row), counts.data_ptr(), _stream(counts))
        return
    if packet.dtype != torch.long or packet.dim() != 2 or packet.stride(1) != 1 or packet.shape[1] < 2 or \
            packet.shape[0] < batch:
        raise ValueError('acceptance_counts: packet must be a (batch, >= 2) int64 tensor with unit column stride')
    _lib.call('speckv_acceptance_counts', packet.data_ptr(), packet.stride(0), int(batch), int(proposed_per_row),
              counts.data_ptr(), _stream(packet))


@_on_device
def mask_bits(mask, bits, first_col, nonbinary):
    """Visibility bits of a dense additive (batch, 1, rows, columns) mask (any strides): bit set
    iff the entry is 0; lowest-value / -inf entries masked; any other value sets nonbinary[0]."""
    _require_cuda(mask, bits, first_col, nonbinary)
    if mask.dim() != 4 or mask.shape[1] != 1 or mask.dtype not in _DTYPE_CODE:
        raise ValueError('mask_bits: mask must be a float (batch, 1, rows, columns) tensor')
    batch, _, rows, cols = mask.shape
    if bits.dtype != torch.int32 or not bits.is_contiguous() or tuple(bits.shape[:2]) != (batch, rows):
        raise ValueError('mask_bits: bits must be a contiguous (batch, rows, words) int32 tensor')
    if first_col.dtype != torch.int32 or first_col.numel() < batch or nonbinary.dtype != torch.int32:
        raise ValueError('mask_bits: first_col / nonbinary must be int32')
    _lib.call('speckv_mask_bits', mask.data_ptr(), _DTYPE_CODE[mask.dtype], batch, rows, cols,
              _lib.i64_array([mask.stride(0), mask.stride(2), mask.stride(3)]), bits.data_ptr(), bits.shape[2],
              first_col.data_ptr(), nonbinary.data_ptr(), _stream(mask))
