"""Preallocated, geometrically growing static KV cache behind the HF ``Cache`` API.

Drop-in for ``helper/opd_static_cache.py`` of the reference: same classes,
methods, attributes, counters and error messages. Each layer keeps its own K
and V pool ``(batch_capacity, heads, capacity, head_dim)``; the visible cache is
the strided view ``pool[:batch_size, :, :length]``.

All row movement runs in libspeckv's sm_100a kernels. Cache-wide operations
(repeat / select / swap-remove, and the B200 additions ``update_layers`` and
``commit_accepted``) move every layer, K and V, in ONE launch instead of the
reference's per-layer launches.

Row tables (``OPDStaticCache(..., row_table=True)``; the reference has none): sequence b
lives in pool row ``row_table[b]`` instead of row b. Releasing finished sequences
(``swap_remove``) and admitting new ones (``admit``) then rewrite the table instead of
moving whole histories; append, commit and the tree-verify attention read through it.
The per-layer views handed to the attention are then the pools' full row range tagged
with the table (``_speckv_rows``), which this package's attention functions follow; an
attention implementation that ignores the tag would read the wrong rows, so the mode is
for callers that run ``tree_attention`` / ``draft_attention``.

Reference semantics followed (file:line in the reference project):
  StaticAppendLayer            helper/opd_static_cache.py:17-174
  OPDStaticCache               helper/opd_static_cache.py:177-244
  swap_remove_plan             helper/opd_static_cache.py:247-254
  persistent_cache             helper/opd_static_cache.py:257-264
"""
import weakref

import torch
from transformers.cache_utils import Cache

try:
    from transformers.cache_utils import CacheLayerMixin
except ImportError:  # older transformers
    CacheLayerMixin = object

from . import _ops

LAYER_COUNTERS = ('pool_allocations', 'full_kv_reallocations', 'full_history_copies', 'full_history_copy_bytes',
                  'row_compactions', 'row_compaction_bytes')


class StaticAppendLayer(CacheLayerMixin):
    """One layer's K/V pools with suffix append, crop, remap and swap-remove."""

    is_compileable = False
    is_sliding = False

    def __init__(self, capacity, owner=None):
        self.key_pool = self.value_pool = None
        self.length = self.batch_size = self.batch_capacity = 0
        # Weak link: the cache owns its layers; a strong back-reference would keep
        # every pool alive until a cyclic GC pass after the rollout.
        self._owner_ref = weakref.ref(owner) if owner is not None else None
        self.stats = {name: 0 for name in LAYER_COUNTERS}
        super().__init__()
        self.capacity = capacity
        self.is_initialized = False
        # (key_states, value_states, position) of rows appended with the owner's fuse_append on
        # and not yet in the pools: the next verify attention over this layer's views stores
        # them (speckv_tree_attention_bits_append); any other use of the pools stores them first
        self._pending = None

    # ---- deferred append (OPDStaticCache(fuse_append=True)) ---------------------
    def _flush(self):
        """Stores rows whose append was deferred to the attention (one append launch)."""
        pending, self._pending = self._pending, None
        if pending is not None:
            k, v, position = pending
            _ops.append_rows([self.key_pool], [self.value_pool], [k], [v], position, row_table=self._table())

    def _fusable(self, key_states, value_states):
        """True when the rows can be left to the fused append + attention kernel: the owner
        asked for it, no row table, head dim 128 in bf16 / fp16, at most 128 rows, CUDA views
        whose bases and strides the kernel's tensor maps can address (16-byte units)."""
        owner = self.owner
        if owner is None or not owner.fuse_append or self._table() is not None:
            return False
        for t in (key_states, value_states):
            if not t.is_cuda or t.dtype not in (torch.bfloat16, torch.float16) or t.dim() != 4 or \
                    t.shape[-1] != 128 or not 1 <= t.shape[-2] <= 128 or t.stride(3) != 1 or \
                    t.data_ptr() % 16 or any(st * t.element_size() % 16 for st in t.stride()[:3]):
                return False
        return True

    # ---- views ---------------------------------------------------------------
    @property
    def owner(self):
        return self._owner_ref() if self._owner_ref is not None else None

    def _table(self):
        owner = self.owner
        return owner._device_rows(self.batch_size) if owner is not None and owner.uses_row_table else None

    def _view(self, pool):
        if pool is None:
            return None
        table = self._table()
        if table is None:
            return pool[:self.batch_size, :, :self.length, :]
        view = pool[:, :, :self.length, :]
        view._speckv_rows = table  # sequence b is pool row table[b]
        return view

    @property
    def keys(self):
        self._flush()
        return self._view(self.key_pool)

    @keys.setter
    def keys(self, value):
        if value is not None:
            self._adopt_view(value, self.key_pool)

    @property
    def values(self):
        self._flush()
        return self._view(self.value_pool)

    @values.setter
    def values(self, value):
        if value is not None:
            self._adopt_view(value, self.value_pool)

    def _adopt_view(self, view, pool):
        # Only views of this layer's own storage may be assigned back (they set
        # the visible length / batch); anything else would silently detach the pool.
        if pool is None:
            raise RuntimeError('cache assignment before initialization')
        self._flush()
        if view.untyped_storage().data_ptr() != pool.untyped_storage().data_ptr():
            raise RuntimeError('use batch_select_indices for row remap; external KV replacement is unsupported')
        self.length = view.shape[-2]
        if self._table() is None:
            self.batch_size = view.shape[0]

    # ---- allocation ----------------------------------------------------------
    def _chunk(self):
        owner = self.owner
        return owner.chunk_size if owner is not None else 256

    def _capacity_for(self, needed):
        chunk = self._chunk()
        return max(self.capacity, -(-needed // chunk) * chunk)

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        self.batch_size = key_states.shape[0]
        owner = self.owner
        self.batch_capacity = max(self.batch_size, owner.batch_capacity if owner is not None else 0)
        self.capacity = self._capacity_for(key_states.shape[-2])
        shape = (self.batch_capacity, key_states.shape[1], self.capacity, key_states.shape[-1])
        self.key_pool = torch.empty(shape, dtype=key_states.dtype, device=key_states.device)
        self.value_pool = torch.empty(shape, dtype=value_states.dtype, device=value_states.device)
        self.stats['pool_allocations'] += 1
        self.is_initialized = True

    def _grow(self, needed, batch_needed=None):
        """Replace the pools when `needed` positions or `batch_needed` rows do not fit.

        Capacity at least doubles (rounded up to the chunk); the live history
        [:batch_size, :, :length] is copied into the new pools.
        """
        batch_needed = self.batch_size if batch_needed is None else batch_needed
        if needed <= self.capacity and batch_needed <= self.batch_capacity:
            return
        self._flush()
        capacity = self._capacity_for(max(needed, 2 * self.capacity)) if needed > self.capacity else self.capacity
        rows = max(batch_needed, self.batch_capacity)
        shape = (rows, self.key_pool.shape[1], capacity, self.key_pool.shape[-1])
        old_keys, old_values = self.keys, self.values
        if self._table() is not None:  # rows are scattered: keep every row in place
            old_keys = self.key_pool[:, :, :self.length]
            old_values = self.value_pool[:, :, :self.length]
        keys = torch.empty(shape, dtype=self.key_pool.dtype, device=self.key_pool.device)
        values = torch.empty(shape, dtype=self.value_pool.dtype, device=self.value_pool.device)
        if self.length and old_keys.shape[0]:
            _ops.append_rows([keys], [values], [old_keys], [old_values], 0)
        self.stats['pool_allocations'] += 1
        self.stats['full_kv_reallocations'] += 1
        if self.length:
            self.stats['full_history_copies'] += 1
            self.stats['full_history_copy_bytes'] += (old_keys.numel() * old_keys.element_size() +
                                                      old_values.numel() * old_values.element_size())
        self.key_pool, self.value_pool = keys, values
        self.capacity, self.batch_capacity = capacity, rows
        owner = self.owner
        if owner is not None and owner.uses_row_table:
            owner._fit_rows(rows)

    # ---- append ----------------------------------------------------------------
    def _prepare_append(self, key_states, value_states):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if key_states.shape[0] != self.batch_size:
            raise ValueError('KV batch differs from live request count')
        end = self.length + key_states.shape[-2]
        self._grow(end)
        if key_states.dtype != self.key_pool.dtype:
            key_states = key_states.to(self.key_pool.dtype)
        if value_states.dtype != self.value_pool.dtype:
            value_states = value_states.to(self.value_pool.dtype)
        return key_states, value_states, end

    def update(self, key_states, value_states, *args, **kwargs):
        self._flush()
        key_states, value_states, end = self._prepare_append(key_states, value_states)
        if self._fusable(key_states, value_states):
            # the rows are stored by the verify attention that reads these views
            # (tree_attention.tree_verify_attention); the views carry the pending append
            self._pending = (key_states, value_states, self.length)
            self.length = end
            keys, values = self._view(self.key_pool), self._view(self.value_pool)
            keys._speckv_pending = values._speckv_pending = (self, self._pending)
            return keys, values
        _ops.append_rows([self.key_pool], [self.value_pool], [key_states], [value_states], self.length,
                         row_table=self._table())
        self.length = end
        return self.keys, self.values

    def update_attend(self, query, key_states, value_states, visibility, scale, out=None):
        """``update(key_states, value_states)`` and the tree-verify attention of ``query`` over
        the updated cache in one launch (speckv_tree_attention_bits_append): the new rows are
        attended straight from ``key_states`` / ``value_states`` and stored into the pools by
        the same kernel. ``visibility`` carries ``bits`` / ``first_col`` over the
        ``length + rows`` columns (``PackedTree.visibility``); returns the attention output
        (batch, rows, q_heads, head_dim). Table-free caches only."""
        if self._table() is not None:
            raise ValueError('the fused append needs a cache without a row table')
        self._flush()
        key_states, value_states, end = self._prepare_append(key_states, value_states)
        rows = self.batch_size
        out = _ops.tree_attention_bits_append(query, self.key_pool[:rows], self.value_pool[:rows], self.length,
                                              key_states, value_states, visibility.bits, visibility.first_col, scale,
                                              out=out)
        self.length = end
        return out

    def get_seq_length(self):
        return self.length

    def get_max_cache_shape(self):
        return self.capacity

    def get_max_length(self):
        return self.capacity

    def get_mask_sizes(self, query_length):
        return self.length + query_length, 0

    def crop(self, length):
        self._flush()
        target = length if length >= 0 else self.length + length
        self.length = max(0, min(self.length, target))

    def reset(self):
        self._pending = None
        self.length = 0

    # ---- remap / release -------------------------------------------------------
    def _count_select(self, new_batch):
        self.stats['row_compactions'] += 1
        moved = new_batch * self.key_pool.shape[1] * self.length * self.key_pool.shape[-1] * (
            self.key_pool.element_size() + self.value_pool.element_size())
        self.stats['row_compaction_bytes'] += moved
        if moved:
            self.stats['full_history_copies'] += 1
            self.stats['full_history_copy_bytes'] += moved
        self.batch_size = new_batch

    def _remap_scratch(self, new_batch):
        elements = _ops.remap_scratch_elements(new_batch, self.key_pool.shape[1], self.key_pool.shape[-1],
                                               self.length, self.key_pool.element_size())
        if not elements:
            return None
        owner = self.owner
        key = ('cuda_live', self.key_pool.dtype, self.key_pool.device)
        scratch = owner._scratch.get(key) if owner is not None else None
        if scratch is None or scratch.numel() < elements:
            scratch = torch.empty(1 << max(0, (elements - 1).bit_length()), dtype=self.key_pool.dtype,
                                  device=self.key_pool.device)
            if owner is not None:
                owner._scratch[key] = scratch
        return scratch

    def batch_select_indices(self, indices):
        if self._table() is not None:
            raise RuntimeError('with a row table, remap rows through the cache (OPDStaticCache.batch_select_indices)')
        new_batch = indices.numel()
        self._flush()
        self._grow(self.length, new_batch)
        _ops.remap_rows([self.key_pool], [self.value_pool], indices, self.length, self._remap_scratch(new_batch))
        self._count_select(new_batch)

    def batch_repeat_interleave(self, repeats):
        if repeats < 1:
            raise ValueError('positive repeats required')
        if repeats != 1:
            self.batch_select_indices(_repeat_indices(self.batch_size, repeats, self.key_pool.device))

    def _count_swap(self, new_batch, count):
        moved = count * self.key_pool.shape[1] * self.length * self.key_pool.shape[-1] * (
            self.key_pool.element_size() + self.value_pool.element_size())
        self.stats['row_compactions'] += 1
        self.stats['row_compaction_bytes'] += moved
        self.stats['full_history_copy_bytes'] += moved
        if moved:
            self.stats['full_history_copies'] += 1
        self.batch_size = new_batch

    def swap_remove(self, new_batch, sources, destinations):
        """Moves disjoint live tail rows into holes below new_batch; survivors stay put."""
        if self._table() is not None:
            raise RuntimeError('with a row table, release rows through the cache (OPDStaticCache.swap_remove)')
        count = sources.numel()
        self._flush()
        if count and self.length:
            _ops.move_rows([self.key_pool], [self.value_pool], sources, destinations, self.length)
        self._count_swap(new_batch, count)


def _repeat_indices(batch, repeats, device):
    return torch.arange(batch, device=device).repeat_interleave(repeats)


class LayerViews:
    """Sequence of per-layer (keys, values) views as of its creation, each built on
    first access: slicing 2 x layers views up front costs more host time than the
    one append launch that precedes them."""

    __slots__ = ('_items',)

    def __init__(self, layers):
        self._items = [(l.key_pool, l.value_pool, l.batch_size, l.length, l._table()) for l in layers]

    def __len__(self):
        return len(self._items)

    def __getitem__(self, index):
        if isinstance(index, slice):
            return [self[i] for i in range(*index.indices(len(self._items)))]
        k, v, b, n, table = self._items[index]
        if table is None:
            return k[:b, :, :n, :], v[:b, :, :n, :]
        k, v = k[:, :, :n, :], v[:, :, :n, :]
        k._speckv_rows = v._speckv_rows = table
        return k, v

    def __iter__(self):
        for i in range(len(self._items)):
            yield self[i]


def _uniform(layers):
    """True when every layer's pools share shape and dtype (one launch can cover them)."""
    first = layers[0]
    return all(layer.key_pool is not None and layer.key_pool.shape == first.key_pool.shape and
               layer.key_pool.dtype == first.key_pool.dtype and layer.value_pool.dtype == first.key_pool.dtype and
               layer.length == first.length and layer.batch_size == first.batch_size for layer in layers)


class OPDStaticCache(Cache):
    """HF ``Cache`` whose layers are StaticAppendLayer pools kept across rollouts.

    ``fuse_append=True`` (no reference counterpart): ``update`` leaves a layer's new rows
    out of the pools and tags the views it returns; the verify attention that reads them
    (``tree_attention.tree_verify_attention``, registered as 'speckv_tree') then attends
    the rows from the projection and stores them in the same launch
    (speckv_tree_attention_bits_append). Every other use of the cache stores pending rows
    first (``flush``). The flag may be switched at any time (e.g. on only for the verify
    forward); a model whose attention is not this package's must not read views of a
    cache with pending rows without calling ``flush()`` first. Until they are stored the
    cache holds references to the ``key_states`` / ``value_states`` given to ``update``:
    they must not be modified in place before the attention (or ``flush``) runs, and it
    should run on the stream that produced them.
    """

    def __init__(self, capacity=256, *, batch_capacity=0, chunk_size=256, row_table=False, fuse_append=False):
        if capacity < 1 or chunk_size < 1 or batch_capacity < 0:
            raise ValueError('positive KV capacity/chunk and nonnegative batch capacity required')
        self.uses_row_table = bool(row_table)
        self.fuse_append = bool(fuse_append)
        # host copy of the table: a permutation of the pool rows, live sequences first
        # (entry b < batch is sequence b's row), the rows free for admission after them
        self._rows = []
        self._rows_dev = None
        try:
            super().__init__(layers=[])
        except TypeError:
            super().__init__()
            self.layers = []
        self.capacity, self.batch_capacity, self.chunk_size = capacity, batch_capacity, chunk_size
        self._scratch = {}
        self.kv_rows_moved = 0

    # ---- row table -----------------------------------------------------------
    def _fit_rows(self, rows):
        """Extends the table to `rows` pool rows (the new rows are free)."""
        if self._rows and rows > len(self._rows):
            self._rows.extend(range(len(self._rows), rows))
            self._upload_rows()

    def _reset_rows(self, rows):
        self._rows = list(range(rows))
        self._upload_rows()

    def _upload_rows(self):
        layer = next((l for l in self.layers if l.key_pool is not None), None)
        if layer is None or not self._rows:
            return
        staged = torch.tensor(self._rows, dtype=torch.long).pin_memory()
        if self._rows_dev is None or self._rows_dev.numel() < len(self._rows) or \
                self._rows_dev.device != layer.key_pool.device:
            self._rows_dev = torch.empty(max(len(self._rows), layer.batch_capacity), dtype=torch.long,
                                         device=layer.key_pool.device)
        self._rows_dev[:len(self._rows)].copy_(staged, non_blocking=True)

    def _device_rows(self, batch):
        if not self._rows and batch:
            first = next((l for l in self.layers if l.key_pool is not None), None)
            if first is None:
                return None
            self._reset_rows(first.batch_capacity)
        if self._rows_dev is None or len(self._rows) < batch:
            raise RuntimeError('row table shorter than the live batch')
        return self._rows_dev[:batch]

    @property
    def row_table(self):
        """Pool row of each live sequence (host list), or None without a row table."""
        if not self.uses_row_table or not self.layers:
            return None
        return list(self._rows[:self.layers[0].batch_size])

    def flush(self):
        """Stores every layer's rows whose append was left to the attention (fuse_append)."""
        for layer in self.layers:
            layer._flush()

    # ---- rollout lifetime ------------------------------------------------------
    def begin_rollout(self, batch, batch_capacity):
        for layer in self.layers:
            layer._pending = None  # the lengths restart at 0: rows of the last rollout are dropped
        self.batch_capacity = max(self.batch_capacity, batch_capacity)
        self.kv_rows_moved = 0
        for layer in self.layers:
            layer.length = 0
            layer.batch_size = batch
            for key in layer.stats:
                layer.stats[key] = 0
        if self.uses_row_table and self.layers and self.layers[0].key_pool is not None:
            self._reset_rows(self.layers[0].batch_capacity)

    def end_rollout(self, max_retained_tokens=0):
        for layer in self.layers:
            layer._pending = None
            layer.length = layer.batch_size = 0
        if max_retained_tokens and any(layer.capacity > max_retained_tokens for layer in self.layers):
            self.layers.clear()
            self._scratch.clear()
            self._rows, self._rows_dev = [], None  # the next pools start with a fresh table

    def scratch(self, pool, shape):
        """Reusable (rows, heads, chunk, dim) tile buffer keyed by device/dtype/geometry."""
        rows = shape[0]
        key = (pool.device, pool.dtype, shape[1], shape[-1])
        buf = self._scratch.get(key)
        if buf is None or any(a < b for a, b in zip(buf.shape, shape)):
            full = (max(shape[0], self.batch_capacity), shape[1], self.chunk_size, shape[-1])
            buf = torch.empty(full, dtype=pool.dtype, device=pool.device)
            self._scratch[key] = buf
        return buf[:rows]

    # ---- HF cache protocol -----------------------------------------------------
    def _layer(self, layer_idx):
        while len(self.layers) <= layer_idx:
            self.layers.append(StaticAppendLayer(self.capacity, self))
        return self.layers[layer_idx]

    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        return self._layer(layer_idx).update(key_states, value_states)

    def update_attend(self, query, key_states, value_states, layer_idx, visibility, scale, out=None):
        """``update(key_states, value_states, layer_idx)`` fused with the verify attention that
        reads the layer right after it (StaticAppendLayer.update_attend); returns its output."""
        return self._layer(layer_idx).update_attend(query, key_states, value_states, visibility, scale, out=out)

    def get_seq_length(self, layer_idx=0):
        return self.layers[layer_idx].length if layer_idx < len(self.layers) else 0

    def get_mask_sizes(self, query_length, layer_idx=0):
        return self.get_seq_length(layer_idx) + query_length, 0

    def get_max_cache_shape(self, layer_idx=0):
        return self.layers[layer_idx].capacity if layer_idx < len(self.layers) else self.capacity

    def crop(self, length):
        for layer in self.layers:
            layer.crop(length)

    def __getitem__(self, index):
        return self.layers[index].keys, self.layers[index].values

    def __iter__(self):
        for layer in self.layers:
            yield layer.keys, layer.values

    def __len__(self):
        return len(self.layers)

    def __bool__(self):
        return bool(self.layers) and self.get_seq_length() > 0

    # ---- cache-wide row movement (one launch for all layers) --------------------
    def _select_all(self, indices):
        layers = self.layers
        if not layers:
            return
        self.flush()
        if self.uses_row_table and layers[0].key_pool is not None:
            # through the table to pool rows, written to rows [0, new_batch): the table is identity after
            indices = self._device_rows(layers[0].batch_size)[indices]
        new_batch = indices.numel()
        for layer in layers:
            layer._grow(layer.length, new_batch)
        if _uniform(layers):
            first = layers[0]
            _ops.remap_rows([l.key_pool for l in layers], [l.value_pool for l in layers], indices, first.length,
                            first._remap_scratch(new_batch))
            for layer in layers:
                layer._count_select(new_batch)
        else:
            for layer in layers:
                _ops.remap_rows([layer.key_pool], [layer.value_pool], indices, layer.length,
                                layer._remap_scratch(new_batch))
                layer._count_select(new_batch)
        if self.uses_row_table:
            self._reset_rows(layers[0].batch_capacity)

    def batch_repeat_interleave(self, repeats):
        if repeats < 1:
            raise ValueError('positive repeats required')
        if repeats != 1 and self.layers:
            first = self.layers[0]
            self._select_all(_repeat_indices(first.batch_size, repeats, first.key_pool.device))
        # Prefill repeat is excluded from kv_rows_moved, as in the reference.

    def batch_select_indices(self, indices):
        self._select_all(indices)
        self.kv_rows_moved += indices.numel()

    def swap_remove(self, new_batch, sources, destinations):
        self.flush()
        layers = self.layers
        if self.uses_row_table and layers and layers[0].key_pool is not None:
            self._swap_remove_rows(new_batch, sources, destinations)
            return
        count = sources.numel()
        if layers and count:
            live = [l for l in layers if l.length]
            if live and _uniform(live):
                _ops.move_rows([l.key_pool for l in live], [l.value_pool for l in live], sources, destinations,
                               live[0].length)
            else:
                for layer in live:
                    _ops.move_rows([layer.key_pool], [layer.value_pool], sources, destinations, layer.length)
        for layer in layers:
            layer._count_swap(new_batch, count)
        self.kv_rows_moved += count

    def _swap_remove_rows(self, new_batch, sources, destinations):
        """swap_remove through the row table: sequence d takes sequence s's pool row for each
        (s, d) pair and the released rows join the free tail; no KV byte moves."""
        sources = sources.tolist() if isinstance(sources, torch.Tensor) else list(sources)
        destinations = destinations.tolist() if isinstance(destinations, torch.Tensor) else list(destinations)
        self._device_rows(self.layers[0].batch_size)  # table initialised
        self._rows = release_rows(self._rows, new_batch, sources, destinations)
        self._upload_rows()
        for layer in self.layers:
            layer.stats['row_compactions'] += 1
            layer.batch_size = new_batch

    # ---- B200 additions ----------------------------------------------------------
    def admit(self, key_states, value_states):
        """Writes the prefixes of k new sequences into rows [batch, batch + k) of every layer.

        ``key_states[l]`` / ``value_states[l]`` are (k, heads, length, dim), already
        left-padded to the cache's shared length; all layers are written in one launch
        and the live batch grows by k. Refills the rows ``swap_remove`` released; the
        reference has no admission step of its own (its rollouts start full).
        """
        layers = self.layers[:len(key_states)]
        if not layers or len(key_states) != len(value_states) or len(layers) != len(self.layers):
            raise ValueError('one key and one value tensor per layer required')
        self.flush()
        count = key_states[0].shape[0]
        length = layers[0].length
        if any(l.length != length or l.batch_size != layers[0].batch_size for l in layers):
            raise ValueError('admission needs every layer at one length and batch size')
        if key_states[0].shape[-2] != length:
            raise ValueError('admitted prefixes must be left-padded to the cache length')
        if count == 0:
            return
        start = layers[0].batch_size
        for layer in layers:
            layer._grow(max(length, 1), batch_needed=start + count)
        if self.uses_row_table:
            # the new sequences take the free rows at the table's positions [start, start + count)
            table = self._device_rows(start + count)[start:]
            if length:
                _ops.append_rows([l.key_pool for l in layers], [l.value_pool for l in layers], list(key_states),
                                 list(value_states), 0, row_table=table)
        elif length:
            _ops.append_rows([l.key_pool[start:] for l in layers], [l.value_pool[start:] for l in layers],
                             list(key_states), list(value_states), 0)
        for layer in layers:
            layer.batch_size = start + count

    def update_layers(self, key_states, value_states, deferred=False, commit=None):
        """Appends key_states[l] / value_states[l] to layer l for every l in one launch.

        Same result as calling ``update(key_states[l], value_states[l], l)`` for each
        layer; returns the per-layer (keys, values) views. With ``deferred=True`` the
        checks, growth and argument marshalling happen now and a callable is returned
        that issues the launch and returns the views; call it before any other change
        to this cache (it lets a caller overlap this host work with a running kernel).

        ``commit = (chosen, past, extension, width)``: the previous round's accepted-suffix
        compaction, left out of its commit (``commit_scheduled(..., compact=False)``), is
        done by the same launch before the new rows land (speckv_append_commit_rows): the
        same cache as ``compact_suffix_inplace`` on every layer followed by this append.
        """
        if len(key_states) != len(value_states):
            raise ValueError('one key and one value tensor per layer required')
        self.flush()
        prepared = []
        for idx, (k, v) in enumerate(zip(key_states, value_states)):
            prepared.append(self._layer(idx)._prepare_append(k, v))
        layers = self.layers[:len(prepared)]
        table = layers[0]._table() if layers else None
        if commit is not None and (table is not None or not _uniform(layers)):
            raise ValueError('a folded commit needs uniform, table-free layers')
        if _uniform(layers):
            launches = [_ops.append_rows([l.key_pool for l in layers], [l.value_pool for l in layers],
                                         [p[0] for p in prepared], [p[1] for p in prepared], layers[0].length,
                                         launch=False, row_table=table, commit=commit)]
        else:
            launches = [_ops.append_rows([layer.key_pool], [layer.value_pool], [k], [v], layer.length, launch=False,
                                         row_table=table)
                        for layer, (k, v, _) in zip(layers, prepared)]

        def launch():
            for go in launches:
                go()
            for layer, (_, _, end) in zip(layers, prepared):
                layer.length = end
            return LayerViews(layers)

        return launch if deferred else launch()

    def commit_accepted(self, chosen, past, extension):
        """Accepted-path commit of every layer in one launch, then crop.

        Equivalent to ``compact_suffix_inplace`` on each layer's views followed by
        ``crop(past + chosen.shape[1])`` (helper/opd_generate.py:632-643).
        """
        width = chosen.shape[1]
        self.flush()
        layers = self.layers
        if layers and extension != width:
            table = layers[0]._table()
            if _uniform(layers):
                first = layers[0]
                _ops.compact_suffix([l.key_pool for l in layers], [l.value_pool for l in layers],
                                    first.batch_size, first.length, chosen, past, extension, width, row_table=table)
            else:
                for layer in layers:
                    _ops.compact_suffix([layer.key_pool], [layer.value_pool], layer.batch_size, layer.length,
                                        chosen, past, extension, width, row_table=table)
        self.crop(past + width)

    def commit_scheduled(self, chosen, past, packet, newly_padded=None, positions=None, past_positions=None,
                         pad_rows=None, owners=None, pad_live=None, deferred=False, compact=True):
        """``commit_accepted`` with width and extension read from the device packet.

        ``chosen`` (and the position operands) are the full-width schedule
        outputs; the launch needs no host value of the round, so it can be
        enqueued before the packet is read back. The caller crops the cache to
        ``past + width`` once it knows the width. With ``deferred=True`` the
        launch is prepared now (the operands' contents may still be written by
        kernels enqueued later) and a callable that issues it is returned. With
        ``compact=False`` only positions / padding are updated: the compaction is then
        the caller's, e.g. folded into the next round's ``update_layers(commit=...)``.
        """
        self.flush()
        layers = [l for l in self.layers if l.key_pool is not None] if compact else []
        pos = dict(newly_padded=newly_padded, positions=positions, past_positions=past_positions,
                   pad_rows=pad_rows, owners=owners, pad_live=pad_live)
        if not layers:
            launches = [_ops.commit_round([], [], packet.shape[0], 0, chosen, past, packet, **pos, launch=False)]
        elif _uniform(layers):
            first = layers[0]
            launches = [_ops.commit_round([l.key_pool for l in layers], [l.value_pool for l in layers],
                                          first.batch_size, first.length, chosen, past, packet, **pos, launch=False,
                                          row_table=first._table())]
        else:
            table = layers[0]._table()
            launches = [_ops.commit_round([layer.key_pool], [layer.value_pool], layer.batch_size, layer.length,
                                          chosen, past, packet, **(pos if i == 0 else {}), launch=False,
                                          row_table=table)
                        for i, layer in enumerate(layers)]

        def launch():
            for go in launches:
                go()

        return launch if deferred else launch()

    def statistics(self):
        totals = {name: sum(layer.stats[name] for layer in self.layers) for name in LAYER_COUNTERS}
        totals['kv_cache_bytes'] = sum(pool.numel() * pool.element_size() for layer in self.layers
                                       for pool in (layer.key_pool, layer.value_pool) if pool is not None)
        totals['kv_compaction_workspace_bytes'] = sum(x.numel() * x.element_size() for x in self._scratch.values())
        totals['kv_rows_moved'] = self.kv_rows_moved
        totals['kv_history_copy_bytes'] = totals['full_history_copy_bytes']
        return totals


def release_rows(rows, new_batch, sources, destinations):
    """Row-table form of swap_remove: `rows` is the table (pool row of each sequence, then the
    free rows). Sequence d < new_batch takes the pool row of sequence s >= new_batch for each
    (s, d) pair, the other sequences below new_batch keep theirs, and every pool row no
    longer referenced joins the free tail. Returns the new table (a permutation of `rows`)."""
    if len(sources) != len(destinations):
        raise ValueError('swap_remove needs one destination per source')
    live = list(rows[:new_batch])
    for src, dst in zip(sources, destinations):
        if not (0 <= dst < new_batch <= src < len(rows)):
            raise ValueError('swap_remove moves rows from the tail into holes below the new batch')
        live[dst] = rows[src]
    kept = set(live)
    return live + [r for r in rows if r not in kept]


def swap_remove_plan(finished):
    """Host plan for releasing finished rows: (keep, tail sources, hole destinations).

    Holes are finished rows below the new batch size; they are filled, in order,
    from the live rows above it taken from the end.
    """
    new_batch = len(finished) - sum(bool(x) for x in finished)
    holes = [i for i in range(new_batch) if finished[i]]
    tail = [i for i in range(len(finished) - 1, new_batch - 1, -1) if not finished[i]]
    keep = list(range(new_batch))
    for destination, source in zip(holes, tail):
        keep[destination] = source
    return keep, tail, holes


def persistent_cache(model, name, batch, responses, device, dtype):
    """Returns the model-owned cache `name`, re-created when device/dtype change."""
    cache = getattr(model, name, None)
    signature = (str(device), dtype)
    if cache is None or getattr(cache, 'runtime_signature', None) != signature:
        cache = OPDStaticCache(256, batch_capacity=batch * responses)
        cache.runtime_signature = signature
        setattr(model, name, cache)
    cache.begin_rollout(batch, batch * responses)
    return cache
