"""Drop-in for helper/opd_history.py: contiguous rollout-history pools.

``ContiguousRolloutHistory`` keeps the reference's attributes (``buffers``, ``lengths``,
``capacities``, ``finished``, ``response_count``), growth rule (capacity max(end, 2 x
capacity), never truncating) and errors; its copies are libspeckv launches:

* ``__init__``: the repeated copy of the initial tensors, one launch for all fields
  (helper/opd_history.py:11-22);
* ``append``: every field's ``index_copy_`` into the owner rows in one launch (:24-42);
  a capacity grow copies the used history with the same kernel;
* ``append_accepted``: the verify round's gather of the accepted target features
  (``feature_states_tree.gather``, helper/opd_generate.py:567-571) fused with the
  history append of :572-579; the gathered features, the next draft step's input,
  are written by the same launch;
* ``finalize``: one pack launch per field (:44-67).
"""
import torch

from . import _ops

MAX_FIELDS = 4


def _launch_groups(fields):
    for k in range(0, len(fields), MAX_FIELDS):
        yield fields[k:k + MAX_FIELDS]


class ContiguousRolloutHistory:
    def __init__(self, initial, *, repeats=1, max_length, reserve_tokens=256):
        if repeats < 1 or max_length < 1:
            raise ValueError('positive history repeats and capacity required')
        sizes = {t.shape[0] for t in initial.values()}
        if len(sizes) != 1:
            raise ValueError('history batch sizes differ')
        self.response_count = sizes.pop() * repeats
        self.buffers = {}
        self.lengths = {}
        self.capacities = {}
        self.finished = {}
        self._launches = {}  # packed launch arguments per field layout (see _ops.history_append)
        fields = []
        for name, tensor in initial.items():
            length = tensor.shape[1]
            capacity = max(length, int(max_length))
            pool = tensor.new_empty((self.response_count, capacity, *tensor.shape[2:]))
            fields.append((pool, tensor, None, None, 0, length))
            self.buffers[name] = pool
            self.lengths[name] = length
            self.capacities[name] = capacity
        if fields and self.response_count:
            device = fields[0][0].device
            owners = torch.arange(self.response_count, device=device)
            sources = torch.div(owners, repeats, rounding_mode='floor')
            for group in _launch_groups(fields):
                _ops.history_append(group, owners, self.response_count, self.response_count, src_rows=sources)

    def _grow(self, name, end):
        pool = self.buffers[name]
        start = self.lengths[name]
        capacity = max(end, pool.shape[1] * 2)
        grown = pool.new_empty((self.response_count, capacity, *pool.shape[2:]))
        if start and self.response_count:
            rows = torch.arange(self.response_count, device=pool.device)
            _ops.history_append([(grown, pool, None, None, 0, start)], rows, self.response_count,
                                self.response_count)
        self.buffers[name] = grown
        self.capacities[name] = capacity
        return grown

    def _owners(self, original_rows, owners, device):
        if owners is None:
            owners = torch.as_tensor(original_rows, device=device, dtype=torch.long)
        if owners.dtype != torch.long or not owners.is_contiguous():
            owners = owners.to(torch.long).contiguous()
        return owners

    def append(self, original_rows, chunks, owners=None):
        if set(chunks) != set(self.buffers):
            raise ValueError('history fields differ')
        owners = self._owners(original_rows, owners, next(iter(chunks.values())).device)
        n = len(original_rows)
        fields = []
        for name, chunk in chunks.items():
            pool = self.buffers[name]
            if chunk.shape[0] != n or chunk.shape[2:] != pool.shape[2:] or chunk.dtype != pool.dtype:
                raise ValueError('history chunk shape/dtype changed')
            start = self.lengths[name]
            end = start + chunk.shape[1]
            if end > pool.shape[1]:
                pool = self._grow(name, end)
            fields.append((pool, chunk, None, None, start, chunk.shape[1]))
        for group in _launch_groups(fields):
            _ops.history_append(group, owners, self.response_count, n, cache=self._launches)
        for name, chunk in chunks.items():
            self.lengths[name] += chunk.shape[1]

    def append_accepted(self, original_rows, next_token, feature_tree, feature_index, owners=None,
                        features_out=None):
        """The verify round's history step in one launch: ``generated_ids`` (and ``input_ids``
        when kept) <- ``next_token`` (B, W); ``features`` (when kept) <- ``feature_tree`` (B, T, D)
        at positions ``feature_index`` (B, W) (= chosen_index - past). Returns the gathered
        features (B, W, D) (``features_out`` if given), the same tensor the reference's
        ``feature_states_tree.gather`` produces."""
        names = set(self.buffers)
        if not names <= {'generated_ids', 'input_ids', 'features'} or 'generated_ids' not in names:
            raise ValueError('history fields differ')
        n, width = next_token.shape[0], next_token.shape[1]
        if n != len(original_rows) or feature_index.shape != next_token.shape or feature_tree.shape[0] != n:
            raise ValueError('history chunk shape/dtype changed')
        owners = self._owners(original_rows, owners, next_token.device)
        if features_out is None:
            features_out = feature_tree.new_empty((n, width, *feature_tree.shape[2:]))
        index = feature_index if feature_index.dtype == torch.long else feature_index.long()
        fields = []
        chunks = {'generated_ids': next_token, 'input_ids': next_token}
        for name in ('generated_ids', 'input_ids'):
            if name in names:
                pool = self.buffers[name]
                chunk = chunks[name]
                if chunk.shape[2:] != pool.shape[2:] or chunk.dtype != pool.dtype:
                    raise ValueError('history chunk shape/dtype changed')
                start = self.lengths[name]
                if start + width > pool.shape[1]:
                    pool = self._grow(name, start + width)
                fields.append((pool, chunk, None, None, start, width))
        pool = None
        start = 0
        if 'features' in names:
            pool = self.buffers['features']
            if feature_tree.shape[2:] != pool.shape[2:] or feature_tree.dtype != pool.dtype:
                raise ValueError('history chunk shape/dtype changed')
            start = self.lengths['features']
            if start + width > pool.shape[1]:
                pool = self._grow('features', start + width)
        fields.append((pool, feature_tree, index, features_out, start, width))
        _ops.history_append(fields, owners, self.response_count, n, cache=self._launches)
        for name in names:
            self.lengths[name] += width
        return features_out

    def mark_finished(self, row):
        if row in self.finished:
            raise ValueError('history row finished twice')
        self.finished[row] = self.lengths.copy()

    def finalize(self):
        """Packs used histories once; output views own only this compact storage."""
        for row in range(self.response_count):
            if row not in self.finished:
                self.mark_finished(row)
        result = [{} for _ in range(self.response_count)]
        for name, pool in self.buffers.items():
            lengths = [self.finished[row][name] for row in range(self.response_count)]
            total = sum(lengths)
            offsets = [0]
            for length in lengths:
                offsets.append(offsets[-1] + length)
            packed = pool.new_empty((total, *pool.shape[2:]))
            if total:
                dev_offsets = torch.tensor(offsets, dtype=torch.long).to(pool.device)
                _ops.history_pack(packed, pool, dev_offsets, self.response_count, max(lengths))
            for row, length in enumerate(lengths):
                result[row][name] = packed[offsets[row]:offsets[row] + length]
        self.buffers.clear()
        return result
