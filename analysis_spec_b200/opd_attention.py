"""Drop-in for helper/opd_attention.py: capacity-reused mask / position buffers of the
draft model's attention, plus the draft expansion mask of one tree step.

``AttentionWorkspace`` keeps the reference's buffer policy (one flat pool per (name,
dtype), grown to a power of two of at least 256 elements, ``allocations`` counting the
growths; helper/opd_attention.py:5-47); its CUDA causal mask is one libspeckv launch.
``expansion_mask`` replaces the zero / fill / scatter / padding sequence of
helper/opd_generate.py:143-162 with one launch.

Both masks are returned carrying their visibility bits (written by the same launch), so
the draft attention (``draft_attention.draft_sdpa``) runs the bits tensor-core kernel
without reading the dense mask or converting it. The bits buffers are private to this
module and not counted in ``allocations`` / ``memory_bytes()``, which follow the
reference's accounting of the mask buffers.
"""
import torch

from . import _ops, opd_attention_kernels
from .tree_attention import DenseMaskVisibility


def _attach_visibility(mask, bits, first_col):
    batch, _, query, columns = mask.shape
    mask._speckv_dense_bits = ((columns, query, batch, mask._version), DenseMaskVisibility(bits, first_col))
    return mask


def _visibility_buffers(store, name, batch, query, columns, device):
    words = _ops.visibility_words(columns)
    count = batch * query * words
    key = (name, 'bits')
    pool = store.get(key)
    if pool is None or pool.numel() < count + batch:
        pool = torch.empty(_capacity(count + batch), dtype=torch.int32, device=device)
        store[key] = pool
    return pool[:count].view(batch, query, words), pool[count:count + batch]


def _capacity(count):
    return 1 << max(8, (max(1, count) - 1).bit_length())


class AttentionWorkspace:
    def __init__(self, device):
        self.device = torch.device(device)
        self.buffers = {}
        self.allocations = 0

    def buffer(self, name, shape, dtype):
        count = 1
        for size in shape:
            count *= size
        key = (name, dtype)
        pool = self.buffers.get(key)
        if pool is None or pool.numel() < count:
            pool = torch.empty(_capacity(count), device=self.device, dtype=dtype)
            self.buffers[key] = pool
            self.allocations += 1
        return pool[:count].view(shape)

    def positions(self, name, past, width):
        out = self.buffer(name, (width,), torch.long)
        key = ('ramp', torch.long)
        ramp = self.buffers.get(key)
        if ramp is None or ramp.numel() < past + width:
            ramp = torch.arange(_capacity(past + width), device=self.device)
            self.buffers[key] = ramp
            self.allocations += 1
        out.copy_(ramp[past:past + width])
        return out

    def causal(self, name, past, query, batch, dtype, padding=None):
        """Causal mask (batch, 1, query, past + query) in the workspace buffer ``name``: one
        libspeckv launch; a workspace on a non-CUDA device raises (no CPU path)."""
        out = self.buffer(name, (batch, 1, query, past + query), dtype)
        if not hasattr(self, '_visibility'):
            self._visibility = {}
        bits, first = _visibility_buffers(self._visibility, name, batch, query, past + query, out.device)
        _ops.causal_mask(out, past, padding, bits, first)
        return _attach_visibility(out, bits, first)

    def memory_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.buffers.values())


def expansion_mask(mask, init_length, seen, padding=None):
    """Draft expansion mask in ``mask`` (batch, 1, query, columns): row r of sequence b sees
    columns below ``init_length`` and column ``seen[b, r, 0]``; padding columns are off.
    ``padding`` is a bool (batch, >= columns) tensor, int64 (n, 2) pairs (b, column), or
    per-sequence lists of padded columns (turned into pairs), the forms of
    helper/opd_generate.py:148-162. Returns ``mask``."""
    if padding is not None and not isinstance(padding, torch.Tensor):
        pairs = [[b, int(c)] for b, cols in enumerate(padding) for c in cols]
        padding = torch.tensor(pairs, device=mask.device, dtype=torch.long) if pairs else None
    pad = padding if isinstance(padding, torch.Tensor) and padding.dtype == torch.bool else None
    batch, _, query, columns = mask.shape
    bits, first = _visibility_buffers({}, None, batch, query, columns, mask.device)
    _ops.expansion_mask(mask, init_length, seen, pad, bits, first)
    _attach_visibility(mask, bits, first)  # a pairs-form fill below advances the version: bits dropped
    if isinstance(padding, torch.Tensor) and padding.dtype != torch.bool and padding.numel():
        mask[padding[:, 0], 0, :, padding[:, 1]] = torch.finfo(mask.dtype).min
    return mask
