"""Drop-in for helper/opd_attention_kernels.py: the causal mask of the draft model's
attention as one libspeckv launch (``speckv_causal_mask``).

``causal_mask(out, past, padding=None)`` fills ``out`` (batch, 1, query, past + query)
with 0 where column c <= past + row and the column is not padding, and with
``torch.finfo(out.dtype).min`` elsewhere (helper/opd_attention_kernels.py:7-22).
"""
from . import _ops


def causal_mask(out, past, padding=None):
    _ops.causal_mask(out, past, padding)
