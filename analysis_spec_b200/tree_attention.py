"""Tree-verify GQA attention as a transformers ``AttentionInterface`` function.

Replaces ``sdpa_attention_forward`` (transformers
``integrations/sdpa_attention.py:40-104``) on the verify forward of
``Qwen2Attention`` (``models/qwen2/modeling_qwen2.py:206-240``). With a 4-D
mask, transformers' SDPA path disables its GQA mode and materialises
``repeat_kv`` copies of K/V for every query head (``sdpa_attention.py:28-37,
56-62``); this kernel reads each KV head of the strided cache views once for
all query heads that share it and applies the additive mask in-kernel. A dense mask
holding only 0 and the dtype's lowest value (transformers' and the reference's masks) is
turned into visibility bits once per forward and every layer runs the bits kernel.

Use: ``register()`` then ``model.config._attn_implementation = 'speckv_tree'``
(or call ``tree_verify_attention`` directly).
"""
import torch

from . import _ops

ATTENTION_NAME = 'speckv_tree'


class DenseMaskVisibility:
    """Visibility bits of a dense 0 / lowest-value mask, built once per mask tensor."""

    def __init__(self, bits, first_col):
        self.bits = bits
        self.first_col = first_col


def dense_mask_visibility(attention_mask, mask, batch, rows, kv_len):
    """Bits for the additive `mask` (`attention_mask` cut to kv_len columns), cached on
    `attention_mask` per (shape, in-place version): every layer of a forward gets the same
    mask tensor, so the conversion (one launch and one 4-byte read-back) runs once per
    forward. Returns None when the mask holds values other than 0 and the dtype's lowest
    value / -inf (such a mask keeps the dense kernel)."""
    key = (kv_len, rows, batch, attention_mask._version)
    cached = getattr(attention_mask, '_speckv_dense_bits', None)
    if cached is not None and cached[0] == key:
        return cached[1]
    dev = mask.device
    bits = torch.empty((batch, rows, _ops.visibility_words(kv_len)), dtype=torch.int32, device=dev)
    first = torch.empty((batch,), dtype=torch.int32, device=dev)
    flag = torch.empty((1,), dtype=torch.int32, device=dev)
    _ops.mask_bits(mask.expand(batch, 1, rows, kv_len), bits, first, flag)
    vis = None if flag.item() else DenseMaskVisibility(bits, first)
    try:
        attention_mask._speckv_dense_bits = (key, vis)
    except (AttributeError, RuntimeError):
        pass
    return vis


def _pending_rows(key):
    """(layer, (key_states, value_states, position)) when `key` is a view of an
    OPDStaticCache(fuse_append=True) layer whose latest rows are not stored yet, else None."""
    tag = getattr(key, '_speckv_pending', None)
    if tag is None or tag[0]._pending is not tag[1]:
        return None
    return tag


def _bits_attention(query, key, value, bits, first_col, scale, rows_table, pending):
    """The visibility-bits kernel, with the layer's pending rows appended by the same launch
    when the views carry them (speckv_tree_attention_bits_append), else after storing them."""
    if pending is not None:
        layer, (k_new, v_new, position) = pending
        if (k_new.shape[-2] == query.shape[2] and position + k_new.shape[-2] == key.shape[-2] and
                k_new.dtype == query.dtype and rows_table is None):
            batch = key.shape[0]
            out = _ops.tree_attention_bits_append(query, layer.key_pool[:batch], layer.value_pool[:batch], position,
                                                  k_new, v_new, bits, first_col, scale)
            layer._pending = None  # stored by that launch
            return out
        layer._flush()
    return _ops.tree_attention_bits(query, key, value, bits, first_col, scale, row_table=rows_table)


def tree_verify_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None,
                          **kwargs):
    """(module, q (B,Hq,R,D), k/v (B,Hkv,L,D), additive mask (B,1,R,L)) -> (out (B,R,Hq,D), None).

    K/V views of an ``OPDStaticCache(fuse_append=True)`` whose latest rows are still pending
    take the fused append + attention kernel on the visibility-bits path; any other path
    stores the rows first."""
    if dropout:
        raise ValueError('tree_verify_attention is an inference kernel (dropout must be 0)')
    scale = scaling if scaling is not None else query.shape[-1] ** -0.5
    rows_table = getattr(key, '_speckv_rows', None)  # K/V of a row-table cache: every pool row
    pending = _pending_rows(key)
    vis = attention_mask if hasattr(attention_mask, 'first_col') else getattr(attention_mask, '_speckv_visibility',
                                                                            None)
    if vis is not None and key.shape[-2] == vis.past + vis.rows and query.shape[2] == vis.rows:
        return _bits_attention(query, key, value, vis.bits, vis.first_col, scale, rows_table, pending), None
    mask = attention_mask
    if mask is not None and mask.shape[-1] > key.shape[-2]:
        mask = mask[:, :, :, :key.shape[-2]]
    causal = is_causal if is_causal is not None else getattr(module, 'is_causal', True)
    if mask is None and causal and query.shape[2] > 1:
        raise ValueError('tree_verify_attention needs an explicit mask for multi-query causal attention')
    if (mask is not None and mask.dim() == 4 and mask.dtype != torch.bool and query.shape[-1] == 128 and
            query.dtype in (torch.bfloat16, torch.float16)):
        batch, rows, kv_len = query.shape[0], query.shape[2], key.shape[-2]
        dense = dense_mask_visibility(attention_mask, mask, batch, rows, kv_len)
        if dense is not None:
            return _bits_attention(query, key, value, dense.bits, dense.first_col, scale, rows_table, pending), None
    if pending is not None:  # the dense-mask and CUDA-core kernels read the rows from the pools
        pending[0]._flush()
    if rows_table is not None:
        raise ValueError('K/V of a row-table cache need a 0 / lowest-valued mask (the visibility-bits kernel), '
                         'head dim 128 and bf16 / fp16')
    return _ops.tree_attention(query, key, value, mask, scale), None


def register(name=ATTENTION_NAME):
    """Registers the kernel with transformers' global attention (and mask) interfaces."""
    from transformers import AttentionInterface
    AttentionInterface.register(name, tree_verify_attention)
    try:
        from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, sdpa_mask
        ALL_MASK_ATTENTION_FUNCTIONS.register(name, sdpa_mask)
    except ImportError:
        pass
    return name
