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


def tree_verify_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None,
                          **kwargs):
    """(module, q (B,Hq,R,D), k/v (B,Hkv,L,D), additive mask (B,1,R,L)) -> (out (B,R,Hq,D), None)."""
    if dropout:
        raise ValueError('tree_verify_attention is an inference kernel (dropout must be 0)')
    scale = scaling if scaling is not None else query.shape[-1] ** -0.5
    rows_table = getattr(key, '_speckv_rows', None)  # K/V of a row-table cache: every pool row
    vis = attention_mask if hasattr(attention_mask, 'first_col') else getattr(attention_mask, '_speckv_visibility',
                                                                            None)
    if vis is not None and key.shape[-2] == vis.past + vis.rows and query.shape[2] == vis.rows:
        return _ops.tree_attention_bits(query, key, value, vis.bits, vis.first_col, scale,
                                        row_table=rows_table), None
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
            return _ops.tree_attention_bits(query, key, value, dense.bits, dense.first_col, scale,
                                            row_table=rows_table), None
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
