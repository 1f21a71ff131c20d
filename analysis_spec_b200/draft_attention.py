"""Attention of the draft model (``CachedDraftAttention.forward``,
helper/fastgrpo_model.py:58-69): ``repeat_kv`` of the cached K/V for every query head
followed by ``F.scaled_dot_product_attention`` with the draft's additive mask (the causal
mask of ``AttentionWorkspace.causal`` on the draft commit, the expansion mask of each
draft step) is one libspeckv attention launch that reads each KV head of the cache views
once for the query heads sharing it. Masks built by ``opd_attention`` carry their
visibility bits, and then the bits kernel runs without reading the dense mask; other
0 / lowest-valued masks are converted once (``tree_attention.dense_mask_visibility``).

``draft_sdpa`` returns what the reference's SDPA call returns, shape (batch, heads,
q_len, head_dim), as a view of a (batch, q_len, heads, head_dim) contiguous result, so
the caller's following ``attn_output.transpose(1, 2).contiguous()`` copies nothing.
"""
import torch

from . import _ops
from .tree_attention import dense_mask_visibility


def draft_sdpa(query_states, key_states, value_states, attention_mask, num_key_value_groups, dropout_p=0.0,
               scale=None):
    """query (B, Hq, R, D); key / value (B, Hkv, L, D) cache views (any strides with unit
    stride on D); attention_mask additive (B, 1, R, >= L) or bool or None (None only for
    R == 1: no causal structure is implied, as SDPA with is_causal=False).
    Hq == Hkv * num_key_value_groups. Returns (B, Hq, R, D)."""
    if dropout_p:
        raise ValueError('draft_sdpa is the rollout (inference) attention: dropout_p must be 0')
    pending = getattr(key_states, '_speckv_pending', None)
    if pending is not None:  # rows an OPDStaticCache(fuse_append=True) left to a verify attention
        pending[0]._flush()
    if query_states.shape[1] != key_states.shape[1] * num_key_value_groups:
        raise ValueError(f'draft_sdpa: {query_states.shape[1]} query heads for {key_states.shape[1]} KV heads '
                         f'x {num_key_value_groups} groups')
    if attention_mask is None and query_states.shape[2] > 1:
        raise ValueError('draft_sdpa: a multi-query draft forward needs its attention mask')
    mask = attention_mask
    if mask is not None and mask.shape[-1] > key_states.shape[-2]:
        mask = mask[..., :key_states.shape[-2]]
    scale = scale if scale is not None else query_states.shape[-1] ** -0.5
    if (mask is not None and mask.dim() == 4 and mask.dtype != torch.bool and query_states.shape[-1] == 128 and
            query_states.dtype in (torch.bfloat16, torch.float16)):
        batch, rows, kv_len = query_states.shape[0], query_states.shape[2], key_states.shape[-2]
        vis = dense_mask_visibility(attention_mask, mask, batch, rows, kv_len)
        if vis is not None:
            return _ops.tree_attention_bits(query_states, key_states, value_states, vis.bits, vis.first_col,
                                            scale, row_table=getattr(key_states, '_speckv_rows', None)
                                            ).transpose(1, 2)
    if getattr(key_states, '_speckv_rows', None) is not None:
        raise ValueError('K/V of a row-table cache need a 0 / lowest-valued mask, head dim 128 and bf16 / fp16')
    out = _ops.tree_attention(query_states, key_states, value_states, mask, scale)
    return out.transpose(1, 2)
