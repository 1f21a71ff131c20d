"""Tree kernel plugin module (pass as ``kernels=``), drop-in for ``helper/tree_kernels.py``.

The reference loads its Triton module with
``importlib.import_module('helper.tree_kernels')`` and hands it to
``PackedTree.attention_mask``, ``trace_verified_path``,
``VerifiedPath.padded_gpu`` and ``schedule``; this module offers the same four
functions backed by libspeckv's CUDA kernels:

  tree_mask          helper/tree_kernels.py:139-155
  trace_path         helper/tree_kernels.py:68-95
  pad_verified_path  helper/tree_kernels.py:97-137 (budget clamped at 0 as the
                     torch branch, helper/tree_verification.py:254-256)
  pad_schedule       helper/tree_kernels.py:7-41

The proposal top-k merge of the reference module is not part of this path.
"""
import torch

from . import _ops


def tree_mask(tree, past_length, mask, pad=None):
    """Additive ancestor mask into ``mask`` (batch, 1, rows, past + rows); optional bool ``pad`` columns."""
    _ops.tree_mask(tree.parents, int(past_length), tree.max_depth + 1, mask, pad)


def trace_path(tree, samples, eos, tokens, indices, contexts, lengths):
    _ops.trace_path(tree.parents, tree.tokens, tree.feedback_contexts, samples, int(eos), tokens, indices, contexts,
                    lengths)


def pad_verified_path(path, past_length, width, eos_token_id, workspace=None):
    batch, capacity = path.tokens.shape
    if workspace is None:
        device = path.tokens.device
        tokens = torch.empty((batch, width), device=device, dtype=torch.long)
        indices = torch.empty_like(tokens)
        mask = torch.empty((batch, width), device=device, dtype=torch.bool)
        last = torch.empty((batch, 1), device=device, dtype=torch.long)
    else:
        tokens, indices, mask = [buffer[:batch, :width] for buffer in workspace[:3]]
        last = workspace[3][:batch, :1]
    _ops.pad_verified_path(path.tokens, path.packed_indices, path.lengths, int(width), int(past_length),
                           int(eos_token_id), tokens, indices, mask, last)
    return tokens, indices, mask, last


def pad_schedule(path, past, eos, tokens, indices, mask, last, packet, snapshot=None):
    _ops.pad_schedule(path.tokens, path.packed_indices, path.lengths, int(past), int(eos), tokens, indices, mask,
                      last, packet, snapshot)
