"""Tensor tree structures of the verify round, drop-in for ``helper/tree_verification.py``.

``PackedTree`` (:12-42), ``pack_tree`` (:45-72), ``VerifiedPath`` (:75-128) and
``trace_verified_path`` (:131-167) keep the reference's signatures. The
reference's ``kernels=None`` branch is a loop of torch ops; here every branch
runs libspeckv's CUDA kernels (``kernels`` defaults to this package's
``tree_kernels`` plugin), so there is one implementation per op.
"""
from dataclasses import dataclass

import torch

from . import _ops
from . import tree_kernels as _default_kernels


@dataclass
class PackedTree:
    parents: torch.Tensor  # [B, packed_nodes + 1], root row 0 has parent -1
    tokens: torch.Tensor
    feedback_contexts: torch.Tensor  # -1 for nodes without a draft-head context
    max_depth: int

    def attention_mask(self, past_length, dtype, padding_positions=None, *, kernels=None, workspace=None):
        """Additive (batch, 1, rows, past + rows) mask: prefix and ancestors visible.

        ``padding_positions`` is the reference's (n, 2) tensor of (sequence, column)
        pairs to hide; a (batch, columns) bool tensor is taken as a padding bitmap
        and fused into the mask kernel.
        """
        batch, rows = self.parents.shape
        shape = (batch, 1, rows, past_length + rows)
        elements = batch * rows * (past_length + rows)
        if workspace is not None and workspace.numel() >= elements:
            mask = workspace[:elements].view(shape)
        else:
            mask = torch.empty(shape, device=self.parents.device, dtype=dtype)
        plugin = kernels if kernels is not None else _default_kernels
        bitmap = None
        if isinstance(padding_positions, torch.Tensor) and padding_positions.dtype == torch.bool:
            bitmap = padding_positions
        if bitmap is not None and plugin is _default_kernels:
            plugin.tree_mask(self, past_length, mask, pad=bitmap)
            return mask
        plugin.tree_mask(self, past_length, mask)
        if bitmap is not None:
            mask.masked_fill_(bitmap[:, None, None, :past_length + rows], torch.finfo(dtype).min)
        elif isinstance(padding_positions, torch.Tensor):
            mask[padding_positions[:, 0], 0, :, padding_positions[:, 1]] = torch.finfo(dtype).min
        return mask

    def visibility(self, past_length, padding=None, *, workspace=None):
        """Bit-packed form of ``attention_mask`` for the tensor-core attention.

        Built once per verify round and shared by every layer: (batch, rows,
        words) int32 bits (bit c of a row = column c visible) plus the first
        visible column of each sequence, so fully padded key tiles are skipped.
        ``padding`` is a (batch, columns) bool bitmap of hidden columns.
        """
        batch, rows = self.parents.shape
        words = _ops.visibility_words(past_length + rows)
        if workspace is not None and workspace[0].numel() >= batch * rows * words and workspace[1].numel() >= batch:
            bits = workspace[0].view(-1)[:batch * rows * words].view(batch, rows, words)
            first = workspace[1].view(-1)[:batch]
        else:
            bits = torch.empty((batch, rows, words), device=self.parents.device, dtype=torch.int32)
            first = torch.empty((batch,), device=self.parents.device, dtype=torch.int32)
        _ops.tree_mask_bits(self.parents, past_length, self.max_depth + 1, bits, first, padding)
        return TreeVisibility(bits, first, int(past_length), rows)


@dataclass
class TreeVisibility:
    """Per-round visibility of the verify forward (see PackedTree.visibility)."""
    bits: torch.Tensor       # (batch, rows, words) int32
    first_col: torch.Tensor  # (batch,) int32
    past: int
    rows: int

    def attach(self, mask):
        """Tags a dense mask so the registered attention reads these bits instead."""
        mask._speckv_visibility = self
        return mask


def pack_tree(full_parents, full_contexts, chosen, all_tokens, max_depth, *, workspace=None):
    """Keeps the sorted confidence-selected nodes, re-indexed with the root as row 0."""
    batch, _ = full_parents.shape
    packed_count = chosen.shape[1]
    device = chosen.device
    if workspace is not None:
        outputs = [w[:batch * (packed_count + 1)].view(batch, packed_count + 1) for w in workspace[1:4]]
    else:
        outputs = [torch.empty((batch, packed_count + 1), device=device, dtype=torch.long) for _ in range(3)]
    _ops.pack_tree(full_parents, full_contexts, all_tokens, chosen, *outputs)
    return PackedTree(*outputs, int(max_depth))


@dataclass
class VerifiedPath:
    tokens: torch.Tensor  # -1 padding; emitted tokens, including the target bonus token
    packed_indices: torch.Tensor  # target-logit rows of those tokens
    feedback_contexts: torch.Tensor
    lengths: torch.Tensor

    def padded_gpu(self, past_length: int, width: int, eos_token_id: int, *, kernels=None, workspace=None):
        """Gap-first padded commit layout on the device: (tokens, indices, mask, last)."""
        _, capacity = self.tokens.shape
        if not 1 <= width <= capacity:
            raise ValueError("invalid committed path width")
        plugin = kernels if kernels is not None else _default_kernels
        return plugin.pad_verified_path(self, past_length, width, eos_token_id, workspace)

    def host_bookkeeping(self, past_length):
        """One small D2H packet: per-sequence lengths, absolute KV indices and tokens."""
        packet = torch.stack((self.tokens, self.packed_indices), dim=1).cpu().tolist()
        tokens, chosen, lengths = [], [], []
        for row_tokens, row_indices in packet:
            length = sum(index >= 0 for index in row_indices)
            tokens.append(row_tokens[:length])
            chosen.append([past_length + index for index in row_indices[:length]])
            lengths.append(length)
        return lengths, chosen, tokens


def trace_verified_path(tree, sampled_tokens, eos_token_id, *, kernels=None, workspace=None):
    """Greedy walk: emit the sampled token, descend to the first child with that token, stop at EOS."""
    batch, rows = sampled_tokens.shape
    if sampled_tokens.shape != tree.parents.shape:
        raise ValueError("sampled tokens do not match the packed tree")
    width = tree.max_depth + 1
    if workspace is None:
        buffers = [torch.empty((batch, width), device=sampled_tokens.device, dtype=torch.long) for _ in range(3)]
        lengths = torch.empty(batch, device=sampled_tokens.device, dtype=torch.long)
    else:
        buffers = [tensor[:batch, :width] for tensor in workspace[:3]]
        lengths = workspace[3][:batch]
    emitted, indices, contexts = buffers
    plugin = kernels if kernels is not None else _default_kernels
    plugin.trace_path(tree, sampled_tokens, eos_token_id, emitted, indices, contexts, lengths)
    return VerifiedPath(emitted, indices, contexts, lengths)
