"""Commit scheduling packet and the in-place accepted-suffix KV compaction.

Drop-in for ``helper/opd_scheduling.py`` (``schedule`` :5-32,
``compact_suffix_inplace`` :35-58). Both always run libspeckv's CUDA kernels;
``kernels`` selects the tree-kernel plugin module (this package's
``tree_kernels`` by default) and, as in the reference, whether the packet row
is the full ``capacity + 3`` layout (plugin given) or the ``width + 3`` layout
(no plugin).
"""
import torch

from . import _ops
from . import tree_kernels as _default_kernels


def schedule(path, past, eos, workspace, packet, kernels=None, opd=None):
    """Pads the verified paths, writes the packet and reads it back (the one D2H per round).

    Returns (rows, tokens, indices, mask, last, width) with rows the host packet
    [length, eos?, extension, pad ids...] per sequence.
    """
    return _schedule(path, past, eos, workspace, packet, kernels, opd, None)


def schedule_commit(path, past, eos, workspace, packet, cache, positions, past_positions, pad_rows=None,
                    owners=None, pad_live=None, kernels=None, opd=None, on_launched=None, compact=True):
    """``schedule`` with the round's commit enqueued on the device before the packet read-back.

    Right after the padded schedule is written, one launch compacts the accepted
    suffix of every layer of ``cache`` and updates positions / padding, taking
    width and extension from the device packet (``speckv_commit_round``); the GPU
    runs the commit while the host waits for the packet. The cache is then
    cropped to ``past + width``. Same result as ``schedule`` followed by
    ``cache.commit_accepted(indices, past, extension)`` and
    ``_ops.position_update(mask, past, positions[:, :width], past_positions, ...)``
    (helper/opd_generate.py:632-650); returns ``schedule``'s tuple.

    ``on_launched()``, when given, is called after these launches and before the host
    waits for the packet (e.g. to enqueue the round's counter reduction, which reads the
    packet on the device), so its host work overlaps the GPU's. With ``compact=False``
    the launch updates positions / padding only and the compaction is the caller's: fold
    it into the next round's append, ``cache.update_layers(..., commit=(indices, past,
    extension, width))``, before the next attention reads the cache.
    """
    def commit(tokens, indices, mask, out_packet):
        # prepared before the schedule kernel is launched and issued right after it, so the
        # host work of the commit overlaps the schedule kernel
        return cache.commit_scheduled(indices, past, out_packet, newly_padded=mask, positions=positions,
                                      past_positions=past_positions, pad_rows=pad_rows, owners=owners,
                                      pad_live=pad_live, deferred=True, compact=compact)

    result = _schedule(path, past, eos, workspace, packet, kernels, opd, commit, on_launched)
    cache.crop(past + result[5])
    return result


def _schedule(path, past, eos, workspace, packet, kernels, opd, commit, on_launched=None):
    b, capacity = path.tokens.shape
    plugin = kernels if kernels is not None else _default_kernels
    if kernels is not None and opd is not None:
        opd.host_sync_count += 1
    if workspace is not None:
        tokens, indices, mask = [x[:b, :capacity] for x in workspace[:3]]
        last = workspace[3][:b, :1]
    else:
        device = path.tokens.device
        tokens = torch.empty((b, capacity), device=device, dtype=torch.long)
        indices = torch.empty_like(tokens)
        mask = torch.empty((b, capacity), device=device, dtype=torch.bool)
        last = torch.empty((b, 1), device=device, dtype=torch.long)
    if packet is None:
        packet = torch.empty((b, capacity + 4), device=path.tokens.device, dtype=torch.long)
    out_packet = packet[:b, :capacity + 3]
    # as in the reference, the OPD runtime's active-count snapshot rides in the packet only on
    # the plugin path; without a plugin `opd` is not read
    reflex = kernels is not None and opd is not None and getattr(opd, 'enabled', True)
    snapshot = None
    if reflex:
        snapshot = (opd.dispatch_snapshot if getattr(opd, 'async_updates', False)
                    else getattr(opd, 'dispatch_count', opd.active_count))
    launch = commit(tokens, indices, mask, out_packet) if commit is not None else None
    plugin.pad_schedule(path, past, eos, tokens, indices, mask, last, out_packet, snapshot=snapshot)
    if launch is not None:
        launch()
    if on_launched is not None:
        on_launched()
    # whole rows of the packet buffer: one contiguous copy, no gather kernel before the D2H
    host = packet[:b].cpu() if packet.is_contiguous() else packet[:b, :capacity + 4].cpu()
    if reflex:
        rows = host[:, :capacity + 4].tolist()
        opd.host_active_count = rows[0][-1]
        rows = [row[:-1] for row in rows]
    else:
        rows = host[:, :capacity + 3].tolist()
    width = max(row[0] for row in rows)
    if kernels is None:
        rows = [row[:3 + width] for row in rows]
    return rows, tokens[:, :width], indices[:, :width], mask[:, :width], last, width


def compact_suffix_inplace(key, value, chosen, past, extension, model):
    """Writes the accepted suffix rows chosen[:, extension:] to [past + extension, past + width).

    ``key`` / ``value`` are (batch, heads, length, dim) views of pools (any
    tensor whose last three strides are (capacity * dim, dim, 1)); the prefix is
    untouched and no scratch is allocated (each (sequence, head) stages its rows
    on chip). Returns the views ``[..., :past + width, :]``.
    """
    width = chosen.shape[1]
    end = past + width
    if extension == width:
        return key[..., :end, :], value[..., :end, :]
    pools = []
    for view in (key, value):
        b, heads, length, dim = view.shape
        if view.stride(3) != 1 or view.stride(2) != dim or view.stride(1) % dim or \
                (b > 1 and view.stride(0) != heads * view.stride(1)):
            raise ValueError('compact_suffix_inplace needs (batch, heads, length, dim) views of a KV pool')
        capacity = view.stride(1) // dim
        pools.append(view.as_strided((b, heads, capacity, dim), (heads * capacity * dim, capacity * dim, dim, 1)))
    _ops.compact_suffix([pools[0]], [pools[1]], key.shape[0], key.shape[2], chosen, past, extension, width)
    return key[..., :end, :], value[..., :end, :]
