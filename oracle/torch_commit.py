"""The reference's torch CPU branch of the KV commit, restated (TEST INFRASTRUCTURE ONLY).

The CPU baseline of the benchmark: the same torch operations, on host tensors,
that the reference runs for one verify round of its static KV cache when no
GPU kernel plugin is given. Only bench.py's CPU-baseline / reference legs and
the tests use it; the product never imports it.

Per round, for every layer:
  append        pool[:B, :, len:len+q].copy_(k) and the same for v
                (helper/opd_static_cache.py:99-109, StaticAppendLayer.update)
  compaction    torch.gather of the accepted rows into a reused scratch, then a
                copy back to [past+e, past+W) (helper/opd_scheduling.py:35-58,
                compact_suffix_inplace, called per layer at
                helper/opd_generate.py:632-643), then crop(past + W)
once per round:
  trace + schedule   the greedy walk and gap-first layout (numpy restatement of
                helper/tree_verification.py:131-167 and helper/opd_scheduling.py:5-32,
                small next to the per-layer copies)
  position update    pad_mask[owners, past:past+W] = newly_padded;
                positions = cumsum(~newly_padded) + past_positions;
                past_positions = positions[:, -1] (helper/opd_generate.py:556-558, 644-650)

Pinned against the reference itself by oracle/pin_torch_commit.py (run in a
container holding the reference checkout): identical caches, and the
restatement's time per round next to the reference's.
"""
import numpy as np
import torch

from . import oracle


class TorchCommit:
    """One workload's caches on host tensors; `round(i)` runs one verify round's commit and
    returns the algorithmic bytes it moved (each moved byte counted once read, once written)."""

    def __init__(self, layers, batch, heads, dim, rows, past, parents, tokens, samples, depth, dtype=torch.bfloat16,
                 seed=7):
        g = torch.Generator().manual_seed(seed)
        self.layers, self.batch, self.heads, self.dim, self.rows, self.past = layers, batch, heads, dim, rows, past
        cap = past + rows
        self.kp = [torch.randn(batch, heads, cap, dim, generator=g).to(dtype) for _ in range(layers)]
        self.vp = [torch.randn(batch, heads, cap, dim, generator=g).to(dtype) for _ in range(layers)]
        # projections laid out (B, q, heads * dim) and viewed (B, heads, q, dim), as the model hands them over
        self.k_src = [torch.randn(batch, rows, heads * dim, generator=g).to(dtype).view(batch, rows, heads, dim)
                      .transpose(1, 2) for _ in range(layers)]
        self.v_src = [torch.randn(batch, rows, heads * dim, generator=g).to(dtype).view(batch, rows, heads, dim)
                      .transpose(1, 2) for _ in range(layers)]
        self.parents, self.tokens, self.samples, self.depth = parents, tokens, samples, depth
        self.scratch = None
        self.pad_mask = torch.zeros(batch, cap, dtype=torch.bool)
        self.past_positions = torch.full((batch,), past, dtype=torch.long)
        self.owners = torch.arange(batch)
        self.es = self.kp[0].element_size()

    def round(self, i, eos):
        B, H, D, R, past = self.batch, self.heads, self.dim, self.rows, self.past
        for l in range(self.layers):  # StaticAppendLayer.update: two copy_ per layer
            self.kp[l][:B, :, past:past + R].copy_(self.k_src[l])
            self.vp[l][:B, :, past:past + R].copy_(self.v_src[l])
        samples = self.samples[i % len(self.samples)]
        pt, pi, _, pl = oracle.trace_path(self.parents, self.tokens, np.zeros_like(self.parents), samples, eos,
                                          self.depth + 1)
        _, idx, newly, _, packet, width = oracle.pad_schedule(pt, pi, pl, past, eos)
        live = packet[packet[:, 1] == 0]
        ext = int(live[:, 2].min()) if len(live) else width
        moved = self.layers * 2 * 2 * B * H * R * D * self.es
        if ext < width:
            chosen = torch.from_numpy(np.ascontiguousarray(idx[:, :width]))
            n = width - ext
            index = chosen[:, ext:][:, None, :, None].expand(B, H, n, D)
            if self.scratch is None or self.scratch[0].numel() < B * H * n * D:
                self.scratch = (torch.empty(B, H, R, D, dtype=self.kp[0].dtype),
                                torch.empty(B, H, R, D, dtype=self.kp[0].dtype))
            k = self.scratch[0].flatten()[:B * H * n * D].view(B, H, n, D)
            v = self.scratch[1].flatten()[:B * H * n * D].view(B, H, n, D)
            end = past + width
            for l in range(self.layers):  # compact_suffix_inplace per layer
                key, value = self.kp[l][:B, :, :past + R], self.vp[l][:B, :, :past + R]
                torch.gather(key, 2, index, out=k)
                torch.gather(value, 2, index, out=v)
                key[..., past + ext:end, :].copy_(k)
                value[..., past + ext:end, :].copy_(v)
            moved += self.layers * 2 * 2 * B * H * n * D * self.es
        newly_t = torch.from_numpy(np.ascontiguousarray(newly[:, :width]))
        self.pad_mask[self.owners[:, None], torch.arange(past, past + width)[None, :]] = newly_t
        positions = torch.cumsum(~newly_t, 1) + self.past_positions[:, None]
        self.past_positions = positions[:, -1].clone()
        return moved
