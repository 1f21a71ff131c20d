"""Seeded synthetic workloads of the verify round (trees, acceptance, ragged prefixes).

Shapes follow the benchmark configurations of the path:
  cpu_commit         1 layer, batch 4, 2 KV heads x 128, fp32, max_len 512, prefix U{32..256},
                     16-node tree (depth 4, top-k 4), accepted length U{1..5}
  qwen25_3b          36 layers, 16 q / 2 KV heads x 128, bf16, batch 64, max_len 4096,
                     prefix U{256..2048}, 60-node tree (depth 6, top-k 10),
                     accepted length ~ geometric(mean 3.5) capped at 7
  qwen25_3b_attn     as qwen25_3b with prefix U{256..3072} and Q/K/V ~ 0.5 N(0, 1)
  qwen25_7b          28 layers, 28 q / 4 KV heads, batch 256 split over the GPUs of the job
                     (strong scaling), max_len 8192, prefix U{512..6144}
  qwen25_14b         48 layers, 40 q / 8 KV heads, batch 16 per GPU (128 over 8 GPUs), max_len
                     16384, prefix log-uniform [128, 14000], 25% of sequences finish per step and
                     as many new ones are admitted; the attention splits the longest sequences'
                     key ranges over several CTAs (key-range chunks)
Sequences share one physical cache length (the longest prefix); shorter
prefixes are left-padded and their padding columns hidden by the padding
bitmap, as the reference's prefill lays them out.
"""
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Workload:
    name: str
    layers: int
    batch: int
    q_heads: int
    kv_heads: int
    dim: int
    dtype: str
    capacity: int
    prefix: tuple  # ('uniform', lo, hi) or ('loguniform', lo, hi)
    nodes: int
    depth: int
    topk: int
    accept: tuple  # ('uniform', lo, hi) or ('geometric', mean, cap)
    finish_fraction: float = 0.0
    qkv_scale: float = 1.0
    extra: dict = field(default_factory=dict)

    @property
    def rows(self):
        return self.nodes + 1


WORKLOADS = {
    'cpu_commit': Workload('cpu_commit', 1, 4, 16, 2, 128, 'float32', 512, ('uniform', 32, 256), 16, 4, 4,
                           ('uniform', 1, 5)),
    'qwen25_3b': Workload('qwen25_3b', 36, 64, 16, 2, 128, 'bfloat16', 4096, ('uniform', 256, 2048), 60, 6, 10,
                          ('geometric', 3.5, 7)),
    'qwen25_3b_attn': Workload('qwen25_3b_attn', 36, 64, 16, 2, 128, 'bfloat16', 4096, ('uniform', 256, 3072), 60, 6,
                               10, ('geometric', 3.5, 7), qkv_scale=0.5),
    'qwen25_7b': Workload('qwen25_7b', 28, 256, 28, 4, 128, 'bfloat16', 8192, ('uniform', 512, 6144), 60, 6, 10,
                          ('geometric', 3.5, 7), extra={'split_batch': True}),
    'qwen25_14b': Workload('qwen25_14b', 48, 16, 40, 8, 128, 'bfloat16', 16384, ('loguniform', 128, 14000), 60, 6,
                           10, ('geometric', 3.5, 7), finish_fraction=0.25, extra={'attention_chunks': True}),
}


def prefix_lengths(rng, spec, batch):
    kind, lo, hi = spec
    if kind == 'uniform':
        return rng.randint(lo, hi + 1, size=batch)
    return np.exp(rng.uniform(np.log(lo), np.log(hi), size=batch)).astype(np.int64)


def left_padding(lengths, past):
    """(batch, past) bool bitmap: True on the left-padding columns of shorter prefixes."""
    cols = np.arange(past)[None, :]
    return cols < (past - np.asarray(lengths))[:, None]


def packed_trees(rng, batch, nodes, depth, topk, vocab=32000):
    """Parent-closed packed trees (root row 0, parent -1): parents[r] < r, depth and fan-out capped."""
    rows = nodes + 1
    parents = np.full((batch, rows), -1, dtype=np.int64)
    for b in range(batch):
        level = np.zeros(rows, dtype=np.int64)
        kids = np.zeros(rows, dtype=np.int64)
        for r in range(1, rows):
            cand = np.nonzero((level[:r] < depth) & (kids[:r] < topk))[0]
            p = cand[rng.randint(len(cand))]
            parents[b, r] = p
            level[r] = level[p] + 1
            kids[p] += 1
    tokens = rng.randint(0, vocab, size=(batch, rows)).astype(np.int64)
    tokens[:, 0] = -1
    return parents, tokens


def accepted_lengths(rng, spec, batch):
    kind, a, b = spec
    if kind == 'uniform':
        return rng.randint(a, b + 1, size=batch)
    return np.minimum(rng.geometric(1.0 / a, size=batch), b)


def samples_for(rng, parents, tokens, accept, vocab=32000, eos=None, eos_prob=0.0):
    """Target samples whose greedy walk emits `accept[b]` tokens where the tree is deep enough.

    Along a random root-to-leaf walk every node samples its chosen child's token;
    the stop node samples a token that matches none of its children (or EOS).
    """
    batch, rows = parents.shape
    samples = rng.randint(0, vocab, size=(batch, rows)).astype(np.int64)
    for b in range(batch):
        children = [[] for _ in range(rows)]
        for r in range(1, rows):
            children[parents[b, r]].append(r)
        node, emitted = 0, 1
        while emitted < accept[b] and children[node]:
            child = children[node][rng.randint(len(children[node]))]
            # first child carrying this token wins the walk: pick tokens unique among siblings
            samples[b, node] = tokens[b, child]
            if any(tokens[b, c] == tokens[b, child] for c in children[node] if c < child):
                break
            node = child
            emitted += 1
        stop = {tokens[b, c] for c in children[node]}
        tok = vocab + 1
        while tok in stop:
            tok += 1
        samples[b, node] = eos if eos is not None and rng.rand() < eos_prob else tok
    return samples
