"""Pins oracle/torch_commit.py (the restated torch CPU branch) to the reference's own code.

Run from the repository root in a container that holds the reference checkout:

    python oracle/pin_torch_commit.py /path/to/analysis_spec

(the path of the reference checkout is required). On the same seeded inputs it
runs, for several verify rounds, the reference's OPDStaticCache.update (append),
trace_verified_path + schedule (torch branch, no kernel plugin),
compact_suffix_inplace per layer and crop, next to TorchCommit.round, checks that
every cache byte is identical, and times both on the host's cores at the
Qwen2.5-3B verify shape (36 layers, batch 64, 2 KV heads x 128, bf16, 61 tree
rows). The result is written to oracle/torch_commit_pin.json; the benchmark's
CPU baseline quotes it.
"""
import json
import os
import sys
import time
from pathlib import Path
from types import SimpleNamespace

if len(sys.argv) < 2:
    sys.exit('usage: python oracle/pin_torch_commit.py /path/to/analysis_spec (the reference checkout)')
REF = Path(sys.argv[1]).resolve()
ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REF))
sys.path.insert(1, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from helper.opd_scheduling import compact_suffix_inplace, schedule  # noqa: E402
from helper.opd_static_cache import OPDStaticCache  # noqa: E402
from helper.tree_verification import PackedTree, trace_verified_path  # noqa: E402

from analysis_spec_b200 import workloads as W  # noqa: E402
from oracle.torch_commit import TorchCommit  # noqa: E402

EOS = 151643


def reference_rounds(tc, rounds, check=True):
    """The reference's own per-round sequence on a copy of tc's initial caches."""
    B, H, D, R, past = tc.batch, tc.heads, tc.dim, tc.rows, tc.past
    cache = OPDStaticCache(capacity=256)
    model = SimpleNamespace()
    for l in range(tc.layers):  # prefill of the prefix: the same bytes TorchCommit starts from
        cache.update(tc.kp[l][:, :, :past].clone(), tc.vp[l][:, :, :past].clone(), l)
    tree = PackedTree(torch.from_numpy(tc.parents), torch.from_numpy(tc.tokens), torch.zeros_like(
        torch.from_numpy(tc.parents)), tc.depth)
    times = []
    for i in range(rounds):
        t0 = time.perf_counter()
        views = [cache.update(tc.k_src[l], tc.v_src[l], l) for l in range(tc.layers)]
        path = trace_verified_path(tree, torch.from_numpy(tc.samples[i % len(tc.samples)]), EOS, kernels=None)
        rows, _, idx, _, _, width = schedule(path, past, EOS, None, None, None)
        live = [r for r in rows if r[1] == 0]
        ext = min(r[2] for r in live) if live else width
        for l in range(tc.layers):
            compact_suffix_inplace(views[l][0], views[l][1], idx, past, ext, model)
        cache.crop(past)  # the stationary benchmark verifies every round at the same length
        times.append(time.perf_counter() - t0)
    return cache, times


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.RandomState(11)
    # equality on a small case: 3 layers, batch 8, several rounds
    batch, rows, depth = 8, 61, 6
    parents, tokens = W.packed_trees(rng, batch, rows - 1, depth, 10)
    samples = [W.samples_for(rng, parents, tokens, W.accepted_lengths(rng, ('geometric', 3.5, 7), batch))
               for _ in range(4)]
    tc = TorchCommit(3, batch, 2, 128, rows, 300, parents, tokens, samples, depth)
    ref, _ = reference_rounds(tc, 4)
    for i in range(4):
        tc.round(i, EOS)
    for l in range(3):
        kr, vr = ref.layers[l].key_pool[:batch, :, :300 + rows], ref.layers[l].value_pool[:batch, :, :300 + rows]
        assert torch.equal(kr.view(torch.int16), tc.kp[l][:, :, :300 + rows].view(torch.int16)), l
        assert torch.equal(vr.view(torch.int16), tc.vp[l][:, :, :300 + rows].view(torch.int16)), l
    # timing at the Qwen2.5-3B verify shape
    wl = W.WORKLOADS['qwen25_3b']
    rng = np.random.RandomState(1000)
    prefix = W.prefix_lengths(rng, wl.prefix, wl.batch)
    parents, tokens = W.packed_trees(rng, wl.batch, wl.nodes, wl.depth, wl.topk)
    samples = [W.samples_for(rng, parents, tokens, W.accepted_lengths(rng, wl.accept, wl.batch)) for _ in range(4)]
    tc = TorchCommit(wl.layers, wl.batch, wl.kv_heads, wl.dim, wl.rows, int(prefix.max()), parents, tokens, samples,
                     wl.depth)
    _, ref_times = reference_rounds(tc, 6)
    ours = []
    for i in range(6):
        t0 = time.perf_counter()
        tc.round(i, EOS)
        ours.append(time.perf_counter() - t0)
    out = {'shape': 'qwen25_3b verify round: 36 layers, batch 64, 2 kv heads x 128, bf16, 61 tree rows, past '
                    f'{tc.past}', 'threads': torch.get_num_threads(), 'cpu': _cpu_model(),
           'reference_s_per_round': round(float(np.median(ref_times[1:])), 4),
           'restatement_s_per_round': round(float(np.median(ours[1:])), 4),
           'caches_identical': True, 'rounds_checked': 4}
    (ROOT / 'oracle' / 'torch_commit_pin.json').write_text(json.dumps(out, indent=1) + '\n')
    print(json.dumps(out))


def _cpu_model():
    try:
        for line in open('/proc/cpuinfo'):
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


if __name__ == '__main__':
    main()
