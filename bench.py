#!/usr/bin/env python
"""Verify-round benchmark of the static-KV-cache / tree-verify path on B200.

One step = one verify round of the Qwen2.5-3B geometry workload (36 layers,
batch 64, 16 query / 2 KV heads x 128, bf16, max_len 4096, prefixes U{256..2048}
left-padded to one shared length, 60-node trees of depth 6 / top-k 10, accepted
length ~ geometric(mean 3.5) capped at 7):

  tree visibility bits (+ padding) -> append the 61 tree rows of all 36 layers (one launch)
  -> 36 x tree-verify attention -> greedy trace -> padded schedule + host packet
  -> accepted-suffix compaction of all layers (one launch) -> crop
  -> position / padding update.

Reported (one JSON line on rank 0):
  value      KV-commit GB/s: algorithmic bytes of append + compaction (each moved
             byte read once and written once) / device time of those kernels
  tree_verify  steps/s = 1 / (visibility build + 36 attention launches) per step; the
             attention launches are replayed from a CUDA graph captured once
             (--no-graph: launched one by one)
  e2e        the same KV-commit metric through the public API with the step's
             inputs copied from pinned host memory and the packet read back
  roofline   the append kernel (dominant commit kernel) vs measured HBM copy peak
  cpu_baseline  the reference's torch CPU branch of the commit, restated on host tensors
             (oracle/torch_commit.py, pinned to the reference's own code), all layers, host cores;
             cpu_baseline_c_port: the C/OpenMP restatement on a sample of the layers
  draft_step   one draft expansion step (mask + attention of one draft layer),
             this library's launches beside the reference's torch sequence
  history_step the accepted-feature gather + rollout-history append of a round,
             one launch beside the reference's gather + index_copy_ sequence
  release_step releasing a quarter of the sequences: the reference's swap_remove
             (history moves) against a row-table cache (table rewrite, no KV bytes)

``--impl reference`` times the reference's torch CPU branch of the commit, restated
(the reference is Python/torch and is not present on the GPU host; the restatement is
pinned to it by oracle/pin_torch_commit.py), on the host cores.
Multi-GPU (torchrun): every rank owns its own batch of sequences (weak scaling)
and one int64 acceptance-counter all_reduce runs per step on a side stream.
"""
import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS = ROOT / 'MEASURED_PEAKS.json'
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS = 6650.0, 1590.0
METRIC = 'KV-commit GB/s (% HBM peak) + tree-verify steps/s, Qwen2.5-3B geom B=64'
EOS = 151643


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--workload', default='qwen25_3b')
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--no-e2e', action='store_true')
    p.add_argument('--layers', type=int, default=None, help='override the layer count (small profiling cases)')
    p.add_argument('--batch', type=int, default=None, help='override the per-GPU batch (small profiling cases)')
    p.add_argument('--fold', action='store_true',
                   help='fold each round\'s compaction into the next round\'s append launch '
                        '(speckv_append_commit_rows); the round\'s commit launch then updates positions only')
    p.add_argument('--no-graph', action='store_true',
                   help="launch the round's attention layer by layer instead of replaying its CUDA graph")
    p.add_argument('--side-only', action='store_true',
                   help='only the draft-step and history-step measurements, on a one-layer cache (profiling)')
    p.add_argument('--row-table', action='store_true',
                   help='rollout workloads: release and admit through a row table instead of moving histories')
    return p.parse_args()


def workload(args):
    from dataclasses import replace
    from analysis_spec_b200.workloads import WORKLOADS
    wl = WORKLOADS[args.workload]
    world = int(os.environ.get('WORLD_SIZE', 1))
    if wl.extra.get('split_batch') and world > 1:  # a job-wide batch sharded over the GPUs (strong scaling)
        wl = replace(wl, batch=wl.batch // world)
    if args.layers:
        wl = replace(wl, layers=args.layers)
    if args.batch:
        wl = replace(wl, batch=args.batch)
    return wl


def peaks():
    if PEAKS.exists():
        d = json.loads(PEAKS.read_text())
        return float(d['hbm_gbs']), float(d['bf16_tflops']), 'measured'
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 'fallback'


def dram_traffic(entry, layers, workload='qwen25_3b'):
    """DRAM bytes per launch of one of this path's kernels from the committed ncu capture
    (scaled to `layers` where the traffic grows with the layer count) and where the figure
    comes from, or (None, reason). The capture records a hash of the kernel's source file; the
    label says whether the source built here still matches it."""
    path = ROOT / 'profiles' / 'dram_traffic_qwen25_3b.json'
    if not path.exists():
        return None, 'no ncu capture committed'
    if workload != 'qwen25_3b':
        return None, 'DRAM traffic captured on the qwen25_3b workload only'
    d = json.loads(path.read_text())
    k = d['kernels'].get(entry)
    if k is None:
        return None, 'kernel not in the ncu capture'
    per = k['dram_read_bytes'] + k['dram_write_bytes']
    src = k.get('source')
    now = hashlib.sha256((ROOT / src).read_bytes()).hexdigest()[:16] if src and (ROOT / src).exists() else None
    same = now is not None and now == d.get('sources', {}).get(src)
    label = (f'ncu dram__bytes_read+write of {k["kernel"]}, {k["captured_layers"]}-layer capture scaled to '
             f'{layers} layers' if k['scale'] != 1.0 else f'ncu dram__bytes_read+write of {k["kernel"]}, one launch')
    label += ('; kernel source unchanged since the capture' if same else
              '; kernel source CHANGED since the capture (figure is stale)')
    return int(per * (layers / k['captured_layers'] if k['scale'] != 1.0 else 1.0)), label


def workload_config(wl, extra=None):
    cfg = {'workload': f'{wl.name}: {wl.layers} layers, batch {wl.batch}, {wl.q_heads}q/{wl.kv_heads}kv heads x '
                       f'{wl.dim}, {wl.dtype}, max_len {wl.capacity}, prefix {wl.prefix}, {wl.nodes}-node tree '
                       f'depth {wl.depth} top-k {wl.topk}, accepted {wl.accept}',
           'layers': wl.layers, 'batch_per_gpu': wl.batch, 'tree_rows': wl.rows,
           'l2': 'inputs larger than L2: each step streams > 4 GB of KV pools'}
    if wl.extra.get('attention_chunks'):
        cfg['attention_chunks'] = 'key ranges of the longest sequences split over several CTAs (row-table runs: off)'
    cfg.update(extra or {})
    return cfg


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    """SM clock and clock-event reasons of this GPU sampled during the timed region: NVML
    every 5 ms from a background thread (read-only queries), nvidia-smi every 20 ms when the
    NVML binding is unavailable."""
    FIELDS = ('uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
    NAMES = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')

    def __init__(self, uuid):
        self.uuid = str(uuid).lower().replace('gpu-', '')
        self.proc = None
        self.file = None
        self.thread = None
        self.samples = []
        self.max_mhz = 0.0

    def start(self):
        try:
            import threading
            import pynvml
            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByUUID('GPU-' + self.uuid)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
            bits = (pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                    pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap)
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                        mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        self.samples.append((mhz, {n for n, bit in zip(self.NAMES, bits) if mask & bit}))
                    except pynvml.NVMLError:
                        pass
                    self._stop.wait(0.005)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-lms', '20'], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            sm = [m for m, _ in self.samples]
            reasons = set().union(*(r for _, r in self.samples))
            return {'sm_mhz': float(np.median(sm)), 'sm_max_mhz': self.max_mhz, 'samples': len(sm),
                    'reasons': sorted(reasons), 'source': 'nvml'}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(', ') for r in Path(self.file.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        uuids = {r[0].strip().lower().replace('gpu-', '') for r in rows if r}
        if self.uuid in uuids:
            rows = [r for r in rows if r[0].strip().lower().replace('gpu-', '') == self.uuid]
        elif len(uuids) != 1:
            return None
        sm, mx, reasons = [], 0.0, set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for name, flag in zip(self.NAMES, r[5:9]):
                    if flag.strip().lower() in ('active', '1'):
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {'sm_mhz': float(np.median(sm)), 'sm_max_mhz': mx, 'samples': len(sm), 'reasons': sorted(reasons),
                'source': 'nvidia-smi'}


# ---------------------------------------------------------------------------
# synthetic verify-round state
# ---------------------------------------------------------------------------
class Round:
    """Device-resident inputs of the stationary verify round (shapes never change)."""

    def __init__(self, wl, device, seed, sample_sets=8, row_table=False):
        import torch
        from analysis_spec_b200 import workloads as W
        from analysis_spec_b200.opd_static_cache import OPDStaticCache
        from analysis_spec_b200.tree_verification import PackedTree
        self.wl = wl
        self.device = device
        dtype = getattr(torch, wl.dtype)
        self.dtype = dtype
        rng = np.random.RandomState(seed)
        B, R, H, D = wl.batch, wl.rows, wl.kv_heads, wl.dim
        self.prefix = W.prefix_lengths(rng, wl.prefix, B)
        self.past = int(self.prefix.max())
        cols = wl.capacity
        pad = np.zeros((B, cols), dtype=bool)
        pad[:, :self.past] = W.left_padding(self.prefix, self.past)
        self.pad = torch.from_numpy(pad).to(device)
        self.pad_commit = torch.zeros_like(self.pad)
        gen = torch.Generator(device=device).manual_seed(seed)
        scale = wl.qkv_scale
        self.cache = OPDStaticCache(wl.capacity, batch_capacity=B, row_table=row_table)
        prefix_k = (scale * torch.randn(B, H, self.past, D, device=device, generator=gen)).to(dtype)
        prefix_v = (scale * torch.randn(B, H, self.past, D, device=device, generator=gen)).to(dtype)
        for l in range(wl.layers):
            self.cache.update(prefix_k, prefix_v, l)
        del prefix_k, prefix_v
        # per-layer projections laid out (B, R, heads * D) and viewed (B, heads, R, D)
        self.k_proj = [(scale * torch.randn(B, R, H * D, device=device, generator=gen)).to(dtype)
                       for _ in range(wl.layers)]
        self.v_proj = [(scale * torch.randn(B, R, H * D, device=device, generator=gen)).to(dtype)
                       for _ in range(wl.layers)]
        self.q_proj = [(scale * torch.randn(B, R, wl.q_heads * D, device=device, generator=gen)).to(dtype)
                       for _ in range(wl.layers)]
        self.keys = [x.view(B, R, H, D).transpose(1, 2) for x in self.k_proj]
        self.values = [x.view(B, R, H, D).transpose(1, 2) for x in self.v_proj]
        self.queries = [x.view(B, R, wl.q_heads, D).transpose(1, 2) for x in self.q_proj]
        self.out = [torch.empty(B, R, wl.q_heads, D, device=device, dtype=dtype) for _ in range(wl.layers)]
        parents, tokens = W.packed_trees(rng, B, wl.nodes, wl.depth, wl.topk)
        self.parents_np, self.tokens_np = parents, tokens
        self.tree = PackedTree(torch.from_numpy(parents).to(device), torch.from_numpy(tokens).to(device),
                               torch.zeros(B, R, dtype=torch.long, device=device), wl.depth)
        self.samples = []
        for _ in range(sample_sets):
            acc = W.accepted_lengths(rng, wl.accept, B)
            self.samples.append(torch.from_numpy(W.samples_for(rng, parents, tokens, acc)).to(device))
        width = wl.depth + 1
        self.path_ws = [torch.empty(B, width, dtype=torch.long, device=device) for _ in range(3)] + \
                       [torch.empty(B, dtype=torch.long, device=device)]
        self.pad_ws = [torch.empty(B, width, dtype=torch.bool if i == 2 else torch.long, device=device)
                       for i in range(3)] + [torch.empty(B, 1, dtype=torch.long, device=device)]
        self.packet = torch.empty(B, width + 4, dtype=torch.long, device=device)
        words = 4 * (-(-(self.past + R) // 128))
        self.vis_ws = (torch.empty(B * R * words, dtype=torch.int32, device=device),
                       torch.empty(B, dtype=torch.int32, device=device))
        self.positions = torch.empty(B, width, dtype=torch.long, device=device)
        self.past_positions = torch.from_numpy(self.prefix.astype(np.int64)).to(device)
        self.owners = torch.arange(B, device=device)
        self.scale = D ** -0.5
        self.counters = torch.zeros(5, dtype=torch.long, device=device)
        es = torch.finfo(dtype).bits // 8
        self.append_bytes = wl.layers * 2 * 2 * B * H * R * D * es
        self.row_bytes = D * es

    def compact_bytes(self, width, extension):
        return self.wl.layers * 2 * 2 * self.wl.batch * self.wl.kv_heads * (width - extension) * self.row_bytes

    def attention_flops(self):
        rows, hq, d = self.wl.rows, self.wl.q_heads, self.wl.dim
        return float(sum(4 * hq * rows * (int(p) + rows) * d for p in self.prefix)) * self.wl.layers


def verify_round(st, i, marks=None, on_launched=None):
    """One verify round; returns (width, extension, rows). `marks` gets CUDA events between phases:
    0 visibility 1 append 2 attention 3 trace + schedule + device commit + packet read-back 4.
    `on_launched` runs once the round's kernels are queued, before the packet read-back."""
    from analysis_spec_b200 import _ops, tree_kernels
    from analysis_spec_b200.opd_scheduling import schedule_commit
    from analysis_spec_b200.tree_verification import trace_verified_path

    def mark(k):
        if marks is not None:
            marks[k].record()

    # with st.fold the previous round's compaction rides on this append (its commit updated
    # positions only); st.folded records the (width, extension) whose compaction this append does
    fold = getattr(st, 'fold', False)
    # with st.fused the append rides on the attention launches (update_attend): no append launch
    fused = getattr(st, 'fused', False)
    pending = getattr(st, 'pending_commit', None) if fold else None
    st.folded = pending[4] if pending is not None else None
    append = None if fused else st.cache.update_layers(st.keys, st.values, deferred=True,  # host work first
                                                       commit=pending[:4] if pending is not None else None)
    mark(0)
    vis = st.tree.visibility(st.past, st.pad, workspace=st.vis_ws)
    mark(1)
    views = append() if append is not None else None
    mark(2)
    if getattr(st, 'attn_graph', None) is not None:
        st.attn_graph.replay()  # the same 36 launches, captured once (capture_attention)
        if fused:  # the host half of update_attend: every layer now holds past + rows positions
            for layer in st.cache.layers:
                layer.length = st.past + st.wl.rows
    elif fused:
        for l in range(st.wl.layers):
            st.cache.update_attend(st.queries[l], st.keys[l], st.values[l], l, vis, st.scale, out=st.out[l])
    else:
        for l in range(st.wl.layers):
            k, v = views[l]
            _ops.tree_attention_bits(st.queries[l], k, v, vis.bits, vis.first_col, st.scale, out=st.out[l],
                                     row_table=getattr(k, '_speckv_rows', None))  # row-table caches only
    mark(3)
    path = trace_verified_path(st.tree, st.samples[i % len(st.samples)], EOS, workspace=st.path_ws)
    rows, _, idx, _, _, width = schedule_commit(path, st.past, EOS, st.pad_ws, st.packet, st.cache, st.positions,
                                                st.past_positions, pad_rows=st.pad_commit, owners=st.owners,
                                                kernels=tree_kernels, on_launched=on_launched, compact=not fold)
    mark(4)
    live = [r for r in rows if r[1] == 0]
    extension = min(r[2] for r in live) if live else width
    if fold:
        st.pending_commit = (idx, st.past, extension, width, (width, extension))
    st.cache.crop(st.past)  # stationary workload: the next round verifies at the same length
    return width, extension, rows


def capture_attention(st):
    """CUDA graph of a round's attention launches, one per layer. The stationary workload keeps
    every operand at the same address each round (the cache pools and their views at
    past + rows, the visibility workspace the round's bits are written into, the query
    projections and the outputs), so replaying it each round runs exactly the launches
    verify_round would make, without host time between them."""
    import torch
    from analysis_spec_b200 import _ops
    vis = st.tree.visibility(st.past, st.pad, workspace=st.vis_ws)
    end = st.past + st.wl.rows
    views = [(l.key_pool[:st.wl.batch, :, :end], l.value_pool[:st.wl.batch, :, :end]) for l in st.cache.layers]
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for l in range(st.wl.layers):
            if getattr(st, 'fused', False):  # the append fused in: pools read up to past, new rows stored
                _ops.tree_attention_bits_append(st.queries[l], st.cache.layers[l].key_pool[:st.wl.batch],
                                                st.cache.layers[l].value_pool[:st.wl.batch], st.past, st.keys[l],
                                                st.values[l], vis.bits, vis.first_col, st.scale, out=st.out[l])
            else:
                _ops.tree_attention_bits(st.queries[l], views[l][0], views[l][1], vis.bits, vis.first_col, st.scale,
                                         out=st.out[l])
    torch.cuda.synchronize()
    return graph


def run_side(args):
    """The draft-step and history-step measurements alone, on a one-layer cache of the workload
    (a small device footprint for kernel profiling); prints one JSON line."""
    import torch
    from dataclasses import replace
    from analysis_spec_b200 import _lib
    from analysis_spec_b200.build import build
    build()
    device = torch.device('cuda', 0)
    torch.cuda.set_device(device)
    _lib.load()
    wl = replace(workload(args), layers=1)
    st = Round(wl, device, seed=1000)
    print(json.dumps({'impl': 'ours', 'side_only': True, 'config': workload_config(wl),
                      'draft_step': measure_draft(st, iters=args.steps, warmup=args.warmup),
                      'history_step': measure_history(st, iters=args.steps, warmup=args.warmup)}), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist
    from analysis_spec_b200 import _lib
    from analysis_spec_b200.build import build
    from analysis_spec_b200.counters import AcceptanceCounters, round_increments

    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    if rank == 0:
        build()
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    if world > 1:
        from datetime import timedelta
        # the job's only collective is a 40-byte counter all_reduce: one NCCL CTA, and the
        # persistent attention leaves that SM free (it runs beside it on a side stream)
        os.environ.setdefault('NCCL_MAX_CTAS', '1')
        dist.init_process_group('nccl', device_id=device, timeout=timedelta(seconds=120))
    _lib.load()
    if world > 1:
        from analysis_spec_b200 import _ops
        _ops.set_attention_ctas(torch.cuda.get_device_properties(device).multi_processor_count -
                                int(os.environ['NCCL_MAX_CTAS']))
    wl = workload(args)
    st = Round(wl, device, seed=1000 + rank)
    st.fold = args.fold
    counters = AcceptanceCounters(device)
    st.counters = counters

    round_rows = []  # the host packet rows of every round, summed after the timed region as a check

    def enqueue_counters():
        # increments computed on the device from the packet, the all_reduce on a side stream;
        # queued before the host waits for the packet, so this host work overlaps the GPU's
        counters.add_device_round(st.packet, wl.batch, wl.nodes)

    def reduce_counters(rows):
        round_rows.append(rows)

    for i in range(args.warmup):
        _, _, rows = verify_round(st, i, on_launched=enqueue_counters)
        reduce_counters(rows)
    torch.cuda.synchronize()
    if not args.no_graph:  # after the warm-up rounds: every first-call set-up has happened
        st.attn_graph = capture_attention(st)
        _, _, rows = verify_round(st, args.warmup, on_launched=enqueue_counters)  # a warm-up round through the graph
        reduce_counters(rows)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = Clocks(f'GPU-{torch.cuda.get_device_properties(device).uuid}') if rank == 0 else None
    if clocks:
        clocks.start()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _lib.profile.reset()
    _lib.profile.enabled = True
    widths = []
    torch.cuda.synchronize()
    start.record()
    for i in range(args.steps):
        w, e, rows = verify_round(st, i, ev[i], on_launched=enqueue_counters)
        reduce_counters(rows)
        widths.append(st.folded if st.fold else (w, e))  # the compaction this step's launches did
    end.record()
    torch.cuda.synchronize()
    _lib.profile.enabled = False
    launches = _lib.profile.calls + (args.steps * wl.layers if not args.no_graph else 0)
    kernel_ms = {name: [s.elapsed_time(e) for s, e in pairs] for name, pairs in _lib.profile.events.items()}
    totals = counters.finish()
    host_totals = [0] * 5
    for rows in round_rows:
        for k, v in enumerate(round_increments(rows, wl.nodes)):
            host_totals[k] += v
    if world > 1:  # the device totals are job-wide: sum the host check over the ranks too
        check = torch.tensor(host_totals, dtype=torch.long, device=device)
        dist.all_reduce(check)
        host_totals = check.tolist()
    totals['matches_host_packet_rows'] = list(totals.values()) == host_totals
    if world > 1:
        dist.barrier()
    clock = clocks.stop() if clocks else None
    total_ms = start.elapsed_time(end)
    # KV commit = the append launch + the device-scheduled commit launch of every step, each timed by
    # CUDA events recorded around the launch on the launching stream
    append_name = 'speckv_append_commit_rows' if st.fold else 'speckv_append_rows'
    commit_ms = sum(kernel_ms[append_name]) + sum(kernel_ms['speckv_commit_round'])
    region_ms = sum(ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps))
    verify_ms = sum(ev[i][0].elapsed_time(ev[i][1]) + ev[i][2].elapsed_time(ev[i][3]) for i in range(args.steps))
    attn_ms = sum(ev[i][2].elapsed_time(ev[i][3]) for i in range(args.steps))
    commit_bytes = sum(st.append_bytes + st.compact_bytes(w, e) for w, e in widths)
    # where a step's device time goes, per phase (ms per step): marks 0-4 of verify_round, and the
    # time from a round's last mark to the next round's first one (host work between rounds,
    # after the packet read-back, while the GPU has nothing queued)
    phases = [sum(ev[i][j].elapsed_time(ev[i][j + 1]) for i in range(args.steps)) / args.steps for j in range(4)]
    between = (sum(ev[i][4].elapsed_time(ev[i + 1][0]) for i in range(args.steps - 1)) / (args.steps - 1)
               if args.steps > 1 else 0.0)
    times = torch.tensor([total_ms, commit_ms, verify_ms, attn_ms, region_ms, *phases, between], device=device,
                         dtype=torch.float64)
    moved = torch.tensor([float(commit_bytes)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(moved)
    total_ms, commit_ms, verify_ms, attn_ms, region_ms, *phases, between = times.tolist()
    job_commit_bytes = moved.item()

    # the same rounds with the append fused into the attention launches (rank 0, after the line)
    # (a rank-0-only measurement: its counters reduce nothing across ranks when the job has several)
    fused = measure_fused(st, args.steps, args.warmup, not args.no_graph,
                          AcceptanceCounters(device) if world == 1 else None) if rank == 0 and not st.fold else None
    if fused is not None:  # DRAM bytes of one fused launch, from the committed ncu capture
        fused['traffic'], fused['traffic_source'] = dram_traffic('speckv_tree_attention_bits_append', wl.layers,
                                                                 wl.name)
    e2e = None if args.no_e2e else measure_e2e(st, args, world)
    draft = measure_draft(st) if rank == 0 else None
    history = measure_history(st) if rank == 0 else None
    release = measure_release(st) if rank == 0 else None
    hbm, tflops, peak_kind = peaks()
    append_ms = float(np.mean(kernel_ms[append_name]))
    # bytes of one launch of that kernel: the append, plus the folded compaction's on average
    append_launch_bytes = st.append_bytes + (np.mean([st.compact_bytes(w, e) for w, e in widths]) if st.fold else 0)
    append_gbs = append_launch_bytes / (append_ms * 1e-3) / 1e9
    if args.no_graph:
        attn_launch_ms = float(np.mean(kernel_ms['speckv_tree_attention_bits']))
    else:  # the graph region holds the layers' launches back to back: its device time / layers
        attn_launch_ms = attn_ms / args.steps / wl.layers
        kernel_ms['speckv_tree_attention_bits'] = [attn_launch_ms]
    attn_tflops = st.attention_flops() / wl.layers / (attn_launch_ms * 1e-3) / 1e12
    value = job_commit_bytes / (commit_ms * 1e-3) / 1e9
    attn_traffic = dram_traffic('speckv_tree_attention_bits', wl.layers, wl.name)
    append_traffic = dram_traffic(append_name, wl.layers, wl.name)
    result = {
        'metric': METRIC, 'value': round(value, 2), 'unit': 'GB/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(total_ms / args.steps, 4), 'higher_is_better': True,
        'scaling': 'strong' if wl.extra.get('split_batch') else 'weak', 'vs_baseline': None, 'dtype': 'bf16',
        'data': 'synthetic (seeded)',
        'config': workload_config(wl, {'parallelism': f'sequence-sharded x{world}',
                                       'global_batch': wl.batch * world}),
        'kv_commit': {'gbs': round(value, 2), 'frac_hbm': round(value / world / hbm, 4), 'peak_gbs': hbm,
                      'ms_per_step': round(commit_ms / args.steps, 4),
                      'bytes_per_step_per_gpu': commit_bytes // args.steps,
                      'launches': [append_name, 'speckv_commit_round'],
                      'compaction': ('folded into the next round\'s append launch; the round\'s own commit launch '
                                     'updates positions / padding only') if st.fold else
                                    'in the round\'s commit launch',
                      'append_region_ms_per_step': round(region_ms / args.steps, 4)},
        'tree_verify': {'steps_per_s': round(world * args.steps / (verify_ms * 1e-3), 3),
                        'ms_per_step': round(verify_ms / args.steps, 4),
                        'attention_tflops': round(attn_tflops, 2),
                        'roofline': {'bound': 'tensor', 'achieved': round(attn_tflops, 2), 'peak': tflops,
                                     'unit': 'TFLOP/s', 'frac': round(attn_tflops / tflops, 4),
                                     'traffic': attn_traffic[0], 'traffic_source': attn_traffic[1],
                                     'peak_kind': peak_kind}},
        'roofline': {'bound': 'hbm', 'kernel': f'{append_name} (all layers)', 'achieved': round(append_gbs, 1),
                     'peak': hbm, 'unit': 'GB/s', 'frac': round(append_gbs / hbm, 4),
                     'traffic': append_traffic[0], 'traffic_source': append_traffic[1],
                     'peak_kind': peak_kind, 'bytes_per_launch': int(append_launch_bytes)},
        'kernel_ms': {k: round(float(np.mean(v)), 5) for k, v in kernel_ms.items()},
        'step_phases_ms': {'visibility': round(phases[0], 4), 'append': round(phases[1], 4),
                           'attention': round(phases[2], 4), 'trace_schedule_commit_readback': round(phases[3], 4),
                           'between_rounds': round(between, 4), 'max_over_ranks': True},
        'gpu_launches': launches,
        'attention_launches': attention_launches(),
        'acceptance': totals,
        'clocks': clock,
        'e2e': e2e,
        'draft_step': draft,
        'history_step': history,
        'release_step': release,
        'fused_append': fused,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result['cpu_baseline'] = cpu_baseline(wl, budget_s=10.0)
        result['cpu_baseline_c_port'] = c_port_baseline(wl, budget_s=6.0)
        result['cpu_baseline_attention'] = cpu_attention_baseline(wl, budget_s=6.0)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def attention_launches():
    """Attention launches the library issued in this process, per kernel family (calls only:
    graph replays are not counted); cuda_core > 0 would mean a shape left the tensor cores."""
    import ctypes
    from analysis_spec_b200 import _lib
    tc, cc = ctypes.c_int64(0), ctypes.c_int64(0)
    _lib.call('speckv_attention_launches', ctypes.byref(tc), ctypes.byref(cc))
    return {'tensor_core': tc.value, 'cuda_core': cc.value}


def time_steps(fn, iters, warmup, spin_ms=8.0):
    """(device µs, launch-bound µs) per call of `fn`. Device: the `iters` calls are queued
    behind a GPU spin of `spin_ms` so the host enqueues them all before the GPU reaches the
    first, and the CUDA events around them see device time only (None if enqueueing took
    longer than the spin). Launch-bound: the same calls back to back on an idle GPU, host
    launch cost included."""
    import torch
    for _ in range(warmup):
        fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(spin_ms * 1e-3 * 2.0e9))
    t0 = time.perf_counter()
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    host_ms = (time.perf_counter() - t0) * 1e3
    torch.cuda.synchronize()
    device = a.elapsed_time(b) * 1e3 / iters if host_ms < 0.8 * spin_ms else None
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return device, a.elapsed_time(b) * 1e3 / iters


def _r(x):
    return None if x is None else round(x, 2)


def measure_draft(st, iters=20, warmup=3):
    """One draft expansion step of one draft layer at the workload's batch, heads and shared
    past (draft K = the tree's top-k): the expansion mask and the draft attention, each as
    this library's launch and as the reference's torch sequence on the same GPU (zero /
    [init:] fill / scatter / padding fill, helper/opd_generate.py:143-162; repeat_kv + SDPA,
    helper/fastgrpo_model.py:58-69), each timed by time_steps; the K/V views (> L2) are
    strided cache views."""
    import torch
    import torch.nn.functional as F
    from analysis_spec_b200.draft_attention import draft_sdpa
    from analysis_spec_b200.opd_attention import expansion_mask
    wl, dev, dtype = st.wl, st.device, st.dtype
    B, Hkv, Hq, D, k = wl.batch, wl.kv_heads, wl.q_heads, wl.dim, wl.topk
    past = st.past
    cols = past + k
    init = past - 2 * k
    gen = torch.Generator(device=dev).manual_seed(11)
    pool_k = torch.randn(B, Hkv, cols + 256, D, device=dev, generator=gen).to(dtype)
    pool_v = torch.randn(B, Hkv, cols + 256, D, device=dev, generator=gen).to(dtype)
    keys, values = pool_k[:, :, :cols], pool_v[:, :, :cols]
    q = torch.randn(B, Hq, k, D, device=dev, generator=gen).to(dtype)
    seen = torch.randint(init, cols, (B, k, 1), device=dev, generator=gen)
    pad = st.pad
    mask = torch.empty(B, 1, k, cols, device=dev, dtype=dtype)
    lowest = torch.finfo(dtype).min
    g = Hq // Hkv

    def ours_mask():
        expansion_mask(mask, init, seen, pad)

    def torch_mask():
        mask.zero_()
        mask[..., init:] = lowest
        mask.scatter_(dim=-1, index=seen.unsqueeze(1), value=0.)
        mask.masked_fill_(pad[:, None, None, :cols], lowest)

    def ours_attn():
        draft_sdpa(q, keys, values, mask, g)

    def torch_attn():
        kk = keys[:, :, None].expand(B, Hkv, g, cols, D).reshape(B, Hq, cols, D)
        vv = values[:, :, None].expand(B, Hkv, g, cols, D).reshape(B, Hq, cols, D)
        F.scaled_dot_product_attention(q, kk, vv, attn_mask=mask)

    torch_mask()
    ref_mask = mask.clone()
    ours_mask()
    same = bool(torch.equal(mask.view(torch.int16), ref_mask.view(torch.int16)))
    t = {name: time_steps(fn, iters, warmup) for name, fn in
         (('mask', ours_mask), ('mask_torch', torch_mask), ('attn', ours_attn), ('attn_torch', torch_attn))}
    out = {'shape': f'batch {B}, draft_k {k}, columns {cols}, {Hq}q/{Hkv}kv x {D}, one draft layer',
           'mask_us': _r(t['mask'][0]), 'mask_us_torch_sequence': _r(t['mask_torch'][0]),
           'attention_us': _r(t['attn'][0]), 'attention_us_torch_sdpa': _r(t['attn_torch'][0]),
           'launch_bound_us': {k2: _r(v[1]) for k2, v in t.items()},
           'timing': 'device time per step (steps queued behind a GPU spin); launch_bound_us: back to back on an '
                     'idle GPU, host launch cost included',
           'mask_bit_exact_vs_torch_sequence': same}
    del pool_k, pool_v
    return out


def measure_history(st, iters=20, warmup=3, hidden=2048):
    """The verify round's history step at the workload's batch (two responses per prompt):
    gather of the accepted target features (hidden size `hidden`, bf16) from the tree's
    hidden states and their append with the emitted tokens to the rollout-history pools,
    as this library's one launch (ContiguousRolloutHistory.append_accepted) and as the
    reference's torch sequence (gather, then one index_copy_ per field,
    helper/opd_generate.py:567-579, helper/opd_history.py:24-42), each timed by time_steps."""
    import torch
    from analysis_spec_b200.opd_history import ContiguousRolloutHistory
    wl, dev, dtype = st.wl, st.device, st.dtype
    B, R, W = wl.batch, wl.rows, wl.depth + 1
    gen = torch.Generator(device=dev).manual_seed(13)
    init = {'generated_ids': torch.randint(0, 150000, (B // 2, 1), device=dev, generator=gen),
            'features': torch.randn(B // 2, 1, hidden, device=dev, generator=gen).to(dtype),
            'input_ids': torch.randint(0, 150000, (B // 2, 1), device=dev, generator=gen)}
    cap = 1 + (warmup + 2 * iters) * W + W
    ours = ContiguousRolloutHistory(init, repeats=2, max_length=cap)
    pools = {k: v.clone() for k, v in ours.buffers.items()}
    tree = torch.randn(B, R, hidden, device=dev, generator=gen).to(dtype)
    index = torch.sort(torch.rand(B, R, device=dev, generator=gen).argsort(dim=1)[:, :W], dim=1).values
    tok = torch.randint(0, 150000, (B, W), device=dev, generator=gen)
    owners = torch.randperm(B, device=dev, generator=gen)
    rows = owners.tolist()
    state = {'start': 1}

    def ours_step():
        ours.append_accepted(rows, tok, tree, index, owners=owners)

    def torch_step():
        start = state['start']
        feats = tree.gather(dim=1, index=index.unsqueeze(-1).expand(B, -1, hidden))
        for name, chunk in (('generated_ids', tok), ('features', feats), ('input_ids', tok)):
            pools[name][:, start:start + W].index_copy_(0, owners, chunk)
        state['start'] = start + W

    (t_ours, lb_ours), (t_torch, lb_torch) = time_steps(ours_step, iters, warmup), time_steps(torch_step, iters,
                                                                                               warmup)
    es = torch.finfo(dtype).bits // 8
    moved = B * W * (hidden * es * 3 + 8 * 2 * 2)  # features read once, written twice; ids read + written
    same = all(torch.equal(ours.buffers[k][:, :state['start']], pools[k][:, :state['start']]) for k in pools)
    return {'shape': f'{B} rows, width {W}, {R}-row trees, hidden {hidden} {wl.dtype}', 'us': _r(t_ours),
            'us_torch_sequence': _r(t_torch), 'bytes_per_step': moved,
            'gbs': None if t_ours is None else round(moved / (t_ours * 1e-6) / 1e9, 1),
            'launch_bound_us': {'ours': _r(lb_ours), 'torch_sequence': _r(lb_torch)},
            'timing': 'device time per step (steps queued behind a GPU spin); launch_bound_us: back to back on an '
                      'idle GPU, host launch cost included',
            'bit_exact_vs_torch_sequence': bool(same)}


def measure_fused(st, steps, warmup, graph, counters=None):
    """The same verify rounds with each layer's append fused into its attention launch
    (speckv_tree_attention_bits_append, through OPDStaticCache.update_attend; with `graph`
    the 36 fused launches replay from a CUDA graph as the line's attention does): the round
    has no append launch, the attention launches store the tree rows. Run after the line's
    timed rounds on the same cache, with the acceptance counters of the line's rounds when
    `counters` is given; device time from CUDA events around the round's phases."""
    import torch
    wl = st.wl
    saved = getattr(st, "attn_graph", None)
    st.fused, st.attn_graph = True, None

    def enqueue():
        counters.add_device_round(st.packet, wl.batch, wl.nodes)

    hook = enqueue if counters is not None else None
    try:
        for i in range(warmup):
            verify_round(st, i, on_launched=hook)
        torch.cuda.synchronize()
        if graph:
            st.attn_graph = capture_attention(st)
            verify_round(st, warmup, on_launched=hook)
            torch.cuda.synchronize()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(steps):
            verify_round(st, i, ev[i], on_launched=hook)
        end.record()
        torch.cuda.synchronize()
    finally:
        st.fused, st.attn_graph = False, saved
    phases = [sum(ev[i][j].elapsed_time(ev[i][j + 1]) for i in range(steps)) / steps for j in range(4)]
    between = (sum(ev[i][4].elapsed_time(ev[i + 1][0]) for i in range(steps - 1)) / (steps - 1)
               if steps > 1 else 0.0)
    per_layer_us = phases[2] / wl.layers * 1e3
    return {'ms_per_step': round(start.elapsed_time(end) / steps, 4),
            'verify_ms_per_step': round(phases[0] + phases[2], 4),
            'attention_with_append_us_per_layer': round(per_layer_us, 2),
            'attention_tflops': round(st.attention_flops() / wl.layers / (per_layer_us * 1e-6) / 1e12, 2),
            'step_phases_ms': {'visibility': round(phases[0], 4), 'append': round(phases[1], 4),
                               'attention_with_append': round(phases[2], 4),
                               'trace_schedule_commit_readback': round(phases[3], 4),
                               'between_rounds': round(between, 4)},
            'append_launches_per_step': 0, 'kv_bytes_stored_by_attention_per_step': st.append_bytes // 2,
            'acceptance_counters': counters is not None,
            'launch': 'speckv_tree_attention_bits_append per layer' + (' (CUDA graph)' if graph else '')}


def measure_release(st, fraction=0.25, spin_ms=8.0):
    """Release of `fraction` of the sequences after the timed rounds, at the workload's layers,
    batch and length: the reference's swap_remove (the surviving tail sequences' whole
    histories moved into the holes, all layers in one move_rows launch; device time with the
    launch queued behind a GPU spin) against a row-table cache, where the release rewrites the
    table (host time of the call, which stages and uploads the table). The table release moves
    no KV bytes whatever the pools' size, so its cache holds a one-position history."""
    import torch
    from analysis_spec_b200.opd_static_cache import OPDStaticCache, swap_remove_plan
    wl, dev = st.wl, st.device
    rng = np.random.RandomState(17)
    batch = st.cache.layers[0].batch_size
    finished = [False] * batch
    for i in rng.choice(batch, size=max(1, int(batch * fraction)), replace=False):
        finished[i] = True
    keep, sources, dests = swap_remove_plan(finished)
    layer = st.cache.layers[0]
    moved = len(sources) * 2 * wl.layers * layer.key_pool.shape[1] * layer.length * layer.key_pool.shape[-1] * \
        layer.key_pool.element_size()
    src = torch.tensor(sources, device=dev, dtype=torch.long)
    dst = torch.tensor(dests, device=dev, dtype=torch.long)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(spin_ms * 1e-3 * 2.0e9))
    a.record()
    st.cache.swap_remove(len(keep), src, dst)
    b.record()
    torch.cuda.synchronize()
    physical_us = a.elapsed_time(b) * 1e3
    table_cache = OPDStaticCache(256, batch_capacity=batch, row_table=True)
    one = torch.zeros(batch, layer.key_pool.shape[1], 1, layer.key_pool.shape[-1], device=dev, dtype=st.dtype)
    table_cache.update_layers([one] * wl.layers, [one] * wl.layers)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    table_cache.swap_remove(len(keep), sources, dests)
    host_us = (time.perf_counter() - t0) * 1e6
    torch.cuda.synchronize()
    return {'released': len(finished) - len(keep), 'moved_by_swap_remove': len(sources),
            'swap_remove_us_device': round(physical_us, 2), 'swap_remove_bytes': moved,
            'swap_remove_gbs': round(moved / (physical_us * 1e-6) / 1e9, 1) if physical_us > 0 else None,
            'row_table_us_host': round(host_us, 2), 'row_table_kv_bytes': 0,
            'shape': f'{wl.layers} layers, batch {batch}, length {layer.length}, {layer.key_pool.shape[1]} kv heads '
                     f'x {layer.key_pool.shape[-1]}'}


def measure_e2e(st, args, world):
    """KV commit through the public API with inputs from pinned host memory and the packet read back.

    Every step's new K/V rows (all layers, one pinned block) are copied host to device on a
    copy stream into one of two device blocks while the previous step's commit runs and the
    host waits for its packet; the append of a step waits for its copy, the copy into a block
    waits until the step that last read it has appended. All copies and read-backs of the
    timed steps happen between the two events."""
    import torch
    from analysis_spec_b200 import tree_kernels
    from analysis_spec_b200.opd_scheduling import schedule_commit
    from analysis_spec_b200.tree_verification import trace_verified_path
    L, (B, R, HD) = st.wl.layers, tuple(st.k_proj[0].shape)
    H = st.wl.kv_heads
    host = torch.empty((2 * L, B, R, HD), dtype=st.k_proj[0].dtype).pin_memory()
    for l in range(L):
        host[l].copy_(st.k_proj[l])
        host[L + l].copy_(st.v_proj[l])
    host_s = [s.cpu().pin_memory() for s in st.samples]
    dev = [torch.empty_like(host, device=st.device) for _ in range(2)]
    dev_s = [torch.empty_like(st.samples[0]) for _ in range(2)]
    views = [([d[l].view(B, R, H, HD // H).transpose(1, 2) for l in range(L)],
              [d[L + l].view(B, R, H, HD // H).transpose(1, 2) for l in range(L)]) for d in dev]
    h2d = host.numel() * host.element_size() + host_s[0].numel() * 8
    d2h = st.packet[:, :st.wl.depth + 4].numel() * 8
    steps = max(2, min(args.steps, 10))
    compute = torch.cuda.current_stream(st.device)
    copy = torch.cuda.Stream(st.device)
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def upload(i, after=None):
        j = i % 2
        with torch.cuda.stream(copy):
            if after is not None:
                copy.wait_event(after)
            if i >= 2:
                copy.wait_event(freed[j])
            dev[j].copy_(host, non_blocking=True)
            dev_s[j].copy_(host_s[i % len(host_s)], non_blocking=True)
            copied[j].record(copy)

    def one(i, resident=False):
        j = 0 if resident else i % 2
        if not resident:
            compute.wait_event(copied[j])
        st.cache.update_layers(*views[j])
        path = trace_verified_path(st.tree, dev_s[j], EOS, workspace=st.path_ws)
        if not resident:
            freed[j].record(compute)
        rows, _, _, _, _, width = schedule_commit(path, st.past, EOS, st.pad_ws, st.packet, st.cache, st.positions,
                                                  st.past_positions, pad_rows=st.pad_commit, owners=st.owners,
                                                  kernels=tree_kernels)
        live = [r for r in rows if r[1] == 0]
        ext = min(r[2] for r in live) if live else width
        st.cache.crop(st.past)
        return st.append_bytes + st.compact_bytes(width, ext)

    def run(n, start=None):
        upload(0, start)
        moved = 0
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            moved += one(i)
        return moved

    run(2)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(compute)
    moved = run(steps, start=s)
    e.record(compute)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    # the same loop with the new rows already on the device: what the API costs without PCIe
    # (host work, launches and the packet read-back of every step)
    s.record(compute)
    moved_r = sum(one(i, resident=True) for i in range(steps))
    e.record(compute)
    torch.cuda.synchronize()
    ms_r = s.elapsed_time(e)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms, ms_r], device=st.device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        m = torch.tensor([float(moved), float(moved_r)], device=st.device, dtype=torch.float64)
        dist.all_reduce(m)
        (ms, ms_r), (moved, moved_r) = t.tolist(), m.tolist()
    return {'value': round(moved / (ms * 1e-3) / 1e9, 3), 'unit': 'GB/s', 'h2d_bytes_per_step': h2d,
            'd2h_bytes_per_step': d2h, 'steps': steps,
            'device_resident': {'value': round(moved_r / (ms_r * 1e-3) / 1e9, 3), 'unit': 'GB/s',
                                'ms_per_step': round(ms_r / steps, 4), 'h2d_bytes_per_step': 0,
                                'd2h_bytes_per_step': d2h,
                                'what': 'the same public-API loop (append of all layers, trace, schedule, device '
                                        'commit, packet read-back) with the new rows already on the GPU'}}


# ---------------------------------------------------------------------------
# CPU: the oracle's restatement of the reference's KV commit
# ---------------------------------------------------------------------------
class CpuCommit:
    """Bounded sample of the KV commit on host cores: `layers` of the workload's layers, full batch."""

    def __init__(self, wl, layers, seed=7):
        from analysis_spec_b200 import workloads as W
        from oracle import oracle
        self.oracle = oracle
        oracle.set_threads(os.cpu_count() or 1)
        rng = np.random.RandomState(seed)
        self.wl, self.layers = wl, layers
        B, R, H, D = wl.batch, wl.rows, wl.kv_heads, wl.dim
        itemsize = 2 if wl.dtype != 'float32' else 4
        dt = np.uint16 if itemsize == 2 else np.float32
        self.past = int(W.prefix_lengths(rng, wl.prefix, B).max())
        cap = self.past + R
        self.kp = [rng.randint(0, 1 << 15, size=(B, H, cap, D)).astype(dt) for _ in range(layers)]
        self.vp = [rng.randint(0, 1 << 15, size=(B, H, cap, D)).astype(dt) for _ in range(layers)]
        self.src = [rng.randint(0, 1 << 15, size=(B, R, H, D)).astype(dt).transpose(0, 2, 1, 3)
                    for _ in range(2 * layers)]
        parents, tokens = W.packed_trees(rng, B, wl.nodes, wl.depth, wl.topk)
        self.parents, self.tokens = parents, tokens
        self.samples = [W.samples_for(rng, parents, tokens, W.accepted_lengths(rng, wl.accept, B)) for _ in range(4)]
        self.append_bytes = layers * 2 * 2 * B * H * R * D * itemsize
        self.row_bytes = D * itemsize

    def step(self, i):
        o, wl = self.oracle, self.wl
        for l in range(self.layers):
            o.append(self.kp[l], self.vp[l], self.src[2 * l], self.src[2 * l + 1], self.past)
        ctx = np.zeros_like(self.parents)
        pt, pi, pc, pl = o.trace_path(self.parents, self.tokens, ctx, self.samples[i % 4], EOS, wl.depth + 1)
        _, idx, _, _, packet, width = o.pad_schedule(pt, pi, pl, self.past, EOS)
        live = packet[packet[:, 1] == 0]
        ext = int(live[:, 2].min()) if len(live) else width
        for l in range(self.layers):
            o.compact_suffix(self.kp[l], self.vp[l], wl.batch, self.past + wl.rows, idx, self.past, ext)
        return self.append_bytes + self.layers * 2 * 2 * wl.batch * wl.kv_heads * (width - ext) * self.row_bytes


def c_port_baseline(wl, budget_s=6.0, layers=4):
    """The C/OpenMP restatement of the commit (a much faster CPU code than the reference's)."""
    cpu = CpuCommit(wl, layers)
    cpu.step(0)
    moved, steps, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        moved += cpu.step(steps)
        steps += 1
    dt = time.perf_counter() - t0
    return {'value': round(moved / dt / 1e9, 4), 'unit': 'GB/s', 'cores': cpu.oracle.max_threads(), 'kind': 'port',
            'sample': f'{layers} of {wl.layers} layers per step (full batch {wl.batch}, {wl.rows} tree rows), '
                      f'{steps} steps in {dt:.1f} s: append + trace + schedule + compaction by the C/OpenMP oracle'}


def torch_commit(wl, seed=7):
    """The reference's torch CPU branch of the commit, restated on host tensors, all layers."""
    import torch
    from analysis_spec_b200 import workloads as W
    from oracle.torch_commit import TorchCommit
    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.RandomState(seed)
    past = int(W.prefix_lengths(rng, wl.prefix, wl.batch).max())
    parents, tokens = W.packed_trees(rng, wl.batch, wl.nodes, wl.depth, wl.topk)
    samples = [W.samples_for(rng, parents, tokens, W.accepted_lengths(rng, wl.accept, wl.batch)) for _ in range(4)]
    return TorchCommit(wl.layers, wl.batch, wl.kv_heads, wl.dim, wl.rows, past, parents, tokens, samples, wl.depth,
                       dtype=getattr(torch, wl.dtype))


def torch_commit_sample(wl, rounds):
    pin = ROOT / 'oracle' / 'torch_commit_pin.json'
    pinned = ''
    if pin.exists():
        p = json.loads(pin.read_text())
        pinned = (f"; pinned against the reference's own code on {p['threads']} threads of {p['cpu']}: "
                  f"caches identical, {p['reference_s_per_round']} s per round for the reference vs "
                  f"{p['restatement_s_per_round']} s for the restatement")
    return (f'{rounds} verify rounds of all {wl.layers} layers (batch {wl.batch}, {wl.rows} tree rows, {wl.dtype}): '
            'the reference torch CPU branch restated (per layer two copy_ appends, torch.gather of the accepted '
            'rows into a reused scratch and a copy back; trace + schedule; position update)' + pinned)


def cpu_baseline(wl, budget_s=10.0):
    import torch
    tc = torch_commit(wl)
    tc.round(0, EOS)
    moved, rounds, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        moved += tc.round(rounds, EOS)
        rounds += 1
    dt = time.perf_counter() - t0
    return {'value': round(moved / dt / 1e9, 4), 'unit': 'GB/s', 'cores': torch.get_num_threads(), 'kind': 'port',
            'sample': torch_commit_sample(wl, rounds) + f', {dt:.1f} s'}


def cpu_attention_baseline(wl, budget_s=6.0):
    """The reference's tree-verify attention on the host cores: transformers'
    sdpa_attention_forward (repeat_kv of K / V, then torch's scaled_dot_product_attention with
    the dense additive tree mask; the call the reference's verify forward makes) over one layer
    of a bounded sample of the workload's sequences, in the workload's dtype. TFLOP/s counts the
    same algorithmic flops as the GPU figure (4 Hq R (P + R) D per sequence)."""
    import torch
    from types import SimpleNamespace
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    from analysis_spec_b200 import workloads as W
    from oracle import oracle
    rng = np.random.RandomState(1000)
    prefix = W.prefix_lengths(rng, wl.prefix, wl.batch)
    parents, _ = W.packed_trees(rng, wl.batch, wl.nodes, wl.depth, wl.topk)
    dtype = getattr(torch, wl.dtype)
    g = torch.Generator().manual_seed(3)
    module = SimpleNamespace(num_key_value_groups=wl.q_heads // wl.kv_heads, is_causal=True, training=False)
    flops, calls, t_all = 0, 0, 0.0
    order = np.argsort(-prefix)  # the sample walks the sequences longest first, then wraps
    while t_all < budget_s:
        b = int(order[calls % wl.batch])
        p = int(prefix[b])
        q = (0.5 * torch.randn(1, wl.q_heads, wl.rows, wl.dim, generator=g)).to(dtype)
        k = (0.5 * torch.randn(1, wl.kv_heads, p + wl.rows, wl.dim, generator=g)).to(dtype)
        v = (0.5 * torch.randn(1, wl.kv_heads, p + wl.rows, wl.dim, generator=g)).to(dtype)
        vis = oracle.tree_visible(parents[b:b + 1], p, wl.depth + 1)
        mask = torch.from_numpy(np.where(vis, 0.0, np.float32(torch.finfo(dtype).min))).to(dtype)[:, None]
        t0 = time.perf_counter()
        sdpa_attention_forward(module, q, k, v, mask, dropout=0.0, scaling=wl.dim ** -0.5)
        t_all += time.perf_counter() - t0
        flops += 4 * wl.q_heads * wl.rows * (p + wl.rows) * wl.dim
        calls += 1
    return {'value': round(flops / t_all / 1e12, 5), 'unit': 'TFLOP/s', 'cores': torch.get_num_threads(),
            'kind': 'reference',
            'sample': f'{calls} single-sequence verify layers (longest prefixes first) through transformers '
                      f'sdpa_attention_forward on the host cores, {wl.dtype}, {t_all:.1f} s'}


def run_reference(args):
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    import torch
    wl = workload(args)
    tc = torch_commit(wl)
    for i in range(args.warmup):
        tc.round(i, EOS)
    moved, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        moved += tc.round(i, EOS)
    dt = time.perf_counter() - t0
    value = moved / dt / 1e9
    print(json.dumps({
        'impl': 'reference', 'metric': METRIC, 'value': round(value, 4), 'unit': 'GB/s', 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(dt * 1e3 / args.steps, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded)',
        'config': workload_config(wl, {'parallelism': f'sequence-sharded x{args.gpus}',
                                       'global_batch': wl.batch * args.gpus}),
        'cpu_baseline': {'value': round(value, 4), 'unit': 'GB/s', 'cores': torch.get_num_threads(), 'kind': 'port',
                         'sample': torch_commit_sample(wl, args.steps)},
        'e2e': {'value': round(value, 4), 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }), flush=True)


def run_rollout(args):
    """Rollout workloads (a fraction of the sequences finishes every step): each timed step is
    a verify round (append, attention of every layer, trace, schedule, device commit, crop)
    followed by the release of the finished sequences (the reference's swap_remove: the
    surviving tail sequences' histories move into the holes; with --row-table a table rewrite)
    and the admission of as many new sequences with fresh prefixes (one append launch for all
    layers into the freed rows). KV-commit GB/s counts append + compaction + release +
    admission bytes (each moved byte read once and written once; admission counts the new
    prefixes' own positions) over the device time of those launches."""
    import torch
    import torch.distributed as dist
    from analysis_spec_b200 import _lib, _ops
    from analysis_spec_b200 import workloads as W
    from analysis_spec_b200.build import build
    from analysis_spec_b200.counters import AcceptanceCounters
    from analysis_spec_b200.opd_static_cache import swap_remove_plan

    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    if rank == 0:
        build()
    torch.cuda.set_device(local)
    device = torch.device('cuda', local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault('NCCL_MAX_CTAS', '1')  # see run_ours
        dist.init_process_group('nccl', device_id=device, timeout=timedelta(seconds=120))
    _lib.load()
    if world > 1:
        _ops.set_attention_ctas(torch.cuda.get_device_properties(device).multi_processor_count -
                                int(os.environ['NCCL_MAX_CTAS']))
    wl = workload(args)
    _ops.set_attention_chunks(wl.extra.get('attention_chunks', False))
    st = Round(wl, device, seed=1000 + rank, row_table=args.row_table)
    counters = AcceptanceCounters(device)
    B, H, D, L = wl.batch, wl.kv_heads, wl.dim, wl.layers
    k_new = max(1, int(round(B * wl.finish_fraction)))
    es = st.dtype.itemsize if hasattr(st.dtype, 'itemsize') else 2
    rng = np.random.RandomState(4242 + rank)
    # fresh prefixes of the admitted sequences, left-padded to the shared length (one source for all layers)
    gen = torch.Generator(device=device).manual_seed(77 + rank)
    fresh_k = (wl.qkv_scale * torch.randn(k_new, H, st.past, D, device=device, generator=gen)).to(st.dtype)
    fresh_v = (wl.qkv_scale * torch.randn(k_new, H, st.past, D, device=device, generator=gen)).to(st.dtype)
    cols = st.pad.shape[1]

    def step(i, ev):
        w, e, rows = verify_round(st, i, on_launched=lambda: counters.add_device_round(st.packet, B, wl.nodes))
        commit = st.append_bytes + st.compact_bytes(w, e)
        finished = [False] * B
        for j in rng.choice(B, size=k_new, replace=False):
            finished[j] = True
        keep, sources, holes = swap_remove_plan(finished)
        length = st.cache.layers[0].length
        ev[0].record()
        st.cache.swap_remove(len(keep), torch.tensor(sources, dtype=torch.long, device=device),
                             torch.tensor(holes, dtype=torch.long, device=device))
        ev[1].record()
        release = 0 if args.row_table else len(sources) * L * 2 * 2 * H * length * D * es
        new_len = W.prefix_lengths(rng, wl.prefix, k_new)
        st.cache.admit([fresh_k] * L, [fresh_v] * L)
        ev[2].record()
        admit = int(new_len.sum()) * L * 2 * 2 * H * D * es
        # the admitted rows' padding: left padding up to their own prefix, nothing in the tree columns
        pad_new = np.zeros((k_new, cols), dtype=bool)
        pad_new[:, :st.past] = W.left_padding(new_len, st.past)
        st.pad[len(keep):].copy_(torch.from_numpy(pad_new), non_blocking=True)
        return commit, release, admit

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        step(i, evs[i])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = Clocks(f'GPU-{torch.cuda.get_device_properties(device).uuid}') if rank == 0 else None
    if clocks:
        clocks.start()
    _lib.profile.reset()
    _lib.profile.enabled = True
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    moved = np.zeros(3)
    torch.cuda.synchronize()
    start.record()
    for i in range(args.steps):
        moved += step(args.warmup + i, evs[args.warmup + i])
    end.record()
    torch.cuda.synchronize()
    _lib.profile.enabled = False
    totals = counters.finish()
    clock = clocks.stop() if clocks else None
    kernel_ms = {name: [a.elapsed_time(b) for a, b in pairs] for name, pairs in _lib.profile.events.items()}
    timed = evs[args.warmup:]
    release_ms = sum(e[0].elapsed_time(e[1]) for e in timed)
    admit_ms = sum(e[1].elapsed_time(e[2]) for e in timed)
    commit_calls = kernel_ms.get('speckv_commit_round', [])
    append_calls = kernel_ms.get('speckv_append_rows', [])
    # append_rows serves both the round's append (deferred plan) and the admission (one call per step)
    round_append_ms = sum(append_calls) - (admit_ms if not args.row_table else 0)
    commit_ms = sum(commit_calls) + max(round_append_ms, 0.0) + release_ms + admit_ms
    attn_ms = sum(kernel_ms.get('speckv_tree_attention_bits', []))
    total_ms = start.elapsed_time(end)
    times = torch.tensor([total_ms, commit_ms, attn_ms], device=device, dtype=torch.float64)
    job = torch.tensor(moved, device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(job)
        dist.barrier()
        dist.destroy_process_group()
    total_ms, commit_ms, attn_ms = times.tolist()
    commit_b, release_b, admit_b = job.tolist()
    value = (commit_b + release_b + admit_b) / (commit_ms * 1e-3) / 1e9
    hbm, tflops, peak_kind = peaks()
    attn_tflops = st.attention_flops() / (attn_ms / args.steps * 1e-3) / 1e12
    if rank == 0:
        print(json.dumps({
            'metric': METRIC, 'value': round(value, 2), 'unit': 'GB/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': round(total_ms / args.steps, 4), 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic (seeded)',
            'config': workload_config(wl, {'parallelism': f'sequence-sharded x{world}',
                                           'release': 'row table' if args.row_table else 'swap_remove (moves)',
                                           'finish_per_step': k_new}),
            'kv_commit': {'gbs': round(value, 2), 'frac_hbm': round(value / world / hbm, 4),
                          'bytes_per_step_job': {'append_compact': commit_b / args.steps,
                                                 'release': release_b / args.steps, 'admit': admit_b / args.steps},
                          'ms_per_step': round(commit_ms / args.steps, 4),
                          'release_ms_per_step': round(release_ms / args.steps, 4),
                          'admit_ms_per_step': round(admit_ms / args.steps, 4)},
            'tree_verify': {'steps_per_s': round(args.steps / (attn_ms * 1e-3), 3),
                            'attention_tflops': round(attn_tflops, 2),
                            'roofline': {'bound': 'tensor', 'achieved': round(attn_tflops, 2), 'peak': tflops,
                                         'unit': 'TFLOP/s', 'frac': round(attn_tflops / tflops, 4),
                                         'peak_kind': peak_kind}},
            'attention_launches': attention_launches(), 'acceptance': totals, 'clocks': clock,
            'gpu_launches': _lib.profile.calls}), flush=True)


if __name__ == '__main__':
    a = parse()
    if a.impl == 'reference':
        run_reference(a)
    elif a.side_only:
        run_side(a)
    else:
        from analysis_spec_b200.workloads import WORKLOADS
        if WORKLOADS[a.workload].finish_fraction > 0:
            run_rollout(a)
        else:
            run_ours(a)
