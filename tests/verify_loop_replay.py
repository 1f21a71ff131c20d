"""Replay of the reference's verify loop, recorded at the drop-in's module boundary.

`tests/golden/make_verify_loop_trace.py` runs the reference's own
`helper.opd_generate.speculative_generate` (opd_reflex, greedy) on a tiny random
Qwen2 and writes, in order, every outermost call the loop and the model make into
the modules this package replaces (static cache, scheduling, tree verification,
rollout history, attention workspace) plus the target model's attention calls, with
arguments, results and the caches' / histories' state after each call.

`replay(trace)` makes the same calls, in the same order, on this package's objects
on the GPU: caches, histories and workspaces are this package's, created by the
recorded constructor calls and carried from call to call, so every cache byte the
loop would read is produced by libspeckv, while the tensors the model produced (new
K/V rows, queries, sampled tokens) come from the trace. After every call the result
and the state are compared with the reference's: bit for bit for every index, mask,
packet and K/V byte (through SHA-256 of the live rows), within the stated tolerance
for the attention outputs (max |err| <= 2e-2, mean <= 2e-3 against the reference's
bf16 SDPA). `kv_compaction_workspace_bytes` is the one statistic that differs by
design: the compaction here stages rows on chip and keeps no scratch (0 bytes).
"""
import hashlib
import json
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

TRACE = Path(__file__).resolve().parent / 'golden' / 'verify_loop_trace.npz'
SCRATCH_STAT = 'kv_compaction_workspace_bytes'


def load_trace(path=TRACE):
    z = np.load(path)
    meta = json.loads(bytes(z['__trace__']).decode())
    return z, meta


def sha(t):
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()[:20]


def array(z, x, device='cpu'):
    a = torch.from_numpy(np.ascontiguousarray(z[x['tensor']]))
    if x['dtype'] == 'bfloat16':
        a = a.view(torch.bfloat16)
    return a.reshape(x['shape']).to(device)


def host_totals(meta):
    """The reference's acceptance counters recomputed from the recorded schedule packets (the
    loop adds them per packet row: opd_generate.py:551-555)."""
    acc = dec = draft = proposed = 0
    calls = meta['calls']
    for i, c in enumerate(calls):
        if c['fn'] != 'opd_scheduling.schedule':
            continue
        rows = [r['list'] for r in c['out']['tuple'][0]['list']]
        tree_rows = _tree_rows_before(calls, i)
        for r in rows:
            acc += r[0]
            dec += 1
            draft += max(r[0] - 1, 0)
            proposed += tree_rows - 1
    return {'total_acc_length': acc, 'total_decoded_token_num': dec, 'total_accepted_draft_tokens': draft,
            'total_proposed_draft_tokens': proposed}


def _tree_rows_before(calls, i):
    for c in reversed(calls[:i]):
        if c['fn'] == 'tree_verification.trace_verified_path':
            return c['args'][0]['PackedTree'][0]['shape'][1]
    raise AssertionError('schedule without a traced tree')


class Replay:
    """Decodes recorded arguments into this package's objects and checks every result."""

    def __init__(self, z, meta, device='cuda', fused=False):
        from analysis_spec_b200 import opd_attention, opd_history, opd_scheduling, opd_static_cache
        from analysis_spec_b200 import tree_attention, tree_verification
        self.z, self.meta, self.device = z, meta, torch.device(device)
        self.osc, self.osch, self.tv = opd_static_cache, opd_scheduling, tree_verification
        self.oh, self.oa, self.ta = opd_history, opd_attention, tree_attention
        self.objects = {}
        self.attention = []  # (layer, max err, mean err)
        self.schedules = []
        self.statistics = {}
        # fused: the loop's caches run with fuse_append on, so each target layer's update is
        # stored by the attention call after it; results that read a layer with rows still
        # pending (the update's returned views, the state check) are checked after that call
        self.fused = fused
        self.deferred = []

    # ---- decoding ---------------------------------------------------------------------
    def view(self, x):
        layer = self.objects[x['view']].layers[x['layer']]
        pool = layer.key_pool if x['kv'] == 0 else layer.value_pool
        return torch.as_strided(pool, x['shape'], x['stride'], pool.storage_offset() + x['offset'])

    def dec(self, x):
        if x is None or isinstance(x, (bool, int, float, str)):
            return x
        if 'tensor' in x:
            return array(self.z, x, self.device)
        if 'view' in x:
            v = self.view(x)
            layer = self.objects[x['view']].layers[x['layer']]
            if self.fused and layer._pending is not None:
                v._speckv_pending = (layer, layer._pending)  # as the views update returned
                return v
            assert sha(v) == x['sha'], f'input view {x["view"]} layer {x["layer"]} differs before the call'
            return v
        if 'empty' in x:
            return torch.empty(x['empty'], dtype=getattr(torch, x['dtype']), device=self.device)
        if 'torch_dtype' in x:
            return getattr(torch, x['torch_dtype'])
        if 'device' in x:
            return self.device
        if 'list' in x:
            return [self.dec(y) for y in x['list']]
        if 'tuple' in x:
            return tuple(self.dec(y) for y in x['tuple'])
        if 'dict' in x:
            return {k: self.dec(v) for k, v in x['dict']}
        if 'PackedTree' in x:
            p, t, c, depth = x['PackedTree']
            return self.tv.PackedTree(self.dec(p), self.dec(t), self.dec(c), depth)
        if 'VerifiedPath' in x:
            return self.tv.VerifiedPath(*[self.dec(f) for f in x['VerifiedPath']])
        if 'object' in x:
            name = x['object']
            if name not in self.objects:
                assert 'opaque' in x, f'{name} used before it was created'
                # the model (holds the persistent caches) or the OPD runtime (schedule's opd=)
                count = torch.zeros(1, dtype=torch.int32, device=self.device)
                self.objects[name] = SimpleNamespace(enabled=True, async_updates=False, active_count=count,
                                                     dispatch_snapshot=count.clone(), host_sync_count=0,
                                                     host_active_count=0)
            return self.objects[name]
        if 'module' in x:
            from analysis_spec_b200 import tree_kernels
            return tree_kernels
        raise AssertionError(f'cannot decode {x}')

    # ---- checking ---------------------------------------------------------------------
    def match(self, exp, got, where):
        if exp is None or isinstance(exp, (bool, int, float, str)):
            assert got == exp, f'{where}: {got!r} != {exp!r}'
            return
        if 'tensor' in exp:
            ref = array(self.z, exp)
            assert isinstance(got, torch.Tensor) and got.dtype == ref.dtype and list(got.shape) == exp['shape'], \
                f'{where}: {getattr(got, "dtype", type(got))} {tuple(getattr(got, "shape", ()))} vs {exp}'
            assert torch.equal(got.cpu(), ref), f'{where}: values differ'
            return
        if 'view' in exp:
            assert list(got.shape) == exp['shape'] and list(got.stride()) == exp['stride'], \
                f'{where}: view {tuple(got.shape)} {got.stride()} vs {exp["shape"]} {exp["stride"]}'
            assert sha(got) == exp['sha'], f'{where}: K/V bytes differ'
            return
        if 'list' in exp or 'tuple' in exp:
            items = exp.get('list', exp.get('tuple'))
            assert len(got) == len(items), f'{where}: {len(got)} items vs {len(items)}'
            for i, (e, g) in enumerate(zip(items, got)):
                self.match(e, g, f'{where}[{i}]')
            return
        if 'dict' in exp:
            keys = [k for k, _ in exp['dict']]
            assert list(got) == keys, f'{where}: keys {list(got)} vs {keys}'
            for k, e in exp['dict']:
                self.match(e, got[k], f'{where}.{k}')
            return
        if 'PackedTree' in exp:
            for e, g, f in zip(exp['PackedTree'], (got.parents, got.tokens, got.feedback_contexts, got.max_depth),
                               ('parents', 'tokens', 'feedback_contexts', 'max_depth')):
                self.match(e, g, f'{where}.{f}')
            return
        if 'VerifiedPath' in exp:
            for e, g, f in zip(exp['VerifiedPath'], (got.tokens, got.packed_indices, got.feedback_contexts, got.lengths),
                               ('tokens', 'packed_indices', 'feedback_contexts', 'lengths')):
                self.match(e, g, f'{where}.{f}')
            return
        if 'object' in exp:
            name = exp['object']
            if name in self.objects:
                assert got is self.objects[name], f'{where}: a different object than {name}'
            return
        raise AssertionError(f'{where}: cannot compare {exp}')

    def check_state(self, state, where):
        for name, st in state.items():
            obj = self.objects[name]
            if 'layers' in st:
                assert len(obj.layers) == len(st['layers']), f'{where}: {name} has {len(obj.layers)} layers'
                for l, (layer, exp) in enumerate(zip(obj.layers, st['layers'])):
                    if exp is None:
                        assert layer.key_pool is None, f'{where}: {name} layer {l} allocated'
                        continue
                    n, b, shape, ksha, vsha = exp
                    assert (layer.length, layer.batch_size, list(layer.key_pool.shape)) == (n, b, shape), \
                        f'{where}: {name} layer {l} (length, batch, pool) = ' \
                        f'{(layer.length, layer.batch_size, tuple(layer.key_pool.shape))} vs {(n, b, shape)}'
                    if layer._pending is not None:  # fused: checked once the attention stored them
                        continue
                    assert sha(layer.key_pool[:b, :, :n]) == ksha, f'{where}: {name} layer {l} K rows differ'
                    assert sha(layer.value_pool[:b, :, :n]) == vsha, f'{where}: {name} layer {l} V rows differ'
                assert obj.kv_rows_moved == st['kv_rows_moved'], f'{where}: {name} kv_rows_moved'
            else:
                assert dict(obj.lengths) == st['lengths'], f'{where}: {name} lengths {obj.lengths}'
                assert sorted(obj.finished) == st['finished'], f'{where}: {name} finished rows'

    # ---- calls ------------------------------------------------------------------------
    def call(self, i, c):
        fn, where = c['fn'], f'call {i} {c["fn"]}'
        self.settle()
        if fn == 'attention':
            return self.attention_call(c, where)
        cls, _, method = fn.partition('.')
        kwargs = {k: self.dec(v) for k, v in c['kwargs'].items()}
        if method == '__init__':
            args = [self.dec(a) for a in c['args'][1:]]
            maker = {'ContiguousRolloutHistory': self.oh.ContiguousRolloutHistory,
                     'AttentionWorkspace': self.oa.AttentionWorkspace}[cls]
            self.objects[c['created']] = maker(*args, **kwargs)
        else:
            args = [self.dec(a) for a in c['args']]
            module = {'opd_static_cache': self.osc, 'opd_scheduling': self.osch,
                      'tree_verification': self.tv}.get(cls)
            target = getattr(module, method) if module is not None else getattr(args.pop(0), method)
            out = target(*args, **kwargs)
            if 'created' in c:
                self.objects[c['created']] = out
                if self.fused and isinstance(out, self.osc.OPDStaticCache):
                    out.fuse_append = True
            if fn == 'opd_scheduling.schedule':
                self.schedules.append(out[0])
            exp = c['out']
            if fn == 'OPDStaticCache.statistics':
                self.statistics[c['args'][0]['object']] = dict(out)
                exp = {'dict': [[k, v] for k, v in exp['dict'] if k != SCRATCH_STAT]}
                out = {k: v for k, v in out.items() if k != SCRATCH_STAT}
            layer = (self.objects[c['args'][0]['object']].layers[c['args'][3]]
                     if fn == 'OPDStaticCache.update' else None)
            if layer is not None and layer._pending is not None:
                self.deferred.append((layer, exp, out, where))
            else:
                self.match(exp, out, where)
        self.check_state(c['state'], where)
        if fn == 'opd_scheduling.compact_suffix_inplace':
            # the loop then stores the returned views back into the layer (_cache_set_layer,
            # opd_generate.py:43-66), which the next call's recorded state includes
            k = c['args'][0]
            layer = self.objects[k['view']].layers[k['layer']]
            layer.keys, layer.values = out

    def attention_call(self, c, where):
        q, k, v, mask = [self.dec(a) for a in c['args']]
        module = SimpleNamespace(layer_idx=c['layer'], training=False, **c['module'])
        out, _ = self.ta.tree_verify_attention(module, q, k, v, mask, **c['kwargs'])
        ref = array(self.z, c['out']).float()
        assert tuple(out.shape) == tuple(ref.shape), f'{where}: shape {tuple(out.shape)}'
        # a query row whose mask hides every column (the prompt's left-padding positions in the
        # prefill) has no defined output: SDPA averages V over the hidden columns, the kernel
        # writes 0; nothing reads it, since that position is hidden from every query
        live = (mask[:, 0, :, :k.shape[-2]] == 0).any(-1).cpu()
        assert live.any(), f'{where}: no visible row'
        err = (out.float().cpu() - ref).abs()[live]
        self.attention.append((c['layer'], float(err.max()), float(err.mean())))
        assert float(err.max()) <= 2e-2 and float(err.mean()) <= 2e-3, \
            f'{where}: attention max {float(err.max()):.3g} mean {float(err.mean()):.3g}'
        self.check_state(c['state'], where)

    def settle(self):
        """Checks the views an update returned with its rows still pending, before the next
        call changes anything: their contents as the loop sees them are the pools' rows with
        the pending rows in place (copies; the cache itself is not touched, so the next call
        still has to store or fuse them, which the state check after it verifies)."""
        for layer, exp, got, at in self.deferred:
            token = layer._pending
            assert token is not None, f'{at}: pending rows stored before the next call'
            k_new, v_new, position = token
            items = exp['tuple']
            assert len(items) == 2 and len(got) == 2, at
            for e, view, rows in zip(items, got, (k_new, v_new)):
                assert list(view.shape) == e['shape'] and list(view.stride()) == e['stride'], at
                logical = view.clone()
                logical[:, :, position:position + rows.shape[-2]] = rows
                assert sha(logical) == e['sha'], f'{at}: K/V bytes differ'
        self.deferred = []


def replay(path=TRACE, fused=False):
    z, meta = load_trace(path)
    r = Replay(z, meta, fused=fused)
    for i, c in enumerate(meta['calls']):
        r.call(i, c)
    torch.cuda.synchronize()
    return r, meta
