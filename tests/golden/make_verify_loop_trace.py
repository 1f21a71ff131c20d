"""Records the reference's own verify loop at its module boundary, for the drop-in replay test.

Usage (from the repository root, in a container holding the reference checkout):

    python tests/golden/make_verify_loop_trace.py /path/to/analysis_spec

The path of the reference checkout is required. The script runs the reference's
`helper.opd_generate.speculative_generate(method='opd_reflex', do_sample=False)`
on a tiny random Qwen2 (2 layers, 4 query / 2 KV heads of dim 128, bf16, vocabulary
97, the draft head of `helper.fastgrpo_model.FastGRPOModel`) on the host's CPU,
with its torch branches (no kernel plugin). Before `helper.opd_generate` is imported,
every entry point of the modules the drop-in replaces is wrapped with a recorder:

    helper.opd_static_cache   persistent_cache, swap_remove_plan, OPDStaticCache methods
    helper.opd_scheduling     schedule, compact_suffix_inplace
    helper.tree_verification  pack_tree, trace_verified_path, PackedTree.attention_mask
    helper.opd_history        ContiguousRolloutHistory (constructor, append, mark_finished, finalize)
    helper.opd_attention      AttentionWorkspace (constructor, positions, causal)

plus the target model's attention calls (transformers' `sdpa` interface). Each
outermost call is written in order with its arguments and its result; tensors that
are views of a cache's K/V pools are written as (cache, layer, K/V, offset, shape,
stride) plus a SHA-256 of their bytes, and after every call the state of each cache
(per layer: length, batch, pool shape and the hash of the live K/V rows) and of each
history (lengths) is written too. The reference's own result (tokens, accepted
lengths, cache statistics) closes the trace.

Output: tests/golden/verify_loop_trace.npz (arrays + the JSON trace under '__trace__').
"""
import hashlib
import json
import sys
from copy import deepcopy
from pathlib import Path
from types import SimpleNamespace

if len(sys.argv) < 2:
    sys.exit('usage: python tests/golden/make_verify_loop_trace.py /path/to/analysis_spec (the reference checkout)')
REF = Path(sys.argv[1]).resolve()
OUT = Path(__file__).resolve().parent / 'verify_loop_trace.npz'
sys.dont_write_bytecode = True
sys.path.insert(0, str(REF))

import numpy as np  # noqa: E402
import torch  # noqa: E402

import helper.opd_attention as ref_attention  # noqa: E402
import helper.opd_history as ref_history  # noqa: E402
import helper.opd_scheduling as ref_scheduling  # noqa: E402
import helper.opd_static_cache as ref_cache  # noqa: E402
import helper.tree_verification as ref_tree  # noqa: E402

EOS = 41  # a token the greedy rollout of two of the four responses emits: they finish and are released
WORKSPACE_ARGS = {'workspace', 'packet'}


def sha(t):
    t = t.detach().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()[:20]


class Recorder:
    def __init__(self):
        self.calls = []
        self.arrays = {}
        self.depth = 0
        self.names = {}      # id(object) -> name
        self.objects = {}    # name -> object (caches, histories, workspaces)
        self.opaque = 0

    # ---- encoding ------------------------------------------------------------------
    def array(self, t):
        t = t.detach().cpu().clone()  # a copy now: the loop reuses and overwrites its buffers in place
        dtype = str(t.dtype).replace('torch.', '')
        a = t.contiguous().view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.contiguous().numpy()
        key = f'a{len(self.arrays)}'
        self.arrays[key] = a
        return {'tensor': key, 'dtype': dtype, 'shape': list(t.shape)}

    def pool_view(self, t):
        for name, obj in self.objects.items():
            if not isinstance(obj, ref_cache.OPDStaticCache):
                continue
            for l, layer in enumerate(obj.layers):
                for kv, pool in enumerate((layer.key_pool, layer.value_pool)):
                    if pool is not None and t.untyped_storage().data_ptr() == pool.untyped_storage().data_ptr():
                        return {'view': name, 'layer': l, 'kv': kv, 'offset': t.storage_offset() - pool.storage_offset(),
                                'shape': list(t.shape), 'stride': list(t.stride()), 'sha': sha(t)}
        return None

    def enc(self, x, workspace=False):
        if x is None or isinstance(x, (bool, int, float, str)):
            return x
        if isinstance(x, torch.Tensor):
            if workspace:
                return {'empty': list(x.shape), 'dtype': str(x.dtype).replace('torch.', '')}
            v = self.pool_view(x)
            return v if v is not None else self.array(x)
        if isinstance(x, torch.dtype):
            return {'torch_dtype': str(x).replace('torch.', '')}
        if isinstance(x, torch.device):
            return {'device': x.type}
        if isinstance(x, (list, tuple)):
            return {'list' if isinstance(x, list) else 'tuple': [self.enc(y, workspace) for y in x]}
        if isinstance(x, dict):
            return {'dict': [[k, self.enc(v, workspace)] for k, v in x.items()]}
        if isinstance(x, ref_tree.PackedTree):
            return {'PackedTree': [self.enc(x.parents), self.enc(x.tokens), self.enc(x.feedback_contexts), x.max_depth]}
        if isinstance(x, ref_tree.VerifiedPath):
            return {'VerifiedPath': [self.enc(x.tokens), self.enc(x.packed_indices), self.enc(x.feedback_contexts),
                                     self.enc(x.lengths)]}
        if id(x) in self.names:
            return {'object': self.names[id(x)]}
        if isinstance(x, type(ref_tree)):
            return {'module': x.__name__}
        # anything else (the model, the OPD runtime) is an opaque host object
        name = f'opaque{self.opaque}'
        self.opaque += 1
        self.names[id(x)] = name
        return {'object': name, 'opaque': type(x).__name__}

    def register(self, obj, prefix):
        name = f'{prefix}{sum(1 for n in self.objects if n.startswith(prefix))}'
        self.names[id(obj)] = name
        self.objects[name] = obj
        return name

    def state(self):
        out = {}
        for name, obj in self.objects.items():
            if isinstance(obj, ref_cache.OPDStaticCache):
                layers = []
                for layer in obj.layers:
                    if layer.key_pool is None:
                        layers.append(None)
                        continue
                    b, n = layer.batch_size, layer.length
                    layers.append([n, b, list(layer.key_pool.shape), sha(layer.key_pool[:b, :, :n]),
                                   sha(layer.value_pool[:b, :, :n])])
                out[name] = {'layers': layers, 'kv_rows_moved': obj.kv_rows_moved}
            elif isinstance(obj, ref_history.ContiguousRolloutHistory):
                out[name] = {'lengths': dict(obj.lengths), 'finished': sorted(obj.finished)}
        return out

    # ---- wrapping ------------------------------------------------------------------
    def record(self, qual, fn, args, kwargs, self_prefix=None, names=()):
        """Runs one outermost call, writing its arguments (before) and result (after)."""
        if self.depth:
            return fn(*args, **kwargs)
        self.depth += 1
        try:
            rec = {'fn': qual}
            init = qual.endswith('__init__')  # the object itself is named once constructed
            rec['args'] = [None if init and i == 0 else self.enc(a, i < len(names) and names[i] in WORKSPACE_ARGS)
                           for i, a in enumerate(args)]
            rec['kwargs'] = {k: self.enc(v, k in WORKSPACE_ARGS) for k, v in kwargs.items()}
            out = fn(*args, **kwargs)
            if init:
                rec['created'] = self.register(args[0], self_prefix)
                rec['out'] = None
            else:
                if isinstance(out, ref_cache.OPDStaticCache) and id(out) not in self.names:
                    rec['created'] = self.register(out, 'cache')
                rec['out'] = self.enc(out)
            rec['state'] = self.state()
            self.calls.append(rec)
            return out
        finally:
            self.depth -= 1


R = Recorder()


def wrap_function(module, name, names=()):
    fn = getattr(module, name)
    qual = f'{module.__name__.split(".")[-1]}.{name}'

    def wrapped(*args, **kwargs):
        return R.record(qual, fn, args, kwargs, names=names)
    setattr(module, name, wrapped)


def wrap_method(cls, name, self_prefix=None, names=()):
    fn = getattr(cls, name)
    qual = f'{cls.__name__}.{name}'

    def wrapped(*args, **kwargs):
        return R.record(qual, fn, args, kwargs, self_prefix=self_prefix, names=('self',) + tuple(names))
    setattr(cls, name, wrapped)


wrap_function(ref_cache, 'persistent_cache')
wrap_function(ref_cache, 'swap_remove_plan')
for m in ('update', 'get_seq_length', 'get_mask_sizes', 'get_max_cache_shape', 'crop', 'batch_repeat_interleave',
          'batch_select_indices', 'swap_remove', 'begin_rollout', 'end_rollout', 'statistics', '__getitem__',
          '__len__'):
    wrap_method(ref_cache.OPDStaticCache, m)
wrap_function(ref_scheduling, 'schedule', names=('path', 'past', 'eos', 'workspace', 'packet'))
wrap_function(ref_scheduling, 'compact_suffix_inplace')
wrap_function(ref_tree, 'pack_tree')
wrap_function(ref_tree, 'trace_verified_path')
wrap_method(ref_tree.PackedTree, 'attention_mask')
wrap_method(ref_history.ContiguousRolloutHistory, '__init__', self_prefix='history')
for m in ('append', 'mark_finished', 'finalize'):
    wrap_method(ref_history.ContiguousRolloutHistory, m)
wrap_method(ref_attention.AttentionWorkspace, '__init__', self_prefix='workspace')
for m in ('positions', 'causal'):
    wrap_method(ref_attention.AttentionWorkspace, m)

from transformers import AttentionInterface, Qwen2Config, Qwen2ForCausalLM  # noqa: E402
from transformers.integrations.sdpa_attention import sdpa_attention_forward  # noqa: E402

TARGET_ATTENTION = set()


def recording_sdpa(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    out = sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling, **kwargs)
    if id(module) in TARGET_ATTENTION and not R.depth:
        R.calls.append({'fn': 'attention', 'layer': module.layer_idx,
                        'module': {'num_key_value_groups': module.num_key_value_groups,
                                   'is_causal': bool(getattr(module, 'is_causal', True))},
                        'args': [R.enc(query), R.enc(key), R.enc(value), R.enc(attention_mask)],
                        'kwargs': {'dropout': dropout, 'scaling': scaling},
                        'out': R.enc(out[0]), 'state': R.state()})
    return out


AttentionInterface.register('recorded_sdpa', recording_sdpa)

from helper.fastgrpo_model import FastGRPOModel  # noqa: E402
from helper.opd_generate import speculative_generate  # noqa: E402


def tiny_model():
    torch.manual_seed(321)
    config = Qwen2Config(vocab_size=97, hidden_size=512, intermediate_size=256, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=128,
                         attention_dropout=0., dtype=torch.bfloat16)
    config._attn_implementation = 'sdpa'
    target = Qwen2ForCausalLM(config).to(dtype=torch.bfloat16).eval()
    dc = deepcopy(config)
    dc.num_hidden_layers = 1
    dc.rope_scaling = None
    model = FastGRPOModel(dc, target).to(dtype=torch.bfloat16).eval()
    model.enable_opd(8)
    target.config._attn_implementation = 'recorded_sdpa'
    for layer in target.model.layers:
        TARGET_ATTENTION.add(id(layer.self_attn))
    return model


def main():
    torch.set_num_threads(8)
    model = tiny_model()
    settings = dict(do_sample=False, repeated_generate_nums=2, max_length=14, verification_capacity=28,
                    max_verification_num=7, max_draft_k=2, max_draft_token_length=3, min_draft_token_length=3,
                    method='opd_reflex')
    prompts, prompt_mask = torch.tensor([[0, 7, 9], [3, 5, 8]]), torch.tensor([[0, 1, 1], [1, 1, 1]])
    with torch.inference_mode():
        result = speculative_generate(model, prompts, prompt_mask, SimpleNamespace(eos_token_id=EOS), **settings)
    summary = {k: v for k, v in result.items() if isinstance(v, (int, float, list, str)) and k != 'total_time_cost'
               and not k.endswith('_time_cost') and not k.endswith('_ms')}
    meta = {'model': 'Qwen2: 2 layers, hidden 512, 4 q / 2 KV heads x 128, bf16, vocabulary 97; draft: '
                     'FastGRPOModel with one layer, opd rank 8',
            'settings': settings, 'prompts': prompts.tolist(), 'prompt_mask': prompt_mask.tolist(), 'eos': EOS,
            'result': summary, 'calls': R.calls}
    arrays = dict(R.arrays)
    arrays['__trace__'] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **arrays)
    counts = {}
    for c in R.calls:
        counts[c['fn']] = counts.get(c['fn'], 0) + 1
    print(json.dumps({'calls': len(R.calls), 'by_function': counts, 'bytes': OUT.stat().st_size,
                      'generated_token_ids': result['generated_token_ids'],
                      'total_acc_length': result['total_acc_length']}))


if __name__ == '__main__':
    main()
