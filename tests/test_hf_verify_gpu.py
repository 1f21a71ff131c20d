"""The drop-in on a real transformers model: a small random-weight Qwen2 (head_dim 128, GQA
4 q / 2 KV heads, bf16) prefills left-padded prompts into OPDStaticCache, then runs the tree
verify forward with the reference's 4-D additive tree mask
(helper/opd_generate.py:470-495) three ways: transformers' SDPA (the reference path), the
registered 'speckv_tree' attention on the dense mask, and on the visibility bits attached to
the mask. Logits must agree within bf16 tolerance and greedy acceptance must be identical."""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops, tree_kernels, workloads as W
from analysis_spec_b200.opd_scheduling import schedule
from analysis_spec_b200.opd_static_cache import OPDStaticCache
from analysis_spec_b200.tree_attention import register
from analysis_spec_b200.tree_verification import PackedTree, trace_verified_path

pytestmark = pytest.mark.gpu

VOCAB, B, PROMPT, ROWS, DEPTH, TOPK = 512, 4, 16, 13, 4, 3


def _model():
    from transformers import Qwen2Config, Qwen2ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen2Config(vocab_size=VOCAB, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      rms_norm_eps=1e-6, tie_word_embeddings=False)
    cfg._attn_implementation = 'sdpa'
    return Qwen2ForCausalLM(cfg).to('cuda', torch.bfloat16).eval()


def _inputs():
    rng = np.random.RandomState(3)
    lengths = np.array([5, 9, 12, 16])
    ids = rng.randint(0, VOCAB, size=(B, PROMPT))
    mask2d = np.zeros((B, PROMPT), dtype=np.int64)
    for b, n in enumerate(lengths):
        mask2d[b, PROMPT - n:] = 1
    parents, tokens = W.packed_trees(rng, B, ROWS - 1, DEPTH, TOPK, vocab=VOCAB)
    tokens[:, 0] = rng.randint(0, VOCAB, size=B)  # root = last committed token
    depth = np.zeros_like(parents)
    for r in range(1, ROWS):
        depth[:, r] = depth[np.arange(B), parents[:, r]] + 1
    positions = lengths[:, None] + depth  # the root follows the last prompt token
    return ids, mask2d, parents, tokens, positions


def _prefill(model, ids, mask2d):
    cache = OPDStaticCache(64, batch_capacity=B)
    am = torch.from_numpy(mask2d).cuda()
    pos = (am.cumsum(-1) - 1).clamp(min=0)
    with torch.no_grad():
        model(input_ids=torch.from_numpy(ids).cuda(), attention_mask=am, position_ids=pos, past_key_values=cache,
              use_cache=True)
    return cache


def _verify(model, cache, tree, tokens, positions, mask, impl):
    model.config._attn_implementation = impl
    for layer in model.model.layers:
        layer.self_attn.config._attn_implementation = impl
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(tokens).cuda(), attention_mask=mask,
                    position_ids=torch.from_numpy(positions).cuda(), past_key_values=cache, use_cache=True)
    return out.logits.float()


def test_tree_verify_forward_matches_sdpa_and_greedy_acceptance():
    name = register()
    model = _model()
    ids, mask2d, parents, tokens, positions = _inputs()
    pad_np = np.zeros((B, PROMPT + ROWS), dtype=bool)
    pad_np[:, :PROMPT] = mask2d == 0
    pad = torch.from_numpy(pad_np).cuda()
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(tokens).cuda(),
                      torch.zeros(B, ROWS, dtype=torch.long, device='cuda'), DEPTH)
    results = {}
    for impl in ('sdpa', 'dense', 'bits'):
        cache = _prefill(model, ids, mask2d)
        assert cache.get_seq_length() == PROMPT
        mask = tree.attention_mask(PROMPT, torch.bfloat16, pad)
        if impl == 'bits':
            mask = tree.visibility(PROMPT, pad).attach(mask)
        logits = _verify(model, cache, tree, tokens, positions, mask, 'sdpa' if impl == 'sdpa' else name)
        assert cache.get_seq_length() == PROMPT + ROWS
        results[impl] = logits
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    ref = results['sdpa']
    scale = ref.abs().max().item()
    for impl in ('dense', 'bits'):
        err = (results[impl] - ref).abs()
        assert err.max().item() <= 2e-2 * max(scale, 1.0), (impl, err.max().item(), scale)
        assert err.mean().item() <= 2e-3 * max(scale, 1.0), (impl, err.mean().item(), scale)
    # greedy acceptance: samples = argmax of each row's logits, traced through the tree
    eos = VOCAB + 1
    lengths = {}
    for impl, logits in results.items():
        samples = logits.argmax(-1)
        path = trace_verified_path(tree, samples, eos)
        rows, *_ = schedule(path, PROMPT, eos, None, None, tree_kernels)
        lengths[impl] = [r[0] for r in rows]
    agree = (results['bits'].argmax(-1) == ref.argmax(-1)).float().mean().item()
    assert agree >= 0.95, agree
    assert lengths['dense'] == lengths['sdpa'] and lengths['bits'] == lengths['sdpa'], lengths


def test_tree_verify_forward_through_a_row_table():
    """A row-table cache on the real model: 2B prompts prefilled, the B decoys among them
    released through the table (no history moved, the survivors scattered over the pool
    rows), then the tree verify forward of the survivors with the registered attention
    matches transformers' SDPA on a table-free cache holding only those prompts."""
    from analysis_spec_b200.opd_static_cache import swap_remove_plan
    name = register()
    model = _model()
    ids, mask2d, parents, tokens, positions = _inputs()
    rng = np.random.RandomState(9)
    real_at = [1, 2, 5, 6]  # where the B real prompts sit among 2B
    all_ids = rng.randint(0, VOCAB, size=(2 * B, PROMPT))
    all_mask = np.ones((2 * B, PROMPT), dtype=np.int64)
    for j, i in enumerate(real_at):
        all_ids[i], all_mask[i] = ids[j], mask2d[j]
    cache = OPDStaticCache(64, batch_capacity=2 * B, row_table=True)
    am = torch.from_numpy(all_mask).cuda()
    pos = (am.cumsum(-1) - 1).clamp(min=0)
    with torch.no_grad():  # the table is still the identity: transformers' SDPA reads the views as they are
        model(input_ids=torch.from_numpy(all_ids).cuda(), attention_mask=am, position_ids=pos,
              past_key_values=cache, use_cache=True)
    keep, sources, dests = swap_remove_plan([i not in real_at for i in range(2 * B)])
    cache.swap_remove(len(keep), sources, dests)
    assert cache.row_table == keep and keep != sorted(keep)
    perm = [real_at.index(k) for k in keep]  # logical sequence -> prompt
    pad_np = np.zeros((B, PROMPT + ROWS), dtype=bool)
    pad_np[:, :PROMPT] = mask2d[perm] == 0
    tree = PackedTree(torch.from_numpy(parents[perm]).cuda(), torch.from_numpy(tokens[perm]).cuda(),
                      torch.zeros(B, ROWS, dtype=torch.long, device='cuda'), DEPTH)
    mask = tree.attention_mask(PROMPT, torch.bfloat16, torch.from_numpy(pad_np).cuda())
    logits = _verify(model, cache, tree, tokens[perm], positions[perm], mask, name)
    assert cache.get_seq_length() == PROMPT + ROWS
    ref_cache = _prefill(model, ids, mask2d)
    ref_pad = np.zeros((B, PROMPT + ROWS), dtype=bool)
    ref_pad[:, :PROMPT] = mask2d == 0
    ref_tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(tokens).cuda(),
                          torch.zeros(B, ROWS, dtype=torch.long, device='cuda'), DEPTH)
    ref_mask = ref_tree.attention_mask(PROMPT, torch.bfloat16, torch.from_numpy(ref_pad).cuda())
    ref = _verify(model, ref_cache, ref_tree, tokens, positions, ref_mask, 'sdpa')[perm]
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    scale = ref.abs().max().item()
    err = (logits - ref).abs()
    assert err.max().item() <= 2e-2 * max(scale, 1.0), (err.max().item(), scale)
    assert err.mean().item() <= 2e-3 * max(scale, 1.0), (err.mean().item(), scale)
    assert (logits.argmax(-1) == ref.argmax(-1)).float().mean().item() >= 0.95


@pytest.mark.parametrize('attach_bits', [True, False])
def test_fused_append_on_the_verify_forward(attach_bits):
    """OPDStaticCache(fuse_append=True) on the real model's verify forward: each decoder layer's
    update leaves its tree rows to the registered attention, which appends them in its own
    launch (speckv_tree_attention_bits_append; no append launch in the forward). Against the
    same forward on a cache without the flag: pools bit-exact, logits within bf16 tolerance,
    identical greedy acceptance; with the dense mask alone (no bits attached) the mask's
    one-time conversion feeds the fused kernel too. The first layer's pools are compared
    bit for bit; deeper layers' tree rows come from hidden states that went through the
    previous layer's attention, whose output agrees to rounding only (the fused kernel splits
    the key tiles differently), so those rows are compared within bf16 tolerance."""
    from analysis_spec_b200 import _lib
    name = register()
    model = _model()
    ids, mask2d, parents, tokens, positions = _inputs()
    pad_np = np.zeros((B, PROMPT + ROWS), dtype=bool)
    pad_np[:, :PROMPT] = mask2d == 0
    pad = torch.from_numpy(pad_np).cuda()
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(tokens).cuda(),
                      torch.zeros(B, ROWS, dtype=torch.long, device='cuda'), DEPTH)
    results, pools, calls = {}, {}, {}
    for fuse in (False, True):
        model.config._attn_implementation = 'sdpa'  # both prefills through transformers' SDPA
        for layer in model.model.layers:
            layer.self_attn.config._attn_implementation = 'sdpa'
        cache = _prefill(model, ids, mask2d)  # the flag goes on after the prefill
        cache.fuse_append = fuse
        mask = tree.attention_mask(PROMPT, torch.bfloat16, pad)
        if attach_bits:
            mask = tree.visibility(PROMPT, pad).attach(mask)
        _lib.profile.reset()
        _lib.profile.enabled = True
        try:
            results[fuse] = _verify(model, cache, tree, tokens, positions, mask, name)
        finally:
            _lib.profile.enabled = False
        calls[fuse] = {k: len(v) for k, v in _lib.profile.events.items()}
        assert cache.get_seq_length() == PROMPT + ROWS
        assert all(layer._pending is None for layer in cache.layers)
        pools[fuse] = [(l.key_pool[:B, :, :PROMPT + ROWS].clone(), l.value_pool[:B, :, :PROMPT + ROWS].clone())
                       for l in cache.layers]
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    layers = len(model.model.layers)
    assert calls[True].get('speckv_tree_attention_bits_append') == layers, calls[True]
    assert 'speckv_append_rows' not in calls[True] and calls[False].get('speckv_append_rows') == layers, calls
    for i, ((k0, v0), (k1, v1)) in enumerate(zip(pools[False], pools[True])):
        end = PROMPT + ROWS if i == 0 else PROMPT
        for a, b in ((k0, k1), (v0, v1)):
            assert torch.equal(a[:, :, :end].view(torch.int16), b[:, :, :end].view(torch.int16)), i
            tail = (a[:, :, PROMPT:].float() - b[:, :, PROMPT:].float()).abs()
            assert tail.max().item() <= 2e-2 * max(a.float().abs().max().item(), 1.0), (i, tail.max().item())
    ref = results[False]
    scale = ref.abs().max().item()
    err = (results[True] - ref).abs()
    assert err.max().item() <= 2e-2 * max(scale, 1.0), (err.max().item(), scale)
    assert err.mean().item() <= 2e-3 * max(scale, 1.0), (err.mean().item(), scale)
    eos = VOCAB + 1
    lengths = {}
    for fuse, logits in results.items():
        path = trace_verified_path(tree, logits.argmax(-1), eos)
        rows, *_ = schedule(path, PROMPT, eos, None, None, tree_kernels)
        lengths[fuse] = [r[0] for r in rows]
    assert lengths[True] == lengths[False], lengths


def test_fused_append_rows_are_stored_before_other_uses():
    """Rows a fuse_append cache left pending are in the pools before anything else reads or
    moves them: a read of the keys / values views, and a remap of the batch."""
    torch.manual_seed(1)
    batch, heads, past, rows = 3, 2, 40, 7
    base = [(0.5 * torch.randn(batch, heads, past, 128, device='cuda')).bfloat16() for _ in range(2)]
    new = [(0.5 * torch.randn(batch, heads, rows, 128, device='cuda')).bfloat16() for _ in range(2)]
    ref = OPDStaticCache(64, batch_capacity=batch)
    ref.update(base[0], base[1], 0)
    keys_ref, values_ref = ref.update(new[0], new[1], 0)
    cache = OPDStaticCache(64, batch_capacity=batch, fuse_append=True)
    cache.update(base[0], base[1], 0)
    cache.update(new[0], new[1], 0)
    layer = cache.layers[0]
    assert layer._pending is not None  # left to the attention
    keys = layer.keys  # a public read stores them
    assert layer._pending is None
    assert torch.equal(keys.view(torch.int16), keys_ref.view(torch.int16))
    cache.update(new[1], new[0], 0)
    assert cache.layers[0]._pending is not None
    idx = torch.tensor([2, 0, 1], device='cuda')
    cache.batch_select_indices(idx)  # a remap stores them first
    ref.update(new[1], new[0], 0)
    ref.batch_select_indices(idx)
    torch.cuda.synchronize()
    assert torch.equal(cache.layers[0].keys.view(torch.int16), ref.layers[0].keys.view(torch.int16))
    assert torch.equal(cache.layers[0].values.view(torch.int16), ref.layers[0].values.view(torch.int16))
    assert _ops.device_error() is None
