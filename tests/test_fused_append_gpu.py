"""The round's append fused into the verify attention (speckv_tree_attention_bits_append).

One launch per layer must leave the pools exactly as the two copy_ calls of
StaticAppendLayer.update (helper/opd_static_cache.py:106-107, here speckv_append_rows) and
return the attention the reference runs over the updated cache right after them
(transformers integrations/sdpa_attention.py:40-104 from helper/opd_generate.py:490), within
the bf16 tolerance (max |err| <= 2e-2, mean |err| <= 2e-3 against the float32 oracle).

The pool positions past `past` hold NaN before the call: the kernel reads the cached
positions only up to `past` (the last cached tile is cut there) and the new rows from the
projection, so a NaN reaching the output or a pool byte written outside [past, past + rows)
fails the test.
"""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _lib, _ops
from analysis_spec_b200.tree_verification import PackedTree
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_ERR, MEAN_ERR = 2e-2, 2e-3


def check(out, expect):
    err = (out.float().cpu() - torch.from_numpy(np.ascontiguousarray(expect))).abs()
    assert err.max().item() <= MAX_ERR, err.max().item()
    assert err.mean().item() <= MEAN_ERR, err.mean().item()


def case(batch, hq, hkv, rows, past, seed, ragged=True, dtype=torch.bfloat16, dim=128):
    rng = np.random.RandomState(seed)
    gen = torch.Generator(device='cuda').manual_seed(seed)
    # projections laid out (B, T, H * D) and viewed as (B, H, T, D), as in Qwen2Attention
    q = (0.5 * torch.randn(batch, rows, hq * dim, device='cuda', generator=gen)).to(dtype)
    q = q.view(batch, rows, hq, dim).transpose(1, 2)
    knew = (0.5 * torch.randn(batch, rows, hkv * dim, device='cuda', generator=gen)).to(dtype)
    vnew = (0.5 * torch.randn(batch, rows, hkv * dim, device='cuda', generator=gen)).to(dtype)
    knew = knew.view(batch, rows, hkv, dim).transpose(1, 2)
    vnew = vnew.view(batch, rows, hkv, dim).transpose(1, 2)
    cap = past + rows + 37
    kpool = torch.full((batch, hkv, cap, dim), float('nan'), device='cuda', dtype=dtype)
    vpool = torch.full((batch, hkv, cap, dim), float('nan'), device='cuda', dtype=dtype)
    kpool[:, :, :past] = (0.5 * torch.randn(batch, hkv, past, dim, device='cuda', generator=gen)).to(dtype)
    vpool[:, :, :past] = (0.5 * torch.randn(batch, hkv, past, dim, device='cuda', generator=gen)).to(dtype)
    parents = np.full((batch, rows), -1, dtype=np.int64)
    for b in range(batch):
        for r in range(1, rows):
            parents[b, r] = rng.randint(max(0, r - 8), r)
    pad = np.zeros((batch, past + rows), dtype=bool)
    if ragged and past:  # left padding of shorter prefixes plus scattered synthetic-EOS columns
        for b in range(batch):
            pad[b, :rng.randint(0, past // 2 + 1)] = True
        pad[:, :past] |= rng.rand(batch, past) < 0.03
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                      torch.from_numpy(parents).cuda(), rows)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    return q, kpool, vpool, knew, vnew, vis, oracle.tree_visible(parents, past, rows, pad=pad)


def same_bits(a, b):
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize('batch,hq,hkv,rows,past,ragged', [
    (4, 16, 2, 61, 700, True),    # the tree fits in the last cached tile's remainder: one tile more
    (3, 16, 2, 61, 2013, True),   # the tree straddles a 128-key boundary
    (2, 16, 2, 61, 256, True),    # past on a tile boundary
    (3, 16, 2, 61, 0, False),     # empty cache: the tree tile alone
    (3, 28, 4, 61, 300, True),    # 7 query heads per KV head
    (2, 40, 8, 61, 260, True),    # 5 query heads per KV head: 3 row tiles
    (2, 8, 1, 128, 129, False),   # the largest tree tile
    (1, 16, 2, 1, 129, False),    # one row
    (3, 16, 2, 10, 2013, True),   # at most 128 packed rows: the split-key kernel
    (2, 16, 2, 16, 31, False),    # split-key, bit offset inside the first visibility word
])
def test_fused_append_matches_append_then_attention(batch, hq, hkv, rows, past, ragged):
    q, kpool, vpool, knew, vnew, vis, visible = case(batch, hq, hkv, rows, past, seed=batch * 17 + rows + past,
                                                     ragged=ragged)
    scale = 128 ** -0.5
    kref, vref = kpool.clone(), vpool.clone()
    _ops.append_rows([kref], [vref], [knew], [vnew], past)
    out_ref = _ops.tree_attention_bits(q, kref[:, :, :past + rows], vref[:, :, :past + rows], vis.bits,
                                       vis.first_col, scale)
    out = _ops.tree_attention_bits_append(q, kpool, vpool, past, knew, vnew, vis.bits, vis.first_col, scale)
    torch.cuda.synchronize()
    # the pools: bit-exact against the append, NaN (untouched) past the new rows
    assert same_bits(kpool, kref) and same_bits(vpool, vref)
    assert torch.isnan(kpool[:, :, past + rows:].float()).all()
    assert not torch.isnan(out.float()).any()
    expect = oracle.attention(q.float().cpu().numpy(), kref[:, :, :past + rows].float().cpu().numpy(),
                              vref[:, :, :past + rows].float().cpu().numpy(),
                              oracle.additive_mask(visible, 'bfloat16'), scale)
    check(out, expect)
    check(out, out_ref.float().cpu().numpy())
    assert _ops.device_error() is None


def test_fused_append_fp16_and_repeat():
    """fp16 operands; a second call on the same pools (the next round at the same length)
    gives the same output and pools."""
    q, kpool, vpool, knew, vnew, vis, visible = case(2, 16, 2, 61, 500, seed=3, dtype=torch.float16)
    scale = 128 ** -0.5
    out1 = _ops.tree_attention_bits_append(q, kpool, vpool, 500, knew, vnew, vis.bits, vis.first_col, scale)
    k1, v1 = kpool.clone(), vpool.clone()
    out2 = _ops.tree_attention_bits_append(q, kpool, vpool, 500, knew, vnew, vis.bits, vis.first_col, scale)
    torch.cuda.synchronize()
    assert torch.equal(out1.view(torch.int16), out2.view(torch.int16))
    assert same_bits(kpool, k1) and same_bits(vpool, v1)
    expect = oracle.attention(q.float().cpu().numpy(), kpool[:, :, :561].float().cpu().numpy(),
                              vpool[:, :, :561].float().cpu().numpy(), oracle.additive_mask(visible, 'float16'),
                              scale)
    check(out1, expect)
    assert _ops.device_error() is None


def test_fused_append_full_size_layer():
    """Qwen2.5-3B tree-verify layer (batch 64, 16q / 2kv x 128, 61 rows, prefixes U{256..2048}
    left-padded to one length): pools bit-exact against the append, outputs of sequence slices
    against the float32 oracle."""
    from analysis_spec_b200 import workloads as W
    rng = np.random.RandomState(8)
    batch, hq, hkv, rows, dim = 64, 16, 2, 61, 128
    prefix = W.prefix_lengths(rng, ('uniform', 256, 2048), batch)
    past = int(prefix.max())
    parents, tokens = W.packed_trees(rng, batch, rows - 1, 6, 10)
    pad = np.zeros((batch, past + rows), dtype=bool)
    pad[:, :past] = W.left_padding(prefix, past)
    gen = torch.Generator(device='cuda').manual_seed(8)
    q = (0.5 * torch.randn(batch, rows, hq * dim, device='cuda', generator=gen)).bfloat16()
    q = q.view(batch, rows, hq, dim).transpose(1, 2)
    qkv = (0.5 * torch.randn(batch, rows, 2 * hkv * dim, device='cuda', generator=gen)).bfloat16()
    knew = qkv[:, :, :hkv * dim].view(batch, rows, hkv, dim).transpose(1, 2)
    vnew = qkv[:, :, hkv * dim:].view(batch, rows, hkv, dim).transpose(1, 2)
    kpool = (0.5 * torch.randn(batch, hkv, 4096, dim, device='cuda', generator=gen)).bfloat16()
    vpool = (0.5 * torch.randn(batch, hkv, 4096, dim, device='cuda', generator=gen)).bfloat16()
    kref, vref = kpool.clone(), vpool.clone()
    _ops.append_rows([kref], [vref], [knew], [vnew], past)
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(tokens).cuda(),
                      torch.zeros(batch, rows, dtype=torch.long, device='cuda'), 6)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    out = _ops.tree_attention_bits_append(q, kpool, vpool, past, knew, vnew, vis.bits, vis.first_col, dim ** -0.5)
    torch.cuda.synchronize()
    assert same_bits(kpool, kref) and same_bits(vpool, vref)
    visible = oracle.tree_visible(parents, past, 7, pad=pad)
    end = past + rows
    for sl in (slice(0, 3), slice(30, 32), slice(61, 64)):
        expect = oracle.attention(q[sl].float().cpu().numpy(), kref[sl, :, :end].float().cpu().numpy(),
                                  vref[sl, :, :end].float().cpu().numpy(), oracle.additive_mask(visible[sl], 'bfloat16'),
                                  dim ** -0.5)
        check(out[sl], expect)
    assert _ops.device_error() is None


def test_cache_update_attend_equals_update_then_attention():
    """OPDStaticCache.update_attend against update + the bits attention over the returned views,
    on a cache that has to grow for the new rows (lazy initialisation and growth unchanged)."""
    from analysis_spec_b200.opd_static_cache import OPDStaticCache
    batch, hq, hkv, rows, past, dim, layers = 4, 16, 2, 61, 200, 128, 2
    gen = torch.Generator(device='cuda').manual_seed(21)
    caches = [OPDStaticCache(256, batch_capacity=batch) for _ in range(2)]
    for layer in range(layers):
        k = (0.5 * torch.randn(batch, hkv, past, dim, device='cuda', generator=gen)).bfloat16()
        v = (0.5 * torch.randn(batch, hkv, past, dim, device='cuda', generator=gen)).bfloat16()
        for c in caches:
            c.update(k, v, layer)
    rng = np.random.RandomState(21)
    parents = np.full((batch, rows), -1, dtype=np.int64)
    for b in range(batch):
        for r in range(1, rows):
            parents[b, r] = rng.randint(max(0, r - 6), r)
    pad = np.zeros((batch, past + rows), dtype=bool)
    for b in range(batch):
        pad[b, :rng.randint(0, past // 2)] = True
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                      torch.from_numpy(parents).cuda(), rows)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    scale = dim ** -0.5
    for layer in range(layers):
        q = (0.5 * torch.randn(batch, rows, hq * dim, device='cuda', generator=gen)).bfloat16()
        q = q.view(batch, rows, hq, dim).transpose(1, 2)
        kv = (0.5 * torch.randn(batch, rows, 2 * hkv * dim, device='cuda', generator=gen)).bfloat16()
        k = kv[:, :, :hkv * dim].view(batch, rows, hkv, dim).transpose(1, 2)
        v = kv[:, :, hkv * dim:].view(batch, rows, hkv, dim).transpose(1, 2)
        out = caches[0].update_attend(q, k, v, layer, vis, scale)
        keys, values = caches[1].update(k, v, layer)
        ref = _ops.tree_attention_bits(q, keys, values, vis.bits, vis.first_col, scale)
        torch.cuda.synchronize()
        a, b = caches[0].layers[layer], caches[1].layers[layer]
        assert a.length == b.length == past + rows and a.capacity == b.capacity
        assert same_bits(a.keys, b.keys) and same_bits(a.values, b.values)
        check(out, ref.float().cpu().numpy())
    assert caches[0].statistics() == caches[1].statistics()
    assert _ops.device_error() is None


def test_fused_append_refusals():
    q, kpool, vpool, knew, vnew, vis, _ = case(2, 16, 2, 61, 100, seed=4)
    cap = kpool.shape[2]
    with pytest.raises(_lib.SpecKVError, match='exceed'):  # past + rows beyond the pools
        _ops.tree_attention_bits_append(q, kpool, vpool, cap - 60, knew, vnew, vis.bits, vis.first_col, 0.1)
    big = case(1, 8, 1, 129, 10, seed=5)
    with pytest.raises(_lib.SpecKVError, match='128-key tile'):
        _ops.tree_attention_bits_append(big[0], big[1], big[2], 10, big[3], big[4], big[5].bits, big[5].first_col,
                                        0.1)
    assert _ops.device_error() is None


def test_fused_append_bounded_wait_runs_out_and_unwinds():
    """A bounded wait of the fused kernel made to run out (test hooks: a 2 ms limit, CTA 0's
    first Q tile withheld): the launch reports 'wait timeout' and returns, every tree-row store
    it issued has completed, and the context stays usable: the next call on restored pools
    appends and attends exactly as before the failure."""
    q, kpool, vpool, knew, vnew, vis, _ = case(16, 16, 2, 61, 1400, seed=31)
    scale = 128 ** -0.5
    k0, v0 = kpool.clone(), vpool.clone()
    ref = _ops.tree_attention_bits_append(q, kpool, vpool, 1400, knew, vnew, vis.bits, vis.first_col, scale)
    kref, vref = kpool.clone(), vpool.clone()
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    kpool.copy_(k0)
    vpool.copy_(v0)
    try:
        _lib.call('speckv_attention_test_hooks', 2_000_000, 1)
        _ops.tree_attention_bits_append(q, kpool, vpool, 1400, knew, vnew, vis.bits, vis.first_col, scale)
        torch.cuda.synchronize()
        err = _ops.device_error()
    finally:
        _lib.call('speckv_attention_test_hooks', 0, 0)
    assert err is not None and err[0] == 'wait timeout', err
    kpool.copy_(k0)
    vpool.copy_(v0)
    again = _ops.tree_attention_bits_append(q, kpool, vpool, 1400, knew, vnew, vis.bits, vis.first_col, scale)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    assert torch.equal(again.view(torch.int16), ref.view(torch.int16))
    assert same_bits(kpool, kref) and same_bits(vpool, vref)
