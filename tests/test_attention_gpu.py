"""Tree-verify attention vs the reference's SDPA outputs and the float32 oracle.

Tolerance (bf16 operands, fp32 accumulation): max |err| <= 2e-2 and mean |err| <= 2e-3
against the float32 reference, the bound the path's correctness criteria state.
"""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200.tree_attention import register, tree_verify_attention
from analysis_spec_b200.tree_verification import PackedTree
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_ERR, MEAN_ERR = 2e-2, 2e-3


def check(out, expect):
    err = (out.float().cpu() - torch.from_numpy(np.ascontiguousarray(expect))).abs()
    assert err.max().item() <= MAX_ERR, err.max().item()
    assert err.mean().item() <= MEAN_ERR, err.mean().item()


class Module:
    def __init__(self, groups):
        self.num_key_value_groups = groups
        self.is_causal = True
        self.training = False


@pytest.mark.parametrize('case', range(3))
@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_golden_attention(golden, case, dtype):
    g = golden('attention')
    a = f'a{case}_'
    q, k, v = (torch.from_numpy(g[a + n]).cuda().to(dtype) for n in ('q', 'k', 'v'))
    mask = torch.from_numpy(g[a + 'mask']).cuda().to(dtype)
    out, _ = tree_verify_attention(Module(q.shape[1] // k.shape[1]), q, k, v, mask, scaling=q.shape[-1] ** -0.5)
    check(out, g[a + 'out'])


def random_case(batch, hq, hkv, rows, past, dim, seed, dtype=torch.bfloat16, ragged=True):
    rng = np.random.RandomState(seed)
    gen = torch.Generator(device='cuda').manual_seed(seed)
    # projections laid out (B, T, H * D) and viewed as (B, H, T, D), as in Qwen2Attention
    q = (0.5 * torch.randn(batch, rows, hq * dim, device='cuda', generator=gen)).to(dtype)
    q = q.view(batch, rows, hq, dim).transpose(1, 2)
    cap = past + rows + 5
    kpool = (0.5 * torch.randn(batch + 1, hkv, cap, dim, device='cuda', generator=gen)).to(dtype)
    vpool = (0.5 * torch.randn(batch + 1, hkv, cap, dim, device='cuda', generator=gen)).to(dtype)
    k, v = kpool[:batch, :, :past + rows], vpool[:batch, :, :past + rows]
    parents = np.full((batch, rows), -1, dtype=np.int64)
    for b in range(batch):
        for r in range(1, rows):
            parents[b, r] = rng.randint(max(0, r - 8), r)
    pad = np.zeros((batch, past + rows), dtype=bool)
    if ragged:  # left padding of shorter prefixes plus scattered synthetic-EOS columns
        for b in range(batch):
            pad[b, :rng.randint(0, past // 2 + 1)] = True
        pad[:, :past] |= rng.rand(batch, past) < 0.03
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                      torch.from_numpy(parents).cuda(), rows)
    mask = tree.attention_mask(past, dtype, torch.from_numpy(pad).cuda())
    return q, k, v, mask, parents, pad


@pytest.mark.parametrize('batch,hq,hkv,rows,past,dim', [(4, 16, 2, 61, 300, 128), (2, 16, 2, 61, 1500, 128),
                                                        (3, 28, 4, 17, 200, 128), (2, 40, 8, 61, 100, 128),
                                                        (5, 4, 4, 9, 33, 64), (2, 6, 2, 7, 19, 40),
                                                        (1, 16, 2, 1, 257, 128)])
def test_random_trees_vs_oracle(batch, hq, hkv, rows, past, dim):
    q, k, v, mask, parents, pad = random_case(batch, hq, hkv, rows, past, dim, seed=batch * 7 + rows)
    out = _ops.tree_attention(q, k, v, mask, dim ** -0.5)
    vis = oracle.tree_visible(parents, past, rows, pad=pad)
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              oracle.additive_mask(vis, 'bfloat16'), dim ** -0.5)
    assert out.shape == (batch, rows, hq, dim) and out.is_contiguous()
    check(out, expect)


def test_visibility_bits_match_mask_rule():
    rng = np.random.RandomState(11)
    for batch, rows, past, depth in ((3, 17, 40, 4), (64, 61, 2048, 6), (2, 130, 7, 20)):
        parents = np.full((batch, rows), -1, dtype=np.int64)
        for b in range(batch):
            for r in range(1, rows):
                parents[b, r] = rng.randint(max(0, r - 5), r)
        pad = np.zeros((batch, past + rows), dtype=bool)
        for b in range(batch):
            pad[b, :rng.randint(0, past + 1)] = True
        tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                          torch.from_numpy(parents).cuda(), depth)
        vis = tree.visibility(past, torch.from_numpy(pad).cuda())
        bits = vis.bits.cpu().numpy().view(np.uint32)
        unpacked = np.unpackbits(bits.view(np.uint8), bitorder='little').reshape(batch, rows, -1)
        expect = oracle.tree_visible(parents, past, depth + 1, pad=pad)
        assert np.array_equal(unpacked[:, :, :past + rows].astype(bool), expect)
        assert not unpacked[:, :, past + rows:].any()
        first = expect.any(axis=1).argmax(axis=1)
        assert np.array_equal(vis.first_col.cpu().numpy(), first)


def test_visibility_bits_scattered_padding():
    # padding committed in earlier rounds is scattered through the prefix (gap-first
    # schedules), and the pad bitmap may cover tree columns too (never the root)
    rng = np.random.RandomState(12)
    for batch, rows, past, depth in ((5, 61, 333, 6), (3, 40, 31, 9), (2, 255, 64, 30)):
        parents = np.full((batch, rows), -1, dtype=np.int64)
        for b in range(batch):
            for r in range(1, rows):
                parents[b, r] = rng.randint(max(0, r - 7), r)
        pad = rng.rand(batch, past + rows) < 0.3
        pad[:, past] = False
        pad[:, past + 1:] &= rng.rand(batch, rows - 1) < 0.5
        tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                          torch.from_numpy(parents).cuda(), depth)
        vis = tree.visibility(past, torch.from_numpy(pad).cuda())
        bits = vis.bits.cpu().numpy().view(np.uint32)
        unpacked = np.unpackbits(bits.view(np.uint8), bitorder='little').reshape(batch, rows, -1)
        expect = oracle.tree_visible(parents, past, depth + 1, pad=pad)
        assert np.array_equal(unpacked[:, :, :past + rows].astype(bool), expect)
        assert not unpacked[:, :, past + rows:].any()
        assert np.array_equal(vis.first_col.cpu().numpy(), expect[:, 0].argmax(axis=1))


@pytest.mark.parametrize('batch,hq,hkv,rows,past,ragged', [(4, 16, 2, 61, 700, True), (3, 28, 4, 61, 300, True),
                                                          (2, 40, 8, 61, 260, True), (2, 16, 2, 17, 3000, True),
                                                          (1, 16, 2, 1, 129, False), (5, 8, 2, 33, 127, False),
                                                          # at most 128 packed rows per (sequence, KV head):
                                                          # the two warpgroups split the key tiles
                                                          (3, 16, 2, 10, 2013, True), (2, 16, 2, 16, 100, False),
                                                          (4, 8, 1, 16, 300, True), (2, 28, 4, 18, 500, True),
                                                          (3, 16, 2, 5, 250, False), (70, 16, 2, 10, 700, True)])
def test_tensor_core_bits_path_vs_oracle(batch, hq, hkv, rows, past, ragged):
    q, k, v, mask, parents, pad = random_case(batch, hq, hkv, rows, past, 128, seed=batch * 13 + hq, ragged=ragged)
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                      torch.from_numpy(parents).cuda(), rows)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    out = _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, 128 ** -0.5)
    dense = _ops.tree_attention(q, k, v, mask, 128 ** -0.5)
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              oracle.additive_mask(oracle.tree_visible(parents, past, rows, pad=pad), 'bfloat16'),
                              128 ** -0.5)
    check(out, expect)
    check(dense, expect)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def test_tensor_core_full_size_tree_verify_layer():
    """Qwen2.5-3B tree-verify layer: batch 64, 16q/2kv x 128, 61 tree rows, prefixes U{256..3072}
    left-padded to one length; checked on a slice of sequences against the float32 oracle."""
    from analysis_spec_b200 import workloads as W
    rng = np.random.RandomState(5)
    batch, hq, hkv, rows, dim = 64, 16, 2, 61, 128
    prefix = W.prefix_lengths(rng, ('uniform', 256, 3072), batch)
    past = int(prefix.max())
    parents, tokens = W.packed_trees(rng, batch, rows - 1, 6, 10)
    pad = np.zeros((batch, past + rows), dtype=bool)
    pad[:, :past] = W.left_padding(prefix, past)
    gen = torch.Generator(device='cuda').manual_seed(5)
    q = (0.5 * torch.randn(batch, rows, hq * dim, device='cuda', generator=gen)).bfloat16()
    q = q.view(batch, rows, hq, dim).transpose(1, 2)
    kpool = (0.5 * torch.randn(batch, hkv, past + rows + 64, dim, device='cuda', generator=gen)).bfloat16()
    vpool = (0.5 * torch.randn(batch, hkv, past + rows + 64, dim, device='cuda', generator=gen)).bfloat16()
    k, v = kpool[:, :, :past + rows], vpool[:, :, :past + rows]
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(tokens).cuda(),
                      torch.zeros(batch, rows, dtype=torch.long, device='cuda'), 6)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    out = _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, dim ** -0.5)
    visible = oracle.tree_visible(parents, past, 7, pad=pad)
    for sl in (slice(0, 3), slice(30, 32), slice(61, 64)):
        expect = oracle.attention(q[sl].float().cpu().numpy(), k[sl].float().cpu().numpy(),
                                  v[sl].float().cpu().numpy(), oracle.additive_mask(visible[sl], 'bfloat16'),
                                  dim ** -0.5)
        check(out[sl], expect)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def test_registered_interface_and_no_mask():
    name = register()
    from transformers import AttentionInterface
    assert AttentionInterface()[name] is tree_verify_attention
    q, k, v, _, _, _ = random_case(2, 8, 2, 1, 50, 128, seed=1, ragged=False)
    out, weights = tree_verify_attention(Module(4), q, k, v, None)
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), None,
                              128 ** -0.5)
    assert weights is None
    check(out, expect)


@pytest.mark.parametrize('batch,hq,hkv,rows,past', [(4, 16, 2, 61, 300), (3, 28, 4, 17, 1100), (2, 16, 2, 1, 257)])
def test_dense_mask_runs_the_bits_kernel(batch, hq, hkv, rows, past):
    """A dense 0 / lowest-value mask (the drop-in path) is converted once into visibility bits
    identical to tree_mask_bits' and every later call with the same mask reuses them."""
    from analysis_spec_b200.tree_attention import dense_mask_visibility
    q, k, v, mask, parents, pad = random_case(batch, hq, hkv, rows, past, 128, seed=rows + past)
    out, _ = tree_verify_attention(Module(hq // hkv), q, k, v, mask, scaling=128 ** -0.5)
    key, dense = mask._speckv_dense_bits
    assert dense is not None
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                      torch.from_numpy(parents).cuda(), rows)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    assert torch.equal(dense.bits, vis.bits)
    assert torch.equal(dense.first_col, vis.first_col)
    vis_np = oracle.tree_visible(parents, past, rows, pad=pad)
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              oracle.additive_mask(vis_np, 'bfloat16'), 128 ** -0.5)
    check(out, expect)
    # a second layer of the same forward: no new conversion
    tree_verify_attention(Module(hq // hkv), q, k, v, mask, scaling=128 ** -0.5)
    assert mask._speckv_dense_bits[1] is dense
    assert dense_mask_visibility(mask, mask, batch, rows, past + rows) is dense
    # an in-place change of the mask invalidates the cached bits
    mask[:, :, :, past + rows - 1] = torch.finfo(mask.dtype).min
    out2, _ = tree_verify_attention(Module(hq // hkv), q, k, v, mask, scaling=128 ** -0.5)
    assert mask._speckv_dense_bits[1] is not dense
    vis_np[:, :, past + rows - 1] = False
    if vis_np.any(axis=-1).all():
        expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                                  oracle.additive_mask(vis_np, 'bfloat16'), 128 ** -0.5)
        check(out2, expect)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def test_non_binary_mask_keeps_the_dense_kernel():
    q, k, v, mask, parents, pad = random_case(3, 16, 2, 17, 200, 128, seed=3)
    soft = mask.clone()
    soft[:, :, :, 200] = -2.5  # the root's column, visible to every tree row: a soft bias
    out, _ = tree_verify_attention(Module(8), q, k, v, soft, scaling=128 ** -0.5)
    assert soft._speckv_dense_bits[1] is None
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              soft.float().cpu().numpy(), 128 ** -0.5)
    check(out, expect)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
