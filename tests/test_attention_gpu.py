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
