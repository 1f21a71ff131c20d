"""Draft-model attention (helper/fastgrpo_model.py:58-69) through ``draft_sdpa`` over
OPDStaticCache views, with the masks the draft forward uses: the causal commit mask of
AttentionWorkspace.causal (left padding on) and the expansion mask of a draft step.

Checked against the float32 oracle attention (repeat_kv + softmax, pinned to the
reference's SDPA outputs) on the oracle's visibility of the same mask; tolerance for
bf16 / fp16 operands with fp32 accumulation: max |err| <= 2e-2, mean |err| <= 2e-3.
"""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from analysis_spec_b200.draft_attention import draft_sdpa
from analysis_spec_b200.opd_attention import AttentionWorkspace, expansion_mask
from analysis_spec_b200.opd_static_cache import OPDStaticCache
from oracle import oracle

pytestmark = pytest.mark.gpu

MAX_ERR, MEAN_ERR = 2e-2, 2e-3
DTYPE_NAME = {torch.bfloat16: 'bfloat16', torch.float16: 'float16'}


def check(out, q, k, v, vis, dtype):
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              oracle.additive_mask(vis, DTYPE_NAME[dtype]), q.shape[-1] ** -0.5)
    got = out.transpose(1, 2).float().cpu()
    err = (got - torch.from_numpy(expect)).abs()
    assert err.max().item() <= MAX_ERR, err.max().item()
    assert err.mean().item() <= MEAN_ERR, err.mean().item()


def draft_cache(batch, hkv, past, dim, dtype, gen, rng):
    cache = OPDStaticCache(1024, batch_capacity=batch)
    k = (0.5 * torch.randn(batch, hkv, past, dim, device='cuda', generator=gen)).to(dtype)
    v = (0.5 * torch.randn(batch, hkv, past, dim, device='cuda', generator=gen)).to(dtype)
    pad = np.zeros((batch, past + 64), dtype=bool)
    for b in range(batch):
        pad[b, :rng.randint(0, past // 3 + 1)] = True
    cache.update(k, v, 0)
    return cache, pad


@pytest.mark.parametrize('batch,hq,hkv,past,rows,dim,dtype', [(4, 16, 2, 300, 7, 128, torch.bfloat16),
                                                              (3, 28, 4, 517, 5, 128, torch.bfloat16),
                                                              (2, 8, 8, 90, 3, 64, torch.float16)])
def test_draft_commit_forward_causal(batch, hq, hkv, past, rows, dim, dtype):
    rng = np.random.RandomState(past)
    gen = torch.Generator(device='cuda').manual_seed(rows)
    cache, pad = draft_cache(batch, hkv, past, dim, dtype, gen, rng)
    new_k = (0.5 * torch.randn(batch, hkv, rows, dim, device='cuda', generator=gen)).to(dtype)
    new_v = (0.5 * torch.randn(batch, hkv, rows, dim, device='cuda', generator=gen)).to(dtype)
    keys, values = cache.update(new_k, new_v, 0)
    assert keys.shape[2] == past + rows and not keys.is_contiguous()  # strided pool views
    q = (0.5 * torch.randn(batch, hq, rows, dim, device='cuda', generator=gen)).to(dtype)
    ws = AttentionWorkspace('cuda')
    mask = ws.causal('draft_commit', past, rows, batch, dtype, torch.from_numpy(pad).cuda())
    out = draft_sdpa(q, keys, values, mask, hq // hkv)
    assert out.shape == (batch, hq, rows, dim)
    flat = out.transpose(1, 2).contiguous()
    assert flat.data_ptr() == out.data_ptr()  # the caller's transpose + contiguous copies nothing
    check(out, q, keys, values, oracle.causal_visible(batch, rows, past, past + rows, pad), dtype)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.parametrize('batch,hq,hkv,past,draft_k,init', [(4, 16, 2, 260, 8, 240), (2, 40, 8, 1100, 4, 1000)])
def test_draft_expansion_step(batch, hq, hkv, past, draft_k, init):
    dim, dtype = 128, torch.bfloat16
    rng = np.random.RandomState(draft_k)
    gen = torch.Generator(device='cuda').manual_seed(past)
    cache, pad = draft_cache(batch, hkv, past, dim, dtype, gen, rng)
    new_k = (0.5 * torch.randn(batch, hkv, draft_k, dim, device='cuda', generator=gen)).to(dtype)
    new_v = (0.5 * torch.randn(batch, hkv, draft_k, dim, device='cuda', generator=gen)).to(dtype)
    keys, values = cache.update(new_k, new_v, 0)
    cols = past + draft_k
    seen = torch.from_numpy(rng.randint(init, cols, size=(batch, draft_k, 1)).astype(np.int64)).cuda()
    ws = AttentionWorkspace('cuda')
    mask = ws.buffer('draft_expansion', (batch, 1, draft_k, cols), dtype)
    expansion_mask(mask, init, seen, torch.from_numpy(pad).cuda())
    q = (0.5 * torch.randn(batch, hq, draft_k, dim, device='cuda', generator=gen)).to(dtype)
    out = draft_sdpa(q, keys, values, mask, hq // hkv)
    vis = oracle.expansion_visible(batch, draft_k, cols, init, seen.cpu().numpy(), pad)
    check(out, q, keys, values, vis, dtype)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def test_draft_sdpa_argument_checks():
    q = torch.zeros(1, 4, 2, 64, device='cuda', dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 5, 64, device='cuda', dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        draft_sdpa(q, k, k, None, 2)
    with pytest.raises(ValueError):
        draft_sdpa(q, k, k, torch.zeros(1, 1, 2, 5, device='cuda', dtype=torch.bfloat16), 3)
    with pytest.raises(ValueError):
        draft_sdpa(q, k, k, torch.zeros(1, 1, 2, 5, device='cuda', dtype=torch.bfloat16), 2, dropout_p=0.1)


def test_draft_expansion_pairs_padding_and_foreign_mask():
    """Pairs-form padding (filled after the mask kernel) and a mask built outside this
    library both reach the right visibility."""
    batch, hq, hkv, past, draft_k, init, dim, dtype = 3, 16, 2, 300, 6, 280, 128, torch.bfloat16
    rng = np.random.RandomState(4)
    gen = torch.Generator(device='cuda').manual_seed(4)
    cache, pad = draft_cache(batch, hkv, past, dim, dtype, gen, rng)
    new = [(0.5 * torch.randn(batch, hkv, draft_k, dim, device='cuda', generator=gen)).to(dtype) for _ in range(2)]
    keys, values = cache.update(new[0], new[1], 0)
    cols = past + draft_k
    seen = torch.from_numpy(rng.randint(init, cols, size=(batch, draft_k, 1)).astype(np.int64)).cuda()
    pairs = np.array([[b, c] for b in range(batch) for c in rng.choice(init, 5, replace=False)], dtype=np.int64)
    mask = torch.empty(batch, 1, draft_k, cols, device='cuda', dtype=dtype)
    expansion_mask(mask, init, seen, torch.from_numpy(pairs).cuda())
    q = (0.5 * torch.randn(batch, hq, draft_k, dim, device='cuda', generator=gen)).to(dtype)
    out = draft_sdpa(q, keys, values, mask, hq // hkv)
    vis = oracle.expansion_visible(batch, draft_k, cols, init, seen.cpu().numpy(), pad_pairs=pairs)
    check(out, q, keys, values, vis, dtype)
    foreign = mask.clone()  # no attached bits: converted once, then cached
    out2 = draft_sdpa(q, keys, values, foreign, hq // hkv)
    assert foreign._speckv_dense_bits[1] is not None
    check(out2, q, keys, values, vis, dtype)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
