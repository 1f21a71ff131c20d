"""Draft-model attention masks: the causal mask of AttentionWorkspace.causal
(helper/opd_attention.py:31-43, kernel helper/opd_attention_kernels.py:7-22) and the
draft expansion mask (helper/opd_generate.py:143-162).

Fixtures: tests/golden/draft_masks.npz, written by tests/golden/make_golden.py from the
reference's CPU branch, its Triton kernel (interpreted) and its expansion op sequence.
Masks are compared bit for bit: visible entries +0, the rest torch.finfo(dtype).min.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

DTYPES = {'float32': torch.float32, 'bfloat16': torch.bfloat16, 'float16': torch.float16}


def causal_cases(g):
    for n in range(int(g['causal_count'])):
        batch, query, past = (int(x) for x in g[f'c{n}_shape'])
        pad = g[f'c{n}_pad']
        yield batch, query, past, DTYPES[str(g[f'c{n}_dtype'])], (pad if pad.size else None), g[f'c{n}_visible']


def expansion_cases(g):
    for n in range(int(g['expansion_count'])):
        batch, k, cols, init = (int(x) for x in g[f'e{n}_shape'])
        pad, pairs = g[f'e{n}_pad'], g[f'e{n}_pairs']
        yield (batch, k, cols, init, DTYPES[str(g[f'e{n}_dtype'])], g[f'e{n}_seen'], (pad if pad.size else None),
               (pairs if pairs.size else None), g[f'e{n}_visible'])


def test_oracle_causal_matches_reference(golden):
    g = golden('draft_masks')
    for batch, query, past, _, pad, visible in causal_cases(g):
        assert np.array_equal(oracle.causal_visible(batch, query, past, past + query, pad), visible)


def test_oracle_expansion_matches_reference(golden):
    g = golden('draft_masks')
    for batch, k, cols, init, _, seen, pad, pairs, visible in expansion_cases(g):
        assert np.array_equal(oracle.expansion_visible(batch, k, cols, init, seen, pad, pairs), visible)


def test_workspace_capacity_policy_host_side():
    """Buffer growth follows helper/opd_attention.py:10-19 (power of two, at least 256
    elements, one allocation per growth) and positions the ramp of :21-29."""
    from analysis_spec_b200.opd_attention import AttentionWorkspace
    ws = AttentionWorkspace('cpu')
    a = ws.buffer('m', (2, 1, 3, 10), torch.float32)
    assert ws.allocations == 1 and ws.buffers[('m', torch.float32)].numel() == 256
    b = ws.buffer('m', (4, 1, 5, 12), torch.float32)
    assert ws.allocations == 1 and b.data_ptr() == a.data_ptr()
    ws.buffer('m', (4, 1, 9, 40), torch.float32)
    assert ws.allocations == 2 and ws.buffers[('m', torch.float32)].numel() == 2048
    ws.buffer('m', (1,), torch.bfloat16)
    assert ws.allocations == 3
    pos = ws.positions('p', 300, 7)
    assert pos.tolist() == list(range(300, 307)) and ws.buffers[('ramp', torch.long)].numel() == 512
    assert ws.memory_bytes() == 2048 * 4 + 256 * 2 + 256 * 8 + 512 * 8
    with pytest.raises(RuntimeError, match='CUDA'):
        ws.causal('c', 3, 2, 1, torch.float32)


def expected_bits(visible, dtype):
    t = torch.where(torch.from_numpy(np.ascontiguousarray(visible)), 0., torch.finfo(dtype).min).to(dtype)
    return t.view(torch.int32 if dtype == torch.float32 else torch.int16)


def bits(mask):
    m = mask.detach().cpu()[:, 0]
    return m.view(torch.int32 if m.dtype == torch.float32 else torch.int16)


@pytest.mark.gpu
def test_causal_kernel_matches_reference(golden):
    from analysis_spec_b200.opd_attention import AttentionWorkspace
    from analysis_spec_b200 import _ops
    g = golden('draft_masks')
    ws = AttentionWorkspace('cuda')
    for batch, query, past, dtype, pad, visible in causal_cases(g):
        padding = None if pad is None else torch.from_numpy(pad).cuda()
        out = ws.causal('draft_causal', past, query, batch, dtype, padding)
        assert torch.equal(bits(out), expected_bits(visible, dtype))
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.gpu
def test_expansion_kernel_matches_reference(golden):
    from analysis_spec_b200.opd_attention import AttentionWorkspace, expansion_mask
    from analysis_spec_b200 import _ops
    g = golden('draft_masks')
    ws = AttentionWorkspace('cuda')
    for batch, k, cols, init, dtype, seen, pad, pairs, visible in expansion_cases(g):
        mask = ws.buffer('draft_expansion', (batch, 1, k, cols), dtype)
        mask.fill_(1.0)  # stale contents must not survive
        padding = None
        if pad is not None:
            padding = torch.from_numpy(pad).cuda()
        elif pairs is not None:
            padding = torch.from_numpy(pairs).cuda()
        expansion_mask(mask, init, torch.from_numpy(seen).cuda(), padding)
        assert torch.equal(bits(mask), expected_bits(visible, dtype))
        if pairs is not None:  # the per-sequence list form builds the same pairs
            lists = [[int(c) for b, c in pairs if b == s] for s in range(batch)]
            mask.fill_(1.0)
            expansion_mask(mask, init, torch.from_numpy(seen).cuda(), lists)
            assert torch.equal(bits(mask), expected_bits(visible, dtype))
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.gpu
@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16, torch.float16])
def test_masks_multi_chunk_strided_padding_vs_oracle(dtype):
    """Columns spanning several 1024-column chunks, padding given as non-contiguous views."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_attention_kernels import causal_mask
    from analysis_spec_b200.opd_attention import expansion_mask
    rng = np.random.RandomState(7)
    batch, query, past = 3, 9, 4100
    cols = past + query
    base = rng.rand(cols + 8, batch + 2) < 0.1
    pad = torch.from_numpy(base).cuda().t()[:batch]  # strides (1, batch + 2)
    out = torch.full((batch, 1, query, cols), 1.0, device='cuda', dtype=dtype)
    causal_mask(out, past, pad)
    expect = oracle.causal_visible(batch, query, past, cols, base.T[:batch])
    assert torch.equal(bits(out), expected_bits(expect, dtype))
    init = 3000
    seen_pool = torch.from_numpy(rng.randint(init, cols, size=(batch + 1, query + 2, 3)).astype(np.int64)).cuda()
    seen = seen_pool[:batch, :query, :1]
    expansion_mask(out, init, seen, pad)
    expect = oracle.expansion_visible(batch, query, cols, init, seen.cpu().numpy(), base.T[:batch])
    assert torch.equal(bits(out), expected_bits(expect, dtype))
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.gpu
def test_expansion_bad_seen_index_reports_device_error():
    """A seen position outside [0, columns) is reported in the device error word; the
    reference's scatter_ would raise. The row keeps only its first init columns."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_attention import expansion_mask
    assert _ops.device_error() is None
    batch, query, cols, init = 2, 3, 40, 30
    seen = torch.tensor([[[31], [32], [33]], [[34], [cols + 5], [35]]], device='cuda', dtype=torch.long)
    mask = torch.empty(batch, 1, query, cols, device='cuda', dtype=torch.bfloat16)
    expansion_mask(mask, init, seen)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('seen index', cols + 5)
    vis = oracle.expansion_visible(batch, query, cols, init, np.array([[31, 32, 33], [34, 0, 35]]))
    vis[1, 1, 0] = True  # column 0 is below init anyway
    assert torch.equal(bits(mask), expected_bits(vis, torch.bfloat16))


@pytest.mark.gpu
def test_masks_empty_and_invalid_arguments():
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_attention_kernels import causal_mask
    causal_mask(torch.empty(0, 1, 4, 8, device='cuda'), 4)
    with pytest.raises(ValueError):
        causal_mask(torch.empty(2, 1, 4, 8, device='cuda', dtype=torch.int32), 4)
    with pytest.raises(ValueError):
        causal_mask(torch.empty(2, 1, 4, 8, device='cuda'), 4, torch.zeros(2, 5, dtype=torch.bool, device='cuda'))
    with pytest.raises(RuntimeError):
        causal_mask(torch.empty(2, 1, 4, 8, device='cuda'), -1)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def unpack_bits(bits, columns):
    words = bits.cpu().numpy().view(np.uint32)
    unpacked = np.unpackbits(words.view(np.uint8), bitorder='little').reshape(words.shape[0], words.shape[1], -1)
    assert not unpacked[:, :, columns:].any()
    return unpacked[:, :, :columns].astype(bool)


@pytest.mark.gpu
def test_masks_carry_their_visibility_bits(golden):
    """The bits written beside each mask (what the draft attention reads) match the mask."""
    from analysis_spec_b200 import _ops
    from analysis_spec_b200.opd_attention import AttentionWorkspace, expansion_mask
    g = golden('draft_masks')
    ws = AttentionWorkspace('cuda')
    for batch, query, past, dtype, pad, visible in causal_cases(g):
        padding = None if pad is None else torch.from_numpy(pad).cuda()
        out = ws.causal('draft_causal', past, query, batch, dtype, padding)
        key, vis = out._speckv_dense_bits
        assert key == (past + query, query, batch, out._version)
        assert np.array_equal(unpack_bits(vis.bits, past + query), visible)
        assert np.array_equal(vis.first_col.cpu().numpy(), visible.any(axis=1).argmax(axis=1))
    for batch, k, cols, init, dtype, seen, pad, pairs, visible in expansion_cases(g):
        mask = ws.buffer('draft_expansion', (batch, 1, k, cols), dtype)
        padding = torch.from_numpy(pad).cuda() if pad is not None else (
            torch.from_numpy(pairs).cuda() if pairs is not None else None)
        expansion_mask(mask, init, torch.from_numpy(seen).cuda(), padding)
        key, vis = mask._speckv_dense_bits
        if pairs is not None:  # filled after the kernel: the attached bits are stale by version
            assert key[3] != mask._version
            continue
        assert key[3] == mask._version
        assert np.array_equal(unpack_bits(vis.bits, cols), visible)
        assert np.array_equal(vis.first_col.cpu().numpy(), visible.any(axis=1).argmax(axis=1))
    torch.cuda.synchronize()
    assert _ops.device_error() is None
