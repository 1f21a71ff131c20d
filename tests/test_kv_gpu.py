"""KV row kernels (append / compact / remap / move) vs the CPU oracle, bit-exact."""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from oracle import oracle
from tests.cpu_ops import _np

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def rand(shape, dtype, gen):
    return torch.randn(shape, device='cuda', generator=gen).to(dtype)


def host(t):
    return _np(t.detach().cpu().contiguous()).copy()


def same(a, b):
    """Bit equality of a CUDA tensor with a numpy array of the oracle."""
    return np.array_equal(host(a), b)


@pytest.mark.parametrize('layers', [1, 3, 66])
@pytest.mark.parametrize('dtype,dim', [(torch.bfloat16, 128), (torch.float32, 37), (torch.float16, 5),
                                       (torch.float32, 128)])
def test_append_from_strided_projection_views(layers, dtype, dim):
    gen = torch.Generator(device='cuda').manual_seed(layers * 1000 + dim)
    b, h, cap, q, length = 5, 2, 96, 13, 40
    kpools = [rand((7, h, cap, dim), dtype, gen) for _ in range(layers)]
    vpools = [rand((7, h, cap, dim), dtype, gen) for _ in range(layers)]
    # (B, q, H*D) projection viewed as (B, H, q, D), as Qwen2Attention hands them over
    ksrc = [rand((b, q, h * dim), dtype, gen).view(b, q, h, dim).transpose(1, 2) for _ in range(layers)]
    vsrc = [rand((b, q, h * dim), dtype, gen).view(b, q, h, dim).transpose(1, 2) for _ in range(layers)]
    expect = []
    for l in range(layers):
        kp, vp = host(kpools[l]), host(vpools[l])
        oracle.append(kp, vp, _np(ksrc[l].cpu()), _np(vsrc[l].cpu()), length)
        expect.append((kp, vp))
    _ops.append_rows(kpools, vpools, ksrc, vsrc, length)
    for l in range(layers):
        assert same(kpools[l], expect[l][0]) and same(vpools[l], expect[l][1])


def path_like_chosen(rng, batch, past, rows, width):
    """Absolute positions of gap-first padded accepted paths (increasing, chosen[j] >= past + j)."""
    chosen = np.empty((batch, width), dtype=np.int64)
    for b in range(batch):
        n = rng.randint(1, width + 1)
        idx = np.sort(rng.choice(np.arange(1, rows), size=n - 1, replace=False)) if n > 1 else np.array([], int)
        idx = np.concatenate([[0], idx])
        budget = width - n
        dest = np.arange(n) + np.minimum(np.maximum(idx - np.arange(n), 0), budget)
        row = np.arange(width) + past
        row[dest] = idx + past
        chosen[b] = row
    return chosen


@pytest.mark.parametrize('dtype,dim,width', [(torch.bfloat16, 128, 7), (torch.float32, 37, 5),
                                             (torch.float32, 128, 40), (torch.float16, 3, 9)])
def test_compact_suffix_matches_gather_then_copy(dtype, dim, width):
    rng = np.random.RandomState(dim + width)
    gen = torch.Generator(device='cuda').manual_seed(dim)
    layers, b, h, past, rows = 3, 9, 2, 50, max(61, width + 2)
    cap = past + rows + 7
    kpools = [rand((b + 2, h, cap, dim), dtype, gen) for _ in range(layers)]
    vpools = [rand((b + 2, h, cap, dim), dtype, gen) for _ in range(layers)]
    for chosen_np, ext in ((path_like_chosen(rng, b, past, rows, width), 1),
                           (rng.randint(past, past + rows, size=(b, width)), 0),
                           (past + np.arange(width)[None].repeat(b, 0), 2)):
        expect = []
        for l in range(layers):
            kp, vp = host(kpools[l]), host(vpools[l])
            assert oracle.compact_suffix(kp, vp, b, past + rows, chosen_np, past, ext) == 0
            expect.append((kp, vp))
        chosen = torch.from_numpy(chosen_np).cuda()
        _ops.compact_suffix(kpools, vpools, b, past + rows, chosen, past, ext, width)
        for l in range(layers):
            assert same(kpools[l], expect[l][0]) and same(vpools[l], expect[l][1])


@pytest.mark.parametrize('new_batch,dim,dtype', [(64, 128, torch.bfloat16), (13, 37, torch.float32),
                                                 (400, 128, torch.float32)])
def test_remap_permutation_with_duplicates(new_batch, dim, dtype):
    rng = np.random.RandomState(new_batch)
    gen = torch.Generator(device='cuda').manual_seed(new_batch)
    layers, h, cap, length = 2, 2, 40, 33
    bcap = new_batch + 3
    kpools = [rand((bcap, h, cap, dim), dtype, gen) for _ in range(layers)]
    vpools = [rand((bcap, h, cap, dim), dtype, gen) for _ in range(layers)]
    ids = rng.randint(0, bcap, size=new_batch)
    elements = _ops.remap_scratch_elements(new_batch, h, dim, length, kpools[0].element_size())
    assert (elements > 0) == (new_batch == 400)
    scratch = torch.empty(max(elements, 1), device='cuda', dtype=dtype) if elements else None
    expect = []
    for l in range(layers):
        kp, vp = host(kpools[l]), host(vpools[l])
        assert oracle.remap_rows(kp, vp, ids, length) == 0
        expect.append((kp, vp))
    _ops.remap_rows(kpools, vpools, torch.from_numpy(ids).cuda(), length, scratch)
    for l in range(layers):
        assert same(kpools[l], expect[l][0]) and same(vpools[l], expect[l][1])


def test_move_rows_tail_to_holes():
    gen = torch.Generator(device='cuda').manual_seed(7)
    layers, b, h, cap, dim, length = 4, 11, 3, 64, 128, 61
    kpools = [rand((b, h, cap, dim), torch.bfloat16, gen) for _ in range(layers)]
    vpools = [rand((b, h, cap, dim), torch.bfloat16, gen) for _ in range(layers)]
    finished = [1, 0, 0, 1, 0, 1, 0, 0, 0, 1, 0]
    keep, tail, holes = oracle.swap_remove_plan(finished)
    expect = []
    for l in range(layers):
        kp, vp = host(kpools[l]), host(vpools[l])
        oracle.move_rows(kp, vp, np.array(tail), np.array(holes), length)
        expect.append((kp, vp))
    _ops.move_rows(kpools, vpools, torch.tensor(tail, device='cuda'), torch.tensor(holes, device='cuda'), length)
    for l in range(layers):
        assert same(kpools[l], expect[l][0]) and same(vpools[l], expect[l][1])


def test_out_of_range_indices_are_reported_not_faulted():
    # Bounds are checked inside the kernels: the bad entry is skipped and the
    # device error word records it; the context stays usable.
    gen = torch.Generator(device='cuda').manual_seed(9)
    kp = rand((4, 2, 16, 8), torch.float32, gen)
    vp = rand((4, 2, 16, 8), torch.float32, gen)
    before = kp.clone()
    _ops.remap_rows([kp], [vp], torch.tensor([0, 9, 1], device='cuda'), 10)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('remap index', 9)
    assert torch.equal(kp[1], before[1]) and torch.equal(kp[0], before[0])
    _ops.compact_suffix([kp], [vp], 4, 12, torch.full((4, 3), 99, device='cuda'), 4, 0, 3)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('compact index', 99)
    _ops.move_rows([kp], [vp], torch.tensor([-1], device='cuda'), torch.tensor([0], device='cuda'), 4)
    torch.cuda.synchronize()
    assert _ops.device_error() == ('move index', -1)
    assert _ops.device_error() is None


def test_full_size_commit_round_properties():
    """Qwen2.5-3B geometry (36 layers, B=64, 2 KV heads, D=128, bf16): append 61 tree rows,
    commit accepted paths; checked by size-independent properties against torch gathers."""
    from analysis_spec_b200.opd_static_cache import OPDStaticCache
    gen = torch.Generator(device='cuda').manual_seed(3)
    rng = np.random.RandomState(3)
    layers, b, h, d, past, rows = 36, 64, 2, 128, 1900, 61
    cache = OPDStaticCache(2048, batch_capacity=b)
    prefix = [rand((b, h, past, d), torch.bfloat16, gen) for _ in range(2)]
    for l in range(layers):
        cache.update(prefix[l % 2], prefix[(l + 1) % 2], l)
    tree_k = [rand((b, rows, h * d), torch.bfloat16, gen).view(b, rows, h, d).transpose(1, 2) for _ in range(layers)]
    tree_v = [rand((b, rows, h * d), torch.bfloat16, gen).view(b, rows, h, d).transpose(1, 2) for _ in range(layers)]
    cache.update_layers(tree_k, tree_v)
    assert cache.get_seq_length() == past + rows
    width = 7
    chosen = torch.from_numpy(path_like_chosen(rng, b, past, rows, width)).cuda()
    before = [(cache[l][0].clone(), cache[l][1].clone()) for l in (0, 17, 35)]
    cache.commit_accepted(chosen, past, 1)
    assert cache.get_seq_length() == past + width
    index = chosen[:, None, :, None].expand(b, h, width, d)
    for (kb, vb), l in zip(before, (0, 17, 35)):
        k, v = cache[l]
        assert torch.equal(k[:, :, :past + 1], kb[:, :, :past + 1])
        assert torch.equal(k[:, :, past:], kb.gather(2, index))
        assert torch.equal(v[:, :, past:], vb.gather(2, index))
