"""The allocation-free remap entry point, speckv_remap_rows_static, against speckv_remap_rows.

Some callers of this library cannot allocate device memory: hosts that hand all
device memory to their own pooling allocator up front (a raw cudaMalloc fails
there), latency-critical loops where cudaMalloc / cudaFree would synchronise the
device, and foreign-language bindings with no access to the framework's
allocator. For them speckv_remap_rows_static does the batch remap through a
fixed scratch array compiled into the library instead of scratch they pass in.

This file checks, through the C ABI, that it leaves every pool byte-identical
to what speckv_remap_rows leaves, on two calls in a row (the second call finds
the first call's data still in the shared array). It is collected last so that
a run stopping at the first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _lib, _ops

pytestmark = pytest.mark.gpu


def c_abi_args(kpools, vpools, indices):
    bcap, heads, capacity, dim = kpools[0].shape
    return (_lib.ptr_array([p.data_ptr() for p in kpools]), _lib.ptr_array([p.data_ptr() for p in vpools]),
            len(kpools), indices.data_ptr(), indices.numel(), bcap, heads, dim, capacity)


def remap_with_scratch(kpools, vpools, indices, length):
    bcap, heads, capacity, dim = kpools[0].shape
    es = kpools[0].element_size()
    nbytes = _lib.load().speckv_remap_scratch_bytes(indices.numel(), heads, dim, length, es)
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device='cuda') if nbytes else None
    _lib.call('speckv_remap_rows', *c_abi_args(kpools, vpools, indices), length,
              None if scratch is None else scratch.data_ptr(), nbytes, es,
              torch.cuda.current_stream().cuda_stream)


def remap_static(kpools, vpools, indices, length):
    _lib.call('speckv_remap_rows_static', *c_abi_args(kpools, vpools, indices), length,
              kpools[0].element_size(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize('new_batch,heads,dim,dtype,length', [
    (64, 2, 128, torch.bfloat16, 2100),   # prefill repeat of a long prompt: several position chunks
    (13, 3, 37, torch.float32, 517),      # odd row size (4-byte vectors), duplicates
    (400, 2, 128, torch.float32, 40),     # where speckv_remap_rows itself needs scratch
])
def test_static_remap_matches_scratch_remap_on_two_calls(new_batch, heads, dim, dtype, length):
    rng = np.random.RandomState(new_batch + dim)
    gen = torch.Generator(device='cuda').manual_seed(length)
    layers, bcap, capacity = 2, new_batch + 3, length + 11
    kpools = [torch.randn(bcap, heads, capacity, dim, device='cuda', generator=gen).to(dtype) for _ in range(layers)]
    vpools = [torch.randn(bcap, heads, capacity, dim, device='cuda', generator=gen).to(dtype) for _ in range(layers)]
    k_static, v_static = [p.clone() for p in kpools], [p.clone() for p in vpools]
    for call in range(2):
        ids = torch.from_numpy(rng.randint(0, bcap, size=new_batch).astype(np.int64)).cuda()
        remap_with_scratch(kpools, vpools, ids, length)
        remap_static(k_static, v_static, ids, length)
        torch.cuda.synchronize()
        for a, b in zip(kpools + vpools, k_static + v_static):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), f'call {call}'
    assert _ops.device_error() is None


def test_static_remap_rejects_rows_beyond_its_scratch():
    # 2 * 1024 rows * 65 heads * 512-byte rows per position exceeds the fixed
    # array: the call is refused on the host before anything is launched.
    tiny = torch.zeros(1, device='cuda')
    one = _lib.ptr_array([tiny.data_ptr()])
    idx = torch.zeros(1024, dtype=torch.long, device='cuda')
    with pytest.raises(_lib.SpecKVError, match='static scratch'):
        _lib.call('speckv_remap_rows_static', one, one, 1, idx.data_ptr(), 1024, 1024, 65, 256, 8, 8, 2,
                  torch.cuda.current_stream().cuda_stream)
