"""Attention dispatch, device ownership and the bounded-wait timeout path, on the GPU.

* Head dim 128 in bf16 runs on the tensor-core kernels only: a view they cannot read
  is refused (SPECKV_ENOSUPPORT), never sent to a slower kernel without a signal; the
  library counts the launches of each kernel family.
* Operands that are plain host memory are refused on the host before any launch.
* Every wait inside the tensor-core kernel is bounded: the test hook withholds one
  arrival (CTA 0's first Q tile, so that no copy or MMA is in flight), the wait runs
  out after a short limit, the kernel records SPECKV_DERR_TIMEOUT and unwinds, and the
  next normal call on the same context gives the same output as before.
"""
import ctypes

import numpy as np
import pytest
import torch

from analysis_spec_b200 import _lib, _ops
from analysis_spec_b200.tree_verification import PackedTree
from tests.test_attention_gpu import check, random_case
from oracle import oracle

pytestmark = pytest.mark.gpu


def launches():
    tc, cc = ctypes.c_int64(0), ctypes.c_int64(0)
    _lib.call('speckv_attention_launches', ctypes.byref(tc), ctypes.byref(cc))
    return tc.value, cc.value


def bits_case(batch=8, hq=16, hkv=2, rows=61, past=900, seed=3):
    q, k, v, mask, parents, pad = random_case(batch, hq, hkv, rows, past, 128, seed=seed)
    tree = PackedTree(torch.from_numpy(parents).cuda(), torch.from_numpy(parents).cuda(),
                      torch.from_numpy(parents).cuda(), rows)
    vis = tree.visibility(past, torch.from_numpy(pad).cuda())
    return q, k, v, vis, parents, pad


def test_launch_counters_and_no_silent_fallback():
    q, k, v, vis, _, _ = bits_case()
    tc0, cc0 = launches()
    _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, 128 ** -0.5)
    tc1, cc1 = launches()
    assert (tc1 - tc0, cc1 - cc0) == (1, 0)
    # fp32 (and head dims other than 128) run on the CUDA-core kernel, counted apart
    qf, kf, vf, mask, _, _ = random_case(2, 8, 2, 5, 40, 64, seed=4, dtype=torch.float32)
    _ops.tree_attention(qf, kf, vf, mask, 64 ** -0.5)
    tc2, cc2 = launches()
    assert (tc2 - tc1, cc2 - cc1) == (0, 1)
    # a bf16 / head-dim-128 query whose base is 2 bytes off a 16-byte boundary: refused
    batch, hq, rows = q.shape[0], q.shape[1], q.shape[2]
    wide = torch.zeros(batch, rows, hq * 128 + 1, dtype=q.dtype, device='cuda')
    wide[..., 1:] = q.transpose(1, 2).reshape(batch, rows, hq * 128)
    skewed = wide[..., 1:].view(batch, rows, hq, 128).transpose(1, 2)
    with pytest.raises(_lib.SpecKVError) as info:
        _ops.tree_attention_bits(skewed, k, v, vis.bits, vis.first_col, 128 ** -0.5)
    assert info.value.status == _lib.SPECKV_ENOSUPPORT
    assert launches() == (tc2, cc2)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


def test_host_memory_operand_is_refused():
    q, k, v, vis, _, _ = bits_case(batch=2)
    out = torch.empty(2, q.shape[2], q.shape[1], 128, dtype=q.dtype, device='cuda')
    host_out = torch.empty_like(out, device='cpu')  # pageable host memory: unreachable from the GPU
    args = lambda o: (q.data_ptr(), _lib.i64_array(q.stride()[:3]), k.data_ptr(),  # noqa: E731
                      _lib.i64_array(k.stride()[:3]), v.data_ptr(), _lib.i64_array(v.stride()[:3]),
                      vis.bits.data_ptr(), vis.bits.shape[2], vis.first_col.data_ptr(), o, 2, q.shape[1],
                      k.shape[1], q.shape[2], k.shape[2], 128, 128 ** -0.5, _lib.BF16, None, 0,
                      torch.cuda.current_stream().cuda_stream)
    with pytest.raises(_lib.SpecKVError, match='host memory') as info:
        _lib.call('speckv_tree_attention_bits', *args(host_out.data_ptr()))
    assert info.value.status == _lib.SPECKV_EINVAL
    _lib.call('speckv_tree_attention_bits', *args(out.data_ptr()))
    idx = torch.zeros(2, dtype=torch.long)  # host index list for a device pool
    pool = torch.zeros(4, 2, 8, 128, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(_lib.SpecKVError, match='host memory'):
        _lib.call('speckv_move_rows', _lib.ptr_array([pool.data_ptr()]), _lib.ptr_array([pool.data_ptr()]), 1,
                  idx.data_ptr(), idx.data_ptr(), 2, 4, 2, 128, 8, 8, 2, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _ops.device_error() is None


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs two GPUs')
def test_operands_of_another_gpu():
    """The front end makes the operands' GPU current; the C ABI refuses a foreign pointer."""
    with torch.cuda.device(1):
        q, k, v, vis, parents, pad = bits_case(batch=2, seed=9)
    assert torch.cuda.current_device() == 0
    out = _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, 128 ** -0.5)
    assert out.device.index == 1
    past = k.shape[2] - q.shape[2]
    visible = oracle.tree_visible(parents, past, q.shape[2], pad=pad)
    expect = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                              oracle.additive_mask(visible, 'bfloat16'), 128 ** -0.5)
    check(out, expect)
    with pytest.raises(_lib.SpecKVError, match='lives on cuda:1'):
        _lib.call('speckv_tree_attention_bits', q.data_ptr(), _lib.i64_array(q.stride()[:3]), k.data_ptr(),
                  _lib.i64_array(k.stride()[:3]), v.data_ptr(), _lib.i64_array(v.stride()[:3]),
                  vis.bits.data_ptr(), vis.bits.shape[2], vis.first_col.data_ptr(), out.data_ptr(), 2, q.shape[1],
                  k.shape[1], q.shape[2], k.shape[2], 128, 128 ** -0.5, _lib.BF16, None, 0,
                  torch.cuda.current_stream(0).cuda_stream)


def test_bounded_wait_runs_out_and_the_kernel_unwinds():
    q, k, v, vis, _, _ = bits_case(batch=16, past=1400, seed=21)
    ref = _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, 128 ** -0.5)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    try:
        _lib.call('speckv_attention_test_hooks', 2_000_000, 1)  # 2 ms limit, withhold one arrival
        _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, 128 ** -0.5)
        torch.cuda.synchronize()
        err = _ops.device_error()
    finally:
        _lib.call('speckv_attention_test_hooks', 0, 0)
    assert err is not None and err[0] == 'wait timeout', err
    # the context is intact: the next call computes every row again, identically
    again = _ops.tree_attention_bits(q, k, v, vis.bits, vis.first_col, 128 ** -0.5)
    torch.cuda.synchronize()
    assert _ops.device_error() is None
    assert torch.equal(again, ref)
