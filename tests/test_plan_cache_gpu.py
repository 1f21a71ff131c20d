"""Prepared append launches are reused for repeated operands (_ops.append_rows, launch=False).

A verify loop appends the same projection buffers into the same pools at the same length each
round; the second preparation must hand back the plan of the first (no new packing or device
checks) and still append the buffers' current contents, while any change of address or length
prepares a new plan. Pools are compared with the oracle's append (StaticAppendLayer.update,
helper/opd_static_cache.py:99-109) bit for bit."""
import numpy as np
import pytest
import torch

from analysis_spec_b200 import _ops
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_repeated_append_reuses_its_plan_and_appends_current_contents():
    torch.manual_seed(3)
    layers, batch, heads, rows, dim, cap = 3, 4, 2, 9, 128, 64
    pools = [torch.zeros(batch, heads, cap, dim, device='cuda', dtype=torch.bfloat16) for _ in range(2 * layers)]
    kp, vp = pools[:layers], pools[layers:]
    src = [torch.empty(batch, heads, rows, dim, device='cuda', dtype=torch.bfloat16) for _ in range(2 * layers)]
    ks, vs = src[:layers], src[layers:]
    plans = []
    for length in (5, 5, 20):
        for t in src:  # new contents in the same buffers
            t.normal_()
        bits = lambda t: np.ascontiguousarray(t.view(torch.int16).cpu().numpy())  # bf16 bit patterns
        expect = [bits(p) for p in pools]
        for l in range(layers):
            oracle.append(expect[l], expect[layers + l], bits(ks[l]), bits(vs[l]), length)
        go = _ops.append_rows(kp, vp, ks, vs, length, launch=False)
        plans.append(go)
        go()
        torch.cuda.synchronize()
        for p, e in zip(pools, expect):
            assert np.array_equal(bits(p), e)
    assert plans[1] is plans[0]  # same operands, same length: the prepared launch is reused
    assert plans[2] is not plans[0]  # another length: prepared anew
    other = [t.clone() for t in ks]  # other addresses
    assert _ops.append_rows(kp, vp, other, vs, 5, launch=False) is not plans[0]
    assert _ops.device_error() is None
