"""LSE merge kernels vs the oracle merge (tests/test_algorithm_cpu.py:51-59 restated)."""

import numpy as np
import pytest
import torch

from gpu_helpers import assert_device_ok, to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-3, torch.float32: 1e-5}


def _partials(T, H, D, dtype, gen, k=2, neg_inf_every=3):
    outs, lses = [], []
    for i in range(k):
        outs.append(torch.randn(T, H, D, generator=gen).to(dtype).cuda())
        l = torch.randn(T, H, generator=gen) * 3
        if i > 0 and neg_inf_every:
            l[i::neg_inf_every] = float("-inf")
        lses.append(l.cuda())
    return outs, lses


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T,H,D", [(37, 5, 24), (1000, 8, 128), (64, 2, 64), (37, 5, 8),
                                   (129, 3, 256)])
def test_merge_state_in_place(dtype, T, H, D):
    """One-pass form (a head's vectors in one warp: D 8..256 in 16-bit, D 4..128 in fp32)
    and the two-pass form (D=24, fp32 D=256), with -inf rows in either operand."""
    from fa4_ring.merge import merge_state_in_place
    g = torch.Generator().manual_seed(T + H + D)
    (va, vb), (sa, sb) = _partials(T, H, D, dtype, g)
    sa[1::5] = float("-inf")  # empty accumulator rows: the partial is taken as is
    want_o, want_l = orc.merge(to_np(va), to_np(sa), to_np(vb), to_np(sb))
    merge_state_in_place(va, sa, vb, sb)
    np.testing.assert_allclose(to_np(va), want_o, atol=TOL[dtype], rtol=TOL[dtype])
    np.testing.assert_allclose(to_np(sa), want_l, atol=1e-4, rtol=1e-5)
    assert_device_ok()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("k", [1, 2, 5, 8])
def test_merge_states_k_way(dtype, k):
    from fa4_ring.merge import merge_states
    T, H, D = 513, 4, 128
    g = torch.Generator().manual_seed(k)
    outs, lses = _partials(T, H, D, dtype, g, k=k)
    want_o, want_l = orc.merge_states([to_np(o) for o in outs], [to_np(s) for s in lses])
    got_o, got_l = merge_states(outs, lses)
    np.testing.assert_allclose(to_np(got_o), want_o, atol=TOL[dtype], rtol=TOL[dtype])
    np.testing.assert_allclose(to_np(got_l), want_l, atol=1e-4, rtol=1e-5)
    assert_device_ok()


def test_incremental_and_batched_mergers_agree_with_golden():
    import os
    from conftest import GOLDEN
    from fa4_ring import BatchedMerger, IncrementalMerger
    s = np.load(os.path.join(GOLDEN, "steps.npz"))
    oa, ob = torch.from_numpy(s["merge_oa"]).cuda(), torch.from_numpy(s["merge_ob"]).cuda()
    la, lb = torch.from_numpy(s["merge_la"]).cuda(), torch.from_numpy(s["merge_lb"]).cuda()
    for m in (IncrementalMerger(), BatchedMerger()):
        m.add(oa, la)
        m.add(ob, lb)
        np.testing.assert_allclose(to_np(m.result()), s["merge_out"], atol=1e-5, rtol=1e-5)
    # the incremental merger never writes into the first partial it was given
    np.testing.assert_array_equal(to_np(oa), s["merge_oa"])
    assert_device_ok()


def test_both_neg_inf_rows_stay_defined():
    from fa4_ring.merge import merge_state_in_place
    v = torch.ones(4, 2, 8, device="cuda")
    s = torch.full((4, 2), float("-inf"), device="cuda")
    merge_state_in_place(v, s, torch.zeros_like(v), s.clone())
    assert torch.isneginf(s).all() and torch.isfinite(v).all()
