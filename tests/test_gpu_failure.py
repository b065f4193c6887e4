"""Failure handling of the attention kernel without any GPU fault: a wait that nothing
will satisfy (a withheld K copy) must give up within its bound (~2 s), record a status
code the host can read, drain the CTA's in-flight copies and MMAs, free tensor memory,
and leave the context usable for the next, correct, launch."""

import ctypes
import math

import numpy as np
import pytest
import torch

from gpu_helpers import to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu

GIVE_UP_CODES = {0x101, 0x102, 0x103, 0x104, 0x105, 0x106, 0x107, 0x108, 0x109}


def test_bounded_wait_expires_and_context_stays_usable():
    from fa4_ring import _lib
    from fa4_ring.attn_backend import b200_attn
    lib = _lib.load()
    T = 256
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(T, 1, 128, generator=g).bfloat16().cuda() for _ in range(3))
    out = torch.empty_like(q)
    lse = torch.empty(T, 1, device="cuda")
    cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
    observed = ctypes.c_int32(0)
    rc = lib.fa4cp_selftest_wait_expiry(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                        lse.data_ptr(), cu.data_ptr(), T, ctypes.byref(observed),
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.fa4cp_last_error()
    assert observed.value in GIVE_UP_CODES, hex(observed.value)
    # the status word was cleared, and the next launch runs normally and correctly
    assert _lib.device_status() == 0
    o, l = b200_attn(q, k, v, causal=True)
    want, _ = orc.attn(to_np(q), to_np(k), to_np(v), True, 1.0 / math.sqrt(128))
    np.testing.assert_allclose(to_np(o), want, atol=2e-2, rtol=0)
    assert _lib.device_status() == 0


def test_ring_kernel_hop_wait_expires_and_context_stays_usable():
    """The persistent ring kernel waits for each hop's counter with a wall-time bound.  A
    counter that nothing writes (a peer that never pushes: here a plain device int that stays
    0) must end the wait with status 0x10a within the bound (set to 300 ms for the test), the
    CTAs drain and return, and the next launch runs normally."""
    from fa4_ring import _lib
    from fa4_ring.attn_backend import b200_attn
    lib = _lib.load()
    T, H, Hkv, D, S, rank = 512, 2, 1, 128, 2, 1
    g = torch.Generator().manual_seed(9)
    q = torch.randn(T, H, D, generator=g).bfloat16().cuda()
    k, v = (torch.randn(T, Hkv, D, generator=g).bfloat16().cuda() for _ in range(2))
    slots_k, slots_v = (torch.randn(S - 1, T, Hkv, D, generator=g).bfloat16().cuda() for _ in range(2))
    out = torch.empty_like(q)
    lse = torch.empty(T, H, device="cuda")
    cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")  # never reaches base + 1
    assert lib.fa4cp_ring_set_wait_timeout_ms(300) == 0
    try:
        rc = lib.fa4cp_ring_attn_fused(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), slots_k.data_ptr(), slots_v.data_ptr(),
            T * Hkv * D * 2, out.data_ptr(), lse.data_ptr(), cu.data_ptr(), 1, T, T, H, Hkv, D,
            _lib.DTYPE_BF16, 1.0 / math.sqrt(D), None, None, None, S, rank,
            ctypes.c_void_p(counter.data_ptr()), 0, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.fa4cp_last_error()
        assert _lib.device_status() == 0x10A
    finally:
        assert lib.fa4cp_ring_set_wait_timeout_ms(10000) == 0
    assert _lib.device_status() == 0
    o, _ = b200_attn(q, k, v, causal=True)
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    want, _ = orc.attn(qn, kn, vn, True, 1.0 / math.sqrt(D))
    np.testing.assert_allclose(to_np(o), want, atol=2e-2, rtol=0)
    assert _lib.device_status() == 0
