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
