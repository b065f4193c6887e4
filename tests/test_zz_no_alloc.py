"""The allocation-free kv8 attention entry point (fa4cp_attn_fwd_kv8_noalloc).

It exists for callers that cannot hand the library a device workspace when they call
(engines that have reserved their memory for their own pools, callers that must not
risk a cudaMalloc's synchronisation, bindings that hold only the tensors they were
given): its dequantised K/V live in a fixed scratch array inside the library.

Checked through the C ABI against the workspace-taking fa4cp_attn_fwd_kv8 on the same
inputs, within the attention tests' tolerances (out <= 2e-2, LSE <= 1e-3), on two calls
in a row with different inputs (the shared scratch keeps the first call's contents when
the second starts), plus the size limit.  The file is named to be collected last.
"""

import ctypes
import math

import pytest
import torch

from gpu_helpers import quant_e4m3

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2
LSE_TOL = 1e-3
SCRATCH_ELEMS = 8 * 1024 * 1024  # K (or V) elements the 32 MiB scratch holds in bf16


def _inputs(seed, T, H, Hkv, D):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(T, H, D, generator=g) * 0.5).bfloat16().cuda()
    k8, ks = quant_e4m3(torch.randn(T, Hkv, D, generator=g) * 0.5)
    v8, vs = quant_e4m3(torch.randn(T, Hkv, D, generator=g) * 0.5)
    kd = ks.reshape(1).expand(Hkv).contiguous().cuda()
    vd = vs.reshape(1).expand(Hkv).contiguous().cuda()
    return q, k8.cuda(), v8.cuda(), kd, vd


def _call(lib, noalloc, q, k8, v8, kd, vd, causal):
    T, H, D = q.shape
    Hkv = k8.shape[1]
    out = torch.empty_like(q)
    lse = torch.empty(T, H, dtype=torch.float32, device="cuda")
    cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    args = [q.data_ptr(), k8.data_ptr(), v8.data_ptr(), out.data_ptr(), lse.data_ptr(),
            cu.data_ptr(), cu.data_ptr(), 1, T, T, T, H, Hkv, D, 1, 0, 1 if causal else 0,
            1.0 / math.sqrt(D), kd.data_ptr(), vd.data_ptr(), 0]
    if noalloc:
        rc = lib.fa4cp_attn_fwd_kv8_noalloc(*args, stream)
    else:
        nbytes = lib.fa4cp_attn_kv8_workspace_bytes(T, Hkv, D)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.fa4cp_attn_fwd_kv8(*args, ws.data_ptr(), nbytes, stream)
    assert rc == 0, lib.fa4cp_last_error()
    return out, lse


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from fa4_ring import _lib
    lib = _lib.load()
    cases = [(1, 1000, 8, 2, 128, True), (2, 700, 4, 2, 256, False)]
    for seed, T, H, Hkv, D, causal in cases:  # two calls in a row, different inputs
        q, k8, v8, kd, vd = _inputs(seed, T, H, Hkv, D)
        ref_o, ref_l = _call(lib, False, q, k8, v8, kd, vd, causal)
        got_o, got_l = _call(lib, True, q, k8, v8, kd, vd, causal)
        torch.cuda.synchronize()
        assert float((got_o.float() - ref_o.float()).abs().max()) <= OUT_TOL
        assert float((got_l - ref_l).abs().max()) <= LSE_TOL
    assert _lib.device_status() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from fa4_ring import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(256)
    Hkv, D = 2, 256
    total_k = SCRATCH_ELEMS // (Hkv * D) + 1
    rc = lib.fa4cp_attn_fwd_kv8_noalloc(dummy, dummy, dummy, dummy, dummy, dummy, dummy, 1, 128,
                                        128, total_k, 4, Hkv, D, 1, 0, 1, 0.1, None, None, 0, None)
    assert rc == -1
    assert b"fixed scratch" in lib.fa4cp_last_error()
