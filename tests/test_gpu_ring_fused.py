"""The persistent ring kernel (``fa4cp_ring_attn_fused``): a rank's whole zig-zag ring
forward in one launch, with the online softmax carried across the steps.

Single GPU, through the C ABI: for every rank of a cp group the receive slots are filled
directly with the other ranks' shards -- slot ``i`` holds the K/V of rank
``(r - i - 1) mod cp``, as the copy-engine transport leaves them -- and the kernel runs
with no hop counter (every slot present).  Each rank's output and LSE are checked against
the oracle's ``ring_rank`` on the same (rounded) inputs (out <= 2e-2, LSE <= 1e-3) and the
stitched output against dense causal attention.  One case passes a counter that already
holds its target (the in-kernel wait returns at once).  e4m3: every rank quantises its own
shards (scale = amax/448), the K/V descales are indexed by source rank, and the oracle runs
on the dequantised shards: out <= 6e-2 on every row, LSE <= 1e-3 (the tolerances of the
FP8 path).  Rows that see only a handful of keys are the hard case for an e4m3 P (3 mantissa
bits): the kernel feeds the causal diagonal tile's P to the PV MMA as two e4m3 terms
(P = hi + lo), so those rows are as accurate as the rest.  head_dim 256 runs the one-query-
tile ring kernel, for f16 / bf16 and for a bf16 query with e4m3 K/V
(``fa4cp_ring_attn_fused_mixed``: the K/V as exact bf16 images, descales by source rank).  The
multi-GPU run of the same kernels behind the copy-engine transport is
``tests/dist_ring_check.py``.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from gpu_helpers import assert_device_ok, dequant, quant_e4m3, to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu

OUT_TOL, LSE_TOL = 2e-2, 1e-3


def run_fused(cp, lens, H, Hkv, D, dtype, seed, counter=False, fp8=False, two_pass=False,
              mixed=False):
    from fa4_ring import _lib
    from fa4_ring.zigzag import zigzag_shard_varlen
    lib = _lib.load()
    g = torch.Generator().manual_seed(seed)
    cu_full = [0] + [int(x) for x in np.cumsum(lens)]
    N = cu_full[-1]
    q, k, v = (torch.randn(N, h, D, generator=g).to(dtype).cuda() for h in (H, Hkv, Hkv))
    qs, ks, vs, lcu = [], [], [], None
    for r in range(cp):
        lq, lcu = zigzag_shard_varlen(q, cu_full, r, cp)
        qs.append(lq)
        ks.append(zigzag_shard_varlen(k, cu_full, r, cp)[0])
        vs.append(zigzag_shard_varlen(v, cu_full, r, cp)[0])
    T = qs[0].shape[0]
    max_local = max(lens) // cp
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream().cuda_stream
    qd = kd = vd = None
    out_dt = dtype
    if fp8:  # per-rank quantisation; descales by source rank
        qq = [quant_e4m3(t) for t in qs]
        kq = [quant_e4m3(t) for t in ks]
        vq = [quant_e4m3(t) for t in vs]
        q_np = [dequant(a, b) for a, b in qq]
        k_np = [dequant(a, b) for a, b in kq]
        v_np = [dequant(a, b) for a, b in vq]
        qs, ks, vs = [a.cuda() for a, _ in qq], [a.cuda() for a, _ in kq], [a.cuda() for a, _ in vq]
        kd = torch.stack([b.reshape(1).expand(Hkv) for _, b in kq]).contiguous().cuda()
        vd = torch.stack([b.reshape(1).expand(Hkv) for _, b in vq]).contiguous().cuda()
        qds = [b.reshape(1).expand(Hkv).contiguous().cuda() for _, b in qq]
        dtype, out_dt = torch.float8_e4m3fn, torch.bfloat16
    elif mixed:  # bf16 q; e4m3 K/V quantised per rank, passed as their exact bf16 images
        kq = [quant_e4m3(t) for t in ks]
        vq = [quant_e4m3(t) for t in vs]
        q_np = [to_np(t) for t in qs]
        k_np = [dequant(a, b) for a, b in kq]
        v_np = [dequant(a, b) for a, b in vq]
        ks = [a.to(torch.bfloat16) for a, _ in kq]
        vs = [a.to(torch.bfloat16) for a, _ in vq]
        assert all(torch.equal(a.float(), b.float()) for a, b in zip(ks, (x for x, _ in kq)))
        kd = torch.stack([b.reshape(1).expand(Hkv) for _, b in kq]).contiguous().cuda()
        vd = torch.stack([b.reshape(1).expand(Hkv) for _, b in vq]).contiguous().cuda()
    else:
        q_np = [to_np(t) for t in qs]
        k_np = [to_np(t) for t in ks]
        v_np = [to_np(t) for t in vs]
    elem = 1 if fp8 else 2
    tol_o, tol_l = (6e-2, LSE_TOL) if fp8 else (OUT_TOL, LSE_TOL)
    lcu_list = [int(x) for x in lcu.tolist()]
    outs = []
    for r in range(cp):
        nsl = max(cp - 1, 1)
        slots_k = torch.zeros(nsl, T, Hkv, D, dtype=dtype, device="cuda")
        slots_v = torch.zeros_like(slots_k)
        for i in range(cp - 1):
            src = (r - i - 1) % cp
            slots_k[i].copy_(ks[src])
            slots_v[i].copy_(vs[src])
        out = torch.full((T, H, D), float("nan"), dtype=out_dt, device="cuda")
        lse = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
        ctr, base = None, 0
        if counter:
            base = 1000
            ctr = torch.tensor([base + cp - 1], dtype=torch.int32, device="cuda")
        if mixed:
            rc = lib.fa4cp_ring_attn_fused_mixed(
                qs[r].data_ptr(), ks[r].data_ptr(), vs[r].data_ptr(), slots_k.data_ptr(),
                slots_v.data_ptr(), T * Hkv * D * 2, out.data_ptr(), lse.data_ptr(),
                lcu.data_ptr(), len(lens), max_local, T, H, Hkv, D, scale, _lib.ptr(kd),
                _lib.ptr(vd), cp, r, None if ctr is None else ctypes.c_void_p(ctr.data_ptr()),
                base, stream)
        elif two_pass:
            # step 0 (local K/V, causal) on its own, then the remote steps merged into it
            rc = lib.fa4cp_attn_fwd(
                qs[r].data_ptr(), ks[r].data_ptr(), vs[r].data_ptr(), out.data_ptr(),
                lse.data_ptr(), lcu.data_ptr(), lcu.data_ptr(), len(lens), max_local, T, T, H, Hkv,
                D, _lib.dtype_code(dtype), _lib.dtype_code(out_dt), _lib.PATTERN_VARLEN, 1, scale,
                None, None, None, 0, stream)
            assert rc == 0, _lib.last_error()
            rc = lib.fa4cp_ring_attn_fused_remote(
                qs[r].data_ptr(), ks[r].data_ptr(), vs[r].data_ptr(), slots_k.data_ptr(),
                slots_v.data_ptr(), T * Hkv * D * elem, out.data_ptr(), lse.data_ptr(),
                lcu.data_ptr(), len(lens), max_local, T, H, Hkv, D, _lib.dtype_code(dtype), scale,
                cp, r, None if ctr is None else ctypes.c_void_p(ctr.data_ptr()), base, stream)
        else:
            rc = lib.fa4cp_ring_attn_fused(
                qs[r].data_ptr(), ks[r].data_ptr(), vs[r].data_ptr(), slots_k.data_ptr(),
                slots_v.data_ptr(), T * Hkv * D * elem, out.data_ptr(), lse.data_ptr(),
                lcu.data_ptr(), len(lens), max_local, T, H, Hkv, D, _lib.dtype_code(dtype), scale,
                _lib.ptr(qds[r]) if fp8 else None, _lib.ptr(kd), _lib.ptr(vd), cp, r,
                None if ctr is None else ctypes.c_void_p(ctr.data_ptr()), base, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        want_o, want_l = orc.ring_rank(q_np[r], k_np, v_np, r, cp, scale, lcu_list)
        got_o = to_np(out)
        np.testing.assert_allclose(got_o, want_o, atol=tol_o, rtol=0)
        np.testing.assert_allclose(to_np(lse), want_l, atol=tol_l, rtol=0)
        outs.append(to_np(out))
    if fp8 or mixed:
        assert_device_ok()
        return
    # the stitched output is plain causal attention of every sequence
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    for j in range(len(lens)):
        a, b = cu_full[j], cu_full[j + 1]
        got = orc.zigzag_unshard([o[lcu_list[j]:lcu_list[j + 1]] for o in outs], cp)
        dense, _ = orc.dense_causal(qn[a:b], kn[a:b], vn[a:b], scale)
        np.testing.assert_allclose(got, dense, atol=OUT_TOL, rtol=0)
    assert_device_ok()


@pytest.mark.parametrize("cp,lens,H,Hkv,D,dtype", [
    (1, [512], 4, 2, 128, torch.bfloat16),
    (2, [2 * 2 * 160], 4, 2, 128, torch.bfloat16),
    (4, [2 * 4 * 200], 8, 2, 128, torch.bfloat16),        # half of 200 rows: partial tiles
    (8, [2 * 8 * 256], 4, 1, 128, torch.bfloat16),
    (3, [2 * 3 * 100], 4, 4, 64, torch.float16),          # D = 64, f16, MHA
    (4, [2 * 4 * n for n in (40, 3, 97, 64)], 4, 1, 128, torch.bfloat16),  # packed sequences
])
def test_ring_fused_matches_oracle(cp, lens, H, Hkv, D, dtype):
    run_fused(cp, lens, H, Hkv, D, dtype, seed=cp * 7 + len(lens))


@pytest.mark.parametrize("cp,lens,H,Hkv", [
    (1, [512], 4, 2),
    (4, [2 * 4 * 200], 8, 2),
    (8, [2 * 8 * 128], 4, 1),
    (3, [2 * 3 * n for n in (40, 97)], 4, 2),
])
def test_ring_fused_fp8_per_source_descales(cp, lens, H, Hkv):
    run_fused(cp, lens, H, Hkv, 128, torch.bfloat16, seed=100 + cp, fp8=True)


@pytest.mark.parametrize("cp,lens,H,Hkv,D,dtype", [
    (1, [512], 4, 2, 128, torch.bfloat16),                 # no remote step: step 0 alone
    (2, [2 * 2 * 160], 4, 2, 128, torch.bfloat16),
    (8, [2 * 8 * 256], 4, 1, 128, torch.bfloat16),
    (3, [2 * 3 * 100], 4, 4, 64, torch.float16),
    (4, [2 * 4 * n for n in (40, 3, 97, 64)], 4, 1, 128, torch.bfloat16),  # rows with no remote key
])
def test_ring_remote_walk_merged_into_step0(cp, lens, H, Hkv, D, dtype):
    """The direct-push forward of f16 / bf16: step 0 by fa4cp_attn_fwd, then the ring kernel
    over the remote steps only (fa4cp_ring_attn_fused_remote), merged in its epilogue."""
    run_fused(cp, lens, H, Hkv, D, dtype, seed=40 + cp, two_pass=True)


@pytest.mark.parametrize("cp,lens,H,Hkv,D,dtype", [
    (1, [512], 4, 2, 256, torch.bfloat16),
    (2, [2 * 2 * 160], 4, 2, 256, torch.bfloat16),         # 160-row halves: a partial tile
    (4, [2 * 4 * n for n in (40, 3, 97, 64)], 4, 1, 256, torch.float16),  # packed sequences
])
def test_ring_fused_head_dim_256(cp, lens, H, Hkv, D, dtype):
    """head_dim 256: one 128-row query tile per CTA (fa4cp_ring_attn_fused)."""
    run_fused(cp, lens, H, Hkv, D, dtype, seed=60 + cp)


@pytest.mark.parametrize("cp,lens,H,Hkv", [
    (1, [512], 4, 2),
    (2, [2 * 2 * 160], 4, 2),
    (4, [2 * 4 * 200], 4, 1),
    (8, [2 * 8 * 128], 2, 1),
    (3, [2 * 3 * n for n in (40, 97)], 4, 2),
])
def test_ring_fused_mixed_bf16_q_e4m3_kv(cp, lens, H, Hkv):
    """bf16 q with e4m3 K/V at head_dim 256 (fa4cp_ring_attn_fused_mixed): K/V passed as the
    exact bf16 images of every rank's e4m3 shards, the K/V descales by source rank applied in
    the kernel; against the oracle on the dequantised shards at the bf16 tolerances (out 2e-2,
    LSE 1e-3): no operand is rounded beyond the e4m3 values themselves."""
    run_fused(cp, lens, H, Hkv, 256, torch.bfloat16, seed=80 + cp, mixed=True)


def test_ring_fused_mixed_counter_already_reached():
    run_fused(4, [2 * 4 * 128], 4, 2, 256, torch.bfloat16, seed=6, counter=True, mixed=True)


def test_ring_fused_counter_already_reached():
    run_fused(4, [2 * 4 * 128], 4, 2, 128, torch.bfloat16, seed=5, counter=True)


def test_ring_fused_rejects_unsupported_shapes():
    from fa4_ring import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(256)
    args = [dummy] * 5 + [1 << 20, dummy, dummy, dummy, 1, 64, 128, 4, 2]
    tail = [None, None, None, 2, 0, None, 0, None]
    assert lib.fa4cp_ring_attn_fused(*args, 64, _lib.DTYPE_E4M3, 0.1, *tail) == _lib.ERR_UNSUPPORTED
    assert lib.fa4cp_ring_attn_fused(*args, 96, _lib.DTYPE_BF16, 0.1, *tail) == _lib.ERR_UNSUPPORTED
    # descales with 16-bit operands: only through the e4m3-K/V entry (head_dim 256)
    d = ctypes.c_void_p(256)
    assert lib.fa4cp_ring_attn_fused(*args, 256, _lib.DTYPE_BF16, 0.1, None, d, d,
                                     *tail[3:]) == _lib.ERR_INVALID
    assert lib.fa4cp_ring_attn_fused_mixed(*args, 128, 0.1, d, d, 2, 0, None, 0,
                                           None) == _lib.ERR_INVALID
    assert lib.fa4cp_ring_attn_fused(*args, 128, _lib.DTYPE_F32, 0.1, *tail) == _lib.ERR_UNSUPPORTED
