"""sm_100a attention kernel vs the oracle: out max-abs <= 2e-2 (bf16/fp16) or 6e-2 (e4m3,
vs the dequantised-fp32 oracle), LSE <= 1e-3, on seeded inputs; causal/non-causal, GQA/MQA,
ragged and empty sequences, the three ring step patterns, and the fused merge epilogue."""

import math

import numpy as np
import pytest
import torch

from gpu_helpers import assert_device_ok, dequant, quant_e4m3, to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu

OUT_TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float8_e4m3fn: 6e-2}
LSE_TOL = 1e-3


def _bottom_right_causal(q, k, v, scale):
    """Causal with the FA convention for T_q != T_k: key j visible to query i iff
    j <= i + (T_k - T_q).  Equals the oracle's square tril when T_q == T_k."""
    tq, tk = q.shape[0], k.shape[0]
    if tq == tk:
        return orc.attn(q, k, v, True, scale)
    H, Hkv = q.shape[1], k.shape[1]
    g = H // Hkv
    out = np.zeros(q.shape, np.float32)
    lse = np.full(q.shape[:2], -np.inf, np.float32)
    mask = np.arange(tk)[None, :] <= (np.arange(tq)[:, None] + (tk - tq))
    for h in range(H):
        s = q[:, h, :] @ k[:, h // g, :].T * scale
        s = np.where(mask, s, -np.inf)
        m = s.max(-1, keepdims=True)
        ms = np.where(np.isfinite(m), m, 0)
        p = np.exp(s - ms)
        l = p.sum(-1, keepdims=True)
        with np.errstate(invalid="ignore", divide="ignore"):
            out[:, h, :] = np.where(l > 0, (p @ v[:, h // g, :]) / l, 0)
            lse[:, h] = np.where(l[:, 0] > 0, np.log(l[:, 0]) + ms[:, 0], -np.inf)
    return out, lse


def _run_case(q_lens, k_lens, H, Hkv, D, causal, dtype, seed=0, qscale=1.0):
    from fa4_ring.attn_backend import b200_attn
    g = torch.Generator().manual_seed(seed)
    tq, tk = sum(q_lens), sum(k_lens)
    q = (torch.randn(tq, H, D, generator=g) * qscale).to(dtype)
    k = torch.randn(tk, Hkv, D, generator=g).to(dtype)
    v = torch.randn(tk, Hkv, D, generator=g).to(dtype)
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    out, lse = b200_attn(q.cuda(), k.cuda(), v.cuda(), causal=causal, softmax_scale=scale,
                         cu_seqlens_q=cu_q.cuda(), cu_seqlens_k=cu_k.cuda(),
                         max_seqlen_q=max(q_lens), max_seqlen_k=max(k_lens))
    assert out.dtype == dtype and lse.dtype == torch.float32
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    got_o, got_l = to_np(out), to_np(lse)
    for j in range(len(q_lens)):
        a, b = int(cu_q[j]), int(cu_q[j + 1])
        c, d = int(cu_k[j]), int(cu_k[j + 1])
        if b == a:
            continue
        if causal:
            wo, wl = _bottom_right_causal(qn[a:b], kn[c:d], vn[c:d], scale)
        else:
            wo, wl = orc.attn(qn[a:b], kn[c:d], vn[c:d], False, scale)
        finite = np.isfinite(wl)
        np.testing.assert_allclose(got_o[a:b], wo, atol=OUT_TOL[dtype], rtol=0)
        np.testing.assert_allclose(got_l[a:b][finite], wl[finite], atol=LSE_TOL, rtol=0)
        assert np.all(np.isneginf(got_l[a:b][~finite]))
    assert_device_ok()


CASES = [
    # q_lens, k_lens, H, Hkv, D, causal, dtype
    ([256], [256], 4, 2, 128, True, torch.bfloat16),
    ([128], [128], 1, 1, 128, False, torch.bfloat16),
    ([300], [300], 4, 4, 128, True, torch.bfloat16),
    ([300], [300], 8, 1, 128, False, torch.bfloat16),
    ([128], [1000], 4, 2, 128, False, torch.bfloat16),
    ([1000], [1000], 2, 2, 64, True, torch.bfloat16),
    ([513], [513], 4, 2, 128, True, torch.float16),
    ([100, 0, 256, 37], [100, 0, 256, 37], 4, 2, 128, True, torch.bfloat16),
    ([200, 300], [500, 300], 4, 2, 128, True, torch.bfloat16),
    ([2048], [2048], 2, 1, 128, True, torch.bfloat16),
    ([1], [1], 2, 1, 128, True, torch.bfloat16),
    ([77, 129], [1, 255], 2, 2, 64, False, torch.float16),
]


@pytest.mark.parametrize("case", CASES, ids=[str(i) for i in range(len(CASES))])
def test_attn_vs_oracle(case):
    _run_case(*case)


def test_attn_large_scores_exercise_rescale():
    # scores spread over many e-folds: the running max grows across KV tiles
    _run_case([1024], [1024], 2, 1, 128, True, torch.bfloat16, seed=5, qscale=6.0)
    _run_case([640], [640], 2, 2, 128, False, torch.float16, seed=6, qscale=4.0)


def test_attn_fp8_e4m3_with_descales():
    from fa4_ring.attn_backend import b200_attn
    g = torch.Generator().manual_seed(11)
    T, H, Hkv, D = 700, 4, 2, 128
    q32, k32, v32 = (torch.randn(T, h, D, generator=g) for h in (H, Hkv, Hkv))
    (q8, qs), (k8, ks), (v8, vs) = quant_e4m3(q32), quant_e4m3(k32), quant_e4m3(v32)
    scale = 1.0 / math.sqrt(D)
    out, lse = b200_attn(q8.cuda(), k8.cuda(), v8.cuda(), causal=True, softmax_scale=scale,
                         q_descale=qs.cuda(), k_descale=ks.reshape(1).expand(Hkv).cuda(),
                         v_descale=vs.reshape(1, 1).expand(1, Hkv).cuda())
    assert out.dtype == torch.bfloat16
    wo, wl = orc.attn(dequant(q8, qs), dequant(k8, ks), dequant(v8, vs), True, scale)
    np.testing.assert_allclose(to_np(out), wo, atol=OUT_TOL[torch.float8_e4m3fn], rtol=0)
    np.testing.assert_allclose(to_np(lse), wl, atol=LSE_TOL, rtol=0)
    assert_device_ok()


@pytest.mark.parametrize("pattern", ["front_kv", "back_q"])
@pytest.mark.parametrize("accumulate", [False, True])
def test_ring_step_patterns(pattern, accumulate):
    """One ring step on a packed varlen local shard, rows addressed in place."""
    from fa4_ring.attn_backend import PATTERN_BACK_Q, PATTERN_FRONT_KV, attn_into
    g = torch.Generator().manual_seed(3)
    cu = [0, 256, 256 + 96, 256 + 96 + 300]
    T, H, Hkv, D = cu[-1], 4, 2, 128
    dt = torch.bfloat16
    q = torch.randn(T, H, D, generator=g).to(dt)
    k = torch.randn(T, Hkv, D, generator=g).to(dt)
    v = torch.randn(T, Hkv, D, generator=g).to(dt)
    scale = 1.0 / math.sqrt(D)
    pat = orc.PATTERN_FRONT_KV if pattern == "front_kv" else orc.PATTERN_BACK_Q
    want_o, want_l = orc.ring_step(to_np(q), to_np(k), to_np(v), cu, pat, scale)
    # accumulator: a step-0 style partial covering every row
    acc_o = torch.randn(T, H, D, generator=g).to(dt)
    acc_l = torch.randn(T, H, generator=g)
    if accumulate:
        want_o, want_l = orc.merge(to_np(acc_o), to_np(acc_l), want_o, want_l)
        out, lse = acc_o.cuda(), acc_l.cuda()
    else:
        out = torch.full((T, H, D), 7.0, dtype=dt, device="cuda")   # sentinel: rows not covered
        lse = torch.full((T, H), 7.0, device="cuda")
    cu_d = torch.tensor(cu, dtype=torch.int32, device="cuda")
    attn_into(q.cuda(), k.cuda(), v.cuda(), out, lse, cu_d, cu_d, nseq=len(cu) - 1,
              max_seqlen_q=max(b - a for a, b in zip(cu[:-1], cu[1:])),
              pattern=PATTERN_FRONT_KV if pattern == "front_kv" else PATTERN_BACK_Q,
              causal=False, softmax_scale=scale, accumulate=accumulate)
    got_o, got_l = to_np(out), to_np(lse)
    if accumulate or pattern == "front_kv":
        np.testing.assert_allclose(got_o, want_o, atol=2e-2, rtol=0)
        np.testing.assert_allclose(got_l, want_l, atol=LSE_TOL, rtol=0)
    else:
        covered = np.isfinite(want_l[:, 0])
        np.testing.assert_allclose(got_o[covered], want_o[covered], atol=2e-2, rtol=0)
        np.testing.assert_allclose(got_l[covered], want_l[covered], atol=LSE_TOL, rtol=0)
        assert np.all(got_o[~covered] == 7.0) and np.all(got_l[~covered] == 7.0)
    assert_device_ok()


HD256_CASES = [
    ([300], [300], 2, 1, 256, True, torch.bfloat16),
    ([129, 64], [129, 64], 4, 2, 256, False, torch.float16),
    ([640], [640], 2, 2, 256, True, torch.bfloat16),
]


@pytest.mark.parametrize("case", HD256_CASES, ids=[str(i) for i in range(len(HD256_CASES))])
def test_attn_head_dim_256(case):
    _run_case(*case)


@pytest.mark.parametrize("D,causal", [(128, True), (256, True), (256, False), (64, False)])
def test_attn_bf16_query_e4m3_kv(D, causal):
    """bf16 Q with e4m3 K/V (per-tensor descales): vs the oracle on dequantised K/V."""
    from fa4_ring.attn_backend import b200_attn
    g = torch.Generator().manual_seed(D)
    T, H, Hkv = 333, 4, 2
    q = (torch.randn(T, H, D, generator=g) * 0.5).bfloat16()
    (k8, ks), (v8, vs) = (quant_e4m3(torch.randn(T, Hkv, D, generator=g) * 0.5) for _ in range(2))
    scale = 1.0 / math.sqrt(D)
    out, lse = b200_attn(q.cuda(), k8.cuda(), v8.cuda(), causal=causal, softmax_scale=scale,
                         k_descale=ks.cuda(), v_descale=vs.reshape(1).expand(Hkv).cuda())
    assert out.dtype == torch.bfloat16
    wo, wl = orc.attn(to_np(q), dequant(k8, ks), dequant(v8, vs), causal, scale)
    np.testing.assert_allclose(to_np(out), wo, atol=OUT_TOL[torch.float8_e4m3fn], rtol=0)
    np.testing.assert_allclose(to_np(lse), wl, atol=LSE_TOL, rtol=0)
    assert_device_ok()


def test_quantize_and_dequantize_e4m3():
    from fa4_ring.fp8 import dequantize_e4m3, quantize_e4m3
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(257, 3, 128, generator=g) * 3).bfloat16().cuda()
    x8, scale = quantize_e4m3(x)
    amax = x.float().abs().max()
    assert torch.allclose(scale, amax / 448.0, rtol=0, atol=0)
    want8 = (x.float() / scale).to(torch.float8_e4m3fn)
    assert torch.equal(x8.view(torch.uint8), want8.view(torch.uint8))
    d = dequantize_e4m3(x8, scale)
    assert torch.equal(d, (x8.float() * scale).bfloat16())
    per_head = torch.tensor([0.5, 2.0, 1.0], device="cuda")
    d2 = dequantize_e4m3(x8, per_head)
    assert torch.equal(d2, (x8.float() * per_head[None, :, None]).bfloat16())
    z8, zs = quantize_e4m3(torch.zeros(64, device="cuda", dtype=torch.bfloat16))
    assert float(zs) == 1.0 and torch.all(z8.float() == 0)
    assert_device_ok()


PERSISTENT_CASES = [
    # more tiles than SMs: every CTA of the persistent kernel walks several tiles
    ([4096], [4096], 40, 8, 128, True, torch.bfloat16),
    ([2048], [2048], 64, 8, 64, False, torch.float16),
    # ragged packed batch with empty sequences: padding tiles interleaved in the schedule
    ([300, 0, 2000, 17, 1024, 129], [300, 0, 2000, 17, 1024, 129], 32, 4, 128, True,
     torch.bfloat16),
]


@pytest.mark.parametrize("case", PERSISTENT_CASES, ids=[str(i) for i in range(len(PERSISTENT_CASES))])
def test_attn_persistent_many_tiles_per_cta(case):
    _run_case(*case)


def test_attn_fp8_many_tiles_per_cta():
    from fa4_ring.attn_backend import b200_attn
    g = torch.Generator().manual_seed(12)
    T, H, Hkv, D = 2048, 48, 8, 128
    q32, k32, v32 = (torch.randn(T, h, D, generator=g) for h in (H, Hkv, Hkv))
    (q8, qs), (k8, ks), (v8, vs) = quant_e4m3(q32), quant_e4m3(k32), quant_e4m3(v32)
    scale = 1.0 / math.sqrt(D)
    out, lse = b200_attn(q8.cuda(), k8.cuda(), v8.cuda(), causal=True, softmax_scale=scale,
                         q_descale=qs.cuda(), k_descale=ks.cuda(), v_descale=vs.cuda())
    wo, wl = orc.attn(dequant(q8, qs), dequant(k8, ks), dequant(v8, vs), True, scale)
    np.testing.assert_allclose(to_np(out), wo, atol=OUT_TOL[torch.float8_e4m3fn], rtol=0)
    np.testing.assert_allclose(to_np(lse), wl, atol=LSE_TOL, rtol=0)
    assert_device_ok()
