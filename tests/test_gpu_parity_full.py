"""Parity at the BASELINE configurations' full sizes -- the sizes bench.py times.

Each case runs the CUDA path at a configuration's full size on one GPU and checks sampled
query rows against ``oracle.ring_oracle.dense_causal_rows`` (the reference's dense causal
attention, tests/test_algorithm_cpu.py:93-95, evaluated on those rows only), for out AND
LSE, at the north-star tolerances: out <= 2e-2 (bf16), out <= 6e-2 (e4m3 operands, against
the dequantised fp32 oracle), LSE <= 1e-3.  Sampled rows: the first rows of every half of
every sequence (they see the fewest keys), the last rows (the most keys: long-row effects
such as the lazy rescale and the fp32 row sum over 10^5 keys), and seeded random rows; all
heads of each.  A multi-rank configuration runs chosen ranks of a cp=8 ring on one GPU with
their receive slots filled as the copy-engine transport leaves them (slot i = the K/V of rank
(r - i - 1) mod cp), so every step, source-rank descale and step boundary is exercised; a
rank's local row maps to its global position through the zig-zag layout.

* cfg2 (bf16, N=32768, Hq=32, Hkv=8, D=128): cp=1 through ``ring_flash_attn_with_lse``;
  cp=8 ranks 0 and 7 through the ring kernel.
* cfg3 (e4m3 q/k/v, N=131072, Hq=32, Hkv=8, D=128): cp=1 (per-tensor amax/448) through the
  public call; cp=8 ranks 0 and 5 through the e4m3 ring kernel (per-rank quantisation,
  k/v descales by source rank).
* cfg4 (16 packed sequences of U[1024, 16384] tokens, Hq=16, Hkv=2): cp=8 rank 3.
* cfg5 (bf16 q x e4m3 k/v, N=262144, Hq=16, Hkv=2, D=256, 0.5 N(0,1)): cp=8 rank 2 through
  the per-step ring path (``ring_forward``).
"""

import math

import numpy as np
import pytest
import torch

import bench
from gpu_helpers import assert_device_ok, to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu

OUT_TOL = {"bf16": 2e-2, "e4m3": 6e-2, "mixed": 6e-2}
LSE_TOL = 1e-3


def _full(n, h, d, gen, amp=1.0):
    x = torch.randn(n, h, d, generator=gen, device="cuda", dtype=torch.bfloat16)
    return x.mul_(amp) if amp != 1.0 else x


def _sample_rows(half_lens, n_rand, seed):
    """Local rows of a zig-zag shard: the first 4 and last 2 rows of every half of every
    sequence plus ``n_rand`` seeded random rows.  ``half_lens[j]`` = h_j; sequence j occupies
    local rows [2 * sum(h_<j), 2 * sum(h_<=j))."""
    rows, start = [], 0
    for h in half_lens:
        for a in (start, start + h):
            rows += list(range(a, a + min(4, h))) + list(range(a + max(0, h - 2), a + h))
        start += 2 * h
    rng = np.random.default_rng(seed)
    rows += rng.integers(0, start, size=n_rand).tolist()
    return np.unique(np.asarray(rows, dtype=np.int64))


def _check(got_o, got_l, rows, lcu, lens, r, cp, q_rows_np, k_np, v_np, scale, kind):
    """got_*: the rank's full local output; rows: sampled local rows; q_rows_np: the oracle's
    query rows (already dequantised); k_np / v_np: the FULL packed K/V [sum(lens), Hkv, D]."""
    got_o = _rows(got_o, rows)
    got_l = _rows(got_l, rows)
    want_o = np.empty(got_o.shape, np.float64)
    want_l = np.empty(got_l.shape, np.float64)
    full_cu = np.concatenate([[0], np.cumsum(lens)])
    for j, n in enumerate(lens):
        sel = (rows >= lcu[j]) & (rows < lcu[j + 1])
        if not sel.any():
            continue
        pos = orc.zigzag_rows(n, r, cp)[rows[sel] - lcu[j]]
        a, b = full_cu[j], full_cu[j + 1]
        want_o[sel], want_l[sel] = orc.dense_causal_rows(q_rows_np[sel], pos, k_np[a:b], v_np[a:b],
                                                         scale)
    err_o = float(np.abs(got_o - want_o).max())
    err_l = float(np.abs(got_l - want_l).max())
    assert err_o <= OUT_TOL[kind], f"out max |err| {err_o:.3e} > {OUT_TOL[kind]} ({kind})"
    assert err_l <= LSE_TOL, f"lse max |err| {err_l:.3e} > {LSE_TOL}"
    return err_o, err_l


def _shards(x, full_cu, cp):
    from fa4_ring.zigzag import zigzag_shard_varlen
    out, lcu = [], None
    for r in range(cp):
        s, lcu = zigzag_shard_varlen(x, full_cu, r, cp)
        out.append(s)
    return out, [int(c) for c in lcu.tolist()]


def _quant_per_rank(shards):
    from fa4_ring.fp8 import quantize_e4m3
    q8, sc = zip(*(quantize_e4m3(s) for s in shards))
    return list(q8), list(sc)


def _dequant_full(q8s, scales, full_cu, cp):
    """The full packed tensor rebuilt from every rank's e4m3 shard times its descale (fp32)."""
    from fa4_ring.zigzag import zigzag_unshard_varlen
    deq = [(a.float() * s).to(torch.float32) for a, s in zip(q8s, scales)]
    return to_np(zigzag_unshard_varlen(deq, full_cu, cp))


def _ring_kernel_rank(qs, ks, vs, r, cp, lcu, max_local, Hq, Hkv, D, dtype, scale, qd=None,
                      kd=None, vd=None):
    """Rank r's whole ring forward in one launch of the ring kernel, slots pre-filled."""
    from fa4_ring import _lib
    lib = _lib.load()
    T = qs[r].shape[0]
    elem = qs[r].element_size()
    slots_k = torch.empty(max(cp - 1, 1), T, Hkv, D, dtype=ks[r].dtype, device="cuda")
    slots_v = torch.empty_like(slots_k)
    for i in range(cp - 1):
        slots_k[i].copy_(ks[(r - i - 1) % cp])
        slots_v[i].copy_(vs[(r - i - 1) % cp])
    out_dt = torch.bfloat16 if dtype == torch.float8_e4m3fn else dtype
    out = torch.empty(T, Hq, D, dtype=out_dt, device="cuda")
    lse = torch.empty(T, Hq, dtype=torch.float32, device="cuda")
    cu = torch.tensor(lcu, dtype=torch.int32, device="cuda")
    rc = lib.fa4cp_ring_attn_fused(
        qs[r].data_ptr(), ks[r].data_ptr(), vs[r].data_ptr(), slots_k.data_ptr(),
        slots_v.data_ptr(), T * Hkv * D * elem, out.data_ptr(), lse.data_ptr(), cu.data_ptr(),
        len(lcu) - 1, max_local, T, Hq, Hkv, D, _lib.dtype_code(dtype), scale, _lib.ptr(qd),
        _lib.ptr(kd), _lib.ptr(vd), cp, r, None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    return out, lse


def _rows(t, rows):
    """Rows of a device tensor as fp32 numpy (e4m3 gathered through a byte view)."""
    idx = torch.from_numpy(rows).to(t.device)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8)[idx].view(torch.float8_e4m3fn).float().cpu().numpy()
    return t[idx].float().cpu().numpy()


def _halves(lens, cp):
    return [n // (2 * cp) for n in lens]


@pytest.mark.parametrize("cp,ranks", [(1, [0]), (8, [0, 7])])
def test_cfg2_full_size(cp, ranks):
    C = bench.CONFIGS["cfg2"]
    N, Hq, Hkv, D = C["lens"][0], C["Hq"], C["Hkv"], C["D"]
    g = torch.Generator(device="cuda").manual_seed(1234)
    q, k, v = _full(N, Hq, D, g), _full(N, Hkv, D, g), _full(N, Hkv, D, g)
    scale = 1.0 / math.sqrt(D)
    k_np, v_np = to_np(k), to_np(v)
    full_cu = [0, N]
    qs, lcu = _shards(q, full_cu, cp)
    ks, _ = _shards(k, full_cu, cp)
    vs, _ = _shards(v, full_cu, cp)
    for r in ranks:
        if cp == 1:
            from fa4_ring import RingConfig
            from fa4_ring.ring_attention import ring_flash_attn_with_lse
            out, lse = ring_flash_attn_with_lse(qs[0], ks[0], vs[0], RingConfig(1, 0))
        else:
            out, lse = _ring_kernel_rank(qs, ks, vs, r, cp, lcu, N // cp, Hq, Hkv, D,
                                         torch.bfloat16, scale)
        rows = _sample_rows(_halves([N], cp), 48, seed=r)
        _check(out, lse, rows, lcu, [N], r, cp, _rows(qs[r], rows), k_np, v_np, scale, "bf16")
    assert_device_ok()


@pytest.mark.parametrize("cp,ranks", [(1, [0]), (8, [0, 5])])
def test_cfg3_e4m3_full_size(cp, ranks):
    from fa4_ring import Descales, RingConfig
    from fa4_ring.ring_attention import ring_flash_attn_with_lse
    C = bench.CONFIGS["cfg3"]
    N, Hq, Hkv, D = C["lens"][0], C["Hq"], C["Hkv"], C["D"]
    g = torch.Generator(device="cuda").manual_seed(77)
    full_cu = [0, N]
    qs, lcu = _shards(_full(N, Hq, D, g), full_cu, cp)
    ks, _ = _shards(_full(N, Hkv, D, g), full_cu, cp)
    vs, _ = _shards(_full(N, Hkv, D, g), full_cu, cp)
    q8, qsc = _quant_per_rank(qs)
    k8, ksc = _quant_per_rank(ks)
    v8, vsc = _quant_per_rank(vs)
    del qs, ks, vs
    k_np = _dequant_full(k8, ksc, full_cu, cp)
    v_np = _dequant_full(v8, vsc, full_cu, cp)
    scale = 1.0 / math.sqrt(D)
    for r in ranks:
        if cp == 1:
            out, lse = ring_flash_attn_with_lse(q8[0], k8[0], v8[0], RingConfig(1, 0),
                                                descales=Descales(q=qsc[0], k=ksc, v=vsc))
        else:
            kd = torch.stack([s.reshape(1).expand(Hkv) for s in ksc]).contiguous()
            vd = torch.stack([s.reshape(1).expand(Hkv) for s in vsc]).contiguous()
            qd = qsc[r].reshape(1).expand(Hkv).contiguous()
            out, lse = _ring_kernel_rank(q8, k8, v8, r, cp, lcu, N // cp, Hq, Hkv, D,
                                         torch.float8_e4m3fn, scale, qd, kd, vd)
        rows = _sample_rows(_halves([N], cp), 24, seed=10 + r)
        q_np = _rows(q8[r], rows) * float(qsc[r])
        _check(out, lse, rows, lcu, [N], r, cp, q_np, k_np, v_np, scale, "e4m3")
    assert_device_ok()


def test_cfg4_varlen_full_size():
    C = bench.CONFIGS["cfg4"]
    cp, r = 8, 3
    lens = bench.config_lens("cfg4", cp)
    Hq, Hkv, D = C["Hq"], C["Hkv"], C["D"]
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    g = torch.Generator(device="cuda").manual_seed(4321)
    q, k, v = _full(N, Hq, D, g), _full(N, Hkv, D, g), _full(N, Hkv, D, g)
    qs, lcu = _shards(q, full_cu, cp)
    ks, _ = _shards(k, full_cu, cp)
    vs, _ = _shards(v, full_cu, cp)
    scale = 1.0 / math.sqrt(D)
    out, lse = _ring_kernel_rank(qs, ks, vs, r, cp, lcu, max(lens) // cp, Hq, Hkv, D,
                                 torch.bfloat16, scale)
    rows = _sample_rows(_halves(lens, cp), 32, seed=4)
    _check(out, lse, rows, lcu, lens, r, cp, _rows(qs[r], rows), to_np(k), to_np(v), scale, "bf16")
    assert_device_ok()


def test_cfg5_bf16_query_e4m3_kv_full_size():
    from fa4_ring import Descales, RingConfig
    from fa4_ring.ring_attention import ring_forward
    C = bench.CONFIGS["cfg5"]
    N, Hq, Hkv, D, amp = C["lens"][0], C["Hq"], C["Hkv"], C["D"], C["amp"]
    cp, r = 8, 2
    g = torch.Generator(device="cuda").manual_seed(55)
    full_cu = [0, N]
    qs, lcu = _shards(_full(N, Hq, D, g, amp), full_cu, cp)
    ks, _ = _shards(_full(N, Hkv, D, g, amp), full_cu, cp)
    vs, _ = _shards(_full(N, Hkv, D, g, amp), full_cu, cp)
    k8, ksc = _quant_per_rank(ks)
    v8, vsc = _quant_per_rank(vs)
    del ks, vs
    k_np = _dequant_full(k8, ksc, full_cu, cp)
    v_np = _dequant_full(v8, vsc, full_cu, cp)
    T = N // cp
    cu = torch.tensor(lcu, dtype=torch.int32, device="cuda")
    out, lse = ring_forward(qs[r], lambda s: (k8[(r - s) % cp], v8[(r - s) % cp]), lambda s: None,
                            RingConfig(cp_size=cp, cp_rank=r), cu=cu, nseq=1, max_seqlen=T,
                            descales=Descales(k=ksc, v=vsc), return_lse=True)
    scale = 1.0 / math.sqrt(D)
    rows = _sample_rows(_halves([N], cp), 16, seed=5)
    _check(out, lse, rows, lcu, [N], r, cp, _rows(qs[r], rows), k_np, v_np, scale, "mixed")
    assert_device_ok()
