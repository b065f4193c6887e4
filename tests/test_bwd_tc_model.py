"""CPU checks of the staged tcgen05 backward kernel (fa4-cp_b200/csrc/attn_bwd_tc.cuh), which
is not yet part of the library nor run on a GPU:

* it compiles for sm_100a (nvcc, no GPU needed);
* a numpy model of its data flow -- shared-memory tiles with the 128-byte swizzle a
  SWIZZLE_128B tensor-map copy produces, UMMA SW128 descriptors decoded K-major / MN-major,
  TMEM column maps, the TMEM-A operand packing and the hand-swizzled dS^T rows -- run with the
  header's own tile sizes and TMEM columns reproduces the oracle's gradients (bf16 P and dS:
  about 2e-3 relative), and a planted mistake (dS^T rows written without the swizzle) is
  caught.  The model follows the same layout rules as the forward kernel's
  descriptors; the hardware semantics of the one form the forward does not use (an MN-major A
  operand) are checked only on the GPU.
"""

import math
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

from oracle import bwd_oracle as bo
from oracle import ring_oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "fa4-cp_b200", "csrc", "attn_bwd_tc.cuh")


def _constants():
    text = open(HEADER).read()
    c = {}
    for name in ("D", "BN", "BMQ"):
        c[name] = int(re.search(r"constexpr int %s = (\d+);" % name, text).group(1))
    m = re.search(r"TM_ST = (\d+), TM_DPT = (\d+), TM_DV = (\d+), TM_DK = (\d+), "
                  r"TM_DQT = (\d+);", text)
    c.update(zip(("TM_ST", "TM_DPT", "TM_DV", "TM_DK", "TM_DQT"), map(int, m.groups())))
    return c


_C = _constants()
D, BN, BMQ = _C["D"], _C["BN"], _C["BMQ"]
TM_ST, TM_DPT, TM_DV, TM_DK, TM_DQT = (_C[k] for k in ("TM_ST", "TM_DPT", "TM_DV", "TM_DK", "TM_DQT"))
K_CHUNK_BYTES, Q_CHUNK_BYTES = BN * 128, BMQ * 128
KV_BYTES, Q_BYTES, DS_BYTES = BN * D * 2, BMQ * D * 2, BN * BMQ * 2
OFF_K, OFF_V = 0, KV_BYTES
OFF_Q = OFF_V + KV_BYTES
OFF_O = OFF_Q + 2 * Q_BYTES
OFF_DS = OFF_O + 2 * Q_BYTES


def bf16(x):
    x = np.asarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def swz(addr):
    """128-byte swizzle of an absolute (1024-aligned-base) smem byte address."""
    return addr ^ (((addr >> 7) & 7) << 4)


class Smem:
    def __init__(self, nbytes):
        self.v = np.zeros(nbytes // 2, np.float32)  # one value per 16-bit element

    def put(self, addr, val):  # addr: logical (pre-swizzle) byte address of a 16-bit element
        self.v[swz(addr) // 2] = val

    def get(self, addr):
        return self.v[swz(addr) // 2]


def tma_load(sm, dst, tile):  # tile: [rows, 64] values -> rows of 128 B at dst
    rows = tile.shape[0]
    for r in range(rows):
        for e in range(64):
            sm.put(dst + r * 128 + e * 2, tile[r, e])


def desc_kmajor(sm, start, rows, sbo=1024):
    """[rows, 16] operand, K-major SW128: element (m, k) at start + (m/8)*SBO + (m%8)*128 + 2k."""
    out = np.zeros((rows, 16))
    for m in range(rows):
        for k in range(16):
            out[m, k] = sm.get(start + (m // 8) * sbo + (m % 8) * 128 + 2 * k)
    return out


def desc_mnmajor(sm, start, n, lbo, sbo=1024):
    """[16, n] operand (k rows, n contiguous), MN-major SW128: element (k, n) at
    start + (n/64)*LBO + (k/8)*SBO + (k%8)*128 + 2*(n%64)."""
    out = np.zeros((16, n))
    for k in range(16):
        for j in range(n):
            out[k, j] = sm.get(start + (j // 64) * lbo + (k // 8) * sbo + (k % 8) * 128 + 2 * (j % 64))
    return out


def tmem_a(tm, col0):
    """TS operand: A[m][k] (16-bit pairs packed per 32-bit column) from 8 TMEM columns."""
    return np.stack([tm[:, col0 + k // 2, k % 2] for k in range(16)], 1)


def run(q, k, v, do, lse, delta, qs, ql, ks, kl, k0, hk, group, causal, scale, swizzle_ds=True):
    """One CTA of the draft; returns (dq contributions, dk rows, dv rows) as the kernel adds."""
    sm = Smem(OFF_DS + 2 * DS_BYTES)
    tm = np.zeros((128, 512, 2))  # [lane, column, half] (fp32 columns use half 0)
    # producer: K / V tiles (rows past kl read what memory holds; the kernel masks them)
    for c in range(2):
        tma_load(sm, OFF_K + c * K_CHUNK_BYTES, k[ks + k0: ks + k0 + BN, hk, 64 * c: 64 * c + 64])
        tma_load(sm, OFF_V + c * K_CHUNK_BYTES, v[ks + k0: ks + k0 + BN, hk, 64 * c: 64 * c + 64])
    q_first = 0
    if causal:
        q_first = max(0, k0 - (kl - ql)) // BMQ * BMQ
    n_qt = (ql - q_first + BMQ - 1) // BMQ
    dq = np.zeros(q.shape)
    dk_acc = np.zeros((BN, D))
    dv_acc = np.zeros((BN, D))
    scale_log2 = scale * math.log2(math.e)
    for t in range(group * n_qt):
        b = t & 1
        q0 = q_first + (t % n_qt) * BMQ
        hq = hk * group + t // n_qt
        for c in range(2):
            tma_load(sm, OFF_Q + b * Q_BYTES + c * Q_CHUNK_BYTES, q[qs + q0: qs + q0 + BMQ, hq, 64 * c: 64 * c + 64])
            tma_load(sm, OFF_O + b * Q_BYTES + c * Q_CHUNK_BYTES, do[qs + q0: qs + q0 + BMQ, hq, 64 * c: 64 * c + 64])
        sQ, sO, sDS = OFF_Q + b * Q_BYTES, OFF_O + b * Q_BYTES, OFF_DS + b * DS_BYTES
        # S^T, dP^T: SS, both K-major
        st = np.zeros((128, BMQ))
        dpt = np.zeros((128, BMQ))
        for kk in range(D // 16):
            off = kk * 32
            ca = (off // 128) * K_CHUNK_BYTES + off % 128
            cb = (off // 128) * Q_CHUNK_BYTES + off % 128
            a_k = desc_kmajor(sm, OFF_K + ca, 128)
            a_v = desc_kmajor(sm, OFF_V + ca, 128)
            b_q = desc_kmajor(sm, sQ + cb, BMQ)   # B K-major: [N rows, 16] -> B = b_q^T
            b_o = desc_kmajor(sm, sO + cb, BMQ)
            st += a_k @ b_q.T
            dpt += a_v @ b_o.T
        tm[:, TM_ST:TM_ST + BMQ, 0] = st
        tm[:, TM_DPT:TM_DPT + BMQ, 0] = dpt
        # softmax warps (lane r = key)
        lse2 = np.array([(lse[qs + q0 + i, hq] * math.log2(math.e)
                          if (q0 + i < ql and np.isfinite(lse[qs + q0 + i, hq])) else np.inf)
                         if q0 + i < ql else np.inf for i in range(BMQ)])
        dl = np.array([delta[qs + q0 + i, hq] if q0 + i < ql else 0.0 for i in range(BMQ)])
        pw = np.zeros((128, BMQ))
        dw = np.zeros((128, BMQ))
        for r in range(128):
            key = k0 + r
            for qi in range(BMQ):
                vis = key < kl and (not causal or key <= q0 + qi + (kl - ql))
                x = tm[r, TM_ST + qi, 0] * scale_log2 - lse2[qi]
                pr = 2.0 ** x if vis else 0.0
                pw[r, qi] = pr
                dw[r, qi] = pr * (tm[r, TM_DPT + qi, 0] - dl[qi])
        pw, dw = bf16(pw), bf16(dw)
        for r in range(128):  # dS^T row r -> smem, chunk c at (c ^ (r & 7))
            for c in range(8):
                for e in range(8):
                    # the kernel writes physical addresses itself: r*128 + ((c ^ (r&7))*16) + 2e
                    cc = (c ^ (r & 7)) if swizzle_ds else c
                    phys = sDS + r * 128 + cc * 16 + 2 * e
                    sm.v[phys // 2] = dw[r, 8 * c + e]
        for col in range(BMQ // 2):  # P^T, dS^T packed into TMEM columns [0,32)
            tm[:, TM_ST + col, 0] = pw[:, 2 * col]
            tm[:, TM_ST + col, 1] = pw[:, 2 * col + 1]
            tm[:, TM_DPT + col, 0] = dw[:, 2 * col]
            tm[:, TM_DPT + col, 1] = dw[:, 2 * col + 1]
        # dV += P^T dO, dK += dS^T Q: TS with dO / Q as MN-major B
        for kk in range(BMQ // 16):
            bo_ = desc_mnmajor(sm, sO + kk * 16 * 128, D, Q_CHUNK_BYTES)
            bq_ = desc_mnmajor(sm, sQ + kk * 16 * 128, D, Q_CHUNK_BYTES)
            dv_acc += tmem_a(tm, TM_ST + kk * 8) @ bo_
            dk_acc += tmem_a(tm, TM_DPT + kk * 8) @ bq_
        # dQ^T = K^T dS^T: A = K MN-major ([16 keys, 128 d] -> A = that^T), B = dS^T MN-major
        dqt = np.zeros((D, BMQ))
        for kk in range(BN // 16):
            a_kt = desc_mnmajor(sm, OFF_K + kk * 16 * 128, D, K_CHUNK_BYTES)   # [16 keys, D]
            b_ds = desc_mnmajor(sm, sDS + kk * 16 * 128, BMQ, DS_BYTES)         # [16 keys, BMQ]
            dqt += a_kt.T @ b_ds
        for qi in range(min(BMQ, ql - q0)):
            dq[qs + q0 + qi, hq] += dqt[:, qi] * scale
    return dq, dk_acc * scale, dv_acc


def _errors(T, Hq, Hkv, causal, seed, swizzle_ds=True):
    rng = np.random.default_rng(seed)
    q, do = bf16(rng.standard_normal((T, Hq, D))), bf16(rng.standard_normal((T, Hq, D)))
    k, v = bf16(rng.standard_normal((T, Hkv, D))), bf16(rng.standard_normal((T, Hkv, D)))
    scale = 1 / math.sqrt(D)
    out, lse = orc.attn(q, k, v, True, scale, np.float64)
    delta = bo.row_delta(bf16(out), do)
    # rows past the end read zeros (a tensor-map copy fills out-of-range rows)
    pad = lambda x: np.concatenate([x, np.zeros((2 * BN,) + x.shape[1:], x.dtype)])  # noqa: E731
    qp, kp, vp, dop, lsep, dlp = (pad(x) for x in (q, k, v, do, lse, delta))
    group = Hq // Hkv
    dq, dk, dv = np.zeros(qp.shape), np.zeros(kp.shape), np.zeros(vp.shape)
    for hk in range(Hkv):
        for k0 in range(0, T, BN):
            a, b_, c_ = run(qp, kp, vp, dop, lsep, dlp, 0, T, 0, T, k0, hk, group, causal, scale,
                            swizzle_ds)
            dq += a
            n = min(BN, T - k0)
            dk[k0:k0 + n, hk] += b_[:n]
            dv[k0:k0 + n, hk] += c_[:n]
    want = bo.attn_bwd_chunk(q, k, v, do, lse, delta, causal, scale)
    return [float(np.abs(g - w).max() / max(1.0, np.abs(w).max()))
            for g, w in zip((dq[:T], dk[:T], dv[:T]), want)]


@pytest.mark.parametrize("T,Hq,Hkv,causal", [(160, 2, 1, True), (200, 4, 2, True),
                                             (200, 4, 2, False)])
def test_model_of_the_staged_kernel_matches_the_oracle(T, Hq, Hkv, causal):
    assert max(_errors(T, Hq, Hkv, causal, seed=T + Hq)) < 1e-2


def test_model_catches_a_planted_layout_mistake():
    assert _errors(160, 2, 1, True, seed=3, swizzle_ds=False)[0] > 0.1


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not found")
def test_staged_kernel_compiles_for_sm100a(tmp_path):
    res = subprocess.run(["nvcc", "-x", "cu", "-gencode", "arch=compute_100a,code=sm_100a",
                          "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-c", HEADER, "-o",
                          str(tmp_path / "tc.o")], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-2000:]


def test_softmax_warps_reach_every_named_barrier_after_a_give_up():
    """The staged kernel's four softmax warps share named barrier 1 (128 threads) once per
    query tile.  If one warp's bounded wait expires while the others' succeed, the warp that
    gave up must still reach every later named_sync, or the others wait there forever.  The
    loop is modelled trip by trip (named_sync, then the waits, which expire for the chosen warp
    at the chosen trip, or for every warp once the CTA's abort flag is up); every warp must
    arrive at the barrier exactly n_tiles times for every choice.  A source guard keeps the
    loop free of `break`."""
    import itertools
    import re

    src = open(os.path.join(ROOT, "fa4-cp_b200", "csrc", "attn_bwd_tc.cuh")).read()
    loop = src[src.index("Every softmax warp runs every trip"):src.index("dK / dV of this key row")]
    assert "named_sync(1, 128)" in loop and not re.search(r"\bbreak\b", loop)

    n_tiles, warps = 5, 4
    for bad_warp, bad_trip, which in itertools.product(range(warps), range(n_tiles), (0, 1)):
        arrivals = [0] * warps
        aborted = [False] * warps
        cta_abort = False
        for t in range(n_tiles):
            for w in range(warps):
                arrivals[w] += 1  # named_sync(1, 128)
                if aborted[w]:
                    continue
                # s_full wait, then (t >= 2) the ds_free wait; a wait gives up when its own
                # limit expires or when another warp already raised the CTA's abort flag
                for k, needed in ((0, True), (1, t >= 2)):
                    if not needed or aborted[w]:
                        continue
                    expired = (w == bad_warp and t == bad_trip and k == which) or cta_abort
                    if expired:
                        aborted[w] = True
                        cta_abort = True
        assert arrivals == [n_tiles] * warps, (bad_warp, bad_trip, which, arrivals)
