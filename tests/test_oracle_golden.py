"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py``, which imports the
reference's ``fa4_ring/zigzag.py`` and the CPU ring simulation of its
``tests/test_algorithm_cpu.py``.  Zig-zag indices must match bit-exactly; the fp32
attention/ring outputs within the reference's own tolerance (atol=rtol=1e-4,
``tests/test_algorithm_cpu.py:181,195``).
"""

import math
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import ring_oracle as orc

TOL = dict(atol=1e-4, rtol=1e-4)


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _inputs(n, H, Hkv, D, seed=0):
    torch.manual_seed(seed)
    q, k, v = torch.randn(n, H, D), torch.randn(n, Hkv, D), torch.randn(n, Hkv, D)
    return q, k, v


def _check_sums(sums, tensors):
    got = np.asarray([float(t.double().sum()) for t in tensors])
    np.testing.assert_allclose(got, sums, rtol=0, atol=1e-6)


def test_zigzag_shard_rows_bit_exact():
    z = _load("zigzag.npz")
    n_checked = 0
    for key in z.files:
        if not key.startswith("shard_"):
            continue
        _, n, cp, r = key.split("_")
        n, cp, r = int(n[1:]), int(cp[2:]), int(r[1:])
        assert np.array_equal(orc.zigzag_rows(n, r, cp), z[key]), key
        x = np.arange(n).reshape(n, 1)
        assert np.array_equal(orc.zigzag_shard(x, r, cp).ravel(), z[key])
        n_checked += 1
    assert n_checked > 50


def test_zigzag_roundtrip():
    for cp in (1, 2, 4, 8):
        n = 4 * cp * 3
        x = np.arange(n).reshape(n, 1)
        shards = [orc.zigzag_shard(x, r, cp) for r in range(cp)]
        assert np.array_equal(orc.zigzag_unshard(shards, cp), x)


def test_zigzag_varlen_and_half_index_bit_exact():
    z = _load("zigzag.npz")
    n_checked = 0
    for key in z.files:
        if not (key.startswith("varlen_") and key.endswith("_rows")):
            continue
        _, name, cp, r, _ = key.split("_")
        cp, r = int(cp[2:]), int(r[1:])
        full_cu = z[f"varlen_{name}_full_cu"]
        rows, lcu = orc.zigzag_varlen_rows(full_cu, r, cp)
        assert np.array_equal(rows, z[key])
        assert np.array_equal(lcu, z[f"varlen_{name}_cp{cp}_r{r}_cu"])
        assert np.array_equal(orc.get_half_index(lcu, True), z[f"varlen_{name}_cp{cp}_r{r}_front"])
        assert np.array_equal(orc.get_half_index(lcu, False), z[f"varlen_{name}_cp{cp}_r{r}_back"])
        n_checked += 1
    assert n_checked >= 10


def test_reference_known_answers_zigzag():
    # tests/test_zigzag.py:51-78 of the reference, restated.
    assert orc.get_half_index([0, 4, 12], True).tolist() == [0, 1, 4, 5, 6, 7]
    assert orc.get_half_index([0, 4, 12], False).tolist() == [2, 3, 8, 9, 10, 11]
    for rank in range(2):
        rows, lcu = orc.zigzag_varlen_rows([0, 8, 24], rank, 2)
        assert lcu.tolist() == [0, 4, 12] and rows.shape[0] == 12


@pytest.mark.parametrize("i", range(7))
def test_oracle_matches_reference_ring_and_dense(i):
    a = _load("algo.npz")
    n, H, Hkv, D, cp = a[f"case{i}_dims"].tolist()
    q, k, v = _inputs(n, H, Hkv, D)
    _check_sums(a[f"case{i}_input_sums"], (q, k, v))
    q, k, v = q.numpy(), k.numpy(), v.numpy()
    scale = 1.0 / math.sqrt(D)
    do, dl = orc.dense_causal(q, k, v, scale)
    np.testing.assert_allclose(do, a[f"case{i}_dense_out"], **TOL)
    np.testing.assert_allclose(dl, a[f"case{i}_dense_lse"], **TOL)
    ro, rl = orc.simulate_ring(q, k, v, cp, scale)
    np.testing.assert_allclose(ro, a[f"case{i}_ring_out"], **TOL)
    np.testing.assert_allclose(rl, a[f"case{i}_dense_lse"], **TOL)


@pytest.mark.parametrize("i", range(4))
def test_oracle_matches_reference_ring_varlen(i):
    a = _load("algo.npz")
    H, Hkv, D, cp = a[f"varlen{i}_dims"].tolist()
    lens = a[f"varlen{i}_lens"].tolist()
    torch.manual_seed(0)
    seqs = [(torch.randn(n, H, D), torch.randn(n, Hkv, D), torch.randn(n, Hkv, D)) for n in lens]
    np.testing.assert_allclose([sum(float(t.double().sum()) for t in s) for s in seqs],
                               a[f"varlen{i}_input_sums"], atol=1e-6, rtol=0)
    seqs = [tuple(t.numpy() for t in s) for s in seqs]
    recon = orc.simulate_ring_varlen(seqs, cp, 1.0 / math.sqrt(D))
    for j, r in enumerate(recon):
        np.testing.assert_allclose(r, a[f"varlen{i}_seq{j}_ring_out"], **TOL)


def test_oracle_ring_steps_and_merge_match_reference():
    s = _load("steps.npz")
    n, H, Hkv, D, cp = s["dims"].tolist()
    q, k, v = _inputs(n, H, Hkv, D, seed=3)
    _check_sums(s["input_sums"], (q, k, v))
    q, k, v = q.numpy(), k.numpy(), v.numpy()
    scale = 1.0 / math.sqrt(D)
    rank, src = int(s["rank"]), int(s["src"])
    lq = orc.zigzag_shard(q, rank, cp)
    rk, rv = orc.zigzag_shard(k, src, cp), orc.zigzag_shard(v, src, cp)
    lk, lv = orc.zigzag_shard(k, rank, cp), orc.zigzag_shard(v, rank, cp)
    T = lq.shape[0]
    h = T // 2
    cu = [0, T]
    o, l = orc.ring_step(lq, lk, lv, cu, orc.PATTERN_LOCAL_CAUSAL, scale)
    np.testing.assert_allclose(o, s["local_causal_out"], **TOL)
    np.testing.assert_allclose(l, s["local_causal_lse"], **TOL)
    o, l = orc.ring_step(lq, rk, rv, cu, orc.PATTERN_FRONT_KV, scale)
    np.testing.assert_allclose(o, s["front_kv_out"], **TOL)
    np.testing.assert_allclose(l, s["front_kv_lse"], **TOL)
    o, l = orc.ring_step(lq, rk, rv, cu, orc.PATTERN_BACK_Q, scale)
    np.testing.assert_allclose(o[h:], s["back_q_out"], **TOL)
    np.testing.assert_allclose(l[h:], s["back_q_lse"], **TOL)
    assert np.all(o[:h] == 0) and np.all(np.isneginf(l[:h]))
    mo, ml = orc.merge(s["merge_oa"], s["merge_la"], s["merge_ob"], s["merge_lb"])
    np.testing.assert_allclose(mo, s["merge_out"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(ml, s["merge_lse"], atol=1e-5, rtol=1e-5)
    # the k-way form agrees with pairwise merging
    ko, kl = orc.merge_states([s["merge_oa"], s["merge_ob"]], [s["merge_la"], s["merge_lb"]])
    np.testing.assert_allclose(ko, s["merge_out"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(kl, s["merge_lse"], atol=1e-5, rtol=1e-5)


def test_oracle_cfg1_matches_reference():
    c = _load("cfg1.npz")
    n, H, Hkv, D, cp = c["dims"].tolist()
    q, k, v = _inputs(n, H, Hkv, D, seed=0)
    _check_sums(c["input_sums"], (q, k, v))
    q, k, v = q.numpy(), k.numpy(), v.numpy()
    scale = 1.0 / math.sqrt(D)
    ro, rl = orc.simulate_ring(q, k, v, cp, scale)
    rows = c["rows"]
    np.testing.assert_allclose(ro[rows], c["ring_out_rows"], **TOL)
    np.testing.assert_allclose(rl[rows], c["dense_lse_rows"], **TOL)
    assert abs(float(ro.astype(np.float64).sum()) - float(c["ring_out_sum"])) < 1e-2
    assert abs(float(np.abs(ro.astype(np.float64)).sum()) - float(c["ring_out_abs_sum"])) < 1e-1
    assert abs(float(rl.astype(np.float64).sum()) - float(c["dense_lse_sum"])) < 1e-1


def test_row_oracle_matches_reference_rows():
    """dense_causal_rows (the full-size parity checker) on the sampled rows of BASELINE
    the reference's ring output and dense LSE at those rows, and the whole-matrix
    oracle on a GQA case with ragged row positions."""
    c = _load("cfg1.npz")
    n, H, Hkv, D, cp = c["dims"].tolist()
    q, k, v = (t.numpy() for t in _inputs(n, H, Hkv, D, seed=0))
    rows = c["rows"]
    ro, rl = orc.dense_causal_rows(q[rows], rows, k, v, 1.0 / math.sqrt(D))
    np.testing.assert_allclose(ro, c["ring_out_rows"], **TOL)
    np.testing.assert_allclose(rl, c["dense_lse_rows"], **TOL)
    rng = np.random.default_rng(3)
    q2, k2, v2 = (rng.standard_normal((300, h, 64)).astype(np.float32) for h in (6, 2, 2))
    pos = np.array([0, 1, 2, 17, 128, 129, 250, 299])
    want_o, want_l = orc.dense_causal(q2, k2, v2, 0.125)
    got_o, got_l = orc.dense_causal_rows(q2[pos], pos, k2, v2, 0.125, chunk=3)
    np.testing.assert_allclose(got_o, want_o[pos], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(got_l, want_l[pos], atol=1e-5, rtol=1e-5)


def test_planted_mistake_is_caught():
    """A wrong ring schedule (the reference GPU path's off-by-one rotation) fails the pin."""
    a = _load("algo.npz")
    n, H, Hkv, D, cp = a["case1_dims"].tolist()
    q, k, v = (t.numpy() for t in _inputs(n, H, Hkv, D))
    scale = 1.0 / math.sqrt(D)
    ks = [orc.zigzag_shard(k, r, cp) for r in range(cp)]
    vs = [orc.zigzag_shard(v, r, cp) for r in range(cp)]
    outs = []
    for rank in range(cp):
        lq = orc.zigzag_shard(q, rank, cp)
        acc = None
        for (step, src, pat) in orc.ring_schedule(rank, cp):
            wrong_src = (src + 1) % cp if step > 0 else src   # attends rank-s+1's KV
            o, l = orc.ring_step(lq, ks[wrong_src], vs[wrong_src], [0, lq.shape[0]], pat, scale)
            acc = (o, l) if acc is None else orc.merge(acc[0], acc[1], o, l)
        outs.append(acc[0])
    bad = orc.zigzag_unshard(outs, cp)
    assert not np.allclose(bad, a["case1_ring_out"], **TOL)


def test_gdn_cp_indices_match_reference_golden():
    """oracle/gdn_oracle.py restates build_gdn_cp_metadata; bit-exact against the fixtures the
    reference itself wrote (tests/golden/gdn_meta.npz)."""
    from oracle import gdn_oracle
    z = np.load(os.path.join(GOLDEN, "gdn_meta.npz"))
    for ci in range(int(z["n_cases"])):
        lens, cp = z[f"c{ci}_lens"].tolist(), int(z[f"c{ci}_cp"])
        for r in range(cp):
            restore, extract, cu = gdn_oracle.gdn_cp_indices(lens, cp, r)
            np.testing.assert_array_equal(restore, z[f"c{ci}_r{r}_restore"])
            np.testing.assert_array_equal(extract, z[f"c{ci}_r{r}_extract"])
            np.testing.assert_array_equal(cu, z[f"c{ci}_r{r}_cu"])


def test_gdn_cp_extract_is_the_ring_sharding():
    """GDN CP and the ring use one sharding: extract_idx == the zig-zag varlen rows."""
    from oracle import gdn_oracle
    for cp, lens in [(2, [12]), (4, [32, 16, 48]), (8, [64, 16])]:
        cu = [0] + list(np.cumsum(lens))
        for r in range(cp):
            _, extract, _ = gdn_oracle.gdn_cp_indices(lens, cp, r)
            rows, _ = orc.zigzag_varlen_rows(cu, r, cp)
            np.testing.assert_array_equal(extract, rows)
            restore, _, _ = gdn_oracle.gdn_cp_indices(lens, cp, 0)
            gathered = np.concatenate([orc.zigzag_varlen_rows(cu, rr, cp)[0] for rr in range(cp)])
            np.testing.assert_array_equal(gathered[restore], np.arange(cu[-1]))


# ---------------------------------------------------------------------------
# backward: the oracle against autograd through the reference's dense forward
# ---------------------------------------------------------------------------

def _bwd_case(b, i):
    n, H, Hkv, D, cp = (int(x) for x in b[f"case{i}_dims"])
    q, k, v = _inputs(n, H, Hkv, D)
    torch.manual_seed(1)
    dout = torch.randn(n, H, D)
    _check_sums(b[f"case{i}_input_sums"], (q, k, v, dout))
    return (n, H, Hkv, D, cp), [t.numpy() for t in (q, k, v, dout)]


@pytest.mark.parametrize("i", range(7))
def test_bwd_oracle_matches_reference_autograd(i):
    from oracle import bwd_oracle as bo
    b = _load("bwd.npz")
    (n, H, Hkv, D, cp), (q, k, v, dout) = _bwd_case(b, i)
    scale = 1.0 / math.sqrt(D)
    dense = bo.attn_bwd(q, k, v, dout, True, scale)
    ring = bo.simulate_ring_bwd(q, k, v, dout, cp, scale)
    for name, d, r in zip(("dq", "dk", "dv"), dense, ring):
        want = b[f"case{i}_{name}"]
        np.testing.assert_allclose(d, want, **TOL, err_msg=f"dense {name}")
        np.testing.assert_allclose(r, want, **TOL, err_msg=f"ring cp={cp} {name}")


def test_bwd_oracle_varlen_ring_equals_dense_per_sequence():
    from oracle import bwd_oracle as bo
    rng = np.random.default_rng(5)
    H, Hkv, D, cp = 6, 2, 16, 4
    lens = [16, 40, 8]
    full_cu = [0] + list(np.cumsum(lens))
    N = full_cu[-1]
    q, dout = rng.standard_normal((N, H, D)), rng.standard_normal((N, H, D))
    k, v = rng.standard_normal((N, Hkv, D)), rng.standard_normal((N, Hkv, D))
    scale = 1.0 / math.sqrt(D)
    # dense, per sequence
    want = [np.zeros_like(x) for x in (q, k, v)]
    outs, lses = np.zeros((N, H, D)), np.zeros((N, H))
    for a, e in zip(full_cu[:-1], full_cu[1:]):
        g = bo.attn_bwd(q[a:e], k[a:e], v[a:e], dout[a:e], True, scale)
        for w, x in zip(want, g):
            w[a:e] = x
        outs[a:e], lses[a:e] = orc.attn(q[a:e], k[a:e], v[a:e], True, scale, np.float64)
    # ring over packed zig-zag shards
    shard = lambda x, r: orc.zigzag_shard_varlen(x, full_cu, r, cp)[0]  # noqa: E731
    lcu = orc.zigzag_shard_varlen(q, full_cu, 0, cp)[1]
    ks = [shard(k, r) for r in range(cp)]
    vs = [shard(v, r) for r in range(cp)]
    got_q = [None] * cp
    got_k = [np.zeros_like(x) for x in ks]
    got_v = [np.zeros_like(x) for x in vs]
    for rank in range(cp):
        dq, dkv = bo.ring_rank_bwd(shard(q, rank), ks, vs, shard(dout, rank), shard(outs, rank),
                                   shard(lses, rank), rank, cp, scale, cu=lcu)
        got_q[rank] = dq
        for src, (b2, c2) in dkv.items():
            got_k[src] += b2
            got_v[src] += c2
    for name, w, got in (("dq", want[0], got_q), ("dk", want[1], got_k), ("dv", want[2], got_v)):
        for r in range(cp):
            np.testing.assert_allclose(got[r], shard(w, r), atol=1e-10, rtol=1e-10,
                                       err_msg=f"{name} rank {r}")


def test_bwd_planted_mistake_is_caught():
    """A backward that uses the step's own LSE instead of the final one is wrong: the
    ring check must see it."""
    from oracle import bwd_oracle as bo
    b = _load("bwd.npz")
    (n, H, Hkv, D, cp), (q, k, v, dout) = _bwd_case(b, 2)
    scale = 1.0 / math.sqrt(D)
    ks = [orc.zigzag_shard(k, r, cp) for r in range(cp)]
    vs = [orc.zigzag_shard(v, r, cp) for r in range(cp)]
    rank = 1
    lq, ldo = orc.zigzag_shard(q, rank, cp), orc.zigzag_shard(dout, rank, cp)
    dq = np.zeros(lq.shape)
    out, lse = orc.attn(q, k, v, True, scale, np.float64)
    delta = bo.row_delta(orc.zigzag_shard(out, rank, cp), ldo)
    for (_s, src, pat) in orc.ring_schedule(rank, cp):
        _o, step_lse = orc.ring_step(lq, ks[src], vs[src], [0, lq.shape[0]], pat, scale,
                                     np.float64)
        dq += bo.ring_step_bwd(lq, ks[src], vs[src], ldo, step_lse, delta, [0, lq.shape[0]], pat,
                               scale)[0]
    want = orc.zigzag_shard(b["case2_dq"], rank, cp)
    assert np.abs(dq - want).max() > 1e-2
