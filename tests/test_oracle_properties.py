"""Property tests of the oracle (CPU, hypothesis): on random shapes, cp sizes and packings,
the zig-zag ring decomposition reproduces the dense causal attention and its gradient.

These tie the oracle's ring restatement (``oracle/ring_oracle.py``, the reference's
``tests/test_algorithm_cpu.py:62-168``) and its backward (``oracle/bwd_oracle.py``) to the
dense definitions on many more cases than the golden fixtures hold, and check the index
invariants the kernels rely on (zig-zag shard / unshard are inverse permutations; the three
step patterns of every rank tile each (query, key) pair of the causal triangle exactly once).
"""

import math

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import bwd_oracle as bo
from oracle import ring_oracle as orc

SETTINGS = settings(max_examples=25, deadline=None, derandomize=True)


@st.composite
def ring_problem(draw):
    cp = draw(st.sampled_from([1, 2, 3, 4]))
    hkv = draw(st.sampled_from([1, 2]))
    group = draw(st.sampled_from([1, 2, 3]))
    d = draw(st.sampled_from([4, 8]))
    nseq = draw(st.integers(1, 3))
    lens = [2 * cp * draw(st.integers(0, 4)) for _ in range(nseq)]
    if sum(lens) == 0:
        lens[0] = 2 * cp
    seed = draw(st.integers(0, 2 ** 16))
    return cp, hkv * group, hkv, d, lens, seed


def _inputs(H, Hkv, D, N, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((N, H, D)), rng.standard_normal((N, Hkv, D)),
            rng.standard_normal((N, Hkv, D)), rng.standard_normal((N, H, D)))


@SETTINGS
@given(ring_problem())
def test_ring_forward_equals_dense(prob):
    cp, H, Hkv, D, lens, seed = prob
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    q, k, v, _ = _inputs(H, Hkv, D, full_cu[-1], seed)
    scale = 1.0 / math.sqrt(D)
    seqs = [(q[a:b], k[a:b], v[a:b]) for a, b in zip(full_cu[:-1], full_cu[1:])]
    got = orc.simulate_ring_varlen(seqs, cp, scale, np.float64)
    for (qs, ks, vs), g in zip(seqs, got):
        want, _ = orc.dense_causal(qs, ks, vs, scale, np.float64)
        np.testing.assert_allclose(g, want, atol=1e-10, rtol=1e-10)


@SETTINGS
@given(ring_problem())
def test_ring_backward_equals_dense_gradient(prob):
    cp, H, Hkv, D, lens, seed = prob
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    q, k, v, dout = _inputs(H, Hkv, D, N, seed)
    scale = 1.0 / math.sqrt(D)
    want = [np.zeros(x.shape) for x in (q, k, v)]
    out, lse = np.zeros(q.shape), np.zeros(q.shape[:2])
    for a, b in zip(full_cu[:-1], full_cu[1:]):
        for w, x in zip(want, bo.attn_bwd(q[a:b], k[a:b], v[a:b], dout[a:b], True, scale)):
            w[a:b] = x
        out[a:b], lse[a:b] = orc.attn(q[a:b], k[a:b], v[a:b], True, scale, np.float64)
    shard = lambda x, r: orc.zigzag_shard_varlen(x, full_cu, r, cp)[0]  # noqa: E731
    lcu = orc.zigzag_shard_varlen(q, full_cu, 0, cp)[1]
    ks = [shard(k, r) for r in range(cp)]
    vs = [shard(v, r) for r in range(cp)]
    dk = [np.zeros(x.shape) for x in ks]
    dv = [np.zeros(x.shape) for x in vs]
    for rank in range(cp):
        dq, dkv = bo.ring_rank_bwd(shard(q, rank), ks, vs, shard(dout, rank), shard(out, rank),
                                   shard(lse, rank), rank, cp, scale, cu=lcu)
        np.testing.assert_allclose(dq, shard(want[0], rank), atol=1e-10, rtol=1e-9)
        for src, (b2, c2) in dkv.items():
            dk[src] += b2
            dv[src] += c2
    for r in range(cp):
        np.testing.assert_allclose(dk[r], shard(want[1], r), atol=1e-10, rtol=1e-9)
        np.testing.assert_allclose(dv[r], shard(want[2], r), atol=1e-10, rtol=1e-9)


@SETTINGS
@given(st.integers(1, 8), st.integers(1, 6), st.integers(0, 3))
def test_zigzag_shard_unshard_are_inverse_permutations(cp, h, extra_seqs):
    lens = [2 * cp * h] + [2 * cp * (i + 1) for i in range(extra_seqs)]
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    rows = np.concatenate([orc.zigzag_varlen_rows(full_cu, r, cp)[0] for r in range(cp)])
    assert np.array_equal(np.sort(rows), np.arange(N))  # a permutation of all rows
    x = np.arange(N).reshape(N, 1)
    shards = [orc.zigzag_shard_varlen(x, full_cu, r, cp)[0] for r in range(cp)]
    lcu = orc.zigzag_shard_varlen(x, full_cu, 0, cp)[1]
    for j in range(len(lens)):
        parts = [s[lcu[j]:lcu[j + 1]] for s in shards]
        assert np.array_equal(orc.zigzag_unshard(parts, cp),
                              x[full_cu[j]:full_cu[j + 1]])


@SETTINGS
@given(st.integers(1, 8), st.integers(1, 5))
def test_step_patterns_tile_the_causal_triangle_once(cp, h):
    """Over all ranks and steps, every (query, key) pair with key <= query of the full
    sequence is attended exactly once, and no pair with key > query is."""
    n = 2 * cp * h
    count = np.zeros((n, n), dtype=np.int64)
    local = [orc.zigzag_rows(n, r, cp) for r in range(cp)]
    T = 2 * h
    for rank in range(cp):
        for (_s, src, pattern) in orc.ring_schedule(rank, cp):
            for (qs, ql, ks_, kl) in orc.pattern_ranges([0, T], pattern):
                qrows = local[rank][qs:qs + ql]
                krows = local[src][ks_:ks_ + kl]
                if pattern == orc.PATTERN_LOCAL_CAUSAL:
                    for i in range(ql):
                        count[qrows[i], krows[:i + 1]] += 1
                else:
                    count[np.ix_(qrows, krows)] += 1
    assert np.array_equal(count, np.tril(np.ones((n, n), dtype=np.int64)))


@pytest.mark.parametrize("causal,tq,tk", [(True, 1024, 1024), (False, 512, 1536),
                                          (True, 300, 300)])
def test_threaded_attention_equals_one_thread(causal, tq, tk, monkeypatch):
    """Large attention blocks run split by query rows over a thread pool (the CPU baseline's
    speed); the rows are independent, so the result equals the single-threaded computation."""
    rng = np.random.default_rng(3)
    H, Hkv, D = 8, 2, 64
    q = rng.standard_normal((tq, H, D), dtype=np.float32)
    k = rng.standard_normal((tk, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((tk, Hkv, D), dtype=np.float32)
    monkeypatch.setattr(orc, "_PARALLEL_MIN_SCORES", 1)
    monkeypatch.setattr(orc, "ATTN_WORKERS", 4)
    o4, l4 = orc.attn(q, k, v, causal, 0.125)
    monkeypatch.setattr(orc, "ATTN_WORKERS", 1)
    o1, l1 = orc.attn(q, k, v, causal, 0.125)
    np.testing.assert_allclose(o4, o1, atol=1e-6, rtol=0)
    np.testing.assert_allclose(l4, l1, atol=1e-6, rtol=0)
