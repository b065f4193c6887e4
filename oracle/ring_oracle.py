"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the reference's CPU ring algorithm.

Nothing in the product imports this module.  It exists so the CUDA path can be
checked against the algorithm the reference defines, on the same seeded inputs.

Each function names the reference code it restates (paths relative to the
hxy0118/fa4-cp project root):

* zig-zag index math  -> ``fa4_ring/zigzag.py:26-97``
* per-chunk attention -> ``tests/test_algorithm_cpu.py:36-48`` (``cpu_attn``)
* LSE merge           -> ``tests/test_algorithm_cpu.py:51-59`` (``merge``)
* ring simulation     -> ``tests/test_algorithm_cpu.py:62-90`` and ``:114-168``
* dense reference     -> ``tests/test_algorithm_cpu.py:93-95`` and
  ``fa4_ring/reference.py:46-54``

The ring schedule here is the *intended* one the reference's CPU simulation
runs (step ``s`` attends the KV that originated on ``(rank - s) mod S``), not
the GPU orchestration in ``fa4_ring/ring_attention.py:125-171``, whose KV
rotation attends the wrong source shard.  LSE is natural log throughout.

Pinned against golden vectors produced by importing the reference itself:
``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``
(checked by ``tests/test_oracle_golden.py``).
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor
from typing import List, Sequence, Tuple

import numpy as np

# Large attention blocks are split by query rows over this many threads (softmax rows are
# independent, so the result is the same); numpy's elementwise ops (mask, exp, sums) are
# single-threaded, and the reference's torch CPU code uses every host thread.  Threads, not
# processes: nothing here forks.
ATTN_WORKERS = max(1, os.cpu_count() or 1)
_PARALLEL_MIN_SCORES = 1 << 22   # score elements per kv head below which one thread runs it

# Step patterns of the zig-zag ring (fa4_ring/ring_attention.py:11-16).
PATTERN_LOCAL_CAUSAL = 0   # step 0: local causal over [early | late]
PATTERN_FRONT_KV = 1       # step <= rank: all local Q x early half of the source KV
PATTERN_BACK_Q = 2         # step  > rank: late half of local Q x all of the source KV


# ----------------------------------------------------------------------------
# zig-zag index math  (fa4_ring/zigzag.py)
# ----------------------------------------------------------------------------

def local_seqlen(n: int, cp_size: int) -> int:
    """fa4_ring/zigzag.py:26-28."""
    assert n % (2 * cp_size) == 0, f"seqlen {n} must be divisible by 2*cp_size={2 * cp_size}"
    return n // cp_size


def zigzag_rows(n: int, cp_rank: int, cp_size: int) -> np.ndarray:
    """Row indices (into the full [n] sequence) of rank ``cp_rank``'s local shard.

    Chunk ``r`` then chunk ``2S-1-r`` of ``2S`` equal chunks (fa4_ring/zigzag.py:31-39).
    """
    assert n % (2 * cp_size) == 0, f"seqlen {n} must be divisible by 2*cp_size={2 * cp_size}"
    h = n // (2 * cp_size)
    j = 2 * cp_size - 1 - cp_rank
    return np.concatenate([np.arange(cp_rank * h, (cp_rank + 1) * h),
                           np.arange(j * h, (j + 1) * h)]).astype(np.int64)


def zigzag_shard(x: np.ndarray, cp_rank: int, cp_size: int) -> np.ndarray:
    """fa4_ring/zigzag.py:31-39."""
    return np.ascontiguousarray(x[zigzag_rows(x.shape[0], cp_rank, cp_size)])


def zigzag_unshard(shards: Sequence[np.ndarray], cp_size: int) -> np.ndarray:
    """fa4_ring/zigzag.py:42-50 (inverse of zigzag_shard)."""
    assert len(shards) == cp_size
    h = shards[0].shape[0] // 2
    chunks = [None] * (2 * cp_size)
    for i, loc in enumerate(shards):
        chunks[i] = loc[:h]
        chunks[2 * cp_size - 1 - i] = loc[h:]
    return np.concatenate(chunks, axis=0)


def get_half_index(cu: Sequence[int], front: bool) -> np.ndarray:
    """fa4_ring/zigzag.py:65-79: long indices of each packed sequence's front/back half."""
    cu = [int(c) for c in cu]
    parts = []
    for i in range(len(cu) - 1):
        start, end = cu[i], cu[i + 1]
        assert (end - start) % 2 == 0, "each local sequence length must be even (zig-zag)"
        mid = (start + end) // 2
        parts.append(np.arange(start, mid) if front else np.arange(mid, end))
    return np.concatenate(parts).astype(np.int64) if parts else np.zeros(0, np.int64)


def zigzag_varlen_rows(full_cu: Sequence[int], cp_rank: int, cp_size: int):
    """Row indices of the packed local shard and its local cu (fa4_ring/zigzag.py:82-97)."""
    full_cu = [int(c) for c in full_cu]
    rows, local_cu = [], [0]
    for j in range(len(full_cu) - 1):
        n = full_cu[j + 1] - full_cu[j]
        r = zigzag_rows(n, cp_rank, cp_size) + full_cu[j]
        rows.append(r)
        local_cu.append(local_cu[-1] + r.shape[0])
    rows = np.concatenate(rows) if rows else np.zeros(0, np.int64)
    return rows.astype(np.int64), np.asarray(local_cu, dtype=np.int32)


def zigzag_shard_varlen(x: np.ndarray, full_cu: Sequence[int], cp_rank: int, cp_size: int):
    """fa4_ring/zigzag.py:82-97 -> (local_packed, local_cu int32)."""
    rows, local_cu = zigzag_varlen_rows(full_cu, cp_rank, cp_size)
    return np.ascontiguousarray(x[rows]), local_cu


# ----------------------------------------------------------------------------
# attention + merge  (tests/test_algorithm_cpu.py:36-59)
# ----------------------------------------------------------------------------

def attn(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool, scale: float,
         dtype=np.float32) -> Tuple[np.ndarray, np.ndarray]:
    """tests/test_algorithm_cpu.py:36-48 (``cpu_attn``).

    q:[Tq,H,D], k/v:[Tk,Hkv,D] -> out:[Tq,H,D], lse:[Tq,H] (natural log).
    GQA maps query head ``hq`` to kv head ``hq // (H/Hkv)`` (``repeat_interleave``).
    The causal mask is the square top-left ``tril`` the reference uses.
    """
    tq, H, D = q.shape
    tk, Hkv, _ = k.shape
    assert H % Hkv == 0
    g = H // Hkv
    out = np.zeros((tq, H, D), dtype)
    lse = np.full((tq, H), -np.inf, dtype)
    if tq == 0:
        return out, lse
    if tk == 0:
        return out, lse
    qf = q.astype(dtype)
    kf = k.astype(dtype)
    vf = v.astype(dtype)
    key_idx = np.arange(tk)

    def rows(qh, kh, vh, r0, r1):
        """Query rows [r0, r1) of one kv head's group: (o [g, r, D], lse [g, r])."""
        s = np.matmul(qh[:, r0:r1], kh.T) * dtype(scale)   # [g, r, Tk]
        if causal:  # the reference's square top-left tril: key j visible to row i iff j <= i
            s = np.where((key_idx[None, :] <= np.arange(r0, r1)[:, None])[None], s, -np.inf)
        m = s.max(axis=-1, keepdims=True)
        m_safe = np.where(np.isfinite(m), m, 0)
        p = np.exp(s - m_safe)
        l = p.sum(axis=-1, keepdims=True)
        with np.errstate(divide="ignore", invalid="ignore"):
            lse_h = (np.log(l) + m_safe)[..., 0]            # [g, r]
            o = np.matmul(p, vh) / l                        # [g, r, D]
        o = np.where(l > 0, o, 0)
        lse_h = np.where(l[..., 0] > 0, lse_h, -np.inf)
        return o, lse_h

    workers = ATTN_WORKERS if g * tq * tk >= _PARALLEL_MIN_SCORES else 1
    bounds = np.linspace(0, tq, min(workers * 2, tq) + 1).astype(int) if workers > 1 else [0, tq]
    pool = ThreadPoolExecutor(max_workers=workers) if workers > 1 else None
    blas_limit = None
    if pool is not None:  # one BLAS thread per worker: the parallelism is over row blocks
        from threadpoolctl import threadpool_limits
        blas_limit = threadpool_limits(limits=1, user_api="blas")
    try:
        for hk in range(Hkv):
            kh = kf[:, hk, :]                                  # [Tk, D]
            vh = vf[:, hk, :]
            qh = qf[:, hk * g:(hk + 1) * g, :].transpose(1, 0, 2)   # [g, Tq, D]
            spans = list(zip(bounds[:-1], bounds[1:]))
            parts = (list(pool.map(lambda b: rows(qh, kh, vh, *b), spans)) if pool is not None
                     else [rows(qh, kh, vh, r0, r1) for r0, r1 in spans])
            for (r0, r1), (o, lse_h) in zip(spans, parts):
                out[r0:r1, hk * g:(hk + 1) * g, :] = o.transpose(1, 0, 2)
                lse[r0:r1, hk * g:(hk + 1) * g] = lse_h.T
    finally:
        if blas_limit is not None:
            blas_limit.restore_original_limits()
        if pool is not None:
            pool.shutdown()
    return out, lse


def attn_varlen(q, k, v, cu_q, cu_k, causal, scale, dtype=np.float32):
    """tests/test_algorithm_cpu.py:100-111: per-segment attention over packed sequences."""
    H, D = q.shape[1], q.shape[2]
    out = np.zeros((q.shape[0], H, D), dtype)
    lse = np.full((q.shape[0], H), -np.inf, dtype)
    for j in range(len(cu_q) - 1):
        qs, qe = int(cu_q[j]), int(cu_q[j + 1])
        ks, ke = int(cu_k[j]), int(cu_k[j + 1])
        o, l = attn(q[qs:qe], k[ks:ke], v[ks:ke], causal, scale, dtype)
        out[qs:qe] = o
        lse[qs:qe] = l
    return out, lse


def merge(out_a, lse_a, out_b, lse_b):
    """tests/test_algorithm_cpu.py:51-59: online-softmax merge, natural-log LSE.

    ``-inf`` rows of b contribute nothing; ``denom`` is clamped at 1e-20 as in
    the reference.
    """
    m = np.maximum(lse_a, lse_b)
    m_safe = np.where(np.isfinite(m), m, 0)
    with np.errstate(invalid="ignore"):
        ea = np.exp(lse_a - m_safe)
        eb = np.exp(lse_b - m_safe)
    denom = np.maximum(ea + eb, 1e-20)
    out = (out_a * ea[..., None] + out_b * eb[..., None]) / denom[..., None]
    lse = np.logaddexp(lse_a, lse_b)
    return out.astype(out_a.dtype), lse.astype(lse_a.dtype)


def merge_states(outs: Sequence[np.ndarray], lses: Sequence[np.ndarray]):
    """k-way form of :func:`merge` (what ``fa4_ring/merge.py:67-86`` computes in one kernel)."""
    lse = np.stack(lses, 0)                     # [k, T, H]
    m = lse.max(axis=0)
    m_safe = np.where(np.isfinite(m), m, 0)
    w = np.exp(lse - m_safe[None])              # [k, T, H]
    denom = w.sum(axis=0)
    acc = sum(o * wi[..., None] for o, wi in zip(outs, w))
    with np.errstate(invalid="ignore", divide="ignore"):
        out = acc / np.maximum(denom, 1e-20)[..., None]
        lse_out = np.log(denom) + m_safe
    lse_out = np.where(denom > 0, lse_out, -np.inf)
    return out.astype(outs[0].dtype), lse_out.astype(lses[0].dtype)


# ----------------------------------------------------------------------------
# ring schedule + simulation  (tests/test_algorithm_cpu.py:62-168)
# ----------------------------------------------------------------------------

def ring_schedule(rank: int, cp_size: int) -> List[Tuple[int, int, int]]:
    """(step, src, pattern) for every step of ``rank`` (tests/test_algorithm_cpu.py:70-88)."""
    sched = [(0, rank, PATTERN_LOCAL_CAUSAL)]
    for s in range(1, cp_size):
        src = (rank - s) % cp_size
        sched.append((s, src, PATTERN_BACK_Q if s > rank else PATTERN_FRONT_KV))
    return sched


def pattern_ranges(cu: Sequence[int], pattern: int):
    """Per-sequence (q_start, q_len, k_start, k_len) of one ring step.

    ``cu`` is the LOCAL cu_seqlens; both Q and the source KV use that packing
    (every rank's local shard of sequence j has the same length).  Restates the
    row selections of fa4_ring/ring_attention.py:89-92,139-166.
    """
    res = []
    for j in range(len(cu) - 1):
        s, e = int(cu[j]), int(cu[j + 1])
        n = e - s
        hh = n // 2
        if pattern == PATTERN_LOCAL_CAUSAL:
            res.append((s, n, s, n))
        elif pattern == PATTERN_FRONT_KV:
            res.append((s, n, s, hh))
        elif pattern == PATTERN_BACK_Q:
            res.append((s + hh, n - hh, s, n))
        else:
            raise ValueError(pattern)
    return res


def ring_step(q_loc, k_src, v_src, cu, pattern, scale, dtype=np.float32):
    """One ring step as a full-size partial (rows not covered get out 0, lse -inf)."""
    T, H, D = q_loc.shape
    out = np.zeros((T, H, D), dtype)
    lse = np.full((T, H), -np.inf, dtype)
    for (qs, ql, ks, kl) in pattern_ranges(cu, pattern):
        o, l = attn(q_loc[qs:qs + ql], k_src[ks:ks + kl], v_src[ks:ks + kl],
                    causal=(pattern == PATTERN_LOCAL_CAUSAL), scale=scale, dtype=dtype)
        out[qs:qs + ql] = o
        lse[qs:qs + ql] = l
    return out, lse


def ring_rank(q_loc, k_by_src, v_by_src, rank, cp_size, scale, cu=None, dtype=np.float32):
    """Everything one rank computes: returns (out[T,H,D], lse[T,H]) for its local rows."""
    T = q_loc.shape[0]
    if cu is None:
        cu = [0, T]
    acc_o = acc_l = None
    for (_step, src, pattern) in ring_schedule(rank, cp_size):
        o, l = ring_step(q_loc, k_by_src[src], v_by_src[src], cu, pattern, scale, dtype)
        if acc_o is None:
            acc_o, acc_l = o, l
        else:
            acc_o, acc_l = merge(acc_o, acc_l, o, l)
    return acc_o, acc_l


def simulate_ring(q, k, v, cp_size, scale, dtype=np.float32):
    """tests/test_algorithm_cpu.py:62-90 -> (reconstructed out [N,H,D], lse [N,H])."""
    ks = [zigzag_shard(k, r, cp_size) for r in range(cp_size)]
    vs = [zigzag_shard(v, r, cp_size) for r in range(cp_size)]
    outs, lses = [], []
    for rank in range(cp_size):
        o, l = ring_rank(zigzag_shard(q, rank, cp_size), ks, vs, rank, cp_size, scale, None, dtype)
        outs.append(o)
        lses.append(l)
    return zigzag_unshard(outs, cp_size), zigzag_unshard(lses, cp_size)


def simulate_ring_varlen(full_seqs, cp_size, scale, dtype=np.float32):
    """tests/test_algorithm_cpu.py:114-168 -> list of per-sequence reconstructed outputs."""
    lens = [s[0].shape[0] for s in full_seqs]
    full_cu = [0]
    for n in lens:
        full_cu.append(full_cu[-1] + n)
    Q = np.concatenate([s[0] for s in full_seqs], 0)
    K = np.concatenate([s[1] for s in full_seqs], 0)
    V = np.concatenate([s[2] for s in full_seqs], 0)
    ks, vs, local_cu = [], [], None
    for r in range(cp_size):
        kl, local_cu = zigzag_shard_varlen(K, full_cu, r, cp_size)
        vl, _ = zigzag_shard_varlen(V, full_cu, r, cp_size)
        ks.append(kl)
        vs.append(vl)
    rank_outs = []
    for rank in range(cp_size):
        lq, lcu = zigzag_shard_varlen(Q, full_cu, rank, cp_size)
        o, _ = ring_rank(lq, ks, vs, rank, cp_size, scale, lcu, dtype)
        rank_outs.append(o)
    recon = []
    for j in range(len(lens)):
        shards = [rank_outs[r][local_cu[j]:local_cu[j + 1]] for r in range(cp_size)]
        recon.append(zigzag_unshard(shards, cp_size))
    return recon


def dense_causal(q, k, v, scale, dtype=np.float32):
    """tests/test_algorithm_cpu.py:93-95 -> (out, lse)."""
    return attn(q, k, v, True, scale, dtype)


def dense_causal_rows(q_rows, pos, k, v, scale, chunk=32):
    """tests/test_algorithm_cpu.py:93-95 (the dense causal reference) evaluated on chosen query
    rows of ONE sequence: ``q_rows [R, H, D]`` holds the rows at positions ``pos [R]`` of the
    sequence, ``k``/``v [N, Hkv, D]`` the whole sequence; row ``pos[i]`` sees keys
    ``[0, pos[i]]`` (GQA: head h reads kv head ``h // (H / Hkv)``).  Returns
    ``(out [R, H, D], lse [R, H])`` in float64, equal to :func:`dense_causal` on those rows,
    without forming the ``[N, N]`` score matrix, so that full-size configurations (N up to
    262144) can be checked row by row.  Scores are float32 products (BLAS), the softmax and
    the P V sum run in float64."""
    pos = np.asarray(pos, dtype=np.int64)
    R, H, D = q_rows.shape
    Hkv = k.shape[1]
    g = H // Hkv
    n_max = int(pos.max()) + 1 if R else 0
    out = np.zeros((R, H, D), np.float64)
    lse = np.full((R, H), -np.inf, np.float64)
    for kh in range(Hkv):
        kk = np.ascontiguousarray(k[:n_max, kh, :], dtype=np.float32)
        vv = np.ascontiguousarray(v[:n_max, kh, :], dtype=np.float64)
        for h in range(kh * g, (kh + 1) * g):
            for a in range(0, R, chunk):
                b = min(R, a + chunk)
                s = (np.asarray(q_rows[a:b, h, :], np.float32) @ kk.T).astype(np.float64) * scale
                s[np.arange(n_max)[None, :] > pos[a:b, None]] = -np.inf
                m = s.max(-1, keepdims=True)
                p = np.exp(s - m)
                l = p.sum(-1, keepdims=True)
                out[a:b, h, :] = (p @ vv) / l
                lse[a:b, h] = (np.log(l) + m)[:, 0]
    return out, lse


def default_scale(head_dim: int) -> float:
    """fa4_ring/fa4_backend.py:88-89: softmax_scale=None -> 1/sqrt(D)."""
    return 1.0 / math.sqrt(head_dim)


def causal_flops(seq_lens: Sequence[int], num_heads_q: int, head_dim: int) -> float:
    """Algorithmic causal FLOPs, N^2/2 convention: sum_j 2 * N_j^2 * Hq * D."""
    return float(sum(2.0 * n * n * num_heads_q * head_dim for n in seq_lens))
