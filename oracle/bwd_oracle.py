"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the attention BACKWARD and of the zig-zag
ring backward, the checker of the CUDA backward kernels.  Nothing in the product imports it.

The reference is forward-only ("forward-only (inference). No backward", README.md:142), so
there is no reference backward to restate line by line.  This module differentiates the
reference's forward instead:

* per-chunk attention ``cpu_attn`` (tests/test_algorithm_cpu.py:36-48): out = softmax(scale *
  q k^T [causal tril]) v per query head, GQA head ``hq -> hq // (H / Hkv)``;
* the ring decomposition of the forward (tests/test_algorithm_cpu.py:62-90, the three step
  patterns of fa4_ring/ring_attention.py:109-166): because every partial of the ring is taken
  with the FINAL log-sum-exp, its gradient is the chunk gradient with that LSE, and the
  per-step gradients add up.

Pinned against golden vectors made by running torch autograd through the reference's own dense
forward ``full_causal_reference(backend="torch")`` (fa4_ring/reference.py:29-54), written by
``tests/golden/make_golden.py`` into ``tests/golden/bwd.npz`` and checked by
``tests/test_oracle_golden.py``.

Math (natural log; per query row i and key j of one head):
    P_ij = exp(scale * q_i.k_j - LSE_i)            (0 where masked)
    D_i  = sum_d dO_id * O_id
    dV_j = sum_i P_ij dO_i
    dS_ij = P_ij * (dO_i.v_j - D_i)
    dQ_i = scale * sum_j dS_ij k_j,    dK_j = scale * sum_i dS_ij q_i
GQA sums dK / dV over the query heads of a group.
"""

from __future__ import annotations

from typing import Dict, Sequence, Tuple

import numpy as np

from .ring_oracle import (PATTERN_LOCAL_CAUSAL, attn, pattern_ranges, ring_schedule,
                          zigzag_shard, zigzag_unshard)


def attn_bwd_chunk(q, k, v, dout, lse, delta, causal: bool, scale: float, dtype=np.float64):
    """Gradient contribution of one attention chunk, given the row statistics of the WHOLE
    attention the chunk is part of.

    q, dout: [Tq, H, D]; k, v: [Tk, Hkv, D]; lse, delta: [Tq, H] (natural-log LSE of the
    final output and rowsum(dO * O)).  Causal = the square top-left ``tril`` of the forward.
    Returns (dq [Tq,H,D], dk [Tk,Hkv,D], dv [Tk,Hkv,D]).  Rows with LSE -inf contribute
    nothing.
    """
    tq, H, D = q.shape
    tk, Hkv, _ = k.shape
    g = H // Hkv
    dq = np.zeros((tq, H, D), dtype)
    dk = np.zeros((tk, Hkv, D), dtype)
    dv = np.zeros((tk, Hkv, D), dtype)
    if tq == 0 or tk == 0:
        return dq, dk, dv
    qf, kf, vf, dof = (x.astype(dtype) for x in (q, k, v, dout))
    lsef = lse.astype(dtype)
    deltaf = delta.astype(dtype)
    mask = np.tril(np.ones((tq, tk), dtype=bool)) if causal else None
    for hk in range(Hkv):
        sl = slice(hk * g, (hk + 1) * g)
        qh = qf[:, sl, :].transpose(1, 0, 2)        # [g, Tq, D]
        doh = dof[:, sl, :].transpose(1, 0, 2)      # [g, Tq, D]
        lh = lsef[:, sl].T[..., None]               # [g, Tq, 1]
        dh = deltaf[:, sl].T[..., None]
        kh, vh = kf[:, hk, :], vf[:, hk, :]         # [Tk, D]
        s = np.matmul(qh, kh.T) * dtype(scale)      # [g, Tq, Tk]
        finite = np.isfinite(lh)
        with np.errstate(invalid="ignore", over="ignore"):
            p = np.where(finite, np.exp(s - np.where(finite, lh, 0)), 0)
        if mask is not None:
            p = np.where(mask[None], p, 0)
        dp = np.matmul(doh, vh.T)                   # [g, Tq, Tk]
        ds = p * (dp - dh)
        dq[:, sl, :] = (np.matmul(ds, kh) * dtype(scale)).transpose(1, 0, 2)
        dk[:, hk, :] = np.matmul(ds.transpose(0, 2, 1), qh).sum(0) * dtype(scale)
        dv[:, hk, :] = np.matmul(p.transpose(0, 2, 1), doh).sum(0)
    return dq, dk, dv


def row_delta(out, dout, dtype=np.float64):
    """D_i = sum_d dO_id * O_id per (row, head)."""
    return (out.astype(dtype) * dout.astype(dtype)).sum(-1)


def attn_bwd(q, k, v, dout, causal: bool, scale: float, dtype=np.float64):
    """Dense gradient of ``ring_oracle.attn`` (the reference's ``cpu_attn``) -> dq, dk, dv."""
    out, lse = attn(q, k, v, causal, scale, dtype)
    return attn_bwd_chunk(q, k, v, dout, lse, row_delta(out, dout, dtype), causal, scale, dtype)


def attn_bwd_varlen(q, k, v, dout, lse, delta, cu_q, cu_k, causal, scale, dtype=np.float64):
    """Per-sequence :func:`attn_bwd_chunk` over packed sequences."""
    dq = np.zeros(q.shape, dtype)
    dk = np.zeros(k.shape, dtype)
    dv = np.zeros(v.shape, dtype)
    for j in range(len(cu_q) - 1):
        qs, qe = int(cu_q[j]), int(cu_q[j + 1])
        ks, ke = int(cu_k[j]), int(cu_k[j + 1])
        a, b, c = attn_bwd_chunk(q[qs:qe], k[ks:ke], v[ks:ke], dout[qs:qe], lse[qs:qe],
                                 delta[qs:qe], causal, scale, dtype)
        dq[qs:qe] += a
        dk[ks:ke] += b
        dv[ks:ke] += c
    return dq, dk, dv


def ring_step_bwd(q_loc, k_src, v_src, dout_loc, lse_loc, delta_loc, cu, pattern, scale,
                  dtype=np.float64):
    """Gradient of one ring step (the rows its pattern selects, as the forward's ring_step):
    returns (dq [T,H,D] of the local rows, dk, dv [T,Hkv,D] of the SOURCE rank's shard)."""
    T, H, D = q_loc.shape
    dq = np.zeros((T, H, D), dtype)
    dk = np.zeros(k_src.shape, dtype)
    dv = np.zeros(v_src.shape, dtype)
    for (qs, ql, ks, kl) in pattern_ranges(cu, pattern):
        a, b, c = attn_bwd_chunk(q_loc[qs:qs + ql], k_src[ks:ks + kl], v_src[ks:ks + kl],
                                 dout_loc[qs:qs + ql], lse_loc[qs:qs + ql],
                                 delta_loc[qs:qs + ql], pattern == PATTERN_LOCAL_CAUSAL, scale,
                                 dtype)
        dq[qs:qs + ql] += a
        dk[ks:ks + kl] += b
        dv[ks:ks + kl] += c
    return dq, dk, dv


def ring_rank_bwd(q_loc, k_by_src, v_by_src, dout_loc, out_loc, lse_loc, rank, cp_size, scale,
                  cu=None, dtype=np.float64):
    """Everything one rank computes in the ring backward: (dq_local, {src: (dk, dv)})."""
    T = q_loc.shape[0]
    if cu is None:
        cu = [0, T]
    delta = row_delta(out_loc, dout_loc, dtype)
    dq = np.zeros(q_loc.shape, dtype)
    dkv: Dict[int, Tuple[np.ndarray, np.ndarray]] = {}
    for (_step, src, pattern) in ring_schedule(rank, cp_size):
        a, b, c = ring_step_bwd(q_loc, k_by_src[src], v_by_src[src], dout_loc, lse_loc, delta,
                                cu, pattern, scale, dtype)
        dq += a
        dkv[src] = (b, c)
    return dq, dkv


def simulate_ring_bwd(q, k, v, dout, cp_size, scale, dtype=np.float64):
    """Zig-zag ring backward over ``cp_size`` simulated ranks for one sequence.

    The forward statistics (out, LSE) come from the dense forward, zig-zag sharded -- the
    ring forward produces exactly those.  Every rank's dK/dV contributions are summed into
    the owner's shard (what the rotating dK/dV accumulators of the ring deliver).  Returns
    the unsharded (dq, dk, dv).
    """
    out, lse = attn(q, k, v, True, scale, dtype)
    ks = [zigzag_shard(k, r, cp_size) for r in range(cp_size)]
    vs = [zigzag_shard(v, r, cp_size) for r in range(cp_size)]
    dqs = []
    dks = [np.zeros(x.shape, dtype) for x in ks]
    dvs = [np.zeros(x.shape, dtype) for x in vs]
    for rank in range(cp_size):
        dq, dkv = ring_rank_bwd(zigzag_shard(q, rank, cp_size), ks, vs,
                                zigzag_shard(dout, rank, cp_size), zigzag_shard(out, rank, cp_size),
                                zigzag_shard(lse, rank, cp_size), rank, cp_size, scale, None, dtype)
        dqs.append(dq)
        for src, (b, c) in dkv.items():
            dks[src] += b
            dvs[src] += c
    return (zigzag_unshard(dqs, cp_size), zigzag_unshard(dks, cp_size),
            zigzag_unshard(dvs, cp_size))


def bwd_flops(seq_lens: Sequence[int], num_heads_q: int, head_dim: int) -> float:
    """Algorithmic causal backward FLOPs: 2.5x the forward's (five matmuls of the forward's
    size -- S, dP, dV, dK, dQ -- against two), N^2/2 convention: sum_j 5 * N_j^2 * Hq * D."""
    return float(sum(5.0 * n * n * num_heads_q * head_dim for n in seq_lens))
