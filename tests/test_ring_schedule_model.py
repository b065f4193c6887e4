"""CPU model of the ring kernels' tile schedule (csrc/ring_fused.cuh).

The ring kernels map a flat CTA (or persistent-tile) index to (sequence, half, query tile(s),
query head) with ``ring_tile`` / ``ring_grid`` and walk, per CTA, the concatenated K/V of every
ring step (``RingSegs``: step 0 local and causal, step s <= rank the front half of source
(rank - s) mod S, step s > rank all of it for late-half rows only).  This module restates that
index math in Python -- two 128-row query tiles per CTA (``ring_tile_geo``, D 64 / 128) and one
(``ring_tile_geo1``, D 256), with the step bookkeeping of ``ring_fused_1q_kernel`` -- and checks
it against the oracle's definition of the ring (``oracle/ring_oracle.py``, ``pattern_ranges``,
restating fa4_ring/ring_attention.py:109-166):

* every local query row of every head is owned by exactly one CTA of the grid;
* the K/V each CTA walks, step by step, is exactly the key range the reference attends for
  those rows at that step (the causal diagonal of step 0 included, through the tile count).

``BM`` and ``kQtileChunk`` are read from the CUDA source, so the model follows the kernel.
The GPU tests (tests/test_gpu_ring_fused.py) check the kernels' outputs themselves.
"""

import os
import random
import re

import pytest

from conftest import ROOT
from oracle import ring_oracle as orc

_SRC = open(os.path.join(ROOT, "fa4-cp_b200", "csrc", "attn_fwd_sm100.cu")).read()
BM = int(re.search(r"constexpr int BM = (\d+);", _SRC).group(1))
CHUNK = int(re.search(r"constexpr int kQtileChunk = (\d+);", _SRC).group(1))


def ring_tile(tile, n_pairs, Hq, group, nseq):
    """ring_fused.cuh ring_tile: (seq, half, pair, head, kvh) or None (schedule padding)."""
    ch = min(CHUNK, n_pairs)
    chunks_per_half = (n_pairs + ch - 1) // ch
    per_seq = ch * Hq
    per_chunk = per_seq * nseq
    chunk, r = divmod(tile, per_chunk)
    rnd = chunk // chunks_per_half
    chunk -= rnd * chunks_per_half
    seq, r = divmod(r, per_seq)
    kvh, r2 = divmod(r, ch * group)
    qd = chunk * ch + r2 // group
    if qd >= n_pairs or rnd > 1:
        return None
    return seq, 1 - rnd, n_pairs - 1 - qd, kvh * group + r2 % group, kvh


def ring_grid(n_pairs, Hq, nseq):
    ch = min(n_pairs, CHUNK)
    return 2 * ((n_pairs + ch - 1) // ch) * ch * Hq * nseq


class Segs:
    """RingSegs: the K/V of each step of one CTA's walk."""

    def __init__(self, hh, half, k0_len, n0, S, rank):
        self.hh, self.half, self.k0_len, self.n0, self.S, self.rank = hh, half, k0_len, n0, S, rank

    def len(self, s):
        if s == 0:
            return self.k0_len
        return self.hh if s <= self.rank else (2 * self.hh if self.half else 0)

    def tiles(self, s, BN):
        return self.n0 if s == 0 else (self.len(s) + BN - 1) // BN


def geo(cu, tile, S, rank, Hq, group, nseq, n_pairs, BN, rows_per_cta):
    """ring_tile_geo (rows_per_cta = 2 BM) / ring_tile_geo1 (BM): (query rows, Segs, tiles)."""
    t = ring_tile(tile, n_pairs, Hq, group, nseq)
    if t is None:
        return None
    seq, half, pair, head, _kvh = t
    a, L = cu[seq], cu[seq + 1] - cu[seq]
    hh = L // 2
    q_start = a + half * hh
    q_len = L - hh if half else hh
    q0 = pair * rows_per_cta
    if q0 >= q_len:
        return None
    rows = min(rows_per_cta, q_len - q0)
    k0_len = L if half else hh
    diag = k0_len - q_len
    kv_end0 = min(k0_len, q0 + rows + diag)
    g = Segs(hh, half, k0_len, (kv_end0 + BN - 1) // BN, S, rank)
    n = sum(g.tiles(s, BN) for s in range(S))
    return (seq, head, q_start + q0, rows, half), g, n


def walk(g, n, BN):
    """ring_fused_1q_kernel's step bookkeeping: (step, first key of the tile) for j < n."""
    step, step_end, kbase, out = 0, g.tiles(0, BN), -BN, []
    for j in range(n):
        kbase += BN
        if j == step_end:
            while True:
                step += 1
                step_end += g.tiles(step, BN)
                if j < step_end:
                    break
            kbase = 0
        out.append((step, kbase))
    return out


def local_cu(lens, S):
    return [0] + list(__import__("itertools").accumulate(n // S for n in lens))


CASES = [(S, seed) for S in (1, 2, 3, 4, 8) for seed in range(3)]


@pytest.mark.parametrize("S,seed", CASES)
@pytest.mark.parametrize("one_tile", [False, True])
def test_ring_schedule_covers_every_row_once_and_walks_the_reference_steps(S, seed, one_tile):
    rnd = random.Random(seed * 31 + S)
    nseq = rnd.choice([1, 1, 2, 3])
    lens = [2 * S * rnd.choice([1, 3, 40, 64, 97, 128, 200, 300]) for _ in range(nseq)]
    Hkv = rnd.choice([1, 2])
    group = rnd.choice([1, 2, 4])
    Hq = Hkv * group
    BN = 64 if one_tile else 128
    rows_per_cta = BM if one_tile else 2 * BM
    cu = local_cu(lens, S)
    max_local = max(lens) // S
    n_pairs = (max_local // 2 + rows_per_cta - 1) // rows_per_cta  # as the launchers compute
    for rank in range(S):
        owner = {}
        for tile in range(ring_grid(n_pairs, Hq, nseq)):
            x = geo(cu, tile, S, rank, Hq, group, nseq, n_pairs, BN, rows_per_cta)
            if x is None:
                continue
            (seq, head, r0, rows, half), g, n = x
            for r in range(r0, r0 + rows):
                assert (r, head) not in owner, f"row {r} head {head} owned twice"
                owner[(r, head)] = tile
            # the walk against the reference's steps for these rows
            steps = {}
            for step, kb in walk(g, n, BN):
                steps.setdefault(step, []).append(kb)
            for s, (_st, _src, pattern) in enumerate(orc.ring_schedule(rank, S)):
                rng = [rg for rg in orc.pattern_ranges(cu, pattern)
                       if rg[0] <= r0 < rg[0] + rg[1]]
                if not rng:  # these rows attend nothing at this step
                    assert s not in steps, (rank, s, pattern)
                    continue
                qs, ql, ks, kl = rng[0]
                assert r0 + rows <= qs + ql, "a CTA's rows stay inside one step range"
                if s == 0:  # causal: up to the last row's diagonal
                    want = min(kl, (r0 + rows - qs))
                else:
                    want = kl
                got = steps.get(s, [])
                assert got == list(range(0, len(got) * BN, BN)), (rank, s, got[:4])
                assert len(got) == (want + BN - 1) // BN, (rank, s, len(got), want, kl)
                if s == 0:  # early-half rows never see past h under the causal mask
                    assert want <= g.len(0) <= kl, (rank, g.len(0), want, kl)
                else:
                    assert g.len(s) == kl, (rank, s, g.len(s), kl)
        want_rows = {(r, h) for r in range(cu[-1]) for h in range(Hq)}
        assert set(owner) == want_rows, f"rank {rank}: rows not covered"


def test_schedule_takes_late_half_tiles_first():
    """Heaviest first: every late-half tile precedes every early-half one in the grid."""
    S, rank, Hq, group = 4, 1, 8, 4
    cu = local_cu([2 * S * 300], S)
    n_pairs = (cu[-1] // 2 + 2 * BM - 1) // (2 * BM)
    halves = [ring_tile(t, n_pairs, Hq, group, 1) for t in range(ring_grid(n_pairs, Hq, 1))]
    halves = [h[1] for h in halves if h is not None]
    first_early = halves.index(0)
    assert all(h == 1 for h in halves[:first_early]) and all(h == 0 for h in halves[first_early:])
