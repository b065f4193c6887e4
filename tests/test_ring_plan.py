"""The copy-engine ring protocol (``fa4cp_ring_ce_plan``), run on the CPU against a
multi-rank simulator of CUDA streams, events and the 32-bit hop counters.

The plan is the exact sequence of operations ``fa4cp_ring_attn_fwd`` issues per call
(K/V pushes into the right neighbour's receive slot, counter writes into the peers'
memory, waits on the own counters, attention steps).  The simulator runs every rank's
plan for several consecutive calls, in random interleavings of the four streams of every
rank, and also with each rank's streams serialised into one queue in host order (the
worst case the CUDA docs warn of for stream memory operations).  It checks that no
schedule deadlocks, that step ``s`` of rank ``r`` attends the K/V that originated on rank
``(r - s) mod S`` in the same call, that nothing overwrites a slot while it is read or
before its content was attended and forwarded, and that counters only grow.  Copies and
attention steps take time: each is a begin and an end, with the other streams running in
between.  The GPU run of the same plan is the NCCL-free multi-GPU ring test.
"""

import ctypes
import random

import pytest

from fa4_ring import _lib

RECORD, WAIT_EVENT, WAIT_FLAG, WRITE_FLAG, COPY, ATTN = range(6)
ARRIVED, FREED = 0, 1
RIGHT, LEFT = 0, 1


class Op(ctypes.Structure):
    _fields_ = [("stream", ctypes.c_int32), ("kind", ctypes.c_int32), ("a", ctypes.c_int64),
                ("b", ctypes.c_int64), ("c", ctypes.c_int64)]


def plan(S, rank, g0):
    lib = _lib.load()
    n = lib.fa4cp_ring_ce_plan(S, rank, g0, None, 0)
    assert n > 0, _lib.last_error()
    buf = (Op * n)()
    assert lib.fa4cp_ring_ce_plan(S, rank, g0, buf, n) == n
    return [(o.stream, o.kind, o.a, o.b, o.c) for o in buf]


class Part:
    """One K or V part of a receive slot."""

    def __init__(self):
        self.hop = None          # hop whose data the part holds
        self.tag = None          # (origin rank, call) of that data
        self.writing = False
        self.readers = 0
        self.attended = False
        self.forwarded = False
        self.needs_fwd = False


def simulate(S, calls, seed, serial):
    rng = random.Random(seed)
    ranks = []
    for r in range(S):
        ops = []
        for c in range(calls):
            for o in plan(S, r, c * (S - 1)):
                ops.append((c,) + o)
        # resolve each event wait to the latest record of that event before it (host order)
        last_record, waits_on = {}, {}
        for i, (c, st, kind, a, b, cc) in enumerate(ops):
            if kind == RECORD:
                last_record[a] = i
            elif kind == WAIT_EVENT:
                waits_on[i] = last_record.get(a)
        queues = {}
        for i, o in enumerate(ops):
            queues.setdefault(0 if serial else o[1], []).append(i)
        ranks.append(dict(ops=ops, waits_on=waits_on, queues=queues, pos={q: 0 for q in queues},
                          pending={}, done=set(), flags=[0, 0],
                          slots=[[Part(), Part()], [Part(), Part()]]))

    def step_of(hop, c):
        return hop - c * (S - 1)

    def runnable(r, q):
        R = ranks[r]
        if q in R["pending"]:
            return True
        if R["pos"][q] >= len(R["queues"][q]):
            return False
        i = R["queues"][q][R["pos"][q]]
        c, st, kind, a, b, cc = R["ops"][i]
        if kind == WAIT_EVENT:
            ref = R["waits_on"][i]
            return ref is None or ref in R["done"]
        if kind == WAIT_FLAG:
            return R["flags"][a] >= b
        return True

    def begin(r, i):
        R = ranks[r]
        c, st, kind, a, b, cc = R["ops"][i]
        if kind == COPY:
            if b >= 0:
                src = R["slots"][b & 1][a]
                assert src.hop == b and not src.writing, "push reads a slot that is not ready"
                tag = src.tag
                src.readers += 1
            else:
                tag, src = (r, c), None
            dst = ranks[(r + 1) % S]["slots"][cc & 1][a]
            assert dst.readers == 0 and not dst.writing, "push overwrites a slot in use"
            assert dst.hop is None or (dst.attended and (dst.forwarded or not dst.needs_fwd)), \
                "push overwrites data not yet attended / forwarded"
            dst.hop, dst.tag, dst.writing = cc, tag, True
            dst.attended = dst.forwarded = False
            dst.needs_fwd = step_of(cc, c) < S - 1
            return ("copy", src, dst)
        if kind == ATTN:
            want = ((r - a) % S, c)
            if b < 0:
                assert a == 0
                return ("attn", [])
            parts = R["slots"][b & 1]
            for p in parts:
                assert p.hop == b and not p.writing, "attention reads a slot that is not ready"
                assert p.tag == want, f"rank {r} step {a} attends {p.tag}, wants {want}"
                p.readers += 1
            return ("attn", parts)
        return None

    def end(token):
        if token[0] == "copy":
            _, src, dst = token
            if src is not None:
                src.readers -= 1
                src.forwarded = True
            dst.writing = False
        else:
            for p in token[1]:
                p.readers -= 1
                p.attended = True

    def execute(r, q):
        R = ranks[r]
        if q in R["pending"]:
            i, token = R["pending"].pop(q)
            end(token)
            R["done"].add(i)
            R["pos"][q] += 1
            return
        i = R["queues"][q][R["pos"][q]]
        c, st, kind, a, b, cc = R["ops"][i]
        if kind in (COPY, ATTN):
            R["pending"][q] = (i, begin(r, i))
            return
        if kind == WRITE_FLAG:
            peer = ranks[(r + 1) % S] if a == RIGHT else ranks[(r - 1) % S]
            assert cc >= peer["flags"][b], "counters only grow"
            peer["flags"][b] = cc
        R["done"].add(i)
        R["pos"][q] += 1

    total = sum(len(R["ops"]) for R in ranks)
    while sum(len(R["done"]) for R in ranks) < total:
        cands = [(r, q) for r in range(S) for q in ranks[r]["queues"] if runnable(r, q)]
        assert cands, f"deadlock (S={S}, seed={seed}, serial={serial})"
        execute(*rng.choice(cands))
    for R in ranks:  # every call attended every step
        assert sum(1 for o in R["ops"] if o[2] == ATTN) == S * calls


@pytest.mark.parametrize("S", [2, 3, 4, 8])
def test_plan_is_deadlock_free_and_hazard_free(S):
    for seed in range(40 if S < 8 else 12):
        simulate(S, calls=3, seed=seed, serial=False)


@pytest.mark.parametrize("S", [2, 3, 4, 8])
def test_plan_with_streams_serialised_in_host_order(S):
    for seed in range(10):
        simulate(S, calls=3, seed=seed, serial=True)


def test_plan_shape():
    ops = plan(4, 1, 0)
    kinds = [o[1] for o in ops]
    assert kinds.count(ATTN) == 4 and kinds.count(COPY) == 6  # 3 hops x (K, V)
    assert [o for o in ops if o[1] == ATTN][0][3] == -1       # step 0 on the caller's K/V
    assert plan(1, 0, 0) == [(0, ATTN, 0, -1, 0), (0, RECORD, 1, 0, 0)]
    with pytest.raises(AssertionError):
        plan(65, 0, 0)


def test_planted_mistake_is_caught():
    """A plan without the slot-release wait must fail the simulator (checks the checker)."""
    real = plan

    def broken(S, rank, g0):
        return [o for o in real(S, rank, g0) if not (o[1] == WAIT_FLAG and o[2] == FREED)]

    globals()["plan"] = broken
    try:
        with pytest.raises(AssertionError):
            for seed in range(40):
                simulate(4, calls=3, seed=seed, serial=False)
    finally:
        globals()["plan"] = real
