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

RECORD, WAIT_EVENT, WAIT_FLAG, WRITE_FLAG, COPY, ATTN, ATTN_FUSED = range(7)
ARRIVED, FREED = 0, 1
RIGHT, LEFT = 0, 1
# simulator-only expansions of the persistent ring kernel (its in-kernel waits and reads)
SEG_READ, KERNEL_END = 100, 101


class Op(ctypes.Structure):
    _fields_ = [("stream", ctypes.c_int32), ("kind", ctypes.c_int32), ("a", ctypes.c_int64),
                ("b", ctypes.c_int64), ("c", ctypes.c_int64)]


def plan(S, rank, g0, fused=False):
    lib = _lib.load()
    n = lib.fa4cp_ring_ce_plan(S, rank, g0, int(fused), None, 0)
    assert n > 0, _lib.last_error()
    buf = (Op * n)()
    assert lib.fa4cp_ring_ce_plan(S, rank, g0, int(fused), buf, n) == n
    return [(o.stream, o.kind, o.a, o.b, o.c) for o in buf]


class Part:
    """One K or V part of a receive slot."""

    def __init__(self):
        self.tag = None          # (origin rank, call) of the data it holds
        self.writing = False
        self.readers = 0
        self.attended = True     # an empty slot may be filled
        self.forwarded = True
        self.needs_fwd = False


def expand(ops, kernel_waits=True):
    """The fused launch as what it does on the compute queue: step 0 on the local K/V, then
    per step s a wait for ARRIVED >= base + s and the reads of slot s-1, all released at the
    kernel's end."""
    out = []
    for o in ops:
        st, kind, a, b, c = o
        if kind == ATTN_FUSED:
            out.append((st, SEG_READ, 0, -1, 0))
            for s in range(1, a):
                if kernel_waits:
                    out.append((st, WAIT_FLAG, ARRIVED, b + s, 0))
                out.append((st, SEG_READ, s, s - 1, 0))
            out.append((st, KERNEL_END, 0, 0, 0))
        else:
            out.append(o)
    return out


def simulate(S, calls, seed, serial, fused=False, plan_fn=None, kernel_waits=True):
    plan_fn = plan_fn or plan
    rng = random.Random(seed)
    ranks = []
    for r in range(S):
        ops = []
        for c in range(calls):
            for o in expand(plan_fn(S, r, c * (S - 1), fused), kernel_waits):
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
                          pending={}, done=set(), flags=[0, 0], kernel_reads=[],
                          slots=[[Part(), Part()] for _ in range(max(S - 1, 1))]))

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

    def read_slot(r, step, idx, c):
        want = ((r - step) % S, c)
        if idx < 0:
            assert step == 0
            return []
        parts = ranks[r]["slots"][idx]
        for p in parts:
            assert not p.writing and p.tag is not None, "attention reads a slot that is not ready"
            assert p.tag == want, f"rank {r} step {step} attends {p.tag}, wants {want}"
            p.readers += 1
        return parts

    def begin(r, i):
        R = ranks[r]
        c, st, kind, a, b, cc = R["ops"][i]
        if kind == COPY:
            if b >= 0:
                src = R["slots"][b][a]
                assert not src.writing and src.tag is not None, "push reads a slot that is not ready"
                assert src.tag == ((r - (b + 1)) % S, c), "push forwards the wrong shard"
                tag = src.tag
                src.readers += 1
            else:
                tag, src = (r, c), None
            dst = ranks[(r + 1) % S]["slots"][cc][a]
            assert dst.readers == 0 and not dst.writing, "push overwrites a slot in use"
            assert dst.attended and (dst.forwarded or not dst.needs_fwd), \
                "push overwrites data not yet attended / forwarded"
            dst.tag, dst.writing = tag, True
            dst.attended = dst.forwarded = False
            dst.needs_fwd = cc + 2 <= S - 1  # step cc+1's data goes on at push cc+2
            return ("copy", src, dst)
        return ("attn", read_slot(r, a, b, c))

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
        if kind == SEG_READ:
            R["kernel_reads"].append(("attn", read_slot(r, a, b, c)))
        elif kind == KERNEL_END:
            if mode == 1 and rng.random() < 0.9:
                return  # a slow kernel: its reads stay in flight a while longer
            for token in R["kernel_reads"]:
                end(token)
            R["kernel_reads"] = []
        elif kind == WRITE_FLAG:
            peer = ranks[(r + 1) % S] if a == RIGHT else ranks[(r - 1) % S]
            assert cc >= peer["flags"][b], "counters only grow"
            peer["flags"][b] = cc
        R["done"].add(i)
        R["pos"][q] += 1

    # adversarial timing: per seed, attention (or copies, or one whole rank) is slow, so a
    # neighbour can run far ahead while a read or write is still in flight
    mode = seed % 4
    slow_rank = rng.randrange(S)

    def slow(r, q):
        R = ranks[r]
        if mode == 3:
            return r == slow_rank
        if q not in R["pending"]:
            return False
        kind = R["ops"][R["pending"][q][0]][2]
        return (mode == 1 and kind == ATTN) or (mode == 2 and kind == COPY)

    total = sum(len(R["ops"]) for R in ranks)
    while sum(len(R["done"]) for R in ranks) < total:
        cands = [(r, q) for r in range(S) for q in ranks[r]["queues"] if runnable(r, q)]
        assert cands, f"deadlock (S={S}, seed={seed}, serial={serial}, fused={fused})"
        fast = [x for x in cands if not slow(*x)]
        if fast and rng.random() < 0.97:
            cands = fast
        execute(*rng.choice(cands))
    for R in ranks:  # every call attended every step
        n_steps = sum(1 for o in R["ops"] if o[2] in (ATTN, SEG_READ))
        assert n_steps == S * calls


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("S", [2, 3, 4, 8])
def test_plan_is_deadlock_free_and_hazard_free(S, fused):
    for seed in range(30 if S < 8 else 10):
        simulate(S, calls=3, seed=seed, serial=False, fused=fused)


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("S", [2, 3, 4, 8])
def test_plan_with_streams_serialised_in_host_order(S, fused):
    for seed in range(8):
        simulate(S, calls=3, seed=seed, serial=True, fused=fused)


def test_plan_shape():
    ops = plan(4, 1, 0)
    kinds = [o[1] for o in ops]
    assert kinds.count(ATTN) == 4 and kinds.count(COPY) == 6  # 3 hops x (K, V)
    assert [o for o in ops if o[1] == ATTN][0][3] == -1       # step 0 on the caller's K/V
    fused = plan(4, 1, 3, fused=True)
    assert [o[1] for o in fused].count(ATTN_FUSED) == 1
    assert [o for o in fused if o[1] == ATTN_FUSED][0][2:4] == (4, 3)
    assert plan(1, 0, 0) == [(0, ATTN, 0, -1, 0)]
    with pytest.raises(AssertionError):
        plan(65, 0, 0)


@pytest.mark.parametrize("fused,drop", [(False, "freed_wait"), (False, "arrived_wait"),
                                        (False, "release_after_push"), (True, "freed_wait"),
                                        (True, "kernel_wait"), (True, "release_after_push")])
def test_planted_mistake_is_caught(fused, drop):
    """A plan missing one of its waits must fail the simulator (checks the checker)."""
    def broken(S, rank, g0, fused):
        out = []
        for o in plan(S, rank, g0, fused):
            st, kind, a, b, c = o
            if drop == "freed_wait" and kind == WAIT_FLAG and a == FREED:
                continue
            if drop == "arrived_wait" and kind == WAIT_FLAG and a == ARRIVED and st == 0:
                continue
            if drop == "release_after_push" and kind == WAIT_EVENT and st == 3 and a != 1:
                continue
            out.append(o)
        return out

    with pytest.raises(AssertionError):
        for seed in range(40):
            simulate(4, calls=3, seed=seed, serial=False, fused=fused, plan_fn=broken,
                     kernel_waits=drop != "kernel_wait")


# --------------------------------------------------------------------------- direct pushes
COPY_TO, WRITE_PEER, ATTN_FUSED_SLOTS = 7, 8, 9
FLAG_SLOT0, FLAG_PEER_FREED0 = 2, 2 + 2 * 64


def direct_plan(S, rank, call, fused=False):
    lib = _lib.load()
    n = lib.fa4cp_ring_ce_direct_plan(S, rank, call, int(fused), None, 0)
    assert n > 0, _lib.last_error()
    buf = (Op * n)()
    assert lib.fa4cp_ring_ce_direct_plan(S, rank, call, int(fused), buf, n) == n
    return [(o.stream, o.kind, o.a, o.b, o.c) for o in buf]


def expand_direct(ops, kernel_waits=True):
    """The fused launch as what it does: step 0 on the local K/V, then per step s a wait for
    slot (set0 + s - 1)'s flag and the reads of that slot, all released at the kernel's end."""
    out = []
    for o in ops:
        st, kind, a, b, c = o
        if kind == ATTN_FUSED_SLOTS:
            out.append((st, SEG_READ, 0, -1, 0))
            for s in range(1, a):
                if kernel_waits:
                    out.append((st, WAIT_FLAG, FLAG_SLOT0 + c + s - 1, b, 0))
                out.append((st, SEG_READ, s, c + s - 1, 0))
            out.append((st, KERNEL_END, 0, 0, 0))
        else:
            out.append(o)
    return out


def simulate_direct(S, calls, seed, serial, fused=False, plan_fn=None, kernel_waits=True,
                    call_streams=False):
    """Every rank's direct-push plan for `calls` consecutive calls (call numbers 1..calls)
    through a simulator of streams, events, flags and slots, in random (or host-order
    serialised) interleavings with adversarial timing.  Checks: no deadlock; step s of rank r
    in call c reads the K/V of rank (r - s) mod S from call c; no slot is written while read
    or written, or overwritten before the call that filled it attended it; flags only grow.
    call_streams: every call on its own caller's stream (consecutive calls then overlap)."""
    plan_fn = plan_fn or direct_plan
    rng = random.Random(seed)
    ranks = []
    for r in range(S):
        ops = []
        for c in range(1, calls + 1):
            for o in expand_direct(plan_fn(S, r, c, fused), kernel_waits):
                ops.append((c,) + o)
        last_record, waits_on = {}, {}
        for i, (c, st, kind, a, b, cc) in enumerate(ops):
            if kind == RECORD:
                last_record[a] = i
            elif kind == WAIT_EVENT:
                waits_on[i] = last_record.get(a)
        queues = {}
        for i, o in enumerate(ops):
            q = 0 if serial else o[1]
            if call_streams and not serial and o[1] == 0:
                q = 100 + o[0]
            queues.setdefault(q, []).append(i)
        ranks.append(dict(ops=ops, waits_on=waits_on, queues=queues, pos={q: 0 for q in queues},
                          pending={}, done=set(), flags={}, kernel_reads=[],
                          slots=[[Part(), Part()] for _ in range(max(2 * (S - 1), 1))]))

    def flag(R, f):
        return R["flags"].get(f, 0)

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
            return flag(R, a) >= b
        return True

    def read_slot(r, step, idx, c):
        if idx < 0:
            assert step == 0
            return []
        parts = ranks[r]["slots"][idx]
        for p in parts:
            assert not p.writing and p.tag is not None, "attention reads a slot that is not ready"
            assert p.tag == ((r - step) % S, c), f"rank {r} step {step} attends {p.tag}"
            p.readers += 1
        return parts

    def begin(r, i):
        c, st, kind, a, b, cc = ranks[r]["ops"][i]
        if kind == COPY_TO:
            dst = ranks[(r + b) % S]["slots"][cc][a]
            assert dst.readers == 0 and not dst.writing, "push overwrites a slot in use"
            assert dst.attended, "push overwrites data not yet attended"
            dst.tag, dst.writing, dst.attended = (r, c), True, False
            return ("copy", None, dst)
        return ("attn", read_slot(r, a, b, c))

    def end(token):
        if token[0] == "copy":
            token[2].writing = False
        else:
            for p in token[1]:
                p.readers -= 1
                p.attended = True

    mode = seed % 4
    slow_rank = rng.randrange(S)

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
        if kind in (COPY_TO, ATTN):
            R["pending"][q] = (i, begin(r, i))
            return
        if kind == SEG_READ:
            R["kernel_reads"].append(("attn", read_slot(r, a, b, c)))
        elif kind == KERNEL_END:
            if mode == 1 and rng.random() < 0.9:
                return
            for token in R["kernel_reads"]:
                end(token)
            R["kernel_reads"] = []
        elif kind == WRITE_PEER:
            peer = ranks[(r + a) % S]
            assert cc >= flag(peer, b), "flags only grow"
            peer["flags"][b] = cc
        else:
            assert kind in (RECORD, WAIT_EVENT, WAIT_FLAG), kind
        R["done"].add(i)
        R["pos"][q] += 1

    def slow(r, q):
        R = ranks[r]
        if mode == 3:
            return r == slow_rank
        if q not in R["pending"]:
            return False
        kind = R["ops"][R["pending"][q][0]][2]
        return (mode == 1 and kind == ATTN) or (mode == 2 and kind == COPY_TO)

    total = sum(len(R["ops"]) for R in ranks)
    while sum(len(R["done"]) for R in ranks) < total:
        cands = [(r, q) for r in range(S) for q in ranks[r]["queues"] if runnable(r, q)]
        assert cands, f"deadlock (S={S}, seed={seed}, serial={serial}, fused={fused})"
        fast = [x for x in cands if not slow(*x)]
        if fast and rng.random() < 0.97:
            cands = fast
        execute(*rng.choice(cands))
    for R in ranks:
        n_steps = sum(1 for o in R["ops"] if o[2] in (ATTN, SEG_READ))
        assert n_steps == S * calls


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("S", [2, 3, 4, 8])
def test_direct_plan_is_deadlock_free_and_hazard_free(S, fused):
    for seed in range(30 if S < 8 else 10):
        simulate_direct(S, calls=4, seed=seed, serial=False, fused=fused)


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("S", [2, 3, 8])
def test_direct_plan_with_a_stream_per_call(S, fused):
    """Consecutive calls on different caller streams overlap; the releases still keep every
    slot set safe."""
    for seed in range(20 if S < 8 else 8):
        simulate_direct(S, calls=5, seed=seed, serial=False, fused=fused, call_streams=True)


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("S", [2, 3, 4, 8])
def test_direct_plan_with_streams_serialised_in_host_order(S, fused):
    for seed in range(8):
        simulate_direct(S, calls=4, seed=seed, serial=True, fused=fused)


def test_direct_plan_shape():
    ops = direct_plan(4, 1, 1)
    kinds = [o[1] for o in ops]
    assert kinds.count(ATTN) == 4 and kinds.count(COPY_TO) == 6  # 3 peers x (K, V)
    # pushes go to peers 1, 2, 3 (step order), alternating copy pairs; set 1 for odd calls
    assert [(o[3], o[4]) for o in ops if o[1] == COPY_TO and o[2] == 0] == [(1, 3), (2, 4), (3, 5)]
    assert {o[0] for o in ops if o[1] == COPY_TO} == {1, 2, 4, 5}
    fused = direct_plan(4, 1, 2, fused=True)
    assert [o for o in fused if o[1] == ATTN_FUSED_SLOTS][0][2:] == (4, 2, 0)
    # from call 3 on a push waits for the release of call n - 2 of the same slot set
    assert not [o for o in direct_plan(4, 0, 2) if o[1] == WAIT_FLAG and o[2] >= FLAG_PEER_FREED0]
    w = [o for o in direct_plan(4, 0, 3) if o[1] == WAIT_FLAG and o[2] >= FLAG_PEER_FREED0]
    assert sorted({(o[2] - FLAG_PEER_FREED0, o[3]) for o in w}) == [(1, 1), (2, 1), (3, 1)]
    assert direct_plan(1, 0, 1) == [(0, ATTN, 0, -1, 0)]
    with pytest.raises(AssertionError):
        direct_plan(4, 0, 0)


@pytest.mark.parametrize("fused,drop", [(False, "freed_wait"), (False, "arrived_wait"),
                                        (False, "release_before_done"), (True, "freed_wait"),
                                        (True, "kernel_wait"), (True, "one_slot_set")])
def test_direct_planted_mistake_is_caught(fused, drop):
    """A direct plan missing one of its waits, or using a single slot set, must fail."""
    def broken(S, rank, call, fused):
        out = []
        for o in direct_plan(S, rank, call, fused):
            st, kind, a, b, c = o
            if drop == "freed_wait" and kind == WAIT_FLAG and a >= FLAG_PEER_FREED0:
                continue
            if drop == "arrived_wait" and kind == WAIT_FLAG and st == 0:
                continue
            if drop == "release_before_done" and kind == WAIT_EVENT and st == 3:
                continue
            if drop == "one_slot_set":
                # every call in set 0, still waiting for call n - 2's release only
                if kind == COPY_TO:
                    o = (st, kind, a, b, c - (S - 1) if c >= S - 1 else c)
                elif kind == WRITE_PEER and b < FLAG_PEER_FREED0 and b >= FLAG_SLOT0 + S - 1:
                    o = (st, kind, a, b - (S - 1), c)
                elif kind == ATTN_FUSED_SLOTS:
                    o = (st, kind, a, b, 0)
            out.append(o)
        return out

    # with one caller stream, call n + 2's pushes already follow call n + 1's attention, which
    # needed the destination's own call n + 1 pushes: a missing release wait only shows when
    # calls run on their own streams
    with pytest.raises(AssertionError):
        for seed in range(60):
            simulate_direct(4, calls=5, seed=seed, serial=False, fused=fused, plan_fn=broken,
                            kernel_waits=drop != "kernel_wait",
                            call_streams=drop in ("freed_wait", "one_slot_set",
                                                  "release_before_done"))
