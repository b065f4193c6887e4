"""Multi-process (world_size 2..4, gloo on CPU) tests of the ring's host-side rotation:
every rank must see the K/V of source ``(rank - s) mod S`` at step ``s``, with exactly
``S - 1`` hops, through the same :class:`fa4_ring.comm.KVRing` the GPU path uses."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path[:0] = q["paths"]
    from fa4_ring.comm import KVRing
    from fa4_ring.ring_attention import ring_schedule
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        T, H, D = 6, 2, 4
        k = torch.full((T, H, D), float(rank))
        v = torch.full((T, H, D), float(100 + rank))
        ring = KVRing(k, v, rank, world)
        ring.start()
        seen = []
        for step, src, _ in ring_schedule(rank, world):
            kk, vv = ring.get(step)
            seen.append((step, src, float(kk[0, 0, 0]), float(vv[0, 0, 0])))
            ring.done(step)
        assert ring.hops_issued == world - 1
        for step, src, ks, vs in seen:
            assert ks == float(src) and vs == float(100 + src), (rank, step, src, ks)
        # user's buffers are never overwritten by the rotation
        assert float(k[0, 0, 0]) == float(rank)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_kv_ring_rotation_gloo(world):
    import sys
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, {"paths": sys.path[:3]}))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes


def _liveness_worker(rank, world, port, q):
    """Ranks enter two ring calls together; then the last rank leaves (between calls) and the
    others' next call must raise, naming it, within the timeout -- not wait forever."""
    import sys
    import time
    sys.path[:0] = q["paths"]
    from fa4_ring.comm import _ring_liveness
    import fa4_ring.comm as comm
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    comm.RING_LIVENESS_TIMEOUT_S = 2.0
    live = _ring_liveness(None, rank, world)
    assert live is not None and live.peers == sorted({(rank - 1) % world, (rank + 1) % world})
    for _ in range(2):
        live.enter()
    assert live.calls == 2
    leaver = world - 1
    dist.barrier()  # every rank has entered call 2 before the leaver goes
    if rank == leaver:
        os._exit(0)  # leaves between calls, without any collective clean-up
    t0 = time.monotonic()
    if leaver in live.peers:
        try:
            live.enter()
        except RuntimeError as e:
            named = str(e).split("neighbour rank ")[1].split(" has")[0].split(", ")
            assert str(leaver) in named, str(e)
            assert 1.9 < time.monotonic() - t0 < 30.0
        else:
            raise AssertionError("a call with a departed neighbour did not raise")
    else:
        live.enter()  # both of its neighbours are still there and enter the call
        assert live.calls == 3
    os._exit(0)  # the process group still counts the leaver: skip its teardown


@pytest.mark.parametrize("world", [2, 4])
def test_ring_liveness_detects_a_departed_neighbour(world):
    import sys
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_liveness_worker, args=(r, world, port, {"paths": sys.path[:3]}))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
