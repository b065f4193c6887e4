"""Chain-forward KV rotation for the zig-zag ring (replaces fa4_ring/ring_attention.py:121-171).

At step ``s`` a rank attends the K/V that originated on rank ``(rank - s) mod S``.
Hop ``s`` (``s = 1 .. S-1``) therefore sends the K/V used at step ``s-1`` to
``rank + 1`` and receives the K/V of step ``s`` from ``rank - 1``; there are exactly
``S - 1`` transfers and every received shard is attended (the reference's loop
computes on the shard it holds while labelling it with the next source, so it
attends its own KV twice and never the shard of ``rank + 1``).

On CUDA the hops run as NCCL send/recv (``torch.distributed.batch_isend_irecv``)
issued from a dedicated high-priority comm stream into two persistent receive
buffers (ping-pong).  Ordering is by CUDA events only, no host blocking:

* hop 1 waits for the caller's stream (which produced the local K/V it sends);
* hop ``s`` waits for the compute of step ``s - 2`` (the last reader of the buffer it
  overwrites); the previous hop is ordered by the comm stream itself;
* the compute stream waits for hop ``s`` right before step ``s``.

Hop ``s + 1`` is issued as soon as step ``s`` is enqueued, so it overlaps step ``s``'s
attention.  With a CPU process group (gloo) the same schedule runs with blocking
hops; that path exists to test the rotation logic without a GPU.
"""

from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

_COMM_STREAMS: Dict[int, torch.cuda.Stream] = {}


def comm_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _COMM_STREAMS.get(idx)
    if st is None:
        lo, hi = torch.cuda.Stream.priority_range()
        st = torch.cuda.Stream(device=torch.device("cuda", idx), priority=hi)
        _COMM_STREAMS[idx] = st
    return st


def nccl_pg_options(cta_policy: str = "default"):
    """Options for the NCCL process group the ring runs on: high-priority NCCL streams.

    The attention kernel fills every SM (one CTA holds an SM's whole register file), so
    the KV hop's NCCL kernel only gets SMs as attention CTAs retire; on a high-priority
    stream its CTAs are placed ahead of the queued attention CTAs, so the transfer overlaps
    the step instead of waiting for the end of the attention grid.  Use as
    ``dist.init_process_group("nccl", pg_options=nccl_pg_options(), ...)`` or for the
    ``group`` passed to ``ring_flash_attn``.
    """
    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    if cta_policy == "zero":
        # NCCL 2.28+: communicate without SM CTAs where NCCL supports it (copy engines)
        opts.config.cta_policy = dist.ProcessGroupNCCL.NCCL_CTA_POLICY_ZERO
    elif cta_policy != "default":
        raise ValueError(f"unknown cta_policy {cta_policy!r}")
    return opts


def _global_rank(group, r: int) -> int:
    if group is None:
        return r
    return dist.get_global_rank(group, r)


class KVRing:
    """Rotates one rank's (K, V) shard around the cp group, one hop per ring step."""

    def __init__(self, k: torch.Tensor, v: torch.Tensor, cp_rank: int, cp_size: int,
                 group: Optional["dist.ProcessGroup"] = None):
        assert cp_size >= 2, "a ring needs at least two ranks"
        self.S = cp_size
        self.rank = cp_rank
        self.group = group
        self.send_to = _global_rank(group, (cp_rank + 1) % cp_size)
        self.recv_from = _global_rank(group, (cp_rank - 1) % cp_size)
        self.cuda = k.is_cuda
        nbuf = min(2, cp_size - 1)
        self.bufs = [(torch.empty_like(k), torch.empty_like(v)) for _ in range(nbuf)]
        self.kv: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {0: (k, v)}
        self.hop_done: Dict[int, torch.cuda.Event] = {}
        self.consumed: Dict[int, torch.cuda.Event] = {}
        self.stream = comm_stream(k.device) if self.cuda else None
        self.hops_issued = 0

    def _hop(self, s: int) -> None:
        sk, sv = self.kv[s - 1]
        dk, dv = self.bufs[s % len(self.bufs)]
        ops = [
            dist.P2POp(dist.isend, sk, self.send_to, group=self.group),
            dist.P2POp(dist.irecv, dk, self.recv_from, group=self.group),
            dist.P2POp(dist.isend, sv, self.send_to, group=self.group),
            dist.P2POp(dist.irecv, dv, self.recv_from, group=self.group),
        ]
        if self.cuda:
            with torch.cuda.stream(self.stream):
                prev_reader = self.consumed.get(s - 2)
                if prev_reader is not None:
                    self.stream.wait_event(prev_reader)
                for req in dist.batch_isend_irecv(ops):
                    req.wait()  # comm stream waits for NCCL; the host does not block
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self.hop_done[s] = ev
        else:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        self.kv[s] = (dk, dv)
        self.hops_issued = s

    def start(self) -> None:
        """Issue hop 1 (overlaps the local step 0).  The caller's K/V were produced on
        the current stream, so the comm stream first waits for everything enqueued there."""
        if self.cuda:
            ready = torch.cuda.Event()
            ready.record(torch.cuda.current_stream(self.kv[0][0].device))
            self.stream.wait_event(ready)
        self._hop(1)

    def get(self, s: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """K/V of step ``s``; the current stream is made to wait for its arrival, and
        the next hop is issued so that it overlaps step ``s``."""
        if s == 0:
            return self.kv[0]
        assert s <= self.hops_issued, "hops are issued in order"
        if self.cuda:
            torch.cuda.current_stream(self.kv[0][0].device).wait_event(self.hop_done[s])
        if s + 1 < self.S:
            self._hop(s + 1)
        return self.kv[s]

    def done(self, s: int) -> None:
        """Mark step ``s``'s compute as enqueued; its K/V buffer may be reused after it."""
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.kv[0][0].device))
            self.consumed[s] = ev


class GradRing:
    """The rotating fp32 dK/dV accumulators of the ring backward.

    At step ``s`` a rank computes the gradient contribution of its queries to the K/V of
    source ``(rank - s) mod S`` into a fresh buffer (:meth:`fresh`), then :meth:`pass_on`
    adds the accumulator of the same source that ``rank - 1`` passed on after ITS step
    ``s - 1``, and sends the sum to ``rank + 1``.  A source's accumulator therefore starts
    on the source itself (step 0) and visits every rank once; the pass after step ``S - 1``
    delivers it, complete, to its owner (:meth:`finish`).  ``S`` passes of
    ``2 * T * H_kv * D * 4`` bytes.

    On CUDA every pass is an NCCL send/recv on the comm stream (the one :class:`KVRing`
    uses, so the two rotations are issued in one order on every rank), ordered by events:
    the pass of step ``s`` waits for the step's add on the compute stream; the add of step
    ``s`` waits for the pass of step ``s - 1``, which delivered its input.  Two compute
    buffers alternate, so step ``s + 1`` computes while the pass of step ``s`` is in
    flight; one receive buffer suffices because a pass is issued only after the add that
    read the previous one.  With a CPU group (gloo) the passes block.
    """

    def __init__(self, shape, cp_rank: int, cp_size: int, device: torch.device,
                 group: Optional["dist.ProcessGroup"] = None):
        assert cp_size >= 2, "a ring needs at least two ranks"
        self.S = cp_size
        self.group = group
        self.device = device
        self.send_to = _global_rank(group, (cp_rank + 1) % cp_size)
        self.recv_from = _global_rank(group, (cp_rank - 1) % cp_size)
        self.cuda = device.type == "cuda"
        self.bufs = [torch.empty(shape, dtype=torch.float32, device=device) for _ in range(2)]
        self.recv = torch.empty(shape, dtype=torch.float32, device=device)
        self.stream = comm_stream(device) if self.cuda else None
        self.passed: Dict[int, Optional[torch.cuda.Event]] = {}

    def _current(self):
        return torch.cuda.current_stream(self.device)

    def fresh(self, s: int) -> torch.Tensor:
        """A zeroed fp32 buffer for step ``s``'s contribution."""
        buf = self.bufs[s % 2]
        prev = self.passed.get(s - 2)
        if self.cuda and prev is not None:
            self._current().wait_event(prev)  # its last send (step s - 2) is done
        buf.zero_()
        return buf

    def pass_on(self, s: int, buf: torch.Tensor, add) -> None:
        """``buf`` holds step ``s``'s contribution (enqueued on the current stream): add the
        accumulator received for this source with ``add(dst, src)`` (from step 1 on), send
        the sum to ``rank + 1`` and receive the accumulator of the next step's source."""
        if s > 0:
            if self.cuda:
                self._current().wait_event(self.passed[s - 1])
            add(buf, self.recv)
        ops = [dist.P2POp(dist.isend, buf, self.send_to, group=self.group),
               dist.P2POp(dist.irecv, self.recv, self.recv_from, group=self.group)]
        if self.cuda:
            ready = torch.cuda.Event()
            ready.record(self._current())
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ready)
                for req in dist.batch_isend_irecv(ops):
                    req.wait()
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self.passed[s] = ev
        else:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
            self.passed[s] = None

    def finish(self) -> torch.Tensor:
        """The complete accumulator of this rank's own K/V (after the pass of step S-1)."""
        assert (self.S - 1) in self.passed, "every step must be passed on first"
        if self.cuda:
            self._current().wait_event(self.passed[self.S - 1])
        return self.recv


# Seconds a native ring call waits on the host for its neighbours to enter the same call
# before it raises (RingLiveness); None turns the check off.
RING_LIVENESS_TIMEOUT_S: Optional[float] = 60.0


class RingLiveness:
    """Host-side check, before a ring call queues device waits on its neighbours, that both
    neighbours are still there.

    The native ring's device-side waits on a neighbour (the copy-engine transport's hop
    counters, ``cuStreamWaitValue32``; NCCL send/recv on the executor's communicator) have no
    time limit: a neighbour that left between calls would block this rank's streams until
    the process ends.  So call ``n`` first sets this rank's key for call ``n`` in the process
    group's key-value store and waits (server side, ``store.wait``) for both neighbours' keys
    of call ``n``; if one is missing after ``timeout_s`` seconds, the call raises
    ``RuntimeError`` naming it, before anything is queued on the GPU.  Three store round trips
    per call (set, wait, and deleting this rank's key of call ``n - 2``, which both neighbours
    have read: they entered call ``n - 1``).  A neighbour that dies while a call runs is not
    caught here (the ring kernel's own wait for a hop counter is bounded; the stream waits are
    not).
    """

    def __init__(self, store, prefix: str, rank: int, size: int, timeout_s: float):
        self.store, self.prefix, self.rank, self.size = store, prefix, rank, size
        self.timeout_s = float(timeout_s)
        self.calls = 0
        self.peers = sorted({(rank - 1) % size, (rank + 1) % size} - {rank})

    def _key(self, r: int, n: int) -> str:
        return f"{self.prefix}/{r}/{n}"

    def enter(self) -> None:
        import datetime

        self.calls += 1
        n = self.calls
        self.store.set(self._key(self.rank, n), "1")
        keys = [self._key(peer, n) for peer in self.peers]
        try:
            self.store.wait(keys, datetime.timedelta(seconds=self.timeout_s))
        except Exception as e:  # the store's timeout error
            gone = [peer for peer, k in zip(self.peers, keys) if not self.store.check([k])]
            raise RuntimeError(
                f"ring rank {self.rank}: neighbour rank {', '.join(map(str, gone or self.peers))} "
                f"has not entered ring call {n} within {self.timeout_s:.0f} s (it left or "
                "stalled); the call was not queued") from e
        if n > 2:
            self.store.delete_key(self._key(self.rank, n - 2))


_RING_SERIAL: Dict[Tuple, int] = {}


def _ring_liveness(group, cp_rank: int, cp_size: int) -> Optional[RingLiveness]:
    """A RingLiveness on the default store for a ring being created (collectively) on
    ``group``; None when the check is off or there is no store."""
    if RING_LIVENESS_TIMEOUT_S is None or cp_size < 2:
        return None
    try:
        from torch.distributed.distributed_c10d import _get_default_store
        store = _get_default_store()
    except Exception:  # no default store (a process group without one): no check
        return None
    ranks = tuple(dist.get_process_group_ranks(group)) if group is not None else tuple(
        range(dist.get_world_size()))
    serial = _RING_SERIAL.get(ranks, 0)  # every rank creates its rings in the same order
    _RING_SERIAL[ranks] = serial + 1
    prefix = "fa4cp_ring/" + "_".join(map(str, ranks)) + f"/{serial}"
    return RingLiveness(store, prefix, cp_rank, cp_size, RING_LIVENESS_TIMEOUT_S)


class NativeRing:
    """The library's native ring executor (``fa4cp_ring_*``) for one cp group on one GPU.

    One :meth:`forward` call issues a rank's whole ring forward (every K/V hop and every
    attention step) from C++, so the host cost per step is a few CUDA API calls instead of
    a Python loop over ``torch.distributed`` P2P ops.  Transports:

    * ``"copy_engine"`` (default): at the start of a call every rank pushes its own K/V with
      ``cudaMemcpyAsync`` straight into every peer's receive slot over NVSwitch (CUDA IPC
      mappings exchanged over ``group``), in step order, and sets that slot's arrival flag in
      the peer's memory (``cuStreamWriteValue32``); the attention waits for each slot's flag
      (the ring kernel in-kernel, per-step launches with ``cuStreamWaitValue32``).  Slots come
      in two sets used by alternate calls.  The transfer uses no SM;
    * ``"copy_engine_chain"``: the reference's chain-forward rotation on the copy engines --
      hop ``s`` forwards the K/V attended at step ``s - 1`` into the right neighbour's slot,
      with one arrival and one release hop counter per rank;
    * ``"nccl"``: NCCL send/recv on the executor's own communicator (created collectively
      from a unique id that cp rank 0 broadcasts over ``group``).

    Call :func:`close_native_rings` on every rank before ``destroy_process_group``.
    """

    TRANSPORTS = ("copy_engine", "copy_engine_chain", "nccl")

    def __init__(self, cp_rank: int, cp_size: int, device: torch.device,
                 group: Optional["dist.ProcessGroup"] = None, transport: str = "copy_engine"):
        import ctypes

        from . import _lib

        if transport not in self.TRANSPORTS:
            raise ValueError(f"unknown ring transport {transport!r}")
        self.lib = _lib.load()
        self.rank, self.size, self.device, self.group = cp_rank, cp_size, device, group
        self.transport = transport
        self.kv_capacity = 0
        uid = None
        if transport == "nccl" and cp_size > 1:
            uid = (ctypes.c_uint8 * 128)()
            if cp_rank == 0:
                _lib.check(self.lib.fa4cp_ring_unique_id(uid), "ring_unique_id")
            on_gpu = dist.get_backend(group) == "nccl"
            t = torch.tensor(list(uid), dtype=torch.uint8,
                             device=device if on_gpu else torch.device("cpu"))
            dist.broadcast(t, src=_global_rank(group, 0), group=group)
            uid = (ctypes.c_uint8 * 128)(*t.cpu().tolist())
        h = ctypes.c_int64(0)
        with torch.cuda.device(device):
            _lib.check(self.lib.fa4cp_ring_comm_init(uid, cp_size, cp_rank, ctypes.byref(h)),
                       "ring_comm_init")
        self.handle = h.value
        self.copy_engine = transport.startswith("copy_engine")
        if self.copy_engine:
            _lib.check(self.lib.fa4cp_ring_set_direct(self.handle,
                                                      int(transport == "copy_engine")),
                       "ring_set_direct")
        self.liveness = _ring_liveness(group, cp_rank, cp_size)

    def ensure_capacity(self, kv_bytes: int) -> None:
        """Copy-engine transport: make the receive slots hold ``kv_bytes`` per K (and V).
        Collective over the group when it grows (all ranks pass the same size)."""
        import ctypes

        from . import _lib

        if not self.copy_engine or self.size < 2 or kv_bytes <= self.kv_capacity:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            dist.barrier(group=self.group)  # no peer is still writing into the old areas
            _lib.check(self.lib.fa4cp_ring_ipc_close(self.handle), "ring_ipc_close")
            dist.barrier(group=self.group)  # nobody maps an area that is about to be freed
            mine = (ctypes.c_uint8 * 64)()
            _lib.check(self.lib.fa4cp_ring_ipc_alloc(self.handle, int(kv_bytes), mine),
                       "ring_ipc_alloc")
            handles = [None] * self.size
            dist.all_gather_object(handles, (bytes(mine), int(kv_bytes)), group=self.group)
            assert all(hb[1] == kv_bytes for hb in handles), "ranks disagree on the K/V size"
            if self.transport == "copy_engine":  # direct pushes: every peer's area
                allh = (ctypes.c_uint8 * (64 * self.size))(*b"".join(hb[0] for hb in handles))
                _lib.check(self.lib.fa4cp_ring_ipc_open_all(self.handle, allh),
                           "ring_ipc_open_all")
            else:
                left = (ctypes.c_uint8 * 64)(*handles[(self.rank - 1) % self.size][0])
                right = (ctypes.c_uint8 * 64)(*handles[(self.rank + 1) % self.size][0])
                _lib.check(self.lib.fa4cp_ring_ipc_open(self.handle, left, right),
                           "ring_ipc_open")
            dist.barrier(group=self.group)  # every area is mapped before the first push
        self.kv_capacity = int(kv_bytes)

    def forward(self, q, k, v, out, lse, cu, *, nseq: int, max_seqlen: int, softmax_scale: float,
                q_descale=None, k_descales=None, v_descales=None, kv_bufs=None,
                workspace=None) -> None:
        """Run the ring forward on the current stream into ``out``/``lse`` (see
        ``fa4cp_ring_attn_fwd``).  ``k_descales``/``v_descales``: ``[cp_size, H_kv]`` fp32."""
        from . import _lib

        T, Hq, D = q.shape
        Hkv = k.shape[1]
        if self.liveness is not None:
            self.liveness.enter()  # raises if a neighbour left: nothing is queued then
        rc = self.lib.fa4cp_ring_attn_fwd(
            self.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.ptr(kv_bufs),
            0 if kv_bufs is None else kv_bufs.numel() * kv_bufs.element_size(), out.data_ptr(),
            lse.data_ptr(), cu.data_ptr(), nseq, max_seqlen, T, Hq, Hkv, D,
            _lib.dtype_code(q.dtype), _lib.dtype_code(k.dtype), float(softmax_scale),
            _lib.ptr(q_descale), _lib.ptr(k_descales), _lib.ptr(v_descales), _lib.ptr(workspace),
            0 if workspace is None else workspace.numel(), _lib.stream_of(q))
        _lib.check(rc, "ring_attn_fwd")

    def start_timing(self, max_launches: int) -> None:
        """Time the next ``max_launches`` attention launches with CUDA events."""
        from . import _lib

        _lib.check(self.lib.fa4cp_ring_timing(self.handle, int(max_launches)), "ring_timing")

    def set_fused(self, mode: int) -> None:
        """Ring kernel: 0 never, 1 for f16 / bf16 (D 64, 128), 2 also for e4m3 (the library
        default), 3 also at head_dim 256 (f16 / bf16, and bf16 q with e4m3 K/V)."""
        from . import _lib

        if getattr(self, "_fused", None) != int(mode):
            _lib.check(self.lib.fa4cp_ring_set_fused(self.handle, int(mode)), "ring_set_fused")
            self._fused = int(mode)

    def set_sm_reserve(self, n: int) -> None:
        """SMs the persistent attention grid leaves free for the hop's NCCL kernel."""
        from . import _lib

        _lib.check(self.lib.fa4cp_ring_set_sm_reserve(self.handle, int(n)), "ring_set_sm_reserve")

    def timeline(self, max_entries: int = 4096):
        """``(attention, hops)``: lists of ``(start_ms, end_ms)`` of the timed launches and
        hops in issue order, relative to the first timed launch (call before
        :meth:`read_timing`, which starts over)."""
        import ctypes

        from . import _lib

        a = (ctypes.c_float * (2 * max_entries))()
        h = (ctypes.c_float * (2 * max_entries))()
        na, nh = ctypes.c_int32(0), ctypes.c_int32(0)
        _lib.check(self.lib.fa4cp_ring_timeline(self.handle, a, max_entries, h, max_entries,
                                                ctypes.byref(na), ctypes.byref(nh)),
                   "ring_timeline")
        return ([(a[2 * i], a[2 * i + 1]) for i in range(na.value)],
                [(h[2 * i], h[2 * i + 1]) for i in range(nh.value)])

    def read_timing(self):
        """``(summed ms, launches)`` of the launches timed since :meth:`start_timing`."""
        import ctypes

        from . import _lib

        ms, n = ctypes.c_double(0.0), ctypes.c_int32(0)
        _lib.check(self.lib.fa4cp_ring_timing_read(self.handle, ctypes.byref(ms), ctypes.byref(n)),
                   "ring_timing_read")
        return ms.value, n.value

    def unmap_peers(self) -> None:
        """Unmap the neighbours' receive areas (waits for this GPU's work)."""
        from . import _lib

        if self.handle and self.kv_capacity:
            with torch.cuda.device(self.device):
                _lib.check(self.lib.fa4cp_ring_ipc_close(self.handle), "ring_ipc_close")

    def close(self) -> None:
        if self.handle:
            self.lib.fa4cp_ring_comm_destroy(self.handle)
            self.handle = 0


_NATIVE_RINGS: Dict[Tuple, Tuple[object, NativeRing]] = {}


def native_ring(cp_rank: int, cp_size: int, device: torch.device,
                group: Optional["dist.ProcessGroup"] = None,
                transport: str = "copy_engine") -> NativeRing:
    """The :class:`NativeRing` of ``group`` on ``device`` (created collectively on first use)."""
    g = group if group is not None else dist.group.WORLD
    key = (id(g), device.index, cp_rank, cp_size, transport)
    hit = _NATIVE_RINGS.get(key)
    if hit is not None and hit[0] is g:
        return hit[1]
    ring = NativeRing(cp_rank, cp_size, device, group, transport)
    _NATIVE_RINGS[key] = (g, ring)  # holds the group so its id stays unique
    return ring


def close_native_rings() -> None:
    """Free every native ring (its NCCL communicator or receive areas).  Collective: all
    ranks call it, before the process group is destroyed.  Every rank unmaps its
    neighbours' receive areas before any rank frees its own (freeing memory another
    process still maps is undefined behaviour in CUDA IPC)."""
    rings = [ring for _, ring in _NATIVE_RINGS.values()]
    for ring in rings:
        ring.unmap_peers()
    if any(r.copy_engine and r.size > 1 for r in rings) and dist.is_initialized():
        dist.barrier()
    for ring in rings:
        ring.close()
    _NATIVE_RINGS.clear()  # a later call on the same group builds a new ring
    _NATIVE_RINGS.clear()
