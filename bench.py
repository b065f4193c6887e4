"""Benchmark of the zig-zag causal ring-attention forward on B200.

Workload ("cfg2"): one causal ring-attention forward over a
bf16 sequence of N=32768 tokens, Hq=32, Hkv=8, D=128, softmax scale 1/sqrt(128),
q/k/v ~ N(0,1) from a seed, cp = number of GPUs, merge_mode incremental.  The
total work is fixed as cp grows ("strong" scaling).  Metric: causal FLOPs
(2*N^2*Hq*D per forward) per second, whole job, in TFLOP/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

One JSON line on rank 0.  ``value``: device time with inputs resident in HBM, max
over ranks, L2 flushed (256 MiB write) before every timed step.  ``e2e``: the same
forward through the public API with the step's Q/K/V shards copied in from pinned
host memory and the output copied back, inside the timed region.  ``roofline``:
the attention kernel (the dominant kernel) -- algorithmic FLOPs / its CUDA-event
time, against the measured bf16 peak.  ``cpu_baseline``: the numpy restatement of
the reference's CPU ring simulation (``oracle/``) on rank 0's share of the ring at
cp=8 (a bounded sample), on the host cores.  ``--impl reference`` times that CPU
path alone (the reference is pure Python over third-party GPU kernels that are not
installed here and its GPU orchestration attends wrong KV shards; its own CPU
simulation is the path that runs).

``--bwd`` measures the ring BACKWARD instead (not in the reference, which is forward-only):
``ring_flash_attn_backward`` on bf16 cfg2 / cfg4 shards with the forward's (out, lse) and a
seeded upstream gradient, FLOPs = 2.5x the forward's (5 matmuls of the forward's size, N^2/2
convention), one JSON line with ``metric`` "causal ring-attn backward TFLOP/s".
"""

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fa4-cp_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "causal ring-attn prefill TFLOP/s/GPU @cp=1/2/4/8; % tensor peak; exposed comm %"
CFG2 = dict(N=32768, Hq=32, Hkv=8, D=128)
L2_FLUSH_BYTES = 256 << 20

# BASELINE.json configs[1..4]; "kind": operand types (bf16 | e4m3 q/k/v | bf16 q + e4m3 k/v)
CONFIGS = {
    "cfg2": dict(kind="bf16", lens=[32768], Hq=32, Hkv=8, D=128, amp=1.0,
                 text="bf16 single sequence, N=32768, Hq=32, Hkv=8, D=128"),
    "cfg3": dict(kind="e4m3", lens=[131072], Hq=32, Hkv=8, D=128, amp=1.0,
                 text="FP8 e4m3 q/k/v quantised per rank (scale=amax/448), N=131072, Hq=32, "
                      "Hkv=8, D=128, k/v descales all-gathered by source rank"),
    "cfg4": dict(kind="bf16", lens="varlen16", Hq=16, Hkv=2, D=128, amp=1.0,
                 text="packed varlen bf16, 16 sequences N_j ~ U[1024,16384] (seed 0) rounded up "
                      "to a multiple of 2*cp, Hq=16, Hkv=2, D=128"),
    "cfg5": dict(kind="mixed", lens=[262144], Hq=16, Hkv=2, D=256, amp=0.5,
                 text="bf16 q with e4m3 k/v (per rank amax/448), N=262144, Hq=16, Hkv=2, D=256, "
                      "q/k/v ~ 0.5*N(0,1)"),
}


def config_lens(name, cp, seq_len=None):
    c = CONFIGS[name]
    if c["lens"] == "varlen16":
        rng = np.random.default_rng(0)
        raw = rng.integers(1024, 16385, size=16)
        m = 2 * cp
        return [int((n + m - 1) // m * m) for n in raw]
    return [seq_len if seq_len else c["lens"][0]]


def measure_fp8_peak(dev):
    """Dense e4m3 GEMM throughput on this GPU (torch._scaled_mm, 8192^3, best of 10)."""
    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.tensor(1.0, device=dev)
    for _ in range(3):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


def causal_flops(N, Hq, D):
    return 2.0 * N * N * Hq * D


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons of this GPU, sampled by NVML every 10 ms in a
    background thread while the timed region runs.  NVML is initialised, and the first sample
    taken, before ``__enter__`` returns: initialising it inside the timed region stalled the
    main thread's kernel launches while the GPU drained its queue (cfg4 at cp=1: 7.77 ms per
    step against 6.2 ms for the same launches timed without the sampler)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index, interval=0.01):
        self.dev = device_index
        self.interval = interval
        self.samples = []
        self.max_mhz = None
        self.error = None

    def _handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            prop = torch.cuda.get_device_properties(self.dev)
            bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def _sample(self):
        nv, h = self._nv, self._h
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        try:
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except AttributeError:
            rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        self.samples.append((sm, rs))

    def _run(self):
        try:
            while not self._stop.wait(self.interval):
                self._sample()
        except Exception as e:
            self.error = repr(e)

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        self._t = None
        try:
            self._nv, self._h = self._handle()
            self.max_mhz = self._nv.nvmlDeviceGetMaxClockInfo(self._h, self._nv.NVML_CLOCK_SM)
            self._sample()  # the first query warms NVML up; it is not a sample of the run
            self.samples.clear()
        except Exception as e:  # NVML missing: report it instead of guessing
            self.error = repr(e)
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join(5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz,
                    "reasons": [f"no samples: {self.error}"]}
        sm = [a for a, _ in self.samples]
        busy = [a for a in sm if self.max_mhz and a > 0.3 * self.max_mhz] or sm
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- CPU baseline
def cpu_sample(rank_steps=None, threads=None, min_seconds=10.0):
    """Time the oracle (numpy restatement of the reference's CPU ring simulation) on rank 0's
    share of the cfg2 ring at cp=8: every step of rank 0, repeated until ``min_seconds`` of
    work (or the given subset of steps once), all heads.  Returns (flops, seconds, threads)."""
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import ring_oracle as orc
    threads = threads or os.cpu_count() or 1
    limiter = threadpool_limits(limits=threads)
    info = threadpool_info()
    threads = max([i.get("num_threads", 1) for i in info if i.get("user_api") == "blas"] or [1])
    N, Hq, Hkv, D = CFG2["N"], CFG2["Hq"], CFG2["Hkv"], CFG2["D"]
    cp, rank = 8, 0
    T = N // cp
    rng = np.random.default_rng(0)
    q = rng.standard_normal((T, Hq, D), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, D), dtype=np.float32)
    scale = 1.0 / math.sqrt(D)
    sched = orc.ring_schedule(rank, cp)
    if rank_steps is not None:
        sched = [sched[i % len(sched)] for i in rank_steps]
    flops = 0.0
    t0 = time.perf_counter()
    # the rank's ring, repeated until about 10 s of CPU work (at least one pass)
    while True:
        acc = None
        for (_step, _src, pat) in sched:
            o, l = orc.ring_step(q, k, v, [0, T], pat, scale)
            acc = (o, l) if acc is None else orc.merge(acc[0], acc[1], o, l)
            # local causal T x T (N^2/2 convention) and T x T/2 non-causal both count 2*T^2*Hq*D
            flops += 2.0 * T * T * Hq * D
        if rank_steps is not None or time.perf_counter() - t0 >= min_seconds:
            break
    dt = time.perf_counter() - t0
    limiter.restore_original_limits()
    return flops, dt, threads


def cpu_sample_bwd(threads=None, heads=32, steps=1):
    """Time the backward oracle (the gradient of the reference's CPU ring algorithm,
    ``oracle/bwd_oracle.py``, fp32) on a bounded sample of the cfg2 ring backward at cp=8:
    the first ``steps`` steps of rank 0 for ``heads`` query heads.  Returns (flops, seconds,
    threads); flops count 5 matmuls of the step's size (2.5x the forward's)."""
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import bwd_oracle as bo
    from oracle import ring_oracle as orc
    threads = threads or os.cpu_count() or 1
    limiter = threadpool_limits(limits=threads)
    info = threadpool_info()
    threads = max([i.get("num_threads", 1) for i in info if i.get("user_api") == "blas"] or [1])
    N, Hq, Hkv, D = CFG2["N"], CFG2["Hq"], CFG2["Hkv"], CFG2["D"]
    cp, rank = 8, 0
    T = N // cp
    hq = min(heads, Hq)
    hkv = max(1, hq * Hkv // Hq)
    rng = np.random.default_rng(0)
    q, dout = (rng.standard_normal((T, hq, D), dtype=np.float32) for _ in range(2))
    k, v = (rng.standard_normal((T, hkv, D), dtype=np.float32) for _ in range(2))
    lse = rng.standard_normal((T, hq), dtype=np.float32) + 8.0
    delta = rng.standard_normal((T, hq), dtype=np.float32)
    scale = 1.0 / math.sqrt(D)
    sched = orc.ring_schedule(rank, cp)[:steps]
    flops = 0.0
    t0 = time.perf_counter()
    for (_step, _src, pat) in sched:
        bo.ring_step_bwd(q, k, v, dout, lse, delta, [0, T], pat, scale, np.float32)
        flops += 2.5 * 2.0 * T * T * hq * D
    dt = time.perf_counter() - t0
    limiter.restore_original_limits()
    return flops, dt, threads


# --------------------------------------------------------------------------- GPU arm
def gpu_main(args, rank, world, local_rank):
    from fa4_ring import RingConfig, ring_flash_attn, zigzag_shard
    from fa4_ring import _lib, attn_backend, ring_attention
    from fa4_ring.ring_attention import ring_flash_attn_with_lse
    from fa4_ring.comm import native_ring

    from fa4_ring import Descales
    from fa4_ring.fp8 import allgather_descales, quantize_e4m3
    from fa4_ring.zigzag import zigzag_shard_varlen

    dev = torch.device("cuda", local_rank)
    C = CONFIGS[args.config]
    Hq, Hkv, D = C["Hq"], C["Hkv"], C["D"]
    cp = world
    lens = config_lens(args.config, cp, args.seq_len)
    for n in lens:
        assert n % (2 * cp) == 0, f"sequence length {n} not divisible by 2*cp"
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    g = torch.Generator(device=dev).manual_seed(1234)
    shards, lcu = [], None
    for h in (Hq, Hkv, Hkv):
        full = torch.randn(N, h, D, generator=g, device=dev, dtype=torch.bfloat16)
        if C["amp"] != 1.0:
            full.mul_(C["amp"])
        loc, lcu = zigzag_shard_varlen(full, full_cu, rank, cp)
        shards.append(loc)
        del full
    lq, lk, lv = shards
    varlen = len(lens) > 1
    cu_arg = lcu if varlen else None
    max_local = max(lens) // cp
    desc = None
    if C["kind"] in ("e4m3", "mixed"):
        # per-rank quantisation (amax/448); k/v descales all-gathered once, by source rank
        lk, ks = quantize_e4m3(lk)
        lv, vs = quantize_e4m3(lv)
        qs = None
        if C["kind"] == "e4m3":
            lq, qs = quantize_e4m3(lq)
        if world > 1:
            ks_all, vs_all = allgather_descales(ks), allgather_descales(vs)
        else:
            ks_all, vs_all = [ks], [vs]
        desc = Descales(q=qs, k=ks_all, v=vs_all)
    cfg = RingConfig(cp_size=cp, cp_rank=rank, merge_mode=args.merge)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    step_flops = float(sum(causal_flops(n, Hq, D) for n in lens))  # whole job, per step

    def barrier():
        if world > 1:
            dist.barrier()

    def run():
        return ring_flash_attn_with_lse(lq, lk, lv, cfg, descales=desc, cu_seqlens=cu_arg,
                                        max_seqlen=max_local if varlen else None)

    # ---- warm-up
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    _lib.device_status()

    # ---- timed: K steps, L2 flushed before each (untimed), per-step CUDA events
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    launches = []
    attn_backend.launch_timer = launches  # attention launches issued from Python
    nring = None
    if world > 1 and ring_attention.use_native_executor() and args.merge == "incremental":
        nring = native_ring(rank, cp, dev, transport=ring_attention.RING_TRANSPORT)  # from warm-up
        if args.sm_reserve is not None:
            nring.set_sm_reserve(args.sm_reserve)
            for _ in range(2):
                run()
        nring.start_timing(args.steps * cp)
    barrier()
    torch.cuda.synchronize()
    n_launch0 = _lib.launch_count
    host_s = 0.0
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record()
            h0 = time.perf_counter()
            timed_out = run()
            host_s += time.perf_counter() - h0
            ev[i][1].record()
        torch.cuda.synchronize()
        barrier()
    attn_backend.launch_timer = None
    gpu_launches = _lib.launch_count - n_launch0
    clocks = clk.summary()
    ms_local = sum(a.elapsed_time(b) for a, b in ev)
    timeline = None
    if nring is not None:
        if args.timeline:
            a, h = nring.timeline()
            na, nh = len(a) // args.steps, len(h) // args.steps  # per forward
            a, h = a[(args.steps - 1) * na:], h[(args.steps - 1) * nh:]  # the last forward
            t0 = a[0][0]
            timeline = {"rank": rank,
                        "attn": [[round(x - t0, 3), round(y - t0, 3)] for x, y in a],
                        "hops": [[round(x - t0, 3), round(y - t0, 3)] for x, y in h]}
        attn_ms_local, n_attn_local = nring.read_timing()
        nring.start_timing(0)
    else:
        attn_ms_local = sum(a.elapsed_time(b) for a, b, _ in launches)
        n_attn_local = len(launches)
    status = _lib.device_status()
    # exposed communication: the share of the step in which no attention kernel ran
    # (K/V hops not hidden under attention, plus launch gaps), this rank; max over ranks
    exposed_local = max(0.0, (ms_local - attn_ms_local) / ms_local * 100.0) if world > 1 else 0.0

    parity = sampled_parity(timed_out, C, lens, rank, cp, dev, desc, world)
    del timed_out
    exposed_8d_local = 0.0
    local_ms = None
    if world > 1:
        fused = nring is not None and n_attn_local == args.steps
        local_ms = local_schedule_ms(lq, lk, lv, cfg, desc, lcu, len(lens), max_local, fused,
                                     flush, max(3, min(args.steps, 10)), world)
        step_ms = ms_local / args.steps
        exposed_8d_local = max(0.0, (step_ms - local_ms) / step_ms * 100.0)

    if args.quick:  # profiling runs: timed loop only
        vals = torch.tensor([ms_local, attn_ms_local, exposed_local, exposed_8d_local],
                            dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        if timeline is not None:
            tls = [None] * world
            dist.all_gather_object(tls, timeline)
            if rank == 0:
                for t in tls:
                    print(json.dumps(t), file=sys.stderr, flush=True)
        if rank == 0:
            ms_step = vals[0].item() / args.steps
            return {"quick": True, "config": args.config, "seq_len": N, "cp": cp,
                    "ms_per_step": round(ms_step, 4),
                    "value": round(step_flops / (ms_step * 1e-3) / 1e12, 2),
                    "attn_ms": round(vals[1].item() / args.steps, 4), "gpu_launches": gpu_launches,
                    "exposed_comm_pct": round(vals[3].item(), 2),
                    "exposed_no_attn_pct": round(vals[2].item(), 2),
                    "host_issue_ms_per_step": round(host_s * 1e3 / args.steps, 3),
                    "parity": parity, "device_status": status}
        return None

    # ---- end to end through the public API: pinned host in, host out
    hq, hk, hv = (t.cpu().pin_memory() for t in (lq, lk, lv))
    out_dt = torch.bfloat16 if lq.dtype == torch.float8_e4m3fn else lq.dtype
    houts = [torch.empty(lq.shape, dtype=out_dt).pin_memory() for _ in range(2)]
    dsets = [tuple(torch.empty_like(t) for t in (lq, lk, lv)) for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    copy_in, copy_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def forward(dq, dk, dv):
        return ring_flash_attn(dq, dk, dv, cfg, descales=desc, cu_seqlens=cu_arg,
                               max_seqlen=max_local if varlen else None)

    def run_serial():  # copy in, compute, copy out, one step at a time
        dq, dk, dv = dsets[0]
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        houts[0].copy_(forward(dq, dk, dv), non_blocking=True)

    def run_pipelined(n):
        """n steps with double-buffered device inputs: the host->device copy of step i+1 and
        the device->host copy of step i run on their own streams beside step i's forward
        (every step still copies its own inputs in and its output back).  The L2 is flushed
        on the compute stream before each forward."""
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(copy_in)
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(copy_in):  # one stream: a second one measured slower
                if i >= 2:
                    copy_in.wait_event(ev_done[b])  # step i-2 no longer reads this set
                for d, h in zip(dsets[b], (hq, hk, hv)):
                    d.copy_(h, non_blocking=True)
                ev_in[b].record(copy_in)
            comp.wait_event(ev_in[b])
            flush.zero_()
            out = forward(*dsets[b])
            ev_done[b].record(comp)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_done[b])
                houts[b].copy_(out, non_blocking=True)
                out.record_stream(copy_out)
        end.record(copy_out)
        return start, end

    for _ in range(2):
        run_serial()
    run_pipelined(2)
    torch.cuda.synchronize()
    # as many steps as the timed loop (the pipeline's fill -- the first step's copy in -- and
    # drain -- the last copy out -- are then spread over the same count), capped near 5 s from
    # the FLOP count (the same on every rank, so all ranks run the same steps)
    est_ms = step_flops / world / 1.0e15 * 1e3
    e2e_steps = max(2, min(args.steps, int(5000.0 / max(est_ms, 1e-3))))
    ev3 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(e2e_steps)]
    barrier()
    torch.cuda.synchronize()
    for i in range(e2e_steps):
        flush.zero_()
        ev3[i][0].record()
        run_serial()
        ev3[i][1].record()
    torch.cuda.synchronize()
    e2e_serial_ms_local = sum(a.elapsed_time(b) for a, b in ev3) / e2e_steps
    barrier()
    torch.cuda.synchronize()
    st_ev, en_ev = run_pipelined(e2e_steps)
    torch.cuda.synchronize()
    barrier()
    e2e_ms_local = st_ev.elapsed_time(en_ev) / e2e_steps
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = houts[0].numel() * houts[0].element_size()

    # ---- reduce over ranks (max)
    vals = torch.tensor([ms_local, attn_ms_local, e2e_ms_local, exposed_local, float(status),
                         e2e_serial_ms_local, exposed_8d_local, local_ms or 0.0],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    (ms_total, attn_ms, e2e_ms, exposed, status_max, e2e_serial_ms, exposed_8d,
     local_ms_max) = vals.tolist()

    if rank != 0:
        return None
    ms_step = ms_total / args.steps
    value = step_flops / (ms_step * 1e-3) / 1e12
    peaks, peaks_kind = load_peaks()
    # attention roofline: every attention launch of one rank in the timed region;
    # algorithmic FLOPs of one rank per step = (sum_j 2*N_j^2*Hq*D) / cp (zig-zag balance)
    attn_flops_rank = step_flops / cp * args.steps
    achieved = attn_flops_rank / (attn_ms * 1e-3) / 1e12 if attn_ms > 0 else None
    if C["kind"] == "e4m3":
        peak = round(measure_fp8_peak(dev), 1)
        peak_kind = "measured on this GPU now: e4m3 torch._scaled_mm 8192^3 (burst)"
    else:
        peak = peaks["bf16_tflops"]
        peak_kind = f"{peaks_kind} bf16 dense (burst)"
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": {"bf16": "bf16", "e4m3": "e4m3", "mixed": "bf16 q, e4m3 k/v"}[C["kind"]],
        "data": "synthetic: q/k/v ~ N(0,1) bf16 from seed 1234"
                + (f" x {C['amp']}" if C["amp"] != 1.0 else ""),
        "config": {"workload": f"{args.config}: causal ring-attention forward, {C['text']}, "
                               f"scale=1/sqrt(D), cp={cp}, merge={args.merge}",
                   "seq_len": N, "num_seqs": len(lens), "num_heads_q": Hq, "num_heads_kv": Hkv,
                   "head_dim": D,
                   "cp": cp, "merge_mode": args.merge, "parallelism": f"cp{cp} zig-zag ring",
                   "transport": args.transport if world > 1 else None,
                   "ring_kernel": args.ring_kernel if world > 1 else None,
                   "l2": "flushed before every timed step (256 MiB write, untimed)"},
        "per_gpu_tflops": round(value / world, 2),
        "pct_tensor_peak": round(value / world / peak * 100.0, 2),
        "exposed_comm_pct": round(exposed_8d, 2) if world > 1 else None,
        "exposed_comm_def": "100 * (ring step time - the same schedule with the transfers "
                            "skipped) / ring step time, max over ranks; the no-transfer time "
                            "runs this rank's forward with every step's K/V already local "
                            "(all-gathered beforehand, untimed)",
        "no_transfer_ms_per_step": round(local_ms_max, 4) if world > 1 else None,
        "exposed_no_attn_pct": round(exposed, 2) if world > 1 else None,
        "exposed_no_attn_def": "100 * (step time - summed attention-launch time) / step time, "
                               "max over ranks (blind to hop waits inside the ring kernel)",
        "executor": (f"native (fa4cp_ring_attn_fwd), {nring.transport} transport, "
                     f"{'the ring kernel once per forward (e4m3: a main and a split pass)' if n_attn_local == args.steps else 'per-step kernels'}"
                     if nring is not None else "python step loop"),
        "roofline": {"bound": "tensor", "kernel": "fa4cp attn_fwd (tcgen05)",
                     "achieved": None if achieved is None else round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind,
                     "unit": "TFLOP/s",
                     "frac": None if achieved is None else round(achieved / peak, 4),
                     "launches_per_step": n_attn_local // max(args.steps, 1),
                     "traffic": None},
        "e2e": {"value": round(step_flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 3),
                "how": f"{e2e_steps} ring_flash_attn calls from pinned host Q/K/V to a pinned "
                       "host output, every step copying its own inputs in and output back; "
                       "inputs double-buffered on the device so step i+1's host->device copy "
                       "and step i's device->host copy overlap step i's forward; L2 flushed "
                       "before each forward; device time from the first copy to the last",
                "serial": {"value": round(step_flops / (e2e_serial_ms * 1e-3) / 1e12, 2),
                           "ms_per_step": round(e2e_serial_ms, 3),
                           "how": "copy in, forward, copy out, one step at a time"}},
        "parity": parity,
        "gpu_launches": gpu_launches,
        "host_issue_ms_per_step": round(host_s * 1e3 / args.steps, 3),
        "clocks": clocks,
        "device_status": int(status_max),
    }
    if world == 1:
        flops_cpu, secs_cpu, threads = cpu_sample()
        line["cpu_baseline"] = {
            "value": round(flops_cpu / secs_cpu / 1e12, 5), "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": "oracle (numpy restatement of the reference's CPU ring simulation) on "
                      "rank 0 of cfg2 at cp=8: all 8 ring steps, 32 heads, T=4096 local "
                      f"tokens, repeated to about 10 s; {flops_cpu:.3e} FLOP in {secs_cpu:.1f} s",
            "vs_reference_cpu_code": _cpu_speed_pin()}
    if world == 1:
        line["hbm_kernels"] = hbm_kernels(dev)
    traffic, traffic_src = _traffic_from_profile(args.config, world)
    if traffic is not None:
        line["roofline"]["traffic"] = traffic
        line["roofline"]["traffic_source"] = traffic_src
    return line


def local_schedule_ms(lq, lk, lv, cfg, desc, lcu, nseq, max_local, fused, flush, steps, world):
    """Exposed communication defined as ring time minus the same schedule run with the
    transfers skipped.  Every rank's K/V shard is all-gathered first (untimed), so
    each step's K/V is already in this GPU's memory; then this rank's forward is timed exactly
    as the ring ran it -- the ring kernel through its public C entry point with every receive
    slot filled and no hop counter (``fa4cp_ring_attn_fused``, arrived = NULL), or the
    per-step kernels through ``ring_forward`` -- L2 flushed before each step, CUDA events.
    Returns this rank's ms per forward."""
    from fa4_ring import _lib
    from fa4_ring.attn_backend import norm_descale
    from fa4_ring.ring_attention import ring_forward
    S, rank = cfg.cp_size, cfg.cp_rank
    T, Hq, D = lq.shape
    Hkv = lk.shape[1]
    gath = []
    for t in (lk, lv):
        parts = [torch.empty_like(t.view(torch.uint8)) for _ in range(world)]
        dist.all_gather(parts, t.contiguous().view(torch.uint8))
        gath.append([x.view(t.dtype) for x in parts])
    ks, vs = gath
    scale = 1.0 / math.sqrt(D)
    lib = _lib.load()
    st = _lib.stream_of(lq)
    if fused:
        # slot i holds the K/V of rank (rank - i - 1) mod S, as the copy-engine transport leaves it
        slots_k = torch.stack([ks[(rank - i - 1) % S].view(torch.uint8) for i in range(S - 1)])
        slots_v = torch.stack([vs[(rank - i - 1) % S].view(torch.uint8) for i in range(S - 1)])
        out = torch.empty(T, Hq, D, dtype=torch.bfloat16 if lq.dtype == torch.float8_e4m3fn
                          else lq.dtype, device=lq.device)
        lse = torch.empty(T, Hq, dtype=torch.float32, device=lq.device)
        kv8 = lk.dtype == torch.float8_e4m3fn
        qd = norm_descale(desc.q, Hkv, lq.device) if (desc and desc.q is not None) else None
        kds = torch.stack([norm_descale(d, Hkv, lq.device) for d in desc.k]) if (kv8 and desc) else None
        vds = torch.stack([norm_descale(d, Hkv, lq.device) for d in desc.v]) if (kv8 and desc) else None

        def one():
            _lib.check(lib.fa4cp_ring_attn_fused(
                lq.data_ptr(), lk.data_ptr(), lv.data_ptr(), slots_k.data_ptr(), slots_v.data_ptr(),
                slots_k[0].numel(), out.data_ptr(), lse.data_ptr(), lcu.data_ptr(), nseq, max_local,
                T, Hq, Hkv, D, _lib.dtype_code(lq.dtype), scale, _lib.ptr(qd), _lib.ptr(kds),
                _lib.ptr(vds), S, rank, None, 0, st), "ring_attn_fused")
        if kv8 and lq.dtype == torch.bfloat16:
            # bf16 q x e4m3 K/V: as the executor runs it, this rank converts its K/V to their
            # exact bf16 images (timed) and every slot already holds a peer's bf16 images
            slots_k = torch.stack([ks[(rank - i - 1) % S].to(torch.bfloat16) for i in range(S - 1)])
            slots_v = torch.stack([vs[(rank - i - 1) % S].to(torch.bfloat16) for i in range(S - 1)])
            kb = torch.empty(lk.shape, dtype=torch.bfloat16, device=lq.device)
            vb = torch.empty_like(kb)

            def one():
                for x8, xb in ((lk, kb), (lv, vb)):
                    _lib.check(lib.fa4cp_dequant_e4m3(x8.data_ptr(), None, xb.data_ptr(), T, Hkv,
                                                      D, st), "dequant_e4m3")
                _lib.check(lib.fa4cp_ring_attn_fused_mixed(
                    lq.data_ptr(), kb.data_ptr(), vb.data_ptr(), slots_k.data_ptr(),
                    slots_v.data_ptr(), slots_k[0].numel() * slots_k.element_size(),
                    out.data_ptr(), lse.data_ptr(), lcu.data_ptr(), nseq, max_local, T, Hq, Hkv, D,
                    scale, _lib.ptr(kds), _lib.ptr(vds), S, rank, None, 0, st),
                    "ring_attn_fused_mixed")
    else:
        def one():
            ring_forward(lq, lambda s: (ks[(rank - s) % S], vs[(rank - s) % S]), lambda s: None,
                         cfg, cu=lcu, nseq=nseq, max_seqlen=max_local, descales=desc)
    for _ in range(2):
        one()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        one()
        e1.record()
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / steps


def zigzag_positions(n, rank, cp, local_rows):
    """Global positions, within a sequence of n tokens, of local rows of a zig-zag shard
    (rank r holds chunks r and 2*cp-1-r of h = n / (2*cp) tokens)."""
    h = n // (2 * cp)
    local_rows = np.asarray(local_rows, dtype=np.int64)
    return np.where(local_rows < h, rank * h + local_rows, (2 * cp - 1 - rank) * h + local_rows - h)


def sampled_parity(result, C, lens, rank, cp, dev, desc, world, n_rand=24):
    """Checks the timed forward's own output: sampled local rows (the first 4 and last 2 rows
    of each half of each sequence, plus seeded random rows) x all heads, out and LSE, against
    dense causal attention of those rows computed here in float64 with torch on the device
    from the same seeded inputs (e4m3 operands: dequantised, per-rank scales as the run used
    them).  Returns the max errors over ranks and whether they meet the tolerances (out 2e-2
    bf16 / 6e-2 e4m3 operands, LSE 1e-3)."""
    from fa4_ring.fp8 import quantize_e4m3
    from fa4_ring.zigzag import zigzag_shard_varlen
    out, lse = result
    Hq, Hkv, D = C["Hq"], C["Hkv"], C["D"]
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    g = torch.Generator(device=dev).manual_seed(1234)  # the inputs gpu_main made
    full = []
    for h in (Hq, Hkv, Hkv):
        x = torch.randn(N, h, D, generator=g, device=dev, dtype=torch.bfloat16)
        full.append(x.mul_(C["amp"]) if C["amp"] != 1.0 else x)

    def operand(x, quant, r_only=None):
        """x as the kernels saw it, in float64: bf16, or each rank's e4m3 shard x its scale."""
        if not quant:
            return x.double()
        y = torch.empty(x.shape, dtype=torch.float64, device=dev)
        for r in range(cp) if r_only is None else [r_only]:
            rows = torch.from_numpy(np.concatenate(
                [a + zigzag_positions(b - a, r, cp, np.arange((b - a) // cp))
                 for a, b in zip(full_cu[:-1], full_cu[1:])])).to(dev)
            x8, sc = quantize_e4m3(zigzag_shard_varlen(x, full_cu, r, cp)[0])
            y[rows] = x8.double() * sc.double()
        return y

    kv8 = C["kind"] in ("e4m3", "mixed")
    qf = operand(full[0], C["kind"] == "e4m3", r_only=rank)
    kf, vf = operand(full[1], kv8), operand(full[2], kv8)
    del full
    rng = np.random.default_rng(rank)
    scale = 1.0 / math.sqrt(D)
    err_o = err_l = 0.0
    n_rows = 0
    lstart = 0
    n_rand_seq = max(1, n_rand // len(lens))
    for j, n in enumerate(lens):
        h = n // (2 * cp)
        loc = sorted(set(list(range(min(4, h))) + list(range(max(0, h - 2), h))
                         + list(range(h, h + min(4, h))) + list(range(2 * h - 2, 2 * h))
                         + rng.integers(0, 2 * h, size=n_rand_seq).tolist()))
        pos = torch.from_numpy(zigzag_positions(n, rank, cp, loc)).to(dev)
        lrows = torch.tensor(loc, device=dev) + lstart
        a = full_cu[j]
        R, grp = len(loc), Hq // Hkv
        q = qf[pos + a].view(R, Hkv, grp, D)                      # head = kv head * grp + i
        s = torch.einsum("rkgd,nkd->kgrn", q, kf[a:a + n]) * scale
        s.masked_fill_(torch.arange(n, device=dev) > pos[:, None], -math.inf)
        want_l = torch.logsumexp(s, dim=-1)                      # [Hkv, grp, R]
        s.sub_(want_l[..., None]).exp_()
        want_o = torch.einsum("kgrn,nkd->rkgd", s, vf[a:a + n]).reshape(R, Hq, D)
        err_o = max(err_o, float((out[lrows].double() - want_o).abs().max()))
        err_l = max(err_l, float((lse[lrows].double() - want_l.reshape(Hq, R).t()).abs().max()))
        n_rows += R
        lstart += 2 * h
        del s
    vals = torch.tensor([err_o, err_l], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    err_o, err_l = vals.tolist()
    tol_o = 2e-2 if C["kind"] == "bf16" else 6e-2
    return {"max_abs_out": round(err_o, 6), "max_abs_lse": round(err_l, 6),
            "rows_per_rank": n_rows, "heads": Hq, "tol_out": tol_o, "tol_lse": 1e-3,
            "pass": bool(err_o <= tol_o and err_l <= 1e-3),
            "how": "the last timed forward's output on sampled rows (first/last rows of every "
                   "half of every sequence + seeded random rows) x all heads, against float64 "
                   "dense causal attention of the same seeded inputs computed with torch on the "
                   "device; max over ranks"}


def bwd_main(args, rank, world, local_rank):
    """The ring backward, timed like the forward (L2 flushed, CUDA events, max over ranks)."""
    from fa4_ring import RingConfig, _lib
    from fa4_ring.ring_attention import ring_flash_attn_with_lse
    from fa4_ring.ring_backward import ring_flash_attn_backward
    from fa4_ring.zigzag import zigzag_shard_varlen

    dev = torch.device("cuda", local_rank)
    C = CONFIGS[args.config]
    if C["kind"] != "bf16":
        raise SystemExit("--bwd runs the bf16 configurations (cfg2, cfg4)")
    Hq, Hkv, D = C["Hq"], C["Hkv"], C["D"]
    cp = world
    lens = config_lens(args.config, cp, args.seq_len)
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    g = torch.Generator(device=dev).manual_seed(1234)
    shards, lcu = [], None
    for h in (Hq, Hkv, Hkv, Hq):  # q, k, v, dout
        full = torch.randn(N, h, D, generator=g, device=dev, dtype=torch.bfloat16)
        loc, lcu = zigzag_shard_varlen(full, full_cu, rank, cp)
        shards.append(loc)
        del full
    lq, lk, lv, ldo = shards
    varlen = len(lens) > 1
    kw = dict(cu_seqlens=lcu if varlen else None, max_seqlen=max(lens) // cp if varlen else None)
    cfg = RingConfig(cp_size=cp, cp_rank=rank)
    out, lse = ring_flash_attn_with_lse(lq, lk, lv, cfg, **kw)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    step_flops = 2.5 * float(sum(causal_flops(n, Hq, D) for n in lens))

    def run():
        return ring_flash_attn_backward(ldo, lq, lk, lv, out, lse, cfg, **kw)

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    n0 = _lib.launch_count
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record()
            run()
            ev[i][1].record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    launches = _lib.launch_count - n0
    ms = torch.tensor([sum(a.elapsed_time(b) for a, b in ev) / args.steps], dtype=torch.float64,
                      device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    status = _lib.device_status()
    if rank != 0:
        return None
    ms_step = ms.item()
    value = step_flops / (ms_step * 1e-3) / 1e12
    peaks, peaks_kind = load_peaks()
    peak = peaks["bf16_tflops"]
    return {
        "metric": "causal ring-attn backward TFLOP/s (dq, dk, dv; 2.5x forward FLOPs)",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded randn q, k, v, dout)",
        "config": {"workload": f"{args.config} backward: {C['text']}", "cp": cp,
                   "tokens": N,
                   "l2": "flushed (256 MiB write) before every timed step"},
        "roofline": {"bound": "tensor", "achieved": round(value / world, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(value / world / peak, 4),
                     "traffic": None, "note": f"whole backward step per GPU (all kernels), "
                     f"of {peaks_kind} bf16 burst peak"},
        "gpu_launches": launches, "clocks": clk.summary(), "device_status": int(status),
        **({"cpu_baseline": _bwd_cpu_baseline()} if world == 1 else {}),
    }


def _cpu_speed_pin():
    """The port's speed against the reference's own CPU ring code on one sample, measured
    where the reference checkout exists (``oracle/cpu_speed_pin.py`` writes
    ``oracle/cpu_speed_pin.json``); None when absent."""
    try:
        with open(os.path.join(ROOT, "oracle", "cpu_speed_pin.json")) as f:
            pin = json.load(f)
    except (OSError, ValueError):
        return None
    return {"port_over_reference": pin.get("port_over_reference"),
            "reference_gflops": pin.get("reference_gflops"), "port_gflops": pin.get("port_gflops"),
            "threads": pin.get("threads"), "sample": pin.get("sample"),
            "how": "oracle/cpu_speed_pin.py: the reference's cpu_attn / merge driven as its "
                   "simulate_ring, and this port, on the same sample in the build container "
                   "(the reference checkout is not on the GPU box); > 1 means the port is the "
                   "faster, so the reported CPU baseline does not understate the reference"}


def _bwd_cpu_baseline():
    flops, secs, threads = cpu_sample_bwd()
    return {"value": round(flops / secs / 1e12, 5), "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": "backward oracle (gradient of the reference's CPU ring algorithm, fp32) "
                      "on rank 0 of cfg2 at cp=8: its first ring step (local causal), all 32 "
                      "query heads, "
                      f"T=4096 local tokens; {flops:.3e} FLOP in {secs:.1f} s"}


def _traffic_from_profile(config, world):
    """(DRAM bytes per attention launch, provenance) recorded from an ncu capture of this
    workload (profiles/attn_fwd_traffic.json: ncu cannot run inside the timed bench), or
    (None, None) when none was captured.  The provenance names the commit of the capture, so
    a figure older than the kernel shows as such."""
    path = os.path.join(ROOT, "profiles", "attn_fwd_traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
    except (OSError, ValueError):
        return None, None
    v = t.get(f"{config}_cp{world}")
    if v is None:
        return None, None
    return v, (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
               f"workload, captured at commit {t.get('captured_at_commit', '?')} "
               f"(profiles/attn_fwd_traffic.json)")


# --------------------------------------------------------------------------- HBM-bound kernels
def hbm_kernels(dev, iters=10):
    """HBM roofline of the merge and zig-zag kernels on cfg2-sized tensors (T=32768 rows,
    Hq=32, D=128, bf16), each timed alone with CUDA events (inputs larger than L2, flushed
    before every launch).  Algorithmic bytes: incremental merge 2*(T*H*D*2 + T*H*4) read +
    (T*H*D*2 + T*H*4) written; k-way merge k*(T*H*D*2 + T*H*4) read + T*H*D*2 + T*H*4
    written; zig-zag shard / unshard 2 * bytes moved."""
    from fa4_ring import _lib
    from fa4_ring.merge import merge_state_in_place, merge_states
    from fa4_ring.zigzag import zigzag_shard, zigzag_unshard
    peaks, kind = load_peaks()
    hbm = peaks["hbm_gbs"]
    T, H, D, K = 32768, 32, 128, 8
    g = torch.Generator(device=dev).manual_seed(5)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    vs = [torch.randn(T, H, D, device=dev, generator=g).bfloat16() for _ in range(K)]
    ss = [torch.randn(T, H, device=dev, generator=g) * 3 for _ in range(K)]
    acc_v, acc_s = vs[0].clone(), ss[0].clone()
    out_v = torch.empty_like(vs[0])
    out_s = torch.empty_like(ss[0])
    x = torch.randn(4 * T, H, D, device=dev, generator=g).bfloat16()  # a 131072-token sequence
    shards = [zigzag_shard(x, r, 2) for r in range(2)]

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        return tot / iters

    row = T * H * D * 2 + T * H * 4
    cases = {
        "merge_state_inplace": (lambda: merge_state_in_place(acc_v, acc_s, vs[1], ss[1]), 3 * row),
        f"merge_states_k{K}": (lambda: merge_states(vs, ss, out=out_v, lse_out=out_s), (K + 1) * row),
        "zigzag_shard_cp2": (lambda: zigzag_shard(x, 0, 2), 2 * x.numel() * 2 // 2),
        "zigzag_unshard_cp2": (lambda: zigzag_unshard(shards, 2), 2 * x.numel() * 2),
    }
    res = {}
    for name, (fn, nbytes) in cases.items():
        ms = timed(fn)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"ms": round(ms, 4), "bytes": int(nbytes), "achieved": round(gbs, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4)}
    status = _lib.device_status()
    return {"kernels": res, "peak_kind": f"{kind} hbm_gbs (copy)", "device_status": status,
            "shape": f"T={T}, Hq={H}, D={D}, bf16 out, fp32 LSE; zig-zag over 131072 rows"}


# --------------------------------------------------------------------------- library comparison
def library_compare(dev, lens=(32768, 8192), iters=10):
    """This repo's attention kernel beside a library tcgen05 kernel on the same inputs:
    flashinfer's CUTLASS SM100 FMHA (``flashinfer.prefill.fmha_varlen``; the reference's GPU
    kernel, FA4's ``flash_attn.cute``, is not installed in this image).  Causal bf16, Hq=32,
    Hkv=8, D=128 (cfg2's heads), one sequence of each length; best of ``iters`` with the L2
    flushed before each launch, CUDA events.  flashinfer builds the module on first use
    (minutes; FLASHINFER_WORKSPACE_BASE selects its cache).  Comparison only: nothing here is
    on the product path."""
    try:
        from flashinfer.prefill import fmha_varlen
    except Exception as e:  # the library is missing or cannot load: say so
        return {"unavailable": f"flashinfer fmha_varlen: {type(e).__name__}: {e}"}
    from fa4_ring.attn_backend import b200_attn
    Hq, Hkv, D = 32, 8, 128
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    res = {}
    for N in lens:
        g = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn(N, Hq, D, device=dev, generator=g, dtype=torch.bfloat16)
        k = torch.randn(N, Hkv, D, device=dev, generator=g, dtype=torch.bfloat16)
        v = torch.randn(N, Hkv, D, device=dev, generator=g, dtype=torch.bfloat16)
        cu = torch.tensor([0, N], dtype=torch.int32, device=dev)
        sc = 1.0 / math.sqrt(D)
        fns = {"flashinfer_cutlass_sm100_fmha": lambda: fmha_varlen(q, k, v, cu, cu, causal=True,
                                                                    sm_scale=sc, max_qo_len=N),
               "fa4cp_attn_fwd_2q_kernel": lambda: b200_attn(q, k, v, causal=True,
                                                             softmax_scale=sc)[0]}
        outs, row = {}, {}
        for name, fn in fns.items():
            for _ in range(3):
                o = fn()
            torch.cuda.synchronize()
            best = float("inf")
            for _ in range(iters):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                o = fn()
                e1.record()
                torch.cuda.synchronize()
                best = min(best, e0.elapsed_time(e1))
            outs[name] = o[0] if isinstance(o, tuple) else o
            row[name] = {"ms": round(best, 4),
                         "tflops": round(causal_flops(N, Hq, D) / (best * 1e-3) / 1e12, 1)}
        a, b = outs.values()
        row["max_abs_diff"] = float((a.float() - b.float()).abs().max())
        res[f"N={N}"] = row
    return res


# --------------------------------------------------------------------------- reference arm
def reference_main(args):
    """The reference's CPU ring simulation (restated in numpy, ``oracle/``) on the host
    cores: each step is a bounded sample -- one ring step of rank 0 of cfg2 at cp=8."""
    threads = os.cpu_count() or 1
    for i in range(args.warmup):
        cpu_sample(rank_steps=[i], threads=threads)
    flops = secs = 0.0
    for i in range(args.steps):
        f, s, _ = cpu_sample(rank_steps=[i], threads=threads)
        flops += f
        secs += s
    value = flops / secs / 1e12
    return {
        "metric": METRIC, "impl": "reference", "value": round(value, 5), "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg2 (N=32768, Hq=32, Hkv=8, D=128) ring at cp=8, rank 0; one "
                               "ring step per bench step", "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port",
                         "sample": "one ring step (T=4096 local tokens, 32 heads) of rank 0 of "
                                   "cfg2 at cp=8 per bench step, cycling through the 8 steps",
                         "vs_reference_cpu_code": _cpu_speed_pin()},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--merge", choices=["incremental", "batched"], default="incremental")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="cfg2",
                    help="BASELINE workload (cfg2 is the headline metric's configuration)")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="override the single-sequence length (smaller only for profiling)")
    ap.add_argument("--nccl-cta-policy", choices=["default", "zero"], default="default",
                    help="NCCL CTA policy of the ring's process group (zero: no SM CTAs)")
    ap.add_argument("--transport", choices=["copy_engine", "copy_engine_chain", "nccl"],
                    default="copy_engine",
                    help="K/V transport of the native ring executor (N > 1): direct pushes to "
                         "every peer (copy_engine), the chained rotation on the copy engines, "
                         "or NCCL send/recv")
    ap.add_argument("--ring-kernel", choices=["fused", "fused-16bit", "fused-all", "steps"],
                    default="fused",
                    help="copy-engine ring: one ring-kernel launch per forward (fused; "
                         "fused-16bit: not for e4m3; fused-all: also head_dim 256, cfg5) or one "
                         "attention launch per step")
    ap.add_argument("--sm-reserve", type=int, default=None,
                    help="SMs the persistent attention grid leaves to NCCL during a ring call "
                         "(native executor; default: the library's)")
    ap.add_argument("--timeline", action="store_true",
                    help="with --quick: print each rank's launch/hop timeline of the last "
                         "forward to stderr")
    ap.add_argument("--library-compare", action="store_true",
                    help="only time flashinfer's CUTLASS SM100 FMHA beside this repo's attention "
                         "kernel on the same causal bf16 inputs (comparison, not a bench line)")
    ap.add_argument("--aux", action="store_true",
                    help="only the HBM-bound kernels (merges, zig-zag) against the HBM peak")
    ap.add_argument("--bwd", action="store_true",
                    help="time the ring backward (bf16 cfg2 / cfg4) instead of the forward")
    ap.add_argument("--quick", action="store_true",
                    help="profiling run: timed loop only (no e2e, no CPU baseline)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(reference_main(args)), flush=True)
        return 0

    torch.cuda.set_device(local_rank)
    if args.library_compare:
        if rank == 0:
            print(json.dumps({"library_compare": library_compare(torch.device("cuda", local_rank))}),
                  flush=True)
        return 0
    if args.aux:
        if rank == 0:
            print(json.dumps({"aux": True, "hbm_kernels": hbm_kernels(torch.device("cuda", local_rank))}),
                  flush=True)
        return 0
    if world > 1:
        from fa4_ring.comm import nccl_pg_options
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank),
                                pg_options=nccl_pg_options(args.nccl_cta_policy))
    from fa4_ring import ring_attention
    ring_attention.RING_TRANSPORT = args.transport
    ring_attention.RING_FUSED = {"fused": True, "fused-16bit": "16bit", "fused-all": "all",
                                 "steps": False}[args.ring_kernel]
    try:
        line = (bwd_main if args.bwd else gpu_main)(args, rank, world, local_rank)
    finally:
        if world > 1:
            from fa4_ring.comm import close_native_rings
            close_native_rings()
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
