"""Zig-zag causal ring attention on B200 (mirrors ``fa4_ring/ring_attention.py:43-174``).

Each rank holds ``2h`` local tokens ``[early half | late half]`` per sequence (see
:mod:`.zigzag`) and runs ``cp_size`` steps; step ``s`` attends the K/V that
originated on rank ``src = (rank - s) mod cp_size``:

* step 0 (``src == rank``): causal attention over the local tokens;
* ``s <= rank`` (``src`` is earlier): all local Q x the early half of the source KV;
* ``s > rank``  (``src`` is later):  the late half of local Q x all of the source KV.

Per step, one launch of the sm_100a attention kernel does the step's attention on
the rows the pattern selects, in place (no ``index_select`` / ``index_copy_``
staging), and in ``incremental`` mode merges the partial into the running
``(out, lse)`` in its epilogue.  ``batched`` mode keeps every partial and runs one
k-way merge kernel at the end.  The K/V rotation overlaps each step's attention with
the next hop's transfer.  Over an NCCL group, ``incremental`` mode runs as one call of
the library's native ring executor (:class:`.comm.NativeRing`: NCCL hops and attention
steps issued from C++); ``batched`` mode, and any other group, runs the Python step
loop over :class:`.comm.KVRing`, which follows the same schedule.
"""

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .attn_backend import (PATTERN_BACK_Q, PATTERN_FRONT_KV, PATTERN_VARLEN, _check_qkv,
                           attn_into, is_mixed, norm_descale, out_dtype_for)
from .comm import KVRing, native_ring
from .config import RingConfig
from .merge import merge_states


@dataclass
class Descales:
    """FP8 descales (fa4_ring/ring_attention.py:43-52).  ``k``/``v`` are indexed by the
    SOURCE rank whose KV is being attended (all-gather them once before the call).
    Each entry is a float32 tensor: a scalar, ``[H_kv]`` or ``(1, H_kv)``."""

    q: Optional[torch.Tensor] = None
    k: Optional[List[torch.Tensor]] = None
    v: Optional[List[torch.Tensor]] = None


def ring_schedule(rank: int, cp_size: int) -> List[Tuple[int, int, int]]:
    """``(step, src, pattern)`` for every step of ``rank``."""
    sched = [(0, rank, PATTERN_VARLEN)]
    for s in range(1, cp_size):
        src = (rank - s) % cp_size
        sched.append((s, src, PATTERN_BACK_Q if s > rank else PATTERN_FRONT_KV))
    return sched


_CU_CACHE: Dict[Tuple[int, int], torch.Tensor] = {}


def _single_cu(total: int, device: torch.device) -> torch.Tensor:
    key = (device.index if device.index is not None else -1, total)
    cu = _CU_CACHE.get(key)
    if cu is None:
        cu = torch.tensor([0, total], dtype=torch.int32, device=device)
        _CU_CACHE[key] = cu
    return cu


def _validate_cu(cu) -> None:
    vals = [int(c) for c in (cu.tolist() if torch.is_tensor(cu) else cu)]
    assert vals and vals[0] == 0, "cu_seqlens must start at 0"
    for a, b in zip(vals[:-1], vals[1:]):
        assert b >= a, "cu_seqlens must be non-decreasing"
        assert (b - a) % 2 == 0, "each local sequence length must be even (zig-zag)"


def ring_flash_attn(
    local_q: torch.Tensor,   # [T, H, D]   zig-zag local shard
    local_k: torch.Tensor,   # [T, H_kv, D]
    local_v: torch.Tensor,   # [T, H_kv, D]
    cfg: RingConfig,
    *,
    group: Optional["dist.ProcessGroup"] = None,
    descales: Optional[Descales] = None,
    cu_seqlens: Optional[torch.Tensor] = None,  # local int32 [num_seq+1]; None -> one sequence
    max_seqlen: Optional[int] = None,
) -> torch.Tensor:
    """Causal ring attention; returns this rank's local output ``[T, H, D]``.

    One sequence per rank: leave ``cu_seqlens=None``.  Packed sequences: pass the
    LOCAL ``cu_seqlens`` (each entry already the zig-zag ``2*h_j`` shard length) and
    ``max_seqlen`` (max local shard length).  ``cu_seqlens`` given on the host is
    validated (even lengths); a CUDA ``cu_seqlens`` is trusted, to avoid a sync.
    Output dtype: the input dtype, or bf16 for e4m3 inputs.

    Differentiable (not in the reference, which is forward-only): when grad mode is on and
    any of q, k, v requires grad (f16 / bf16, head_dim 64 or 128), the call records the
    ring backward of :mod:`.ring_backward` for autograd.
    """
    if torch.is_grad_enabled() and any(t.requires_grad for t in (local_q, local_k, local_v)):
        return _RingFlashAttnFn.apply(local_q, local_k, local_v, cfg, group, descales,
                                      cu_seqlens, max_seqlen)
    return ring_flash_attn_with_lse(local_q, local_k, local_v, cfg, group=group,
                                    descales=descales, cu_seqlens=cu_seqlens,
                                    max_seqlen=max_seqlen)[0]


def ring_flash_attn_with_lse(local_q, local_k, local_v, cfg: RingConfig, *, group=None,
                             descales: Optional[Descales] = None, cu_seqlens=None,
                             max_seqlen=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """:func:`ring_flash_attn` returning ``(out [T, H, D], lse [T, H])``: the final
    natural-log LSE of every local row (what :func:`.ring_backward.ring_flash_attn_backward`
    takes).  No autograd."""
    _check_qkv(local_q, local_k, local_v)
    S, rank = cfg.cp_size, cfg.cp_rank
    T, Hq, D = local_q.shape
    assert local_k.shape[0] == T, "q and kv shards must have the same token count"
    dev = local_q.device
    cu, nseq, max_seqlen = local_cu_args(T, dev, cu_seqlens, max_seqlen)

    k0 = local_k.contiguous()
    v0 = local_v.contiguous()
    if S > 1 and cfg.merge_mode == "incremental" and use_native_executor(group):
        return _native_forward(local_q.contiguous(), k0, v0, cfg, group, cu=cu, nseq=nseq,
                               max_seqlen=max_seqlen, descales=descales)
    ring = KVRing(k0, v0, rank, S, group) if S > 1 else None
    if ring is not None:
        ring.start()  # hop 1 overlaps the local step

    def kv_at(step):
        return ring.get(step) if (ring is not None and step > 0) else (k0, v0)

    def step_done(step):
        if ring is not None:
            ring.done(step)

    return ring_forward(local_q, kv_at, step_done, cfg, cu=cu, nseq=nseq, max_seqlen=max_seqlen,
                        descales=descales, return_lse=True)


def local_cu_args(T: int, dev, cu_seqlens, max_seqlen) -> Tuple[torch.Tensor, int, int]:
    """``(cu int32 on dev, nseq, max_seqlen)`` of a local shard (one sequence when
    ``cu_seqlens`` is None)."""
    if cu_seqlens is None:
        assert T % 2 == 0, "the local shard length must be even (zig-zag)"
        return _single_cu(T, dev), 1, T
    assert max_seqlen is not None, "max_seqlen required when cu_seqlens is given"
    if not cu_seqlens.is_cuda:
        _validate_cu(cu_seqlens)
    cu = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
    return cu, cu.numel() - 1, int(max_seqlen)


class _RingFlashAttnFn(torch.autograd.Function):
    """Autograd node of :func:`ring_flash_attn`: the forward keeps (q, k, v, out, lse); the
    backward runs the ring backward over the same group."""

    @staticmethod
    def forward(ctx, q, k, v, cfg, group, descales, cu_seqlens, max_seqlen):
        out, lse = ring_flash_attn_with_lse(q, k, v, cfg, group=group, descales=descales,
                                            cu_seqlens=cu_seqlens, max_seqlen=max_seqlen)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.cfg, ctx.group, ctx.cu, ctx.max_seqlen = cfg, group, cu_seqlens, max_seqlen
        return out

    @staticmethod
    def backward(ctx, dout):
        from .ring_backward import ring_flash_attn_backward
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = ring_flash_attn_backward(dout, q, k, v, out, lse, ctx.cfg, group=ctx.group,
                                              cu_seqlens=ctx.cu, max_seqlen=ctx.max_seqlen)
        return dq, dk, dv, None, None, None, None, None


# Run incremental-mode rings over an NCCL group through the native executor
# (fa4cp_ring_attn_fwd); False keeps the Python step loop over KVRing.
NATIVE_EXECUTOR = True
# K/V transport of the native executor: "copy_engine" (each rank pushes its K/V straight into
# every peer's receive slot over NVSwitch, per-slot arrival flags, no SM used),
# "copy_engine_chain" (the chain-forward rotation on the copy engines, hop counters) or "nccl"
# (send/recv on the executor's own communicator)
RING_TRANSPORT = "copy_engine"
# copy engine: run the whole forward as one launch of the ring kernel -- True: for f16 / bf16
# with D 64 or 128 and e4m3 with D 128; "all": also at head_dim 256 (f16 / bf16, and bf16 q
# with e4m3 K/V -- measured 2-5% slower than the per-step kernels at cfg5's sizes, so not the
# default); "16bit": f16 / bf16 (D 64, 128) only; False: one attention launch per step
RING_FUSED = True


def use_native_executor(group=None) -> bool:
    return (NATIVE_EXECUTOR and dist.is_available() and dist.is_initialized()
            and dist.get_backend(group) == "nccl")


def _native_forward(q, k, v, cfg: RingConfig, group, *, cu, nseq, max_seqlen,
                    descales: Optional[Descales]) -> torch.Tensor:
    """The whole ring forward in one native call (NCCL hops + attention steps in C++)."""
    S, rank = cfg.cp_size, cfg.cp_rank
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    dev = q.device
    assert dist.get_rank(group) == rank, "cp_rank must be this process's rank in the cp group"
    assert dist.get_world_size(group) == S, "cp_size must be the size of the cp group"
    scale = cfg.softmax_scale if cfg.softmax_scale is not None else 1.0 / math.sqrt(D)
    fp8 = q.dtype == torch.float8_e4m3fn
    kv8 = k.dtype == torch.float8_e4m3fn
    qd = norm_descale(descales.q, Hkv, dev) if (fp8 and descales and descales.q is not None) else None
    kds = vds = None
    if kv8 and descales and descales.k:
        assert len(descales.k) == S, "one k descale per source rank"
        kds = torch.stack([norm_descale(d, Hkv, dev) for d in descales.k])
    if kv8 and descales and descales.v:
        assert len(descales.v) == S, "one v descale per source rank"
        vds = torch.stack([norm_descale(d, Hkv, dev) for d in descales.v])
    out = torch.empty((T, Hq, D), dtype=out_dtype_for(q.dtype), device=dev)
    lse = torch.empty((T, Hq), dtype=torch.float32, device=dev)
    kv_bytes = k.numel() * k.element_size()
    ring = native_ring(rank, S, dev, group, RING_TRANSPORT)
    # bf16 q x e4m3 K/V at head_dim 256: the ring kernel takes the K/V as exact bf16 images,
    # which the executor converts once and pushes (twice the e4m3 bytes per slot)
    mixed_fused = is_mixed(q, k) and D == 256 and ring.copy_engine and RING_FUSED == "all"
    bufs = None
    if ring.transport == "nccl":
        bufs = torch.empty(4 * kv_bytes, dtype=torch.uint8, device=dev)  # two [K | V] slots
    else:
        ring.ensure_capacity(2 * kv_bytes if mixed_fused else kv_bytes)
        ring.set_fused({"16bit": 1, "all": 3}.get(RING_FUSED, 2 if RING_FUSED else 0))
    ws = None
    if is_mixed(q, k):
        nbytes = _lib.load().fa4cp_attn_kv8_workspace_bytes(T, Hkv, D)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    ring.forward(
        q, k, v, out, lse, cu, nseq=nseq, max_seqlen=max_seqlen, softmax_scale=scale,
        q_descale=qd, k_descales=kds, v_descales=vds, kv_bufs=bufs, workspace=ws)
    fused = (ring.copy_engine and bool(RING_FUSED) and q.dtype == k.dtype
             and ((q.dtype in (torch.float16, torch.bfloat16)
                   and (D in (64, 128) or (D == 256 and RING_FUSED == "all")))
                  or (RING_FUSED in (True, "all") and q.dtype == torch.float8_e4m3fn
                      and D == 128)))
    # the ring kernel: e4m3 runs a main pass and a split pass (rows that see few keys); with
    # direct pushes and S >= 8 f16 / bf16 (D 64, 128) run step 0 in a launch of its own before
    # the remote walk; bf16 x e4m3 K/V converts K and V (two launches) before its one launch
    two_pass = q.dtype == torch.float8_e4m3fn or (ring.transport == "copy_engine" and S >= 8
                                                  and D != 256)
    if mixed_fused:
        _lib.count_launches(3)
    else:
        _lib.count_launches((2 if two_pass else 1) if fused else S * (3 if ws is not None else 1))
    return out, lse


def ring_forward(local_q, kv_at, step_done, cfg: RingConfig, *, cu: torch.Tensor, nseq: int,
                 max_seqlen: int, descales: Optional[Descales] = None, return_lse: bool = False):
    """The per-step compute of :func:`ring_flash_attn` for one rank.

    ``kv_at(step)`` returns the (K, V) that originated on ``(rank - step) mod S`` (the
    ring supplies it after its hop; a single-GPU test supplies every rank's shard
    directly); ``step_done(step)`` is called after the step's kernels are enqueued.
    Returns ``out``, or ``(out, lse)`` with ``return_lse``.
    """
    S, rank = cfg.cp_size, cfg.cp_rank
    T, Hq, D = local_q.shape
    dev = local_q.device
    scale = cfg.softmax_scale if cfg.softmax_scale is not None else 1.0 / math.sqrt(D)
    q = local_q.contiguous()
    k0, _ = kv_at(0)
    Hkv = k0.shape[1]
    fp8 = q.dtype == torch.float8_e4m3fn
    kv8 = k0.dtype == torch.float8_e4m3fn  # e4m3 K/V, with an e4m3 or a bf16 query
    qd = norm_descale(descales.q, Hkv, dev) if (fp8 and descales and descales.q is not None) else None

    def kd(src):
        if kv8 and descales and descales.k:
            return norm_descale(descales.k[src], Hkv, dev)
        return None

    def vd(src):
        if kv8 and descales and descales.v:
            return norm_descale(descales.v[src], Hkv, dev)
        return None

    out_dt = out_dtype_for(q.dtype)
    batched = cfg.merge_mode == "batched"
    out = torch.empty((T, Hq, D), dtype=out_dt, device=dev)
    lse = torch.empty((T, Hq), dtype=torch.float32, device=dev)
    partials = [(out, lse)]
    stream = _lib.stream_of(q)
    lib = _lib.load()

    for step, src, pattern in ring_schedule(rank, S):
        k, v = kv_at(step)
        q_rows = (max_seqlen + 1) // 2 if pattern == PATTERN_BACK_Q else max_seqlen
        if step == 0 or not batched:
            o_t, l_t, acc = out, lse, step > 0
        else:
            o_t = torch.empty((T, Hq, D), dtype=out_dt, device=dev)
            l_t = torch.empty((T, Hq), dtype=torch.float32, device=dev)
            if pattern == PATTERN_BACK_Q:  # rows this step does not cover: identity
                _lib.check(lib.fa4cp_fill_f32(l_t.data_ptr(), l_t.numel(), float("-inf"), stream),
                           "fill_f32")
                _lib.count_launches()
            partials.append((o_t, l_t))
            acc = False
        attn_into(q, k, v, o_t, l_t, cu, cu, nseq=nseq, max_seqlen_q=q_rows, pattern=pattern,
                  causal=(step == 0), softmax_scale=scale, q_descale=qd, k_descale=kd(src),
                  v_descale=vd(src), accumulate=acc)
        step_done(step)

    if batched and len(partials) > 1:
        final = torch.empty((T, Hq, D), dtype=out_dt, device=dev)
        final_lse = torch.empty((T, Hq), dtype=torch.float32, device=dev)
        merge_states([p[0] for p in partials], [p[1] for p in partials], out=final,
                     lse_out=final_lse)
        return (final, final_lse) if return_lse else final
    return (out, lse) if return_lse else out
