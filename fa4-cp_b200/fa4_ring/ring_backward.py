"""Backward of the zig-zag causal ring attention.

Not in the reference, which is forward-only (README.md:142: "forward-only (inference). No
backward").  This is the gradient of its forward (``fa4_ring/ring_attention.py:61-174``):
the ring backward runs the forward's schedule again -- step ``s`` of rank ``r`` attends the
K/V of source ``(r - s) mod S`` with the step's row pattern (local causal; all Q x the
source's front half; the late half of Q x all of the source) -- and, because every forward
partial was taken against the FINAL log-sum-exp, each step's gradient is the chunk gradient
with that final LSE and the steps' gradients add up:

* dQ of the local rows accumulates in fp32 over all steps (``fa4cp_attn_bwd`` adds);
* the K/V rotate as in the forward (:class:`.comm.KVRing`, ``S - 1`` hops);
* dK/dV of each source's K/V accumulate in fp32 while they travel with the ring
  (:class:`.comm.GradRing`, ``S`` passes): every rank adds its contribution and passes the
  sum on, and the last pass delivers it to the owner;
* one rounding to the input dtype at the end.

Kernels: ``fa4cp_attn_bwd_preprocess`` (Delta = rowsum(dO * O)), ``fa4cp_attn_bwd`` per step,
``fa4cp_add_f32`` per pass, ``fa4cp_convert_f32`` for the results.  There is no CPU path.
"""

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .attn_backend import PATTERN_FRONT_KV, PATTERN_VARLEN
from .comm import GradRing, KVRing
from .config import RingConfig
from .ring_attention import local_cu_args, ring_schedule

BWD_HEAD_DIMS = (64, 128)
BWD_DTYPES = (torch.float16, torch.bfloat16)


def _check_bwd(dout, q, k, v, out, lse):
    _lib.require_cuda(dout, q, k, v, out, lse)
    if q.dtype not in BWD_DTYPES:
        raise NotImplementedError(f"the backward takes f16 / bf16 inputs, got {q.dtype}")
    assert k.dtype == v.dtype == q.dtype == out.dtype == dout.dtype, (
        "q, k, v, out and dout must share a dtype")
    assert q.dim() == 3 and k.shape == v.shape and k.shape[0] == q.shape[0]
    assert out.shape == q.shape and dout.shape == q.shape, "out / dout must be [T, H, D]"
    assert lse.shape == q.shape[:2] and lse.dtype == torch.float32, "lse must be fp32 [T, H]"
    H, Hkv, D = q.shape[1], k.shape[1], q.shape[2]
    assert H % Hkv == 0, f"H_q={H} not a multiple of H_kv={Hkv}"
    if D not in BWD_HEAD_DIMS:
        raise NotImplementedError(f"head_dim {D} is not supported by the backward")


def bwd_delta(out: torch.Tensor, dout: torch.Tensor) -> torch.Tensor:
    """Delta[T, H] = sum_d dout * out (fp32)."""
    T, H, D = out.shape
    delta = torch.empty((T, H), dtype=torch.float32, device=out.device)
    _lib.check(_lib.load().fa4cp_attn_bwd_preprocess(
        out.data_ptr(), dout.data_ptr(), delta.data_ptr(), T, H, D, _lib.dtype_code(out.dtype),
        _lib.stream_of(out)), "attn_bwd_preprocess")
    _lib.count_launches()
    return delta


def bwd_step(q, k, v, dout, lse, delta, dq_acc, dk_acc, dv_acc, cu, *, nseq: int,
             max_seqlen_k: int, pattern: int, causal: bool, softmax_scale: float) -> None:
    """Add one step's gradient contributions into the fp32 accumulators
    (``fa4cp_attn_bwd``, current stream)."""
    rc = _lib.load().fa4cp_attn_bwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), dout.data_ptr(), lse.data_ptr(),
        delta.data_ptr(), dq_acc.data_ptr(), dk_acc.data_ptr(), dv_acc.data_ptr(),
        cu.data_ptr(), cu.data_ptr(), nseq, max_seqlen_k, q.shape[0], k.shape[0], q.shape[1],
        k.shape[1], q.shape[2], _lib.dtype_code(q.dtype), pattern, 1 if causal else 0,
        float(softmax_scale), _lib.stream_of(q))
    _lib.check(rc, "attn_bwd")
    _lib.count_launches()


def acc_add(dst: torch.Tensor, src: torch.Tensor) -> None:
    """dst += src (fp32, ``fa4cp_add_f32``)."""
    _lib.check(_lib.load().fa4cp_add_f32(dst.data_ptr(), src.data_ptr(), dst.numel(),
                                         _lib.stream_of(dst)), "add_f32")
    _lib.count_launches()


def acc_to(acc: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The fp32 accumulator rounded to ``dtype`` (``fa4cp_convert_f32``)."""
    out = torch.empty(acc.shape, dtype=dtype, device=acc.device)
    _lib.check(_lib.load().fa4cp_convert_f32(acc.data_ptr(), out.data_ptr(), acc.numel(),
                                             _lib.dtype_code(dtype), _lib.stream_of(acc)),
               "convert_f32")
    _lib.count_launches()
    return out


def step_max_k(pattern: int, max_seqlen: int) -> int:
    """Upper bound on a sequence's key count under ``pattern``."""
    return (max_seqlen + 1) // 2 if pattern == PATTERN_FRONT_KV else max_seqlen


def ring_flash_attn_backward(
    dout: torch.Tensor,      # [T, H, D] gradient of the local output
    local_q: torch.Tensor,   # [T, H, D]
    local_k: torch.Tensor,   # [T, H_kv, D]
    local_v: torch.Tensor,   # [T, H_kv, D]
    out: torch.Tensor,       # [T, H, D] the forward's local output
    lse: torch.Tensor,       # [T, H] fp32, the forward's final natural-log LSE
    cfg: RingConfig,
    *,
    group: Optional["dist.ProcessGroup"] = None,
    cu_seqlens: Optional[torch.Tensor] = None,
    max_seqlen: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients ``(dq, dk, dv)`` of this rank's local shards (input dtype).

    ``out`` and ``lse`` come from :func:`.ring_attention.ring_flash_attn_with_lse` on the same
    inputs and group; ``cu_seqlens`` / ``max_seqlen`` as the forward.  Collective over the cp
    group like the forward.  dQ sums with fp32 atomics, so ``cfg.deterministic=True`` (a
    run-to-run bit-identical backward) is rejected.
    """
    _check_bwd(dout, local_q, local_k, local_v, out, lse)
    if cfg.deterministic:
        raise NotImplementedError("the ring backward adds dQ with fp32 atomics; "
                                  "deterministic=True is not supported")
    T, _, D = local_q.shape
    scale = cfg.softmax_scale if cfg.softmax_scale is not None else 1.0 / math.sqrt(D)
    cu, nseq, max_seqlen = local_cu_args(T, local_q.device, cu_seqlens, max_seqlen)
    q, k, v = local_q.contiguous(), local_k.contiguous(), local_v.contiguous()
    dout, out, lse = dout.contiguous(), out.contiguous(), lse.contiguous()
    delta = bwd_delta(out, dout)
    dq_acc, dkv = ring_backward_accumulate(q, k, v, dout, lse, delta, cfg, cu=cu, nseq=nseq,
                                           max_seqlen=max_seqlen, softmax_scale=scale,
                                           group=group)
    return acc_to(dq_acc, q.dtype), acc_to(dkv[0], k.dtype), acc_to(dkv[1], v.dtype)


def ring_backward_accumulate(q, k, v, dout, lse, delta, cfg: RingConfig, *, cu, nseq: int,
                             max_seqlen: int, softmax_scale: float, group=None,
                             step_fn=None, add_fn=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """The ring schedule of the backward for one rank: returns the fp32 accumulators
    ``(dq [T, H, D], dkv [2, T, H_kv, D])`` (dK, dV of this rank's own K/V, complete).

    ``step_fn`` / ``add_fn`` default to the CUDA kernels (:func:`bwd_step`, :func:`acc_add`);
    the schedule and the two rotations are the same whatever computes the steps.
    """
    step_fn = bwd_step if step_fn is None else step_fn
    add_fn = acc_add if add_fn is None else add_fn
    S, rank = cfg.cp_size, cfg.cp_rank
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    dev = q.device
    dq_acc = torch.zeros((T, Hq, D), dtype=torch.float32, device=dev)
    kw = dict(nseq=nseq, softmax_scale=softmax_scale)
    if S == 1:
        dkv = torch.zeros((2, T, Hkv, D), dtype=torch.float32, device=dev)
        if T > 0:
            step_fn(q, k, v, dout, lse, delta, dq_acc, dkv[0], dkv[1], cu,
                    max_seqlen_k=max_seqlen, pattern=PATTERN_VARLEN, causal=True, **kw)
        return dq_acc, dkv
    kv_ring = KVRing(k, v, rank, S, group)
    kv_ring.start()
    grad_ring = GradRing((2, T, Hkv, D), rank, S, dev, group)
    for step, _src, pattern in ring_schedule(rank, S):
        ks, vs = kv_ring.get(step)
        part = grad_ring.fresh(step)
        if T > 0:
            step_fn(q, ks, vs, dout, lse, delta, dq_acc, part[0], part[1], cu,
                    max_seqlen_k=step_max_k(pattern, max_seqlen), pattern=pattern,
                    causal=(step == 0), **kw)
        kv_ring.done(step)
        grad_ring.pass_on(step, part, add_fn)
    return dq_acc, grad_ring.finish()
