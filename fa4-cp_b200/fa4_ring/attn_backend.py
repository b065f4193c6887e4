"""Per-chunk attention on B200 (replaces ``fa4_ring/fa4_backend.py:58-123``).

``b200_attn`` has the calling convention of the reference's ``fa4_attn``: 3-D varlen
``[total, H, D]`` tensors plus ``cu_seqlens_q/k`` and ``max_seqlen_q/k``, optional
FP8 descales, and returns ``(out[Tq, H, D], lse[Tq, H])`` with LSE in float32 natural
log, already in the ``[T, H]`` layout the mergers use (no transpose copy).  It runs
the hand-written sm_100a kernel of ``fa4cp_attn_fwd`` (tcgen05 MMA, TMEM
accumulators, TMA tiles); FP8 e4m3 inputs produce a bf16 output.

``attn_into`` is the lower-level entry the ring uses: it writes (or, with
``accumulate=True``, merges) a step's partial into caller-owned ``out``/``lse`` for
one of the three zig-zag step patterns, addressing the row halves in place.
"""

import math
from typing import Optional, Tuple

import torch

from . import _lib

PATTERN_VARLEN = _lib.PATTERN_VARLEN
PATTERN_FRONT_KV = _lib.PATTERN_FRONT_KV
PATTERN_BACK_Q = _lib.PATTERN_BACK_Q

SUPPORTED_HEAD_DIMS = {torch.bfloat16: (64, 128, 256), torch.float16: (64, 128, 256),
                       torch.float8_e4m3fn: (128,)}
# bf16 query with e4m3 K/V (K/V dequantised to bf16 in a workspace, then the bf16 kernel)
MIXED_HEAD_DIMS = (64, 128, 256)


def is_mixed(q: torch.Tensor, k: torch.Tensor) -> bool:
    return q.dtype == torch.bfloat16 and k.dtype == torch.float8_e4m3fn


def has_backend() -> bool:
    """True when the CUDA library loads (the reference's ``has_fa4``, fa4_backend.py:41-42)."""
    try:
        _lib.load()
        return True
    except RuntimeError:
        return False


def norm_descale(d: Optional[torch.Tensor], h_kv: int, device) -> Optional[torch.Tensor]:
    """Normalise an FP8 descale (scalar, ``[H_kv]`` or ``(1, H_kv)``) to a contiguous fp32
    ``[H_kv]`` CUDA tensor (fa4_ring/fa4_backend.py:45-55)."""
    if d is None:
        return None
    if not torch.is_tensor(d):
        d = torch.tensor(float(d))
    d = d.to(device=device, dtype=torch.float32)
    if d.dim() == 0:
        d = d.reshape(1).expand(h_kv)
    elif d.dim() == 2:
        d = d.reshape(-1)
    assert d.numel() == h_kv, f"descale must have H_kv={h_kv} entries, got {d.numel()}"
    return d.contiguous()


def out_dtype_for(dt: torch.dtype) -> torch.dtype:
    return torch.bfloat16 if dt == torch.float8_e4m3fn else dt


def _check_qkv(q, k, v):
    _lib.require_cuda(q, k, v)
    assert q.dim() == 3 and k.dim() == 3 and v.dim() == 3, "expected [T, H, D] tensors"
    assert k.dtype == v.dtype, "k and v must share a dtype"
    assert q.dtype == k.dtype or is_mixed(q, k), (
        "q, k, v must share a dtype (or bf16 q with e4m3 k/v)")
    assert k.shape == v.shape, "k and v must have the same shape"
    assert q.shape[2] == k.shape[2], "q and k head_dim differ"
    H, Hkv, D = q.shape[1], k.shape[1], q.shape[2]
    assert H % Hkv == 0, f"H_q={H} not a multiple of H_kv={Hkv}"
    if is_mixed(q, k):
        if D not in MIXED_HEAD_DIMS:
            raise NotImplementedError(f"head_dim {D} is not supported for bf16 q x e4m3 kv")
    elif q.dtype not in SUPPORTED_HEAD_DIMS or D not in SUPPORTED_HEAD_DIMS[q.dtype]:
        raise NotImplementedError(f"head_dim {D} with dtype {q.dtype} is not supported")


# Optional per-launch timing: when set to a list, every attn_into launch appends
# (start_event, end_event, pattern) recorded on the launching stream.
launch_timer = None


def attn_into(q, k, v, out, lse, cu_q, cu_k, *, nseq: int, max_seqlen_q: int, pattern: int,
              causal: bool, softmax_scale: float, q_descale=None, k_descale=None,
              v_descale=None, accumulate: bool = False) -> None:
    """Launch ``fa4cp_attn_fwd`` on the current stream.  All tensors contiguous CUDA."""
    lib = _lib.load()
    timer = launch_timer
    if timer is not None:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
    if is_mixed(q, k):
        ws_bytes = lib.fa4cp_attn_kv8_workspace_bytes(k.shape[0], k.shape[1], k.shape[2])
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=q.device)
        rc = lib.fa4cp_attn_fwd_kv8(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(),
            cu_q.data_ptr(), _lib.ptr(cu_k), nseq, max_seqlen_q, q.shape[0], k.shape[0],
            q.shape[1], k.shape[1], q.shape[2], _lib.dtype_code(q.dtype), pattern,
            1 if causal else 0, float(softmax_scale), _lib.ptr(k_descale), _lib.ptr(v_descale),
            1 if accumulate else 0, ws.data_ptr(), ws.numel(), _lib.stream_of(q))
        _lib.check(rc, "attn_fwd_kv8")
        _lib.count_launches(3)
    else:
        rc = lib.fa4cp_attn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(),
            cu_q.data_ptr(), _lib.ptr(cu_k), nseq, max_seqlen_q, q.shape[0], k.shape[0],
            q.shape[1], k.shape[1], q.shape[2], _lib.dtype_code(q.dtype),
            _lib.dtype_code(out.dtype), pattern, 1 if causal else 0, float(softmax_scale),
            _lib.ptr(q_descale), _lib.ptr(k_descale), _lib.ptr(v_descale),
            1 if accumulate else 0, _lib.stream_of(q))
        _lib.check(rc, "attn_fwd")
        _lib.count_launches()
    if timer is not None:
        ev1.record()
        timer.append((ev0, ev1, pattern))


def b200_attn(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool,
    softmax_scale: Optional[float] = None,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    cu_seqlens_k: Optional[torch.Tensor] = None,
    max_seqlen_q: Optional[int] = None,
    max_seqlen_k: Optional[int] = None,
    q_descale: Optional[torch.Tensor] = None,
    k_descale: Optional[torch.Tensor] = None,
    v_descale: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Varlen attention forward; returns ``(out [T_q,H,D], lse [T_q,H] fp32 natural log)``.

    Causal masking is bottom-right aligned per sequence (key j visible to query i iff
    ``j <= i + T_k - T_q``), which is the square ``tril`` of the reference's CPU
    simulation whenever ``T_q == T_k``.  Rows that see no key get out 0, lse -inf.
    """
    _check_qkv(q, k, v)
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    dev = q.device
    t_q, t_k = q.shape[0], k.shape[0]
    if cu_seqlens_q is None:
        cu_seqlens_q = torch.tensor([0, t_q], device=dev, dtype=torch.int32)
        max_seqlen_q = t_q
    if cu_seqlens_k is None:
        cu_seqlens_k = torch.tensor([0, t_k], device=dev, dtype=torch.int32)
        max_seqlen_k = t_k
    assert max_seqlen_q is not None, "max_seqlen_q required when cu_seqlens_q is given"
    assert cu_seqlens_q.numel() == cu_seqlens_k.numel(), "cu_seqlens_q/k describe different batches"
    cu_q = cu_seqlens_q.to(device=dev, dtype=torch.int32).contiguous()
    cu_k = cu_seqlens_k.to(device=dev, dtype=torch.int32).contiguous()
    h_kv = k.shape[1]
    fp8 = q.dtype == torch.float8_e4m3fn
    kv8 = k.dtype == torch.float8_e4m3fn
    qd = norm_descale(q_descale, h_kv, dev) if fp8 else None
    kd = norm_descale(k_descale, h_kv, dev) if kv8 else None
    vd = norm_descale(v_descale, h_kv, dev) if kv8 else None
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty(q.shape, dtype=out_dtype_for(q.dtype), device=dev)
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device=dev)
    nseq = cu_q.numel() - 1
    if t_q > 0 and nseq > 0:
        # rows outside every sequence of cu_seqlens_q are left unwritten (as in FA4)
        attn_into(q, k, v, out, lse, cu_q, cu_k, nseq=nseq, max_seqlen_q=int(max_seqlen_q),
                  pattern=PATTERN_VARLEN, causal=causal, softmax_scale=softmax_scale,
                  q_descale=qd, k_descale=kd, v_descale=vd, accumulate=False)
    return out, lse


# Drop-in name of the reference's per-chunk entry (fa4_ring/fa4_backend.py:58).
fa4_attn = b200_attn


def b200_attn_paged(
    q: torch.Tensor,            # [T_q, H, D]
    k_pages: torch.Tensor,      # [num_pages, page_size, H_kv, D]
    v_pages: torch.Tensor,      # [num_pages, page_size, H_kv, D]
    block_table: torch.Tensor,  # int32 [num_seqs, max_pages_per_seq]
    *,
    cu_seqlens_q: torch.Tensor,  # int32 [num_seqs + 1]
    cu_seqlens_k: torch.Tensor,  # int32 [num_seqs + 1], logical K/V lengths
    max_seqlen_q: int,
    causal: bool,
    softmax_scale: Optional[float] = None,
    q_descale: Optional[torch.Tensor] = None,
    k_descale: Optional[torch.Tensor] = None,
    v_descale: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Varlen attention over a paged K/V cache (``fa4cp_attn_fwd_paged``): the K/V rows of
    sequence j at logical position r are row ``r % page_size`` of page
    ``block_table[j, r // page_size]``.  ``page_size`` must be a multiple of 128.  Causal
    masking is bottom-right aligned per sequence, as :func:`b200_attn`.  Returns
    ``(out [T_q, H, D], lse [T_q, H] fp32 natural log)``.  Not in the reference, whose K/V is
    contiguous."""
    _lib.require_cuda(q, k_pages, v_pages, block_table)
    assert k_pages.dim() == 4 and k_pages.shape == v_pages.shape, "pools are [pages, page, H_kv, D]"
    assert k_pages.dtype == v_pages.dtype == q.dtype, "q and the pools must share a dtype"
    num_pages, page_size, h_kv, D = k_pages.shape
    assert q.shape[2] == D and q.shape[1] % h_kv == 0
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    dev = q.device
    fp8 = q.dtype == torch.float8_e4m3fn
    qd = norm_descale(q_descale, h_kv, dev) if fp8 else None
    kd = norm_descale(k_descale, h_kv, dev) if fp8 else None
    vd = norm_descale(v_descale, h_kv, dev) if fp8 else None
    q = q.contiguous()
    bt = block_table.to(device=dev, dtype=torch.int32).contiguous()
    cu_q = cu_seqlens_q.to(device=dev, dtype=torch.int32).contiguous()
    cu_k = cu_seqlens_k.to(device=dev, dtype=torch.int32).contiguous()
    assert bt.dim() == 2 and bt.shape[0] == cu_q.numel() - 1 == cu_k.numel() - 1
    out = torch.empty(q.shape, dtype=out_dtype_for(q.dtype), device=dev)
    lse = torch.empty(q.shape[:2], dtype=torch.float32, device=dev)
    lib = _lib.load()
    rc = lib.fa4cp_attn_fwd_paged(
        q.data_ptr(), k_pages.contiguous().data_ptr(), v_pages.contiguous().data_ptr(),
        bt.data_ptr(), page_size, num_pages, bt.shape[1], out.data_ptr(), lse.data_ptr(),
        cu_q.data_ptr(), cu_k.data_ptr(), cu_q.numel() - 1, int(max_seqlen_q), q.shape[0],
        q.shape[1], h_kv, D, _lib.dtype_code(q.dtype), _lib.dtype_code(out.dtype),
        1 if causal else 0, float(softmax_scale), _lib.ptr(qd), _lib.ptr(kd), _lib.ptr(vd),
        _lib.stream_of(q))
    _lib.check(rc, "attn_fwd_paged")
    _lib.count_launches()
    return out, lse
