"""Zig-zag context-parallel sharding on the GPU (mirrors ``fa4_ring/zigzag.py:26-97``).

A sequence of ``N`` tokens is cut into ``2 * cp_size`` chunks of ``h = N / (2 * cp_size)``
rows; rank ``i`` holds chunk ``i`` (early) followed by chunk ``2*cp_size-1-i`` (late), so
every rank does the same share of causal work.  Packed sequences are sharded one by
one and the local shards stay packed in sequence order.

Every function here moves data with the gather/scatter kernels of the CUDA library
(``fa4cp_zigzag_shard``, ``fa4cp_zigzag_unshard``, ``fa4cp_half_index``,
``fa4cp_local_cu``); inputs must be CUDA tensors.  The only host work is validating
sequence lengths, as the reference does with its ``assert``s -- for boundaries given on the
host.  Boundaries given as a CUDA tensor are trusted and never copied to the host (the
reference's ``.tolist()`` at ``fa4_ring/zigzag.py:71`` is a device->host sync): the packed
length comes from the tensors' shapes, or from ``total=`` for :func:`get_half_index`.
"""

import math
from typing import List, Sequence, Union

import torch

from . import _lib


def local_seqlen(n: int, cp_size: int) -> int:
    """fa4_ring/zigzag.py:26-28."""
    assert n % (2 * cp_size) == 0, f"seqlen {n} must be divisible by 2*cp_size={2 * cp_size}"
    return n // cp_size


def _row_bytes(x: torch.Tensor) -> int:
    return math.prod(x.shape[1:]) * x.element_size()


def zigzag_shard(x: torch.Tensor, cp_rank: int, cp_size: int) -> torch.Tensor:
    """Take the full ``[N, ...]`` sequence and return this rank's local ``[2h, ...]`` shard."""
    _lib.require_cuda(x)
    n = x.shape[0]
    assert n % (2 * cp_size) == 0, f"seqlen {n} must be divisible by 2*cp_size={2 * cp_size}"
    assert 0 <= cp_rank < cp_size
    x = x.contiguous()
    out = torch.empty((n // cp_size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if out.numel() == 0:
        return out
    _lib.check(_lib.load().fa4cp_zigzag_shard(
        x.data_ptr(), out.data_ptr(), None, 1, n, cp_rank, cp_size, _row_bytes(x),
        _lib.stream_of(x)), "zigzag_shard")
    _lib.count_launches()
    return out


def zigzag_unshard(local_shards: List[torch.Tensor], cp_size: int) -> torch.Tensor:
    """Inverse of :func:`zigzag_shard`: stitch per-rank ``[2h, ...]`` shards back to ``[N, ...]``."""
    assert len(local_shards) == cp_size
    _lib.require_cuda(*local_shards)
    shards = [s.contiguous() for s in local_shards]
    t0 = shards[0]
    for s in shards[1:]:
        assert s.shape == t0.shape and s.dtype == t0.dtype, "all shards must have the same shape"
    n = t0.shape[0] * cp_size
    assert n % (2 * cp_size) == 0, "each shard must hold an even number of rows"
    out = torch.empty((n,) + tuple(t0.shape[1:]), dtype=t0.dtype, device=t0.device)
    if out.numel() == 0:
        return out
    _lib.check(_lib.load().fa4cp_zigzag_unshard(
        _lib.ptr_array(shards), out.data_ptr(), None, 1, n, cp_size, _row_bytes(t0),
        _lib.stream_of(t0)), "zigzag_unshard")
    _lib.count_launches()
    return out


def _cu_list(cu) -> List[int]:
    return [int(c) for c in (cu.tolist() if torch.is_tensor(cu) else cu)]


def _on_device(cu) -> bool:
    return torch.is_tensor(cu) and cu.is_cuda


def _cu_device(cu, device) -> torch.Tensor:
    if torch.is_tensor(cu) and cu.is_cuda and cu.dtype == torch.int32 and cu.is_contiguous():
        return cu
    if torch.is_tensor(cu):
        return cu.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(cu), dtype=torch.int32, device=device)


def zigzag_shard_varlen(x: torch.Tensor, full_cu_seqlens: Union[torch.Tensor, Sequence[int]],
                        cp_rank: int, cp_size: int):
    """Shard several packed sequences zig-zag for this rank (fa4_ring/zigzag.py:82-97).

    ``full_cu_seqlens`` are the FULL sequence boundaries (int list or tensor).  Returns
    ``(local_packed, local_cu_seqlens)`` with ``local_cu_seqlens`` int32 on ``x.device``.
    """
    _lib.require_cuda(x)
    if _on_device(full_cu_seqlens):
        # trusted (no host copy): the sequences must cover x exactly
        nseq = full_cu_seqlens.numel() - 1
        total = x.shape[0]
        assert total % (2 * cp_size) == 0, "the packed length must be divisible by 2*cp_size"
    else:
        cu = _cu_list(full_cu_seqlens)
        assert len(cu) >= 1 and cu[0] == 0, "cu_seqlens must start at 0"
        for j in range(len(cu) - 1):
            n = cu[j + 1] - cu[j]
            assert n >= 0, "cu_seqlens must be non-decreasing"
            assert n % (2 * cp_size) == 0, f"seqlen {n} must be divisible by 2*cp_size={2 * cp_size}"
        assert cu[-1] <= x.shape[0], "cu_seqlens exceed the packed tensor"
        nseq = len(cu) - 1
        total = cu[-1]
    x = x.contiguous()
    cu_dev = _cu_device(full_cu_seqlens, x.device)
    local_cu = torch.empty(nseq + 1, dtype=torch.int32, device=x.device)
    stream = _lib.stream_of(x)
    lib = _lib.load()
    _lib.check(lib.fa4cp_local_cu(cu_dev.data_ptr(), nseq, cp_size, local_cu.data_ptr(), stream),
               "local_cu")
    out = torch.empty((total // cp_size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if nseq > 0 and out.numel() > 0:
        _lib.check(lib.fa4cp_zigzag_shard(
            x.data_ptr(), out.data_ptr(), cu_dev.data_ptr(), nseq, total, cp_rank, cp_size,
            _row_bytes(x), stream), "zigzag_shard_varlen")
    return out, local_cu


def zigzag_unshard_varlen(local_shards: List[torch.Tensor], full_cu_seqlens, cp_size: int):
    """Stitch per-rank packed varlen shards back into the full packed ``[sum N_j, ...]``."""
    _lib.require_cuda(*local_shards)
    assert len(local_shards) == cp_size
    shards = [s.contiguous() for s in local_shards]
    t0 = shards[0]
    total = t0.shape[0] * cp_size
    if _on_device(full_cu_seqlens):
        nseq = full_cu_seqlens.numel() - 1  # trusted (no host copy)
    else:
        cu = _cu_list(full_cu_seqlens)
        for j in range(len(cu) - 1):
            assert (cu[j + 1] - cu[j]) % (2 * cp_size) == 0
        assert cu[-1] == total, "the shards do not hold the sequences"
        nseq = len(cu) - 1
    out = torch.empty((total,) + tuple(t0.shape[1:]), dtype=t0.dtype, device=t0.device)
    cu_dev = _cu_device(full_cu_seqlens, t0.device)
    if out.numel() > 0:
        _lib.check(_lib.load().fa4cp_zigzag_unshard(
            _lib.ptr_array(shards), out.data_ptr(), cu_dev.data_ptr(), nseq, total, cp_size,
            _row_bytes(t0), _lib.stream_of(t0)), "zigzag_unshard_varlen")
    return out


def get_half_index(cu_seqlens: torch.Tensor, *, front: bool, total: int = None) -> torch.Tensor:
    """int64 indices of the front (early) or back (late) half of every packed local
    sequence (fa4_ring/zigzag.py:65-79), computed by a kernel on ``cu_seqlens.device``.

    ``total`` (keyword, not in the reference): the packed length ``cu_seqlens[-1]``, when the
    caller knows it.  Given, the call reads nothing back from the device (the boundaries are
    trusted); omitted, ``cu_seqlens`` is copied to the host to size the output and check that
    every length is even, as the reference does."""
    _lib.require_cuda(cu_seqlens)
    if total is None:
        cu = _cu_list(cu_seqlens)
        for i in range(len(cu) - 1):
            assert (cu[i + 1] - cu[i]) % 2 == 0, "each local sequence length must be even (zig-zag)"
        total = cu[-1] if cu else 0
    nseq = cu_seqlens.numel() - 1
    assert total % 2 == 0, "the packed local length must be even (zig-zag)"
    out = torch.empty(total // 2, dtype=torch.long, device=cu_seqlens.device)
    if nseq >= 1 and total > 0:
        cu_dev = _cu_device(cu_seqlens, cu_seqlens.device)
        _lib.check(_lib.load().fa4cp_half_index(
            cu_dev.data_ptr(), nseq, total, 1 if front else 0, out.data_ptr(),
            _lib.stream_of(cu_dev)), "half_index")
    return out


def half_indices(local_len: int, device) -> tuple:
    """(first_half_idx, second_half_idx) into a single local ``[2h]`` sequence."""
    cu = torch.tensor([0, local_len], dtype=torch.int32, device=device)
    return (get_half_index(cu, front=True, total=local_len),
            get_half_index(cu, front=False, total=local_len))
