"""GDN context parallelism, Plan A (the reference's ``fa4_ring/gdn_cp/allgather_cp.py:30-56``):
all-gather the local projected inputs, restore natural token order, run the caller's scan,
extract this rank's zig-zag-local output.

``scan_fn(natural_packed [total, F], full_cu_seqlens [nseq+1] int32) -> out [total, Hv, Dv]``
is the caller's GDN recurrence (conv1d + gating + chunked delta rule on the GPU); it is
injected, as in the reference.  Here the all-gather lands in one rank-major buffer
(``all_gather_into_tensor``), and the restore / extract are the zig-zag gather kernels
(``fa4cp_zigzag_unshard`` over the S parts of that buffer, ``fa4cp_zigzag_shard`` of the
scan output) -- one launch each, no ``index_select`` with int64 index tensors, no ``cat``.
"""

import ctypes
from typing import Callable, Optional

import torch
import torch.distributed as dist

from .. import _lib
from .metadata import GdnCpMeta

ScanFn = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


def _restore(packed_full: torch.Tensor, meta: GdnCpMeta) -> torch.Tensor:
    """Rank-major ``[S*L, ...]`` -> natural order ``[total, ...]`` (one kernel)."""
    S, L = meta.cp_size, meta.local_len
    x = packed_full.contiguous()
    assert x.shape[0] == S * L == meta.total_len, "packed_full must hold cp_size * local_len rows"
    row_bytes = x[0].numel() * x.element_size() if x.shape[0] else 0
    out = torch.empty_like(x)
    if x.numel() == 0:
        return out
    ptrs = (ctypes.c_void_p * S)(*[x.data_ptr() + r * L * row_bytes for r in range(S)])
    nseq = meta.full_cu_seqlens.numel() - 1
    _lib.check(_lib.load().fa4cp_zigzag_unshard(ptrs, out.data_ptr(), meta.full_cu_seqlens.data_ptr(),
                                                nseq, meta.total_len, S, row_bytes,
                                                _lib.stream_of(x)), "zigzag_unshard")
    _lib.count_launches()
    return out


def _extract(full_out: torch.Tensor, meta: GdnCpMeta) -> torch.Tensor:
    """Natural ``[total, ...]`` -> this rank's local ``[L, ...]`` (one kernel)."""
    x = full_out.contiguous()
    assert x.shape[0] == meta.total_len, "scan output must have total_len rows"
    out = torch.empty((meta.local_len,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if out.numel() == 0:
        return out
    row_bytes = x[0].numel() * x.element_size()
    nseq = meta.full_cu_seqlens.numel() - 1
    _lib.check(_lib.load().fa4cp_zigzag_shard(x.data_ptr(), out.data_ptr(),
                                              meta.full_cu_seqlens.data_ptr(), nseq,
                                              meta.total_len, meta.cp_rank, meta.cp_size,
                                              row_bytes, _lib.stream_of(x)), "zigzag_shard")
    _lib.count_launches()
    return out


def _gdn_cp_core(packed_full: torch.Tensor, scan_fn: ScanFn, meta: GdnCpMeta) -> torch.Tensor:
    """The collective-free core: rank-major gathered ``[S*L, F]`` -> natural -> scan ->
    local ``[L, Hv, Dv]``."""
    _lib.require_cuda(packed_full)
    natural = _restore(packed_full, meta)
    full_out = scan_fn(natural, meta.full_cu_seqlens)
    local_out = _extract(full_out, meta)
    if not bool(meta.valid_mask.all()):
        local_out = local_out * meta.valid_mask[:, None, None].to(local_out.dtype)
    return local_out


def gdn_cp_allgather(local_packed: torch.Tensor, scan_fn: ScanFn, meta: GdnCpMeta, *,
                     group: Optional["dist.ProcessGroup"] = None) -> torch.Tensor:
    """All-gather + replicate-scan + extract; returns this rank's local output ``[L, Hv, Dv]``."""
    _lib.require_cuda(local_packed)
    world = dist.get_world_size(group)
    assert world == meta.cp_size, "the group size must equal the metadata's cp_size"
    x = local_packed.contiguous()
    gathered = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                           device=x.device)
    dist.all_gather_into_tensor(gathered, x, group=group)
    return _gdn_cp_core(gathered, scan_fn, meta)
