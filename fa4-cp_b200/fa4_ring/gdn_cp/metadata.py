"""GDN context-parallel index metadata (the reference's ``fa4_ring/gdn_cp/metadata.py:34-96``).

Every CP rank holds the same sequences, each zig-zag sharded exactly as
:func:`fa4_ring.zigzag.zigzag_shard_varlen` does (rank r: chunks r and 2S-1-r of
``h_j = N_j / (2S)`` tokens, stored ``[early | late]``).  The local packing concatenates the
sequences' shards (``L = sum_j 2 h_j``); an all-gather gives the rank-major packing
``[rank0 | rank1 | ...]`` of ``S * L = total`` rows.

* ``restore_perm`` [total] int64: ``gathered[restore_perm]`` is the natural order;
* ``extract_idx`` [L] int64: ``natural_out[extract_idx]`` is this rank's local output;
* ``full_cu_seqlens`` [nseq+1] int32: natural-order boundaries (for the scan).

The indices are computed on the device by one kernel (no Python loop over tokens); the
B200 gathers themselves do not need them (see :mod:`.allgather_cp`), they are kept for
callers of the reference's API.
"""

from dataclasses import dataclass
from typing import Sequence

import torch

from .. import _lib


@dataclass
class GdnCpMeta:
    restore_perm: torch.Tensor      # [total] long
    extract_idx: torch.Tensor       # [L] long
    valid_mask: torch.Tensor        # [L] bool (all True: no padding)
    full_cu_seqlens: torch.Tensor   # [num_seq+1] int32 (natural order)
    local_len: int                  # L
    total_len: int                  # total == S * L
    cp_size: int = 1
    cp_rank: int = 0


def build_gdn_cp_metadata(full_seq_lens: Sequence[int], cp_size: int, cp_rank: int,
                          device="cuda") -> GdnCpMeta:
    """Index metadata for this rank.  ``full_seq_lens`` are the FULL (un-sharded) sequence
    lengths; each must be divisible by ``2*cp_size`` (AssertionError otherwise, as the
    reference).  ``device`` must be a CUDA device (there is no CPU path)."""
    S = int(cp_size)
    assert 0 <= cp_rank < S, f"cp_rank {cp_rank} out of range for cp_size {S}"
    lens = [int(n) for n in full_seq_lens]
    assert lens, "at least one sequence"
    for n in lens:
        assert n % (2 * S) == 0, f"seq len {n} must be divisible by 2*cp_size={2 * S}"
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    total = cu[-1]
    L = total // S
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("fa4_ring.gdn_cp needs a CUDA device (no CPU path)")
    full_cu = torch.tensor(cu, dtype=torch.int32).to(dev)
    restore = torch.empty(total, dtype=torch.int64, device=dev)
    extract = torch.empty(L, dtype=torch.int64, device=dev)
    lib = _lib.load()
    _lib.check(lib.fa4cp_gdn_cp_indices(full_cu.data_ptr(), len(lens), S, int(cp_rank), total,
                                        _lib.ptr(restore), _lib.ptr(extract),
                                        _lib.stream_of(full_cu)), "gdn_cp_indices")
    _lib.count_launches()
    return GdnCpMeta(restore_perm=restore, extract_idx=extract,
                     valid_mask=torch.ones(L, dtype=torch.bool, device=dev),
                     full_cu_seqlens=full_cu, local_len=L, total_len=total, cp_size=S,
                     cp_rank=int(cp_rank))
