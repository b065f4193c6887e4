"""Online-softmax mergers of ring partials (mirrors ``fa4_ring/merge.py:45-94``).

Both consume full-size partials ``(out[T,H,D], lse[T,H])``; rows a partial does not
cover carry ``lse = -inf`` and are the identity of the merge (their ``out`` values
are never read).  LSE is float32 natural log.

* ``IncrementalMerger`` -- ``fa4cp_merge_state_inplace`` once per step, O(1) extra
  memory.  (``ring_flash_attn`` goes one step further and fuses this merge into the
  attention kernel's epilogue.)
* ``BatchedMerger``     -- keeps every partial and runs one k-way
  ``fa4cp_merge_states`` over a pointer array at the end (no ``torch.stack`` copy).

Invariant (fa4_ring/merge.py:19-23): the first partial added must cover every row
with a finite LSE (the ring's step 0).  Unlike the flashinfer kernels the reference
calls, rows that are -inf in both operands stay -inf here instead of turning NaN.
"""

from typing import List

import torch

from . import _lib


def _check_pair(out: torch.Tensor, lse: torch.Tensor):
    _lib.require_cuda(out, lse)
    assert out.dim() == 3 and lse.dim() == 2 and out.shape[:2] == lse.shape, (
        "expected out [T,H,D] and lse [T,H]")
    assert lse.dtype == torch.float32, "lse must be float32"


def merge_state_in_place(v: torch.Tensor, s: torch.Tensor, v_other: torch.Tensor,
                         s_other: torch.Tensor) -> None:
    """(v, s) <- merge((v, s), (v_other, s_other)), in place (natural-log LSE)."""
    _check_pair(v, s)
    _check_pair(v_other, s_other)
    assert v.shape == v_other.shape and v.dtype == v_other.dtype
    assert v.is_contiguous() and s.is_contiguous(), "the accumulator must be contiguous"
    v_other, s_other = v_other.contiguous(), s_other.contiguous()
    T, H, D = v.shape
    _lib.check(_lib.load().fa4cp_merge_state_inplace(
        v.data_ptr(), s.data_ptr(), v_other.data_ptr(), s_other.data_ptr(), T, H, D,
        _lib.dtype_code(v.dtype), _lib.stream_of(v)), "merge_state_in_place")
    # one pass when a head's 16-byte vectors are a power of two <= 32, else values + LSE
    vph = D // (4 if v.dtype == torch.float32 else 8)
    if T > 0:
        _lib.count_launches(1 if 0 < vph <= 32 and (vph & (vph - 1)) == 0 else 2)


def merge_states(outs: List[torch.Tensor], lses: List[torch.Tensor], *, out: torch.Tensor = None,
                 lse_out: torch.Tensor = None):
    """k-way merge of partials; returns ``(out [T,H,D], lse [T,H])``."""
    assert outs and len(outs) == len(lses)
    assert len(outs) <= 32, "at most 32 partials per merge"
    outs = [o.contiguous() for o in outs]
    lses = [s.contiguous() for s in lses]
    for o, s in zip(outs, lses):
        _check_pair(o, s)
        assert o.shape == outs[0].shape and o.dtype == outs[0].dtype
    T, H, D = outs[0].shape
    if out is None:
        out = torch.empty_like(outs[0])
    if lse_out is None:
        lse_out = torch.empty((T, H), dtype=torch.float32, device=outs[0].device)
    _lib.check(_lib.load().fa4cp_merge_states(
        _lib.ptr_array(outs), _lib.ptr_array(lses), len(outs), out.data_ptr(), lse_out.data_ptr(),
        T, H, D, _lib.dtype_code(outs[0].dtype), _lib.stream_of(out)), "merge_states")
    _lib.count_launches()
    return out, lse_out


class IncrementalMerger:
    """Accumulate (out, lse) in place, one step at a time (fa4_ring/merge.py:45-64)."""

    def __init__(self):
        self.out = None  # [T, H, D]
        self.lse = None  # [T, H]

    def add(self, out: torch.Tensor, lse: torch.Tensor) -> None:
        _check_pair(out, lse)
        if self.out is None:
            # the first partial seeds the accumulator; copy so later in-place merges
            # never write into the caller's buffers
            self.out = out.clone(memory_format=torch.contiguous_format)
            self.lse = lse.clone(memory_format=torch.contiguous_format)
        else:
            merge_state_in_place(self.out, self.lse, out, lse)

    def result(self) -> torch.Tensor:
        assert self.out is not None, "no partials were added"
        return self.out


class BatchedMerger:
    """Stash every step's (out, lse); combine all at once at the end (fa4_ring/merge.py:67-86)."""

    def __init__(self):
        self.outs: List[torch.Tensor] = []
        self.lses: List[torch.Tensor] = []

    def add(self, out: torch.Tensor, lse: torch.Tensor) -> None:
        _check_pair(out, lse)
        self.outs.append(out)
        self.lses.append(lse)

    def result(self) -> torch.Tensor:
        assert self.outs, "no partials were added"
        if len(self.outs) == 1:
            return self.outs[0]
        out, _ = merge_states(self.outs, self.lses)
        return out


def make_merger(merge_mode: str):
    """fa4_ring/merge.py:89-94."""
    if merge_mode == "incremental":
        return IncrementalMerger()
    if merge_mode == "batched":
        return BatchedMerger()
    raise ValueError(f"unknown merge_mode {merge_mode!r}")
