"""Configuration of the B200 ring attention (mirrors ``fa4_ring/config.py:12-33``)."""

from dataclasses import dataclass
from typing import Optional

# Merge modes (fa4_ring/config.py:12):
#   "incremental" -> each ring step merges into the running (out, lse) inside the
#                    attention kernel's epilogue; O(1) extra memory.
#   "batched"     -> every step's partial is kept; one k-way merge kernel at the end;
#                    O(cp_size) memory.
MERGE_MODES = ("incremental", "batched")


@dataclass
class RingConfig:
    cp_size: int
    cp_rank: int
    causal: bool = True
    softmax_scale: Optional[float] = None  # default: 1/sqrt(head_dim)
    merge_mode: str = "incremental"
    # accepted for API parity (the reference only declares it); the forward kernels are
    # deterministic, the backward sums dQ with atomics and refuses deterministic=True
    deterministic: bool = False

    def __post_init__(self):
        assert self.merge_mode in MERGE_MODES, (
            f"merge_mode must be one of {MERGE_MODES}, got {self.merge_mode}"
        )
        assert self.cp_size >= 1, "cp_size must be >= 1"
        assert 0 <= self.cp_rank < self.cp_size
        assert self.causal, "only the causal ring is implemented (non-causal is not on the path)"
