"""fa4_ring on B200 -- zig-zag context-parallel causal ring attention, sm_100a native.

Drop-in for the reference package ``fa4_ring`` (hxy0118/fa4-cp): the same public
names (``fa4_ring/__init__.py:10-24``) backed by hand-written CUDA kernels for
sm_100a behind the C ABI of ``include/fa4cp_b200.h``:

    RingConfig         - configuration (cp_size, cp_rank, merge_mode, ...)
    ring_flash_attn    - causal ring attention on a zig-zag local shard
    Descales           - optional FP8 per-tensor descales (per source rank)
    zigzag_shard / zigzag_unshard - shard a full sequence / stitch shards back
    IncrementalMerger / BatchedMerger / make_merger - LSE mergers

Beyond the reference (which is forward-only): ``ring_flash_attn`` is differentiable, and
``ring_flash_attn_with_lse`` / ``ring_flash_attn_backward`` run the forward (returning the
LSE) and the ring backward explicitly.

There is no CPU fallback: every op needs the built CUDA library and CUDA tensors.
"""

from .config import MERGE_MODES, RingConfig
from .merge import BatchedMerger, IncrementalMerger, make_merger
from .ring_attention import Descales, ring_flash_attn, ring_flash_attn_with_lse
from .ring_backward import ring_flash_attn_backward
from .zigzag import zigzag_shard, zigzag_unshard

__all__ = [
    "RingConfig",
    "ring_flash_attn",
    "Descales",
    "zigzag_shard",
    "zigzag_unshard",
    "IncrementalMerger",
    "BatchedMerger",
    "make_merger",
    "ring_flash_attn_with_lse",
    "ring_flash_attn_backward",
]
