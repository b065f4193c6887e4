"""GDN (gated delta net / linear attention) context parallelism, Plan A (mirrors the
reference's ``fa4_ring/gdn_cp/__init__.py:1-23``): all-gather the projected GDN inputs,
replicate the recurrence on the full sequence, extract this rank's zig-zag-local output.
It shares the zig-zag sharding of the ring attention (one sharding for the whole model).

On B200 the index metadata is built by a CUDA kernel (``fa4cp_gdn_cp_indices``) and the
restore / extract gathers are the zig-zag gather kernels (``fa4cp_zigzag_unshard`` /
``fa4cp_zigzag_shard``) instead of ``index_select``; the all-gather is one
``all_gather_into_tensor`` into the rank-major buffer (no ``torch.cat``).

The reference's ``gdn_reference`` (a CPU torch recurrence used as ground truth in its tests)
is test infrastructure here: its restatement lives in the repository's ``oracle/``.
"""

from .allgather_cp import _gdn_cp_core, gdn_cp_allgather
from .metadata import GdnCpMeta, build_gdn_cp_metadata
from .state_passing import gdn_cp_state_passing

__all__ = ["build_gdn_cp_metadata", "gdn_cp_allgather", "GdnCpMeta", "gdn_cp_state_passing"]
