"""Import-compatible name of the reference's per-chunk backend module
(``fa4_ring/fa4_backend.py``): ``fa4_attn`` and ``has_fa4`` resolve to the sm_100a
kernel of :mod:`.attn_backend`."""

from .attn_backend import b200_attn as fa4_attn  # noqa: F401
from .attn_backend import has_backend as has_fa4  # noqa: F401
