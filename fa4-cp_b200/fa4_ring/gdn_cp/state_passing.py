"""GDN context parallelism, Plan B (sequential state passing): not implemented, as in the
reference (``fa4_ring/gdn_cp/state_passing.py:1-31``), whose v1 is Plan A (all-gather +
replicate scan, :mod:`.allgather_cp`).  Plan B needs contiguous (not zig-zag) sharding."""


def gdn_cp_state_passing(*args, **kwargs):
    raise NotImplementedError(
        "Plan B (sequential state-passing) is not implemented; use gdn_cp_allgather (Plan A)")
