"""GDN context parallelism, Plan A, on the GPU (fa4_ring.gdn_cp).

* the device index metadata (``fa4cp_gdn_cp_indices``) is bit-exact against the fixtures
  the reference's own ``build_gdn_cp_metadata`` wrote (tests/golden/gdn_meta.npz);
* the collective-free core (restore -> scan -> extract with the zig-zag gather kernels),
  run for every rank of a simulated cp group on one GPU: the stitched per-rank outputs
  equal the single-device scan exactly (the reference's "max_err = 0" check), with the
  oracle's gated-delta-rule recurrence as the scan and with a per-sequence cumulative
  sum on the GPU;
* the all-gather wrapper over NCCL is in tests/dist_ring_check.py (>= 2 GPUs).
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_helpers import assert_device_ok

pytestmark = pytest.mark.gpu


def test_device_indices_match_reference_golden():
    from fa4_ring.gdn_cp import build_gdn_cp_metadata
    z = np.load(os.path.join(GOLDEN, "gdn_meta.npz"))
    for ci in range(int(z["n_cases"])):
        lens, cp = z[f"c{ci}_lens"].tolist(), int(z[f"c{ci}_cp"])
        for r in range(cp):
            m = build_gdn_cp_metadata(lens, cp, r)
            np.testing.assert_array_equal(m.restore_perm.cpu().numpy(), z[f"c{ci}_r{r}_restore"])
            np.testing.assert_array_equal(m.extract_idx.cpu().numpy(), z[f"c{ci}_r{r}_extract"])
            np.testing.assert_array_equal(m.full_cu_seqlens.cpu().numpy(), z[f"c{ci}_r{r}_cu"])
            assert m.local_len * cp == m.total_len == sum(lens)
    assert_device_ok()


def _segment_cumsum(natural, cu):
    """A causal per-sequence scan on the GPU: running sums, reshaped to [T, 2, F/2]."""
    out = torch.empty_like(natural)
    c = [int(x) for x in cu.tolist()]
    for a, b in zip(c[:-1], c[1:]):
        out[a:b] = torch.cumsum(natural[a:b], dim=0)
    return out.reshape(out.shape[0], 2, -1)


def _oracle_scan(Hk, Dk, Hv, Dv):
    from oracle import gdn_oracle

    def scan(natural, cu):
        x = natural.double().cpu().numpy()
        i = 0
        q = x[:, i:i + Hk * Dk].reshape(-1, Hk, Dk); i += Hk * Dk
        k = x[:, i:i + Hk * Dk].reshape(-1, Hk, Dk); i += Hk * Dk
        v = x[:, i:i + Hv * Dv].reshape(-1, Hv, Dv); i += Hv * Dv
        g = x[:, i:i + Hv]; i += Hv
        beta = x[:, i:i + Hv]
        o = gdn_oracle.gdn_scan(q, k, v, g, beta, cu.tolist())
        return torch.from_numpy(o).to(natural.device)
    return scan


@pytest.mark.parametrize("cp,lens", [(2, [24]), (4, [32, 16, 48]), (8, [64, 64]), (3, [6, 18, 30])])
def test_core_equals_single_device_scan(cp, lens):
    from fa4_ring.gdn_cp import _gdn_cp_core, build_gdn_cp_metadata
    from fa4_ring.zigzag import zigzag_shard_varlen
    g = torch.Generator().manual_seed(cp)
    cu = [0] + [int(x) for x in np.cumsum(lens)]
    total = cu[-1]
    Hk, Dk, Hv, Dv = 2, 8, 4, 8
    F = 2 * Hk * Dk + Hv * Dv + 2 * Hv
    natural = torch.randn(total, F, generator=g, dtype=torch.float64)
    natural[:, -2 * Hv:-Hv] = -torch.rand(total, Hv, generator=g, dtype=torch.float64)  # log-decay
    natural[:, -Hv:] = torch.rand(total, Hv, generator=g, dtype=torch.float64)          # beta
    natural = natural.cuda()
    locals_ = [zigzag_shard_varlen(natural, cu, r, cp)[0] for r in range(cp)]
    packed_full = torch.cat(locals_, 0)  # what the all-gather produces (rank-major)
    for scan, ints in ((_oracle_scan(Hk, Dk, Hv, Dv), False), (_segment_cumsum, True)):
        x = packed_full.round() if ints else packed_full  # integer data: exact cumsums
        nat = natural.round() if ints else natural
        full_cu = torch.tensor(cu, dtype=torch.int32, device="cuda")
        want = scan(nat, full_cu)
        for r in range(cp):
            meta = build_gdn_cp_metadata(lens, cp, r)
            got = _gdn_cp_core(x, scan, meta)
            exp = zigzag_shard_varlen(want.reshape(total, -1), cu, r, cp)[0].reshape(got.shape)
            assert torch.equal(got, exp), f"cp={cp} rank={r}"
    assert_device_ok()
