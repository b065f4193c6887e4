"""Zig-zag gather/scatter kernels vs the oracle and the reference's golden indices (bit-exact)."""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from gpu_helpers import assert_device_ok
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cp", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("row_shape,dtype", [((1,), torch.float32), ((4, 128), torch.bfloat16),
                                             ((3, 5), torch.float16), ((7,), torch.uint8)])
def test_shard_unshard_bit_exact(cp, row_shape, dtype):
    from fa4_ring import zigzag_shard, zigzag_unshard
    n = 2 * cp * 37
    x = torch.arange(n * int(np.prod(row_shape)), dtype=torch.int64) % 251
    x = x.reshape((n,) + row_shape).to(dtype).cuda()
    shards = [zigzag_shard(x, r, cp) for r in range(cp)]
    for r in range(cp):
        want = x.cpu()[torch.from_numpy(orc.zigzag_rows(n, r, cp))]
        assert torch.equal(shards[r].cpu(), want)
    assert torch.equal(zigzag_unshard(shards, cp), x)
    assert_device_ok()


def test_golden_shard_rows():
    from fa4_ring import zigzag_shard
    z = np.load(os.path.join(GOLDEN, "zigzag.npz"))
    for key in z.files:
        if not key.startswith("shard_"):
            continue
        _, n, cp, r = key.split("_")
        n, cp, r = int(n[1:]), int(cp[2:]), int(r[1:])
        x = torch.arange(n, dtype=torch.int64).reshape(n, 1).cuda()
        assert np.array_equal(zigzag_shard(x, r, cp).cpu().numpy().ravel(), z[key]), key


def test_golden_varlen_rows_and_half_index():
    from fa4_ring.zigzag import get_half_index, zigzag_shard_varlen, zigzag_unshard_varlen
    z = np.load(os.path.join(GOLDEN, "zigzag.npz"))
    checked = 0
    for key in z.files:
        if not (key.startswith("varlen_") and key.endswith("_rows")):
            continue
        _, name, cps, rs, _ = key.split("_")
        cp, r = int(cps[2:]), int(rs[1:])
        full_cu = z[f"varlen_{name}_full_cu"]
        total = int(full_cu[-1])
        x = torch.arange(total, dtype=torch.int64).reshape(total, 1).cuda()
        for cu_arg in (full_cu.tolist(), torch.from_numpy(full_cu).cuda()):
            loc, lcu = zigzag_shard_varlen(x, cu_arg, r, cp)
            assert np.array_equal(loc.cpu().numpy().ravel(), z[key])
            assert np.array_equal(lcu.cpu().numpy(), z[f"varlen_{name}_cp{cp}_r{r}_cu"])
        assert np.array_equal(get_half_index(lcu, front=True).cpu().numpy(),
                              z[f"varlen_{name}_cp{cp}_r{r}_front"])
        assert np.array_equal(get_half_index(lcu, front=False).cpu().numpy(),
                              z[f"varlen_{name}_cp{cp}_r{r}_back"])
        # with the packed length given, nothing is read back from the device
        for front, tag in ((True, "front"), (False, "back")):
            got = get_half_index(lcu, front=front, total=total // cp)
            assert np.array_equal(got.cpu().numpy(), z[f"varlen_{name}_cp{cp}_r{r}_{tag}"])
        shards = [zigzag_shard_varlen(x, full_cu.tolist(), rr, cp)[0] for rr in range(cp)]
        assert torch.equal(zigzag_unshard_varlen(shards, full_cu.tolist(), cp), x)
        assert torch.equal(zigzag_unshard_varlen(shards, torch.from_numpy(full_cu).cuda(), cp), x)
        checked += 1
    assert checked >= 10
    assert_device_ok()


def test_varlen_with_empty_sequence_and_large_rows():
    from fa4_ring.zigzag import zigzag_shard_varlen, zigzag_unshard_varlen
    cp = 4
    cu = [0, 0, 64, 64, 64 + 8 * 25]
    total = cu[-1]
    x = torch.randn(total, 8, 128, dtype=torch.bfloat16).cuda()
    shards = []
    for r in range(cp):
        loc, lcu = zigzag_shard_varlen(x, cu, r, cp)
        rows, want_cu = orc.zigzag_varlen_rows(cu, r, cp)
        assert torch.equal(loc.cpu(), x.cpu()[torch.from_numpy(rows)])
        assert lcu.cpu().tolist() == want_cu.tolist()
        shards.append(loc)
    assert torch.equal(zigzag_unshard_varlen(shards, cu, cp), x)
    assert_device_ok()


def test_shard_rejects_bad_lengths():
    from fa4_ring import zigzag_shard
    from fa4_ring.zigzag import zigzag_shard_varlen
    x = torch.zeros(10, 2, device="cuda")
    with pytest.raises(AssertionError):
        zigzag_shard(x, 0, 2)
    with pytest.raises(AssertionError):
        zigzag_shard_varlen(torch.zeros(12, 2, device="cuda"), [0, 6, 12], 0, 2)
