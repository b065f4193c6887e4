"""Paged K/V attention (``fa4cp_attn_fwd_paged`` / ``b200_attn_paged``).

Each sequence's K/V is cut into logical pages that are scattered over a shuffled page pool
(with spare pages holding garbage); the kernel must give exactly -- bit for bit -- what the
contiguous kernel gives on the same rows (same tiles, same order; rows past a sequence's end
are masked either way), and the oracle agrees within the bf16 tolerance.
"""

import math

import numpy as np
import pytest
import torch

from gpu_helpers import assert_device_ok, to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu


def _paged(k, lens_k, page_size, gen, spare=3):
    """Scatter [sum(lens_k), Hkv, D] into a shuffled pool; return (pool, block_table)."""
    n_pages = [(n + page_size - 1) // page_size for n in lens_k]
    total_pages = sum(n_pages) + spare
    perm = torch.randperm(total_pages, generator=gen)
    pool = torch.randn((total_pages, page_size) + tuple(k.shape[1:]), generator=gen).to(k.dtype)
    table = torch.full((len(lens_k), max(max(n_pages), 1)), -1, dtype=torch.int32)
    nxt, off = 0, 0
    for j, n in enumerate(lens_k):
        for pg in range(n_pages[j]):
            phys = int(perm[nxt]); nxt += 1
            table[j, pg] = phys
            rows = k[off + pg * page_size: off + min(n, (pg + 1) * page_size)]
            pool[phys, :rows.shape[0]] = rows
        off += n
    return pool, table


CASES = [
    # q_lens, k_lens, H, Hkv, D, causal, dtype, page_size
    ([1000], [1000], 4, 2, 128, True, torch.bfloat16, 128),
    ([100, 300, 37], [100, 300, 37], 4, 1, 128, True, torch.bfloat16, 256),
    ([1, 5], [1000, 777], 8, 2, 128, False, torch.bfloat16, 128),
    ([513], [513], 4, 4, 64, True, torch.float16, 128),
    ([700], [700], 4, 2, 128, True, torch.float8_e4m3fn, 128),
]


@pytest.mark.parametrize("case", CASES, ids=[str(i) for i in range(len(CASES))])
def test_paged_equals_contiguous(case):
    from fa4_ring.attn_backend import b200_attn, b200_attn_paged
    q_lens, k_lens, H, Hkv, D, causal, dt, page = case
    g = torch.Generator().manual_seed(sum(k_lens) + page)
    tq, tk = sum(q_lens), sum(k_lens)
    q = torch.randn(tq, H, D, generator=g).to(dt)
    k = torch.randn(tk, Hkv, D, generator=g).to(dt)
    v = torch.randn(tk, Hkv, D, generator=g).to(dt)
    kp, table = _paged(k, k_lens, page, g)
    vp, table_v = _paged(v, k_lens, page, torch.Generator().manual_seed(sum(k_lens) + page))
    # the same table must describe both pools: re-scatter V with K's table
    vp = torch.zeros_like(kp)
    off = 0
    for j, n in enumerate(k_lens):
        for pg in range((n + page - 1) // page):
            rows = v[off + pg * page: off + min(n, (pg + 1) * page)]
            vp[int(table[j, pg]), :rows.shape[0]] = rows
        off += n
    cu_q = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32).cuda()
    cu_k = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32).cuda()
    kw = {}
    if dt == torch.float8_e4m3fn:
        one = torch.ones(Hkv, device="cuda")
        kw = dict(q_descale=one, k_descale=one, v_descale=one)
    o_p, l_p = b200_attn_paged(q.cuda(), kp.cuda(), vp.cuda(), table.cuda(), cu_seqlens_q=cu_q,
                               cu_seqlens_k=cu_k, max_seqlen_q=max(q_lens), causal=causal, **kw)
    o_c, l_c = b200_attn(q.cuda(), k.cuda(), v.cuda(), causal=causal, cu_seqlens_q=cu_q,
                         cu_seqlens_k=cu_k, max_seqlen_q=max(q_lens), max_seqlen_k=max(k_lens), **kw)
    torch.cuda.synchronize()
    assert torch.equal(o_p, o_c), float((o_p.float() - o_c.float()).abs().max())
    assert torch.equal(l_p, l_c)
    if dt != torch.float8_e4m3fn:  # and the oracle, sequence by sequence
        qn, kn, vn, got = to_np(q), to_np(k), to_np(v), to_np(o_p)
        scale = 1.0 / math.sqrt(D)
        for j in range(len(q_lens)):
            a, b = int(cu_q[j]), int(cu_q[j + 1])
            c, d = int(cu_k[j]), int(cu_k[j + 1])
            if causal:
                want, _ = orc.attn(qn[a:b], kn[c:d], vn[c:d], True, scale) if b - a == d - c else (None, None)
            else:
                want, _ = orc.attn(qn[a:b], kn[c:d], vn[c:d], False, scale)
            if want is not None:
                np.testing.assert_allclose(got[a:b], want, atol=2e-2 if dt == torch.bfloat16 else 2e-3, rtol=0)
    assert_device_ok()


def test_paged_rejects_bad_page_size():
    from fa4_ring.attn_backend import b200_attn_paged
    q = torch.zeros(128, 2, 128, dtype=torch.bfloat16, device="cuda")
    pool = torch.zeros(4, 64, 1, 128, dtype=torch.bfloat16, device="cuda")
    table = torch.zeros(1, 4, dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, 128], dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="page_size"):
        b200_attn_paged(q, pool, pool, table, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=128,
                        causal=True)
