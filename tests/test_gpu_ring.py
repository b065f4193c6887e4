"""Ring attention end to end.

Single GPU: every rank of a cp group is run in turn through the same per-step code as
``ring_flash_attn`` (``ring_forward``), with the source shards supplied directly --
NCCL cannot put two ranks on one GPU.  The stitched output must match the oracle's
dense causal attention (<= 2e-2 for bf16) and the oracle's ring simulation.
With >= 2 GPUs the real NCCL ring runs under torchrun (tests/dist_ring_check.py).
"""

import math
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN, ROOT
from gpu_helpers import assert_device_ok, dequant, quant_e4m3, to_np
from oracle import ring_oracle as orc

pytestmark = pytest.mark.gpu


def simulate_on_gpu(q, k, v, cp, merge_mode="incremental", full_cu=None, descales=None,
                    fp8_scales=None):
    """Run every rank's ring steps on one GPU; return the stitched output [N, H, D] and
    final LSE [N, H]."""
    from fa4_ring import RingConfig
    from fa4_ring.ring_attention import ring_forward
    from fa4_ring.zigzag import zigzag_shard_varlen, zigzag_unshard_varlen
    N = q.shape[0]
    cu_full = full_cu if full_cu is not None else [0, N]
    shards_q, shards_k, shards_v, lcu = [], [], [], None
    for r in range(cp):
        lq, lcu = zigzag_shard_varlen(q, cu_full, r, cp)
        shards_q.append(lq)
        shards_k.append(zigzag_shard_varlen(k, cu_full, r, cp)[0])
        shards_v.append(zigzag_shard_varlen(v, cu_full, r, cp)[0])
    lens = [b - a for a, b in zip(cu_full[:-1], cu_full[1:])]
    max_local = max(lens) // cp
    outs, lses = [], []
    for r in range(cp):
        cfg = RingConfig(cp_size=cp, cp_rank=r, merge_mode=merge_mode)

        def kv_at(step, r=r):
            src = (r - step) % cp
            return shards_k[src], shards_v[src]

        o, l = ring_forward(shards_q[r], kv_at, lambda s: None, cfg, cu=lcu,
                            nseq=len(cu_full) - 1, max_seqlen=max_local, descales=descales,
                            return_lse=True)
        outs.append(o)
        lses.append(l)
    return zigzag_unshard_varlen(outs, cu_full, cp), zigzag_unshard_varlen(lses, cu_full, cp)


@pytest.mark.parametrize("cp", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("merge_mode", ["incremental", "batched"])
def test_ring_single_sequence(cp, merge_mode):
    g = torch.Generator().manual_seed(cp)
    N, H, Hkv, D = 2 * cp * 160, 4, 2, 128
    q, k, v = (torch.randn(N, h, D, generator=g).bfloat16() for h in (H, Hkv, Hkv))
    got, got_l = simulate_on_gpu(q.cuda(), k.cuda(), v.cuda(), cp, merge_mode)
    scale = 1.0 / math.sqrt(D)
    dense, dense_l = orc.dense_causal(to_np(q), to_np(k), to_np(v), scale)
    np.testing.assert_allclose(to_np(got), dense, atol=2e-2, rtol=0)
    np.testing.assert_allclose(to_np(got_l), dense_l, atol=1e-3, rtol=0)
    assert_device_ok()


@pytest.mark.parametrize("cp", [2, 4])
@pytest.mark.parametrize("merge_mode", ["incremental", "batched"])
def test_ring_varlen(cp, merge_mode):
    g = torch.Generator().manual_seed(10 + cp)
    lens = [2 * cp * n for n in (40, 3, 97, 64)]
    cu = [0] + list(np.cumsum(lens))
    H, Hkv, D = 4, 1, 128
    N = cu[-1]
    q, k, v = (torch.randn(N, h, D, generator=g).bfloat16() for h in (H, Hkv, Hkv))
    got, got_l = (to_np(t) for t in simulate_on_gpu(q.cuda(), k.cuda(), v.cuda(), cp, merge_mode,
                                                       full_cu=cu))
    scale = 1.0 / math.sqrt(D)
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    for j in range(len(lens)):
        a, b = cu[j], cu[j + 1]
        dense, dense_l = orc.dense_causal(qn[a:b], kn[a:b], vn[a:b], scale)
        np.testing.assert_allclose(got[a:b], dense, atol=2e-2, rtol=0)
        np.testing.assert_allclose(got_l[a:b], dense_l, atol=1e-3, rtol=0)
    assert_device_ok()


def test_ring_cfg1_against_reference_golden():
    """BASELINE configs[0] (N=4096, Hq=8, Hkv=2, D=128, cp=4, seed 0) in bf16, against the
    reference's own fp32 ring output (golden) and the oracle on the rounded inputs."""
    c = np.load(os.path.join(GOLDEN, "cfg1.npz"))
    n, H, Hkv, D, cp = c["dims"].tolist()
    torch.manual_seed(0)
    q, k, v = torch.randn(n, H, D), torch.randn(n, Hkv, D), torch.randn(n, Hkv, D)
    got, got_l = (to_np(t) for t in simulate_on_gpu(q.bfloat16().cuda(), k.bfloat16().cuda(),
                                                       v.bfloat16().cuda(), cp))
    rows = c["rows"]
    np.testing.assert_allclose(got[rows], c["ring_out_rows"], atol=3e-2, rtol=0)
    qn, kn, vn = (to_np(t.bfloat16()) for t in (q, k, v))
    want, want_l = orc.simulate_ring(qn, kn, vn, cp, 1.0 / math.sqrt(D))
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    np.testing.assert_allclose(got_l, want_l, atol=1e-3, rtol=0)
    assert_device_ok()


def test_ring_fp8_per_source_descales():
    """FP8 e4m3 Q/K/V quantised per rank (scale = amax/448), K/V descales indexed by source."""
    from fa4_ring import Descales
    cp, H, Hkv, D = 4, 4, 2, 128
    N = 2 * cp * 128
    g = torch.Generator().manual_seed(21)
    q, k, v = (torch.randn(N, h, D, generator=g) for h in (H, Hkv, Hkv))
    # quantise each rank's shard with its own scale, then reassemble the full tensors
    qs, ks, vs, q8, k8, v8 = [], [], [], [], [], []
    deq = {"q": [], "k": [], "v": []}
    for r in range(cp):
        rows = torch.from_numpy(orc.zigzag_rows(N, r, cp))
        for name, t, lst8, lsts in (("q", q, q8, qs), ("k", k, k8, ks), ("v", v, v8, vs)):
            t8, s = quant_e4m3(t[rows])
            lst8.append(t8)
            lsts.append(s)
            deq[name].append(dequant(t8, s))
    from fa4_ring import RingConfig
    from fa4_ring.ring_attention import ring_forward
    cu = torch.tensor([0, N // cp], dtype=torch.int32, device="cuda")
    outs, lses = [], []
    for r in range(cp):
        cfg = RingConfig(cp_size=cp, cp_rank=r)
        desc = Descales(q=qs[r].cuda(), k=[s.cuda() for s in ks], v=[s.cuda() for s in vs])

        def kv_at(step, r=r):
            src = (r - step) % cp
            return k8[src].cuda(), v8[src].cuda()

        o, l = ring_forward(q8[r].cuda(), kv_at, lambda s: None, cfg, cu=cu, nseq=1,
                            max_seqlen=N // cp, descales=desc, return_lse=True)
        outs.append(to_np(o))
        lses.append(to_np(l))
    got = orc.zigzag_unshard(outs, cp)
    got_l = orc.zigzag_unshard(lses, cp)
    qf = orc.zigzag_unshard(deq["q"], cp)
    kf = orc.zigzag_unshard(deq["k"], cp)
    vf = orc.zigzag_unshard(deq["v"], cp)
    want, want_l = orc.dense_causal(qf, kf, vf, 1.0 / math.sqrt(D))
    np.testing.assert_allclose(got, want, atol=6e-2, rtol=0)
    np.testing.assert_allclose(got_l, want_l, atol=1e-3, rtol=0)
    assert_device_ok()


def test_ring_flash_attn_cp1_public_api():
    from fa4_ring import RingConfig, ring_flash_attn
    g = torch.Generator().manual_seed(2)
    T, H, Hkv, D = 384, 8, 2, 128
    q, k, v = (torch.randn(T, h, D, generator=g).bfloat16() for h in (H, Hkv, Hkv))
    for mode in ("incremental", "batched"):
        out = ring_flash_attn(q.cuda(), k.cuda(), v.cuda(), RingConfig(1, 0, merge_mode=mode))
        dense, _ = orc.dense_causal(to_np(q), to_np(k), to_np(v), 1.0 / math.sqrt(D))
        np.testing.assert_allclose(to_np(out), dense, atol=2e-2, rtol=0)
    assert_device_ok()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs for the NCCL ring")
def test_nccl_ring_multi_gpu():
    world = min(4, torch.cuda.device_count())
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           "--master-port=29533", os.path.join(ROOT, "tests", "dist_ring_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "RING_OK" in res.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs >= 2 GPUs")
def test_ring_detects_a_departed_neighbour():
    """A rank leaves between calls (nothing in flight); its neighbours' next ring call raises
    on the host instead of queuing waits on it (tests/dist_liveness_check.py, NVLS off)."""
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           "--master-port=29534", os.path.join(ROOT, "tests", "dist_liveness_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "LIVENESS_OK rank 0" in res.stdout, res.stdout[-3000:]


def test_ring_bf16_query_e4m3_kv_head_dim_256():
    """cfg5 in miniature: bf16 Q, e4m3 K/V quantised per rank (amax/448), D=256, cp=4,
    incremental; vs the oracle on the dequantised K/V (<= 6e-2)."""
    from fa4_ring import Descales, RingConfig
    from fa4_ring.fp8 import quantize_e4m3
    from fa4_ring.ring_attention import ring_forward
    cp, H, Hkv, D = 4, 4, 2, 256
    N = 2 * cp * 96
    g = torch.Generator().manual_seed(31)
    q = (torch.randn(N, H, D, generator=g) * 0.5).bfloat16()
    k = (torch.randn(N, Hkv, D, generator=g) * 0.5).bfloat16()
    v = (torch.randn(N, Hkv, D, generator=g) * 0.5).bfloat16()
    T = N // cp
    k8, v8, ks, vs, kd, vd = [], [], [], [], [], []
    for r in range(cp):
        rows = torch.from_numpy(orc.zigzag_rows(N, r, cp))
        a8, a_s = quantize_e4m3(k[rows].cuda())
        b8, b_s = quantize_e4m3(v[rows].cuda())
        k8.append(a8); ks.append(a_s); v8.append(b8); vs.append(b_s)
        kd.append(dequant(a8.cpu(), a_s.cpu())); vd.append(dequant(b8.cpu(), b_s.cpu()))
    cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
    outs, lses = [], []
    for r in range(cp):
        rows = torch.from_numpy(orc.zigzag_rows(N, r, cp))
        desc = Descales(k=ks, v=vs)
        o, l = ring_forward(q[rows].cuda(), lambda s, r=r: (k8[(r - s) % cp], v8[(r - s) % cp]),
                            lambda s: None, RingConfig(cp_size=cp, cp_rank=r), cu=cu,
                            nseq=1, max_seqlen=T, descales=desc, return_lse=True)
        outs.append(to_np(o))
        lses.append(to_np(l))
    got = orc.zigzag_unshard(outs, cp)
    got_l = orc.zigzag_unshard(lses, cp)
    want, want_l = orc.dense_causal(to_np(q), orc.zigzag_unshard(kd, cp), orc.zigzag_unshard(vd, cp),
                                    1.0 / math.sqrt(D))
    np.testing.assert_allclose(got, want, atol=6e-2, rtol=0)
    np.testing.assert_allclose(got_l, want_l, atol=1e-3, rtol=0)
    assert_device_ok()
