"""Ring backward.

CPU (gloo, world 2..4): the host schedule of ``ring_backward_accumulate`` -- the K/V
rotation (KVRing) and the rotating fp32 dK/dV accumulators (GradRing) -- with each step's
gradient computed by the oracle instead of the CUDA kernel, against the oracle's ring
backward.  Checks that every rank ends with dQ of its rows and the complete dK/dV of its own
K/V after exactly S passes.

GPU: ``fa4cp_attn_bwd`` per step pattern against the oracle (bf16 / f16, D 64 / 128, GQA,
ragged and packed sequences), the ring backward of cp = 2 / 4 emulated on one GPU, and
autograd through ``ring_flash_attn``.  Tolerance: max |err| <= 2e-2 * max(1, max |ref|)
(bf16 P and dS feed the tensor cores; a CPU emulation of the kernel's rounding gives about
3e-3), 1e-2 for f16.
"""

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import bwd_oracle as bo
from oracle import ring_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(lens, H, Hkv, D, seed):
    rng = np.random.default_rng(seed)
    N = int(sum(lens))
    q, dout = rng.standard_normal((N, H, D)), rng.standard_normal((N, H, D))
    k, v = rng.standard_normal((N, Hkv, D)), rng.standard_normal((N, Hkv, D))
    return q, k, v, dout


def _dense_stats(q, k, v, full_cu, scale):
    out = np.zeros(q.shape)
    lse = np.zeros(q.shape[:2])
    for a, b in zip(full_cu[:-1], full_cu[1:]):
        out[a:b], lse[a:b] = orc.attn(q[a:b], k[a:b], v[a:b], True, scale, np.float64)
    return out, lse


def _dense_grads(q, k, v, dout, full_cu, scale):
    g = [np.zeros(x.shape) for x in (q, k, v)]
    for a, b in zip(full_cu[:-1], full_cu[1:]):
        for acc, x in zip(g, bo.attn_bwd(q[a:b], k[a:b], v[a:b], dout[a:b], True, scale)):
            acc[a:b] = x
    return g


def _oracle_step(q, k, v, dout, lse, delta, dq_acc, dk_acc, dv_acc, cu, *, nseq, max_seqlen_k,
                 pattern, causal, softmax_scale):
    """CPU stand-in for the kernel, for the host-logic test only."""
    assert causal == (pattern == orc.PATTERN_LOCAL_CAUSAL)
    dq, dk, dv = bo.ring_step_bwd(q.numpy(), k.numpy(), v.numpy(), dout.numpy(), lse.numpy(),
                                  delta.numpy(), [int(c) for c in cu.tolist()], pattern,
                                  softmax_scale)
    dq_acc += torch.from_numpy(dq).float()
    dk_acc += torch.from_numpy(dk).float()
    dv_acc += torch.from_numpy(dv).float()


def _gloo_worker(rank, world, port, args):
    import sys
    sys.path[:0] = args["paths"]
    from fa4_ring.config import RingConfig
    from fa4_ring.ring_backward import ring_backward_accumulate
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        lens, H, Hkv, D = args["lens"], 4, 2, 8
        full_cu = [0] + [int(x) for x in np.cumsum(lens)]
        q, k, v, dout = _problem(lens, H, Hkv, D, seed=11)
        scale = 1.0 / math.sqrt(D)
        out, lse = _dense_stats(q, k, v, full_cu, scale)
        shard = lambda x: orc.zigzag_shard_varlen(x, full_cu, rank, world)[0]  # noqa: E731
        lcu = orc.zigzag_shard_varlen(q, full_cu, rank, world)[1]
        lq, lk, lv, ldo = (torch.from_numpy(shard(x)) for x in (q, k, v, dout))
        llse = torch.from_numpy(shard(lse))
        delta = torch.from_numpy(bo.row_delta(shard(out), shard(dout)))
        cfg = RingConfig(cp_size=world, cp_rank=rank)
        dq, dkv = ring_backward_accumulate(
            lq, lk, lv, ldo, llse, delta, cfg, cu=torch.from_numpy(lcu), nseq=len(lens),
            max_seqlen=int(max(np.diff(lcu))), softmax_scale=scale, step_fn=_oracle_step,
            add_fn=lambda dst, src: dst.add_(src))
        want = _dense_grads(q, k, v, dout, full_cu, scale)
        for name, got, w in (("dq", dq, want[0]), ("dk", dkv[0], want[1]), ("dv", dkv[1], want[2])):
            np.testing.assert_allclose(got.numpy(), shard(w), atol=1e-4, rtol=1e-4,
                                       err_msg=f"rank {rank} {name}")
        assert float(lk[0, 0, 0]) == float(shard(k)[0, 0, 0])  # inputs untouched
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,lens", [(2, [16]), (3, [24, 12]), (4, [16, 40, 8])])
def test_ring_backward_schedule_gloo(world, lens):
    import sys
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker,
                         args=(r, world, port, {"paths": sys.path[:3], "lens": lens}))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes


def test_backward_rejects_without_gpu_path():
    """No CPU fallback: the public backward refuses CPU tensors."""
    from fa4_ring.config import RingConfig
    from fa4_ring.ring_backward import ring_flash_attn_backward
    t = torch.zeros(8, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ring_flash_attn_backward(t, t, t[:, :1], t[:, :1], t, torch.zeros(8, 2),
                                 RingConfig(cp_size=1, cp_rank=0))


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------

def _tol(dtype):
    return 2e-2 if dtype == torch.bfloat16 else 1e-2


def _check(name, got, want, dtype):
    got = got.float().cpu().numpy() if torch.is_tensor(got) else got
    mag = max(1.0, float(np.abs(want).max()))
    err = float(np.abs(got - want).max())
    assert err <= _tol(dtype) * mag, f"{name}: max err {err:.3e} (max |ref| {mag:.3e})"


STEP_CASES = [
    # (lens (local, per sequence), H, Hkv, D, pattern, causal, dtype)
    ([256], 4, 2, 128, 0, True, torch.bfloat16),
    ([200], 2, 2, 64, 0, True, torch.bfloat16),
    ([130, 62, 300], 4, 1, 128, 0, True, torch.float16),
    ([256, 96], 8, 2, 128, 1, False, torch.bfloat16),
    ([256, 96], 8, 2, 128, 2, False, torch.bfloat16),
    ([34, 512], 2, 1, 64, 1, False, torch.float16),
    ([34, 512], 2, 1, 64, 2, False, torch.bfloat16),
    ([0, 64, 0], 2, 2, 64, 0, True, torch.bfloat16),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", STEP_CASES)
def test_gpu_bwd_step_matches_oracle(case):
    from fa4_ring.ring_backward import bwd_delta, bwd_step, step_max_k
    lens, H, Hkv, D, pattern, causal, dtype = case
    cu = [0] + [int(x) for x in np.cumsum(lens)]
    T = cu[-1]
    q, k, v, dout = _problem(lens if T else [1], H, Hkv, D, seed=3)
    q, k, v, dout = (x[:T] for x in (q, k, v, dout))
    # rounding to the input dtype first: the oracle sees the values the kernel sees
    tq, tk, tv, tdo = (torch.from_numpy(x).to(dtype) for x in (q, k, v, dout))
    q, k, v, dout = (t.double().numpy() for t in (tq, tk, tv, tdo))
    scale = 1.0 / math.sqrt(D)
    # final statistics: the local causal attention merged with this step's partial (for the
    # remote patterns), so that the step's P <= 1 as in a real ring
    out, lse = _dense_stats(q, k, v, cu, scale)
    if pattern != 0:
        o_s, l_s = orc.ring_step(q, k, v, cu, pattern, scale, np.float64)
        out, lse = orc.merge(out, lse, o_s, l_s)
    tout = torch.from_numpy(out).to(dtype)
    delta_ref = bo.row_delta(tout.double().numpy(), dout)
    dev = torch.device("cuda")
    gq, gk, gv, gdo, gout = (t.to(dev) for t in (tq, tk, tv, tdo, tout))
    glse = torch.from_numpy(lse).float().to(dev)
    gcu = torch.tensor(cu, dtype=torch.int32, device=dev)
    delta = bwd_delta(gout, gdo)
    _check("delta", delta, delta_ref, torch.float16)
    dq = torch.zeros((T, H, D), dtype=torch.float32, device=dev)
    dk = torch.zeros((T, Hkv, D), dtype=torch.float32, device=dev)
    dv = torch.zeros((T, Hkv, D), dtype=torch.float32, device=dev)
    max_len = max(lens)
    bwd_step(gq, gk, gv, gdo, glse, delta, dq, dk, dv, gcu, nseq=len(lens),
             max_seqlen_k=step_max_k(pattern, max_len), pattern=pattern, causal=causal,
             softmax_scale=scale)
    torch.cuda.synchronize()
    if pattern == 0:
        want = bo.attn_bwd_varlen(q, k, v, dout, lse, delta_ref, cu, cu, causal, scale)
    else:
        want = bo.ring_step_bwd(q, k, v, dout, lse, delta_ref, cu, pattern, scale)
    for name, got, w in zip(("dq", "dk", "dv"), (dq, dk, dv), want):
        _check(name, got, w, dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("cp,lens,H,Hkv,D", [(2, [512], 4, 2, 128), (4, [256, 768], 4, 1, 64)])
def test_gpu_ring_backward_emulated(cp, lens, H, Hkv, D):
    """Every rank's ring backward on one GPU: each rank's steps through ``fa4cp_attn_bwd``,
    dK/dV contributions summed per source as the rotating accumulators do."""
    from fa4_ring.attn_backend import PATTERN_VARLEN
    from fa4_ring.ring_attention import ring_schedule
    from fa4_ring.ring_backward import acc_add, acc_to, bwd_delta, bwd_step, step_max_k
    dtype = torch.bfloat16
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    q, k, v, dout = _problem(lens, H, Hkv, D, seed=9)
    tq, tk, tv, tdo = (torch.from_numpy(x).to(dtype) for x in (q, k, v, dout))
    q, k, v, dout = (t.double().numpy() for t in (tq, tk, tv, tdo))
    scale = 1.0 / math.sqrt(D)
    out, lse = _dense_stats(q, k, v, full_cu, scale)
    want = _dense_grads(q, k, v, dout, full_cu, scale)
    dev = torch.device("cuda")
    shard = lambda x, r: orc.zigzag_shard_varlen(x, full_cu, r, cp)[0]  # noqa: E731
    rows = [torch.from_numpy(orc.zigzag_varlen_rows(full_cu, r, cp)[0]).to(dev)
            for r in range(cp)]
    lcu_np = orc.zigzag_shard_varlen(q, full_cu, 0, cp)[1]
    lcu = torch.tensor(lcu_np, dtype=torch.int32, device=dev)
    max_len = int(max(np.diff(lcu_np)))
    gq, gk, gv, gdo = (t.to(dev) for t in (tq, tk, tv, tdo))
    gout = torch.from_numpy(out).to(dtype).to(dev)
    glse = torch.from_numpy(lse).float().to(dev)
    ks = [gk[rows[r]].contiguous() for r in range(cp)]
    vs = [gv[rows[r]].contiguous() for r in range(cp)]
    dkv = [torch.zeros((2,) + tuple(ks[0].shape), dtype=torch.float32, device=dev)
           for _ in range(cp)]
    for rank in range(cp):
        lq, ldo, lout = (t[rows[rank]].contiguous() for t in (gq, gdo, gout))
        llse = glse[rows[rank]].contiguous()
        delta = bwd_delta(lout, ldo)
        dq = torch.zeros(lq.shape, dtype=torch.float32, device=dev)
        for step, src, pattern in ring_schedule(rank, cp):
            part = torch.zeros_like(dkv[src])
            bwd_step(lq, ks[src], vs[src], ldo, llse, delta, dq, part[0], part[1], lcu,
                     nseq=len(lens), max_seqlen_k=step_max_k(pattern, max_len),
                     pattern=pattern, causal=(step == 0), softmax_scale=scale)
            acc_add(dkv[src], part)
            assert (pattern == PATTERN_VARLEN) == (step == 0)
        _check(f"dq rank {rank}", acc_to(dq, dtype), shard(want[0], rank), dtype)
    for r in range(cp):
        _check(f"dk rank {r}", acc_to(dkv[r][0], dtype), shard(want[1], r), dtype)
        _check(f"dv rank {r}", acc_to(dkv[r][1], dtype), shard(want[2], r), dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gpu_autograd_through_ring_flash_attn(dtype):
    """cp = 1: ``ring_flash_attn`` records the backward; grads match the oracle."""
    from fa4_ring import RingConfig, ring_flash_attn
    lens, H, Hkv, D = [384], 4, 2, 128
    q, k, v, dout = _problem(lens, H, Hkv, D, seed=21)
    dev = torch.device("cuda")
    tq, tk, tv, tdo = (torch.from_numpy(x).to(dtype).to(dev) for x in (q, k, v, dout))
    q, k, v, dout = (t.double().cpu().numpy() for t in (tq, tk, tv, tdo))
    for t in (tq, tk, tv):
        t.requires_grad_(True)
    out = ring_flash_attn(tq, tk, tv, RingConfig(cp_size=1, cp_rank=0))
    assert out.requires_grad
    out.backward(tdo)
    want = bo.attn_bwd(q, k, v, dout, True, 1.0 / math.sqrt(D))
    for name, t, w in zip(("dq", "dk", "dv"), (tq, tk, tv), want):
        assert t.grad is not None and t.grad.dtype == dtype
        _check(name, t.grad, w, dtype)


@pytest.mark.gpu
def test_gpu_backward_rejections():
    from fa4_ring import RingConfig
    from fa4_ring.ring_backward import ring_flash_attn_backward
    dev = torch.device("cuda")
    cfg = RingConfig(cp_size=1, cp_rank=0)
    t = torch.zeros(64, 2, 256, dtype=torch.bfloat16, device=dev)
    lse = torch.zeros(64, 2, device=dev)
    with pytest.raises(NotImplementedError):
        ring_flash_attn_backward(t, t, t, t, t, lse, cfg)  # head_dim 256
    t8 = torch.zeros(64, 2, 128, device=dev).to(torch.float8_e4m3fn)
    with pytest.raises(NotImplementedError):
        ring_flash_attn_backward(t8, t8, t8, t8, t8, lse, cfg)
    t = torch.zeros(64, 2, 128, dtype=torch.bfloat16, device=dev)
    with pytest.raises(NotImplementedError):
        ring_flash_attn_backward(t, t, t, t, t, lse,
                                 RingConfig(cp_size=1, cp_rank=0, deterministic=True))
