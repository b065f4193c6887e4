"""torchrun worker of test_gpu_ring.test_nccl_ring_multi_gpu: the real NCCL ring
(``ring_flash_attn``) on every rank, outputs gathered and checked on rank 0 against the
oracle's dense causal attention, for both merge modes, single and packed sequences."""

import datetime
import math
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fa4-cp_b200")]

from fa4_ring import RingConfig, ring_flash_attn, zigzag_shard  # noqa: E402
from fa4_ring.zigzag import zigzag_shard_varlen, zigzag_unshard, zigzag_unshard_varlen  # noqa: E402
from oracle import ring_oracle as orc  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    from fa4_ring.comm import nccl_pg_options
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            pg_options=nccl_pg_options())
    dev = torch.device("cuda")
    ok = True
    try:
        H, Hkv, D = 8, 2, 128
        scale = 1.0 / math.sqrt(D)
        for num_seqs in (1, 3):
            g = torch.Generator().manual_seed(1234)
            lens = [2 * world * 96] if num_seqs == 1 else [2 * world * n for n in (64, 16, 80)]
            cu = [0] + list(np.cumsum(lens))
            N = cu[-1]
            q, k, v = (torch.randn(N, h, D, generator=g).bfloat16().to(dev) for h in (H, Hkv, Hkv))
            for mode in ("incremental", "batched"):
                cfg = RingConfig(cp_size=world, cp_rank=rank, merge_mode=mode)
                if num_seqs == 1:
                    lq, lk, lv = (zigzag_shard(t, rank, world) for t in (q, k, v))
                    out = ring_flash_attn(lq, lk, lv, cfg)
                else:
                    lq, lcu = zigzag_shard_varlen(q, cu, rank, world)
                    lk, _ = zigzag_shard_varlen(k, cu, rank, world)
                    lv, _ = zigzag_shard_varlen(v, cu, rank, world)
                    out = ring_flash_attn(lq, lk, lv, cfg, cu_seqlens=lcu,
                                          max_seqlen=max(lens) // world)
                gathered = [torch.empty_like(out) for _ in range(world)]
                dist.all_gather(gathered, out.contiguous())
                if rank == 0:
                    full = (zigzag_unshard(gathered, world) if num_seqs == 1
                            else zigzag_unshard_varlen(gathered, cu, world))
                    full = full.float().cpu().numpy()
                    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
                    for j in range(len(lens)):
                        a, b = cu[j], cu[j + 1]
                        ref, _ = orc.dense_causal(qn[a:b], kn[a:b], vn[a:b], scale)
                        err = float(np.abs(full[a:b] - ref).max())
                        print(f"world={world} seqs={num_seqs} mode={mode} seq{j} max_err={err:.3e}")
                        ok &= err <= 2e-2
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    if rank == 0:
        print("RING_OK" if ok else "RING_FAIL")
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
