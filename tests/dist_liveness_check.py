"""torchrun worker (2+ GPUs) of test_gpu_ring.test_ring_detects_a_departed_neighbour.

Every rank runs two native-executor ring forwards (copy-engine transport, the ring kernel)
and checks them against each other; then, with every kernel finished, the last rank leaves
between calls, without any collective clean-up.  Its neighbours' next ``ring_flash_attn``
must raise RuntimeError from the host-side liveness check (``fa4_ring.comm.RingLiveness``,
timeout set to 5 s here) before anything is queued on their GPU, and their GPU must still
answer afterwards.  No GPU fault, trap or hang is provoked: the leaver's GPU is idle when it
exits and no device-side wait on it is ever queued.  Run with NCCL_NVLS_ENABLE=0.
"""

import datetime
import math
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fa4-cp_b200")]

import fa4_ring.comm as comm  # noqa: E402
from fa4_ring import RingConfig, ring_flash_attn, ring_attention, zigzag_shard  # noqa: E402
from fa4_ring.comm import nccl_pg_options  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            pg_options=nccl_pg_options())
    comm.RING_LIVENESS_TIMEOUT_S = 5.0
    ring_attention.RING_TRANSPORT = "copy_engine"
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(3)
    N, H, Hkv, D = 2 * world * 256, 4, 2, 128
    q, k, v = (torch.randn(N, h, D, generator=g).bfloat16().to(dev) for h in (H, Hkv, Hkv))
    lq, lk, lv = (zigzag_shard(t, rank, world) for t in (q, k, v))
    cfg = RingConfig(cp_size=world, cp_rank=rank, softmax_scale=1.0 / math.sqrt(D))
    a = ring_flash_attn(lq, lk, lv, cfg)
    b = ring_flash_attn(lq, lk, lv, cfg)
    ok = bool(torch.equal(a, b)) and bool(torch.isfinite(a.float()).all())
    torch.cuda.synchronize()
    dist.barrier()
    leaver = world - 1
    if rank == leaver:
        print(f"rank {rank}: leaving between calls", flush=True)
        os._exit(0)
    neighbour = rank in ((leaver - 1) % world, (leaver + 1) % world)
    try:
        ring_flash_attn(lq, lk, lv, cfg)
        raised = False
    except RuntimeError as e:
        raised = "neighbour rank" in str(e)
        print(f"rank {rank}: {e}", flush=True)
    torch.cuda.synchronize()  # this GPU still answers; nothing was left waiting on it
    x = torch.ones(1024, device=dev).sum().item()
    ok = ok and x == 1024.0 and (raised or not neighbour)
    print(("LIVENESS_OK" if ok else "LIVENESS_FAIL") + f" rank {rank}", flush=True)
    os._exit(0 if ok else 1)  # the group still counts the leaver: skip its teardown


if __name__ == "__main__":
    main()
