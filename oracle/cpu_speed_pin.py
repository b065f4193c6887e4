"""Pin the speed of the CPU restatement against the reference's own CPU ring code.

Test infrastructure (the timed CPU baseline's calibration), not product code.  ``bench.py``
times ``oracle/ring_oracle.py`` as the CPU baseline because the reference checkout does not
exist on the GPU box; this script, run where the checkout is present, times both on the same
sample and records the ratio in ``oracle/cpu_speed_pin.json`` so the baseline can be read as
a multiple of the reference's own CPU speed.

Sample: rank 0's eight ring steps of cfg2 at cp=8 (T = 4096 local tokens, D = 128), with 8 of
the 32 query heads and 2 kv heads (cfg2's 4:1 GQA ratio; the reference materialises
[H, Tq, Tk] fp32 scores, 2 GiB per tensor for all 32 heads), fp32, seed 0, every host thread
for both (torch intra-op threads for the reference, the BLAS pool for the port).

Reference side: ``cpu_attn`` and ``merge`` of the reference's ``tests/test_algorithm_cpu.py``
(:36-59) and its ``fa4_ring/zigzag.zigzag_shard``, driven exactly as its ``simulate_ring``
(:62-90) drives them for one rank: step 0 local causal, then for r > rank the late-half rows
against the whole source shard, scattered into zero / -inf staging and merged.

Usage:  python oracle/cpu_speed_pin.py --reference <path-to-hxy0118/fa4-cp checkout>
"""

import argparse
import importlib.util
import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

N, HQ, HKV, D, CP, RANK = 32768, 8, 2, 128, 8, 0


def load_reference(root):
    sys.path.insert(0, root)
    import fa4_ring.zigzag as zz  # the reference's module
    spec = importlib.util.spec_from_file_location(
        "ref_test_algorithm_cpu", os.path.join(root, "tests", "test_algorithm_cpu.py"))
    algo = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(algo)
    return zz, algo


def time_reference(zz, algo, q, k, v, scale):
    """One rank of the reference's simulate_ring (tests/test_algorithm_cpu.py:68-89)."""
    h = N // (2 * CP)
    t0 = time.perf_counter()
    lq = zz.zigzag_shard(q, RANK, CP)
    acc_out, acc_lse = algo.cpu_attn(lq, zz.zigzag_shard(k, RANK, CP),
                                     zz.zigzag_shard(v, RANK, CP), causal=True, scale=scale)
    for r in range(1, CP):
        src = (RANK - r) % CP
        rk, rv = zz.zigzag_shard(k, src, CP), zz.zigzag_shard(v, src, CP)
        if r > RANK:
            o, l = algo.cpu_attn(lq[h:], rk, rv, causal=False, scale=scale)
            out_full = torch.zeros(2 * h, HQ, D)
            lse_full = torch.full((2 * h, HQ), float("-inf"))
            out_full[h:] = o
            lse_full[h:] = l
            acc_out, acc_lse = algo.merge(acc_out, acc_lse, out_full, lse_full)
        else:
            o, l = algo.cpu_attn(lq, rk[:h], rv[:h], causal=False, scale=scale)
            acc_out, acc_lse = algo.merge(acc_out, acc_lse, o, l)
    return time.perf_counter() - t0, acc_out.numpy(), acc_lse.numpy()


def time_port(q, k, v, scale):
    """The same rank through oracle/ring_oracle.py, as bench.py's cpu_sample runs it."""
    sys.path.insert(0, ROOT)
    from oracle import ring_oracle as orc
    qn, kn, vn = (x.numpy() for x in (q, k, v))
    t0 = time.perf_counter()
    lq = orc.zigzag_shard(qn, RANK, CP)
    ks = [orc.zigzag_shard(kn, r, CP) for r in range(CP)]
    vs = [orc.zigzag_shard(vn, r, CP) for r in range(CP)]
    T = lq.shape[0]
    acc = None
    for (_step, src, pat) in orc.ring_schedule(RANK, CP):
        o, l = orc.ring_step(lq, ks[src], vs[src], [0, T], pat, scale)
        acc = (o, l) if acc is None else orc.merge(acc[0], acc[1], o, l)
    return time.perf_counter() - t0, acc[0], acc[1]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    ap.add_argument("--repeats", type=int, default=2)
    a = ap.parse_args()
    from threadpoolctl import threadpool_limits
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    threadpool_limits(limits=threads)
    zz, algo = load_reference(a.reference)
    torch.manual_seed(0)
    q, k, v = torch.randn(N, HQ, D), torch.randn(N, HKV, D), torch.randn(N, HKV, D)
    scale = 1.0 / math.sqrt(D)
    T = N // CP
    flops = CP * 2.0 * T * T * HQ * D  # bench.py's count: 2*T^2*Hq*D per step
    t_ref = min(time_reference(zz, algo, q, k, v, scale)[0] for _ in range(a.repeats))
    t_port = min(time_port(q, k, v, scale)[0] for _ in range(a.repeats))
    _, ro, rl = time_reference(zz, algo, q, k, v, scale)
    _, po, pl = time_port(q, k, v, scale)
    res = {
        "sample": f"rank {RANK} of cfg2 at cp={CP}: all {CP} ring steps, T={T} local tokens, "
                  f"Hq={HQ} of 32 query heads, Hkv={HKV}, D={D}, fp32, seed 0",
        "threads": threads,
        "flop": flops,
        "reference_s": round(t_ref, 3), "port_s": round(t_port, 3),
        "reference_gflops": round(flops / t_ref / 1e9, 1),
        "port_gflops": round(flops / t_port / 1e9, 1),
        "port_over_reference": round(t_ref / t_port, 3),
        "max_abs_out_diff": float(np.abs(ro - po).max()),
        "max_abs_lse_diff": float(np.abs(rl - pl).max()),
        "reference_code": "tests/test_algorithm_cpu.py:36-59 (cpu_attn, merge) driven as "
                          "simulate_ring (:62-90); fa4_ring/zigzag.py:31-39 (zigzag_shard)",
    }
    path = os.path.join(HERE, "cpu_speed_pin.json")
    with open(path, "w") as f:
        json.dump(res, f, indent=1)
        f.write("\n")
    print(json.dumps(res))


if __name__ == "__main__":
    main()
