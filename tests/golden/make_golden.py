"""Generate the golden fixtures that pin the oracle, by running the REFERENCE itself.

Usage (in a container that has the reference checkout; it never runs on the GPU box):

    python tests/golden/make_golden.py --reference <path-to-hxy0118/fa4-cp checkout>

It imports the reference's own CPU code -- ``fa4_ring/zigzag.py`` and the CPU ring
simulation in ``tests/test_algorithm_cpu.py`` -- runs it on seeded inputs generated
exactly as the reference's tests generate them (``torch.manual_seed(seed)`` then
``randn`` for q, k, v in that order, ``tests/test_algorithm_cpu.py:172-175,187-190``),
and writes the results as ``.npz`` fixtures next to this script.  Inputs are not
stored: tests regenerate them from the seed and check ``input_sums`` to detect RNG
drift.

Fixtures written:
  zigzag.npz   -- shard row indices, varlen local_cu, get_half_index vectors
  algo.npz     -- the reference's 7 single-sequence + 4 varlen cases: dense out/lse
                  (``cpu_attn``) and the ring simulation output (``simulate_ring``)
  steps.npz    -- one per-step partial for each ring pattern (``cpu_attn`` on the
                  pattern's rows), plus ``merge`` known answers incl. -inf rows
  cfg1.npz     -- BASELINE configs[0] (N=4096, Hq=8, Hkv=2, D=128, cp=4, seed 0):
                  sampled rows + checksums of the ring output and dense LSE
  gdn_meta.npz -- the GDN context-parallel index metadata of the reference's
                  ``fa4_ring/gdn_cp/metadata.py`` (``build_gdn_cp_metadata``): restore_perm,
                  extract_idx, full_cu_seqlens for every rank of GDN_CASES
                  (``--only gdn`` writes just this one)
  bwd.npz      -- gradients of the reference's dense forward
                  (``fa4_ring/reference.py:29-54``, ``full_causal_reference(backend="torch")``)
                  by torch autograd, for the ALGO_CASES shapes: q, k, v from seed 0 as above,
                  the upstream gradient ``randn(N, H, D)`` after ``manual_seed(1)``
                  (``--only bwd`` writes just this one).  The reference has no backward of
                  its own (README.md:142); these pin the backward oracle.
"""

import argparse
import importlib.util
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

ALGO_CASES = [  # tests/test_algorithm_cpu.py:202-211 (N, H, Hkv, D, cp)
    (16, 4, 4, 8, 2),
    (32, 8, 2, 16, 4),
    (64, 8, 8, 16, 4),
    (64, 4, 1, 32, 8),
    (128, 8, 2, 64, 8),
    (48, 6, 3, 16, 2),
    (96, 8, 8, 16, 4),
]
VARLEN_CASES = [  # tests/test_algorithm_cpu.py:217-223 (seq_lens, H, Hkv, D, cp)
    ([16, 32], 4, 4, 8, 2),
    ([32, 16, 48], 8, 2, 16, 4),
    ([64, 64], 4, 1, 16, 8),
    ([48, 24], 6, 3, 16, 2),
]


GDN_CASES = [  # (cp, full sequence lengths); the first three from tests/test_gdn_cp_cpu.py
    (4, [48]),
    (4, [32, 16, 48]),
    (8, [64, 64]),
    (2, [12]),
    (3, [6, 18, 30]),
    (8, [80, 16]),
]


def write_gdn(root):
    from fa4_ring.gdn_cp.metadata import build_gdn_cp_metadata  # the reference's module
    out = {}
    for ci, (cp, lens) in enumerate(GDN_CASES):
        out[f"c{ci}_lens"] = np.asarray(lens)
        out[f"c{ci}_cp"] = np.asarray(cp)
        for r in range(cp):
            m = build_gdn_cp_metadata(lens, cp, r)
            out[f"c{ci}_r{r}_restore"] = m.restore_perm.numpy()
            out[f"c{ci}_r{r}_extract"] = m.extract_idx.numpy()
            out[f"c{ci}_r{r}_cu"] = m.full_cu_seqlens.numpy()
    out["n_cases"] = np.asarray(len(GDN_CASES))
    p = os.path.join(HERE, "gdn_meta.npz")
    np.savez_compressed(p, **out)
    print(f"wrote {p} ({os.path.getsize(p)} bytes)")


def write_bwd(root):
    from fa4_ring.reference import full_causal_reference  # the reference's module
    out = {}
    for i, (n, H, Hkv, D, cp) in enumerate(ALGO_CASES):
        q, k, v = gen_inputs(n, H, Hkv, D)
        torch.manual_seed(1)
        dout = torch.randn(n, H, D)
        qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = full_causal_reference(qg, kg, vg, softmax_scale=1.0 / math.sqrt(D), backend="torch")
        dq, dk, dv = torch.autograd.grad(o, (qg, kg, vg), dout)
        out[f"case{i}_dims"] = np.asarray([n, H, Hkv, D, cp])
        out[f"case{i}_input_sums"] = np.asarray(
            [float(t.double().sum()) for t in (q, k, v, dout)])
        out[f"case{i}_dq"] = dq.numpy()
        out[f"case{i}_dk"] = dk.numpy()
        out[f"case{i}_dv"] = dv.numpy()
    out["n_cases"] = np.asarray(len(ALGO_CASES))
    p = os.path.join(HERE, "bwd.npz")
    np.savez_compressed(p, **out)
    print(f"wrote {p} ({os.path.getsize(p)} bytes)")


def load_reference(root):
    sys.path.insert(0, root)
    import fa4_ring.zigzag as zz  # the reference's module
    spec = importlib.util.spec_from_file_location(
        "ref_test_algorithm_cpu", os.path.join(root, "tests", "test_algorithm_cpu.py"))
    algo = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(algo)
    return zz, algo


def gen_inputs(n, H, Hkv, D, seed=0):
    torch.manual_seed(seed)
    return torch.randn(n, H, D), torch.randn(n, Hkv, D), torch.randn(n, Hkv, D)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    ap.add_argument("--only", choices=["gdn", "bwd"], default=None,
                    help="write one fixture only")
    args = ap.parse_args()
    zz, algo = load_reference(os.path.abspath(args.reference))
    if args.only in (None, "gdn"):
        write_gdn(os.path.abspath(args.reference))
    if args.only in (None, "bwd"):
        write_bwd(os.path.abspath(args.reference))
    if args.only is not None:
        return
    torch.set_num_threads(os.cpu_count() or 1)

    # ---------------- zig-zag known answers ----------------
    z = {}
    for cp in (1, 2, 3, 4, 8):
        for n in (2 * cp, 4 * cp * 3, 64 * cp):
            x = torch.arange(n).reshape(n, 1)
            for r in range(cp):
                z[f"shard_n{n}_cp{cp}_r{r}"] = zz.zigzag_shard(x, r, cp).flatten().numpy()
    varlen_cu = {
        "a": [0, 8, 24],
        "b": [0, 16, 48, 64, 128],
        "c": [0, 32],
        "d": [0, 48, 56, 120, 184, 200],
    }
    for name, cu in varlen_cu.items():
        for cp in (1, 2, 4):
            if any((cu[i + 1] - cu[i]) % (2 * cp) for i in range(len(cu) - 1)):
                continue
            total = cu[-1]
            x = torch.arange(total).reshape(total, 1)
            for r in range(cp):
                loc, lcu = zz.zigzag_shard_varlen(x, torch.tensor(cu, dtype=torch.int32), r, cp)
                z[f"varlen_{name}_cp{cp}_r{r}_rows"] = loc.flatten().numpy()
                z[f"varlen_{name}_cp{cp}_r{r}_cu"] = lcu.numpy()
                z[f"varlen_{name}_cp{cp}_r{r}_front"] = zz.get_half_index(lcu, front=True).numpy()
                z[f"varlen_{name}_cp{cp}_r{r}_back"] = zz.get_half_index(lcu, front=False).numpy()
        z[f"varlen_{name}_full_cu"] = np.asarray(cu, np.int32)
    np.savez_compressed(os.path.join(HERE, "zigzag.npz"), **z)

    # ---------------- algorithm cases (single sequence + varlen) ----------------
    a = {}
    for i, (n, H, Hkv, D, cp) in enumerate(ALGO_CASES):
        q, k, v = gen_inputs(n, H, Hkv, D)
        scale = 1.0 / math.sqrt(D)
        dense_o, dense_l = algo.cpu_attn(q, k, v, causal=True, scale=scale)
        ring_o = algo.simulate_ring(q, k, v, cp, scale)
        a[f"case{i}_dims"] = np.asarray([n, H, Hkv, D, cp])
        a[f"case{i}_input_sums"] = np.asarray([q.double().sum(), k.double().sum(), v.double().sum()])
        a[f"case{i}_dense_out"] = dense_o.numpy()
        a[f"case{i}_dense_lse"] = dense_l.numpy()
        a[f"case{i}_ring_out"] = ring_o.numpy()
    for i, (lens, H, Hkv, D, cp) in enumerate(VARLEN_CASES):
        torch.manual_seed(0)  # tests/test_algorithm_cpu.py:172-175
        seqs = [(torch.randn(n, H, D), torch.randn(n, Hkv, D), torch.randn(n, Hkv, D)) for n in lens]
        scale = 1.0 / math.sqrt(D)
        recon = algo.simulate_ring_varlen(seqs, cp, scale)
        a[f"varlen{i}_dims"] = np.asarray([H, Hkv, D, cp])
        a[f"varlen{i}_lens"] = np.asarray(lens)
        a[f"varlen{i}_input_sums"] = np.asarray(
            [sum(float(t.double().sum()) for t in s) for s in seqs])
        for j, r in enumerate(recon):
            a[f"varlen{i}_seq{j}_ring_out"] = r.numpy()
    np.savez_compressed(os.path.join(HERE, "algo.npz"), **a)

    # ---------------- per-step partials and merge known answers ----------------
    s = {}
    n, H, Hkv, D, cp = 64, 8, 2, 32, 4
    q, k, v = gen_inputs(n, H, Hkv, D, seed=3)
    scale = 1.0 / math.sqrt(D)
    s["dims"] = np.asarray([n, H, Hkv, D, cp])
    s["input_sums"] = np.asarray([q.double().sum(), k.double().sum(), v.double().sum()])
    rank, src = 2, 0
    h = n // (2 * cp)
    lq = zz.zigzag_shard(q, rank, cp)
    rk, rv = zz.zigzag_shard(k, src, cp), zz.zigzag_shard(v, src, cp)
    lk, lv = zz.zigzag_shard(k, rank, cp), zz.zigzag_shard(v, rank, cp)
    o0, l0 = algo.cpu_attn(lq, lk, lv, causal=True, scale=scale)          # step 0
    o1, l1 = algo.cpu_attn(lq, rk[:h], rv[:h], causal=False, scale=scale)  # src earlier
    o2, l2 = algo.cpu_attn(lq[h:], rk, rv, causal=False, scale=scale)      # src later
    s.update(rank=np.asarray(rank), src=np.asarray(src),
             local_causal_out=o0.numpy(), local_causal_lse=l0.numpy(),
             front_kv_out=o1.numpy(), front_kv_lse=l1.numpy(),
             back_q_out=o2.numpy(), back_q_lse=l2.numpy())
    g = torch.Generator().manual_seed(7)
    T, Hm, Dm = 37, 5, 24
    oa, ob = torch.randn(T, Hm, Dm, generator=g), torch.randn(T, Hm, Dm, generator=g)
    la, lb = torch.randn(T, Hm, generator=g) * 4, torch.randn(T, Hm, generator=g) * 4
    lb[::3] = float("-inf")  # uncovered rows, as a back-Q step produces
    mo, ml = algo.merge(oa, la, ob, lb)
    s.update(merge_oa=oa.numpy(), merge_ob=ob.numpy(), merge_la=la.numpy(), merge_lb=lb.numpy(),
             merge_out=mo.numpy(), merge_lse=ml.numpy())
    np.savez_compressed(os.path.join(HERE, "steps.npz"), **s)

    # ---------------- N=4096, Hq=8, Hkv=2, D=128, cp=4, seed 0 ----
    n, H, Hkv, D, cp = 4096, 8, 2, 128, 4
    q, k, v = gen_inputs(n, H, Hkv, D, seed=0)
    scale = 1.0 / math.sqrt(D)
    ring_o = algo.simulate_ring(q, k, v, cp, scale)
    _, dense_l = algo.cpu_attn(q, k, v, causal=True, scale=scale)
    rows = np.sort(np.random.default_rng(0).choice(n, 96, replace=False))
    np.savez_compressed(
        os.path.join(HERE, "cfg1.npz"),
        dims=np.asarray([n, H, Hkv, D, cp]),
        input_sums=np.asarray([q.double().sum(), k.double().sum(), v.double().sum()]),
        rows=rows, ring_out_rows=ring_o[rows].numpy(), dense_lse_rows=dense_l[rows].numpy(),
        ring_out_sum=np.asarray(ring_o.double().sum()),
        ring_out_abs_sum=np.asarray(ring_o.double().abs().sum()),
        dense_lse_sum=np.asarray(dense_l.double().sum()),
    )
    for f in ("zigzag", "algo", "steps", "cfg1"):
        p = os.path.join(HERE, f + ".npz")
        print(f"wrote {p} ({os.path.getsize(p)} bytes)")


if __name__ == "__main__":
    main()
