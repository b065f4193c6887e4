"""The benchmark's workload definitions (CPU): BASELINE configs, FLOP formulas and the
peak table -- what every bench line's `config`, `value` and `roofline` are computed from."""

import json
import os

import pytest

import bench
from oracle import bwd_oracle as bo
from oracle import ring_oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_configs_match_baseline_json():
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        text = json.dumps(json.load(f))
    # the headline configuration is cfg2: bf16, N=32768, Hq=32, Hkv=8, D=128
    c = bench.CONFIGS["cfg2"]
    assert (c["kind"], c["lens"], c["Hq"], c["Hkv"], c["D"]) == ("bf16", [32768], 32, 8, 128)
    assert "32768" in text and "131072" in text and "262144" in text
    assert bench.CONFIGS["cfg3"]["lens"] == [131072] and bench.CONFIGS["cfg3"]["kind"] == "e4m3"
    assert bench.CONFIGS["cfg5"]["D"] == 256 and bench.CONFIGS["cfg5"]["kind"] == "mixed"


@pytest.mark.parametrize("cp", [1, 2, 4, 8])
def test_varlen_config_is_seeded_and_divisible(cp):
    lens = bench.config_lens("cfg4", cp)
    assert len(lens) == 16 and lens == bench.config_lens("cfg4", cp)  # deterministic
    assert all(n % (2 * cp) == 0 and 1024 <= n <= 16384 + 2 * cp for n in lens)


def test_flop_formulas_agree_with_the_oracle():
    assert bench.causal_flops(32768, 32, 128) == orc.causal_flops([32768], 32, 128) == 2 * 32768 ** 2 * 32 * 128
    # the backward line counts 2.5x the forward (five matmuls against two)
    assert bo.bwd_flops([32768], 32, 128) == 2.5 * bench.causal_flops(32768, 32, 128)


def test_peaks_table():
    peaks, kind = bench.load_peaks()
    assert kind in ("measured", "fallback")
    assert peaks["bf16_tflops"] > 1000 and peaks["hbm_gbs"] > 5000


@pytest.mark.parametrize("lens,cp,rank", [([64], 2, 1), ([32, 96, 16], 4, 2)])
def test_bench_parity_checker_agrees_with_the_oracle(lens, cp, rank):
    """bench.sampled_parity (the bench line's `parity` key) on CPU tensors: fed the oracle's
    own rank output for the same seeded inputs, it reports errors at rounding level, and a
    planted error in one sampled row is reported."""
    import math
    import numpy as np
    import torch
    C = dict(kind="bf16", Hq=4, Hkv=2, D=32, amp=1.0)
    dev = torch.device("cpu")
    full_cu = [0] + [int(x) for x in np.cumsum(lens)]
    N = full_cu[-1]
    g = torch.Generator(device=dev).manual_seed(1234)
    q, k, v = (torch.randn(N, h, C["D"], generator=g, dtype=torch.bfloat16).float().numpy()
               for h in (C["Hq"], C["Hkv"], C["Hkv"]))
    scale = 1.0 / math.sqrt(C["D"])
    lq, lcu = orc.zigzag_shard_varlen(q, full_cu, rank, cp)
    ks = [orc.zigzag_shard_varlen(k, full_cu, r, cp)[0] for r in range(cp)]
    vs = [orc.zigzag_shard_varlen(v, full_cu, r, cp)[0] for r in range(cp)]
    o, l = orc.ring_rank(lq, ks, vs, rank, cp, scale, [int(c) for c in lcu], dtype=np.float64)
    res = bench.sampled_parity((torch.from_numpy(o), torch.from_numpy(l)), C, lens, rank, cp, dev,
                               None, 1)
    assert res["pass"] and res["max_abs_out"] < 1e-5 and res["max_abs_lse"] < 1e-5
    o[0, 1, 3] += 0.5  # local row 0 is always sampled
    res = bench.sampled_parity((torch.from_numpy(o), torch.from_numpy(l)), C, lens, rank, cp, dev,
                               None, 1)
    assert not res["pass"] and abs(res["max_abs_out"] - 0.5) < 1e-4
