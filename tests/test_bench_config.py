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
