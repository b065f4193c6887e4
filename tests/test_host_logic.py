"""Host-side logic of the drop-in API, on CPU: config validation, merger selection,
the ring schedule, descale normalisation, error mapping, and the no-fallback rule."""

import pytest
import torch

from oracle import ring_oracle as orc


def test_ring_config_validation_mirrors_reference():
    from fa4_ring import RingConfig
    RingConfig(cp_size=4, cp_rank=3)
    with pytest.raises(AssertionError):
        RingConfig(cp_size=4, cp_rank=4)
    with pytest.raises(AssertionError):
        RingConfig(cp_size=0, cp_rank=0)
    with pytest.raises(AssertionError):
        RingConfig(cp_size=2, cp_rank=0, merge_mode="nope")
    with pytest.raises(AssertionError):
        RingConfig(cp_size=2, cp_rank=0, causal=False)


def test_make_merger():
    from fa4_ring import BatchedMerger, IncrementalMerger, make_merger
    assert isinstance(make_merger("incremental"), IncrementalMerger)
    assert isinstance(make_merger("batched"), BatchedMerger)
    with pytest.raises(ValueError):
        make_merger("other")


@pytest.mark.parametrize("S", [1, 2, 3, 4, 8])
def test_ring_schedule_matches_oracle(S):
    from fa4_ring.ring_attention import ring_schedule
    for r in range(S):
        assert ring_schedule(r, S) == orc.ring_schedule(r, S)
    # every rank attends every source exactly once; S-1 transfers
    for r in range(S):
        assert sorted(src for _, src, _ in ring_schedule(r, S)) == list(range(S))


def test_schedule_balances_causal_work():
    # pairs per rank: step 0 (2h)^2/2 causal + (S-1) * 2h*h -> equal on every rank
    S, h = 4, 16
    works = []
    for r in range(S):
        w = 0
        for _, _, pat in orc.ring_schedule(r, S):
            w += (2 * h) * (2 * h + 1) // 2 if pat == orc.PATTERN_LOCAL_CAUSAL else 2 * h * h
        works.append(w)
    assert len(set(works)) == 1


def test_norm_descale_shapes():
    from fa4_ring.attn_backend import norm_descale
    assert norm_descale(None, 4, "cpu") is None
    assert norm_descale(torch.tensor(0.5), 4, "cpu").tolist() == [0.5] * 4
    assert norm_descale(torch.arange(4.0), 4, "cpu").tolist() == [0, 1, 2, 3]
    assert norm_descale(torch.ones(1, 4), 4, "cpu").shape == (4,)
    with pytest.raises(AssertionError):
        norm_descale(torch.ones(3), 4, "cpu")


def test_status_codes_map_to_reference_exceptions():
    from fa4_ring import _lib
    _lib.check(0, "ok")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")


def test_no_cpu_fallback():
    """CPU tensors are refused loudly instead of being computed on the host."""
    from fa4_ring import RingConfig, ring_flash_attn, zigzag_shard
    x = torch.zeros(8, 2, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        zigzag_shard(x, 0, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        ring_flash_attn(x.bfloat16(), x[:, :1].bfloat16(), x[:, :1].bfloat16(),
                        RingConfig(cp_size=1, cp_rank=0))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from fa4_ring import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="not built"):
        _lib.load()


def test_local_cu_args_validates_like_the_forward():
    import torch

    from fa4_ring.ring_attention import local_cu_args
    dev = torch.device("cpu")
    cu, nseq, mx = local_cu_args(8, dev, None, None)
    assert cu.tolist() == [0, 8] and nseq == 1 and mx == 8
    with pytest.raises(AssertionError, match="even"):
        local_cu_args(7, dev, None, None)
    with pytest.raises(AssertionError, match="max_seqlen"):
        local_cu_args(8, dev, torch.tensor([0, 4, 8], dtype=torch.int32), None)
    with pytest.raises(AssertionError, match="even"):
        local_cu_args(8, dev, torch.tensor([0, 3, 8], dtype=torch.int32), 5)
    cu, nseq, mx = local_cu_args(8, dev, torch.tensor([0, 2, 8]), 6)
    assert cu.dtype == torch.int32 and nseq == 2 and mx == 6


def test_backward_step_key_bounds():
    """The per-step key-count bound sizes the backward grid: half the local length for
    the front-half pattern, the whole length otherwise."""
    from fa4_ring.attn_backend import PATTERN_BACK_Q, PATTERN_FRONT_KV, PATTERN_VARLEN
    from fa4_ring.ring_backward import step_max_k
    assert step_max_k(PATTERN_VARLEN, 512) == 512
    assert step_max_k(PATTERN_BACK_Q, 512) == 512
    assert step_max_k(PATTERN_FRONT_KV, 512) == 256
    assert step_max_k(PATTERN_FRONT_KV, 514) == 257


def test_backward_argument_check_refuses_cpu_tensors():
    import torch

    from fa4_ring.ring_backward import _check_bwd
    t = torch.zeros(4, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _check_bwd(t, t, t, t, t, torch.zeros(4, 2))
