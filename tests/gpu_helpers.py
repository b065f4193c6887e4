"""Shared helpers of the GPU parity tests (inputs, oracle conversion, status check)."""

import numpy as np
import torch


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def randn(shape, dtype, gen, scale=1.0, device="cuda"):
    x = torch.randn(shape, generator=gen, dtype=torch.float32) * scale
    return x.to(dtype).to(device)


def quant_e4m3(x: torch.Tensor):
    """Per-tensor e4m3 quantisation, scale = amax / 448 (the FP8 recipe of the configs)."""
    amax = x.float().abs().max().clamp_min(1e-12)
    scale = (amax / 448.0).float()
    q = (x.float() / scale).to(torch.float8_e4m3fn)
    return q, scale


def dequant(q: torch.Tensor, scale) -> np.ndarray:
    return (q.float().cpu() * float(scale)).numpy()


def assert_device_ok():
    from fa4_ring import _lib
    assert _lib.device_status(clear=True) == 0, "a kernel gave up a bounded wait"
