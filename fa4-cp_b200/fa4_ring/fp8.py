"""FP8 e4m3 helpers for the ring: per-rank quantisation and the per-source descale
all-gather (the step before ``ring_flash_attn`` with ``Descales``; the reference leaves
this to its callers, ``fa4_ring/ring_attention.py:43-52``, ``README.md:110-118``).

Recipe (the FP8 configs of the benchmark): each rank quantises its own shard with a
per-tensor ``scale = amax / 448``; the K and V scales of all ranks are all-gathered once,
so step ``s`` can use the descale of the source rank whose K/V it attends.
"""

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib


def quantize_e4m3(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor e4m3 quantisation on the GPU: returns ``(x_e4m3, scale)`` with
    ``x ~= x_e4m3.float() * scale`` and ``scale = amax(|x|) / 448`` (fp32 0-d tensor)."""
    _lib.require_cuda(x)
    x = x.contiguous()
    assert x.numel() % 2 == 0, "element count must be even"
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty((), dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().fa4cp_quantize_e4m3(x.data_ptr(), _lib.dtype_code(x.dtype), x.numel(),
                                               out.data_ptr(), scale.data_ptr(),
                                               _lib.stream_of(x)), "quantize_e4m3")
    _lib.count_launches(3)
    return out, scale


def dequantize_e4m3(x8: torch.Tensor, descale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``[T, H, D]`` e4m3 -> bf16 times a per-head (or scalar) descale."""
    from .attn_backend import norm_descale
    _lib.require_cuda(x8)
    assert x8.dim() == 3 and x8.dtype == torch.float8_e4m3fn
    x8 = x8.contiguous()
    d = norm_descale(descale, x8.shape[1], x8.device)
    out = torch.empty(x8.shape, dtype=torch.bfloat16, device=x8.device)
    _lib.check(_lib.load().fa4cp_dequant_e4m3(x8.data_ptr(), _lib.ptr(d), out.data_ptr(),
                                              x8.shape[0], x8.shape[1], x8.shape[2],
                                              _lib.stream_of(x8)), "dequant_e4m3")
    _lib.count_launches()
    return out


def allgather_descales(scale: torch.Tensor, group=None) -> List[torch.Tensor]:
    """All-gather one scale per rank (once, before the ring); entry ``r`` is rank ``r``'s."""
    world = dist.get_world_size(group)
    bufs = [torch.empty_like(scale) for _ in range(world)]
    dist.all_gather(bufs, scale.contiguous(), group=group)
    return bufs
