"""Dense single-device references for validating the ring output
(mirrors ``fa4_ring/reference.py:20-54``).

``full_causal_reference`` computes ordinary causal attention over the whole
sequence.  Backends:

* ``"torch"`` -- ``scaled_dot_product_attention`` in fp32 with GQA expanded
  (the reference's math ground truth); a test/validation utility, not used by the
  ring itself;
* ``"b200"``  -- the same sm_100a kernel the ring uses, for an apples-to-apples
  comparison (the reference's ``"fa4"`` backend; ``"fa4"`` is accepted as an alias).
"""

import math
from typing import Optional

import torch
import torch.nn.functional as F


def _expand_kv(k: torch.Tensor, v: torch.Tensor, n_q_heads: int):
    """Expand [T, H_kv, D] -> [T, H_q, D] for GQA/MQA."""
    h_kv = k.shape[1]
    if h_kv == n_q_heads:
        return k, v
    assert n_q_heads % h_kv == 0, f"H_q={n_q_heads} not a multiple of H_kv={h_kv}"
    rep = n_q_heads // h_kv
    return k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)


def full_causal_reference(
    q: torch.Tensor,  # [N, H, D]
    k: torch.Tensor,  # [N, H_kv, D]
    v: torch.Tensor,  # [N, H_kv, D]
    softmax_scale: Optional[float] = None,
    backend: str = "torch",
) -> torch.Tensor:
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    if backend in ("b200", "fa4"):
        from .attn_backend import b200_attn

        out, _ = b200_attn(q, k, v, causal=True, softmax_scale=softmax_scale)
        return out
    assert backend == "torch", f"unknown backend {backend!r}"
    kq, vq = _expand_kv(k, v, q.shape[1])
    qt = q.transpose(0, 1).unsqueeze(0).float()
    kt = kq.transpose(0, 1).unsqueeze(0).float()
    vt = vq.transpose(0, 1).unsqueeze(0).float()
    out = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, scale=softmax_scale)
    return out.squeeze(0).transpose(0, 1).contiguous().to(q.dtype)
