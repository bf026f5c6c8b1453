"""CPU restatements of the layer output epilogues (test infrastructure only).

* ``lane_route``     -- gdn3/gdn3_upgrade.py:842-856: router softmax over the
  lanes, lane-weighted sum, ``F.normalize(p=2, dim=-1, eps=1e-6) * sqrt(V) * norm``.
* ``rms_norm_gated`` -- ``Qwen3_5RMSNormGated.forward`` (transformers
  qwen3_5 modeling; called at gdn3/kmd2_native.py:176) in fp32.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def lane_route(y, router_logits, norm, gate=None):
    """y [B,T,H,M,V], router_logits [B,T,H,M], norm [V] -> [B,T,H,V] (fp32).  With ``gate``
    ([B,T,H,V]) also ``* F.silu(gate)``: gdn3/gdn3_upgrade.py:861-871 when H*V == D."""
    V = y.shape[-1]
    router_weights = F.softmax(router_logits.float(), dim=-1)
    routed = (router_weights.unsqueeze(-1) * y.float()).sum(dim=3)
    routed_normed = F.normalize(routed, p=2, dim=-1, eps=1e-6) * torch.sqrt(torch.tensor(float(V)))
    out = routed_normed * norm.float()
    return out if gate is None else out * F.silu(gate.float())


def rms_norm_gated(y, gate, weight, eps=1e-6):
    """fp32 gated RMS norm over the last dim."""
    h = y.float()
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    h = weight.float() * h
    return h * F.silu(gate.float())
