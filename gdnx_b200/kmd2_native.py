"""Drop-in forward of ``KMD2NativeAttn`` (gdn3/kmd2_native.py:134-183) on the sm_100a kernels.

The layer's GEMMs (``in_proj_qkv``, ``in_proj_z``, ``in_proj_b``, ``in_proj_a``, ``rot_proj``,
``out_proj``) stay torch linear layers; everything between them runs here:

* ``gdnx_kmd2_prologue``: causal conv + SiLU, q/k normalisation and query scale, beta_e /
  beta_w, the per-channel decay, the query-slot scales and the cumulative data-dependent
  rotation of k and the slots (gdn3/kmd2_native.py:140-172);
* the KMD-2 scan (``kmd2_fast_scan.scan``: the general tensor-core kernels);
* ``gdnx_epilogue`` (gated RMS norm, ``Qwen3_5RMSNormGated`` at :176).

The layer object supplies the reference's attribute names (``H``, ``dk``, ``dv``, ``r_out``, the
linear layers, ``conv1d.weight``, ``dt_bias``, ``A_log``, ``decay_chan``, ``bw_off``,
``q_slot_scale``, ``out_mix``, ``norm.weight`` / ``norm.variance_epsilon``).  Inference only: the
prologue and the norm have no backward here, so the call raises under autograd (train through
the reference forward with the scan drop-in, whose backward is ``gdnx_scan_bwd``).  CUDA tensors
only; there is no CPU fallback.
"""
from __future__ import annotations

import types

import torch

from . import kmd2_fast_scan, ops


def kmd2_forward(layer, hidden_states: torch.Tensor, attention_mask=None, **kwargs) -> torch.Tensor:
    """Signature of ``KMD2NativeAttn.forward`` (gdn3/kmd2_native.py:134-135)."""
    if torch.is_grad_enabled() and (hidden_states.requires_grad or
                                    any(p.requires_grad for p in layer.parameters())):
        raise RuntimeError("gdnx_b200.kmd2_native: the fused forward is inference-only (use torch.no_grad())")
    x = hidden_states
    B, T, _ = x.shape
    H, dk, dv, r_out = int(layer.H), int(layer.dk), int(layer.dv), int(layer.r_out)
    mixed = layer.in_proj_qkv(x)
    z = layer.in_proj_z(x)
    b = layer.in_proj_b(x)
    a = layer.in_proj_a(x)
    theta = layer.rot_proj(x)
    q, k, v, g, be, bw = ops.kmd2_prologue(mixed, layer.conv1d.weight, b, a, theta, H=H, dt_bias=layer.dt_bias,
                                           A_log=layer.A_log, decay_chan=layer.decay_chan, bw_off=layer.bw_off,
                                           q_slot_scale=layer.q_slot_scale if r_out > 1 else None, r_out=r_out,
                                           dk=dk, dv=dv)
    y = kmd2_fast_scan.scan(q, k, v, g, be, bw, layer.out_mix if r_out > 1 else None)  # [B,T,H,dv]
    # Qwen3_5RMSNormGated on y cast to z's dtype, output in that dtype
    y = ops.rms_norm_gated(y.to(z.dtype), z.view(B, T, H, dv), layer.norm.weight, eps=layer.norm.variance_epsilon,
                           out_dtype=z.dtype)
    out = layer.out_proj(y.reshape(B, T, H * dv))
    if attention_mask is not None:
        if attention_mask.ndim == 2:
            attention_mask = attention_mask.unsqueeze(-1)
        out = out * attention_mask
    return out


class KMD2ForwardMixin:
    """Put first in the bases of a ``KMD2NativeAttn`` subclass to run its forward here."""
    forward = kmd2_forward


def patch_layer(layer):
    """Bind the fused forward to an existing ``KMD2NativeAttn`` instance (returns it)."""
    layer.forward = types.MethodType(kmd2_forward, layer)
    return layer
