"""Drop-in replacement of the GDN3 recurrent scan of ``GDN3LinearAttn``.

The reference computes the recurrence in ``GDN3LinearAttn._gdn3_recurrent_state``
(gdn3/gdn3_upgrade.py:403-531; frozen semantics gdn3/_reference_recurrence.py:33-94).
This module provides the same method, with the same signature and the same
reads of the layer's attributes (``R``, ``P``, ``a_k``, ``b_k``, ``a_v``,
``b_v``, ``slow_decay``, ``compact_mode``), running on the sm_100a kernels:

* sequences shorter than the compaction period (``T < P``) never compact, so
  the residual buffer is exactly the dense state and the dense scan kernel
  runs (``gdnx_scan_fwd``);
* otherwise the Kronecker-residual kernel with in-kernel compaction runs
  (``gdnx_kr_scan_fwd``), by the layer's ``compact_mode`` ("svd", or "sketch" /
  "sketch_noqr": gdn3/gdn3_upgrade.py:81,579-596).  Its Gaussian sketch is the one
  the reference draws: ``torch.randn(N, b_v*b_k, q)`` from a CPU generator seeded
  1234 (gdn3/gdn3_upgrade.py:679-682 on a CPU layer; q = R in the sketch modes,
  :556-563), uploaded once per (N, q, device).

Use either :func:`patch_layer` on an existing reference layer, or
:class:`GDN3ScanMixin` as the first base of a subclass.  Under autograd,
sequences without compaction (T < P) backpropagate through the exact fp32
backward kernel (``gdnx_scan_bwd``); with compaction backward raises.  Inputs
must be CUDA tensors; there is no CPU fallback.
"""
from __future__ import annotations

import types
from typing import Dict, Tuple

import torch

from . import ops

_SKETCH_CACHE: Dict[Tuple, torch.Tensor] = {}


def reference_sketch(N: int, n: int, q: int, device) -> torch.Tensor:
    """G [N, n, q] exactly as the reference draws it (CPU generator, seed 1234)."""
    key = (N, n, q, str(device))
    G = _SKETCH_CACHE.get(key)
    if G is None:
        gen = torch.Generator(device="cpu").manual_seed(1234)
        G = torch.randn(N, n, q, generator=gen).to(device).contiguous()
        _SKETCH_CACHE[key] = G
    return G


class _NoGrad(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, *inputs):
        return y

    @staticmethod
    def backward(ctx, *grads):
        raise RuntimeError("gdnx_b200: the GDN3 scan kernels are forward-only; backward is not implemented")


def gdn3_recurrent_state(layer, q_features, k_features, v_features, b_gates, w_gates, decay_factors):
    """Signature of ``GDN3LinearAttn._gdn3_recurrent_state`` (gdn3/gdn3_upgrade.py:403-411).

    q/k/b [B,T,H,M,K], v/w [B,T,H,M,V], decay [B,T,H,M] -> Y [B,T,H,M,V] fp32.
    Also sets ``layer._last_comp_err`` (on device) like the reference
    (gdn3/gdn3_upgrade.py:523-528).
    """
    mode = str(getattr(layer, "compact_mode", "svd")).lower()
    if mode not in ("svd", "sketch", "sketch_noqr"):
        raise ValueError(f"gdnx_b200: unknown compact_mode {mode!r} (svd, sketch, sketch_noqr)")
    B, T, H, M, K = q_features.shape
    V = v_features.shape[-1]
    R, P = int(layer.R), int(layer.P)
    dims = (int(layer.a_v), int(layer.a_k), int(layer.b_v), int(layer.b_k))
    f32 = lambda x: x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
    args = [f32(t) for t in (q_features, k_features, v_features, b_gates, w_gates)]
    dec = f32(decay_factors)
    train = torch.is_grad_enabled() and any(t.requires_grad for t in (q_features, k_features, v_features, b_gates,
                                                                     w_gates, decay_factors))
    if T < P:
        if train:  # exact fp32 backward kernel behind autograd (no compaction reaches the outputs)
            y, _ = ops.gdn3_scan_train(*args, dec, decay_kind="gamma")
            layer._last_comp_err = torch.zeros((), device=y.device)
            return y
        y = ops.gdn3_scan(*args, dec, decay_kind="gamma", out_dtype=torch.float32)
        layer._last_comp_err = torch.zeros((), device=y.device)
    else:
        N = B * H * M
        G = reference_sketch(N, dims[2] * dims[3], ops.sketch_width(R, dims, mode), q_features.device)
        st = ops.KRState.zeros(N, R, P, dims, V, K, q_features.device)
        y = ops.gdn3_kr_scan(*args, dec, st, G, P=P, R=R, dims=dims, slow_decay=float(layer.slow_decay),
                             decay_kind="gamma", out_dtype=torch.float32, compact_mode=mode)
        layer._last_comp_err = st.err.sum().clamp(min=0.0)
    grads = [t for t in (q_features, k_features, v_features, b_gates, w_gates, decay_factors) if t.requires_grad]
    if torch.is_grad_enabled() and grads:
        y = _NoGrad.apply(y, *grads)
    return y


class GDN3ScanMixin:
    """Put first in the bases of a ``GDN3LinearAttn`` subclass to run its scan here."""
    _gdn3_recurrent_state = gdn3_recurrent_state


def patch_layer(layer):
    """Bind the sm_100a scan to an existing ``GDN3LinearAttn`` instance (returns it)."""
    layer._gdn3_recurrent_state = types.MethodType(gdn3_recurrent_state, layer)
    return layer
