"""Drop-in replacement of ``gdn3.kmd2_fast_scan`` (gdn3/kmd2_fast_scan.py:163-282).

``scan(q, k, v, g, beta_e, beta_w, out_mix=None)`` and
``scan_with_update_norm(...) -> (y, scores)`` keep the reference's exact
argument names and single ``None`` default (pinned by
tests/ablation/test_fast_scan_api.py:13,30-39 in the reference).  They are plain
functions calling the sm_100a kernels -- no ``torch.compile``, no Triton.

Shapes (research/kernel_ab/ref_scan.py:8-18): q [B,T,H,r_out,dk], k/g
[B,T,H,dk] (g per key channel), v [B,T,H,dv], beta_e/beta_w [B,T,H],
out_mix [H,r_out] when r_out > 1.  Returns y [B,T,H,dv] fp32; scores
[B,T,H] = |k| |beta_w v - beta_e k^T S| (detached), as
research/kmd2_ablation/exact_cache.py:1283-1292.  Under autograd the backward runs
on the exact fp32 backward kernel (``gdnx_scan_bwd``).
"""
from __future__ import annotations

import torch

from . import ops


def _scan_core(q, k, v, g, beta_e, beta_w, out_mix=None, *, return_scores):
    r_out = q.shape[3]
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                       for t in (q, k, v, g, beta_e, beta_w, out_mix)):
        # training: the exact fp32 backward kernel (gdnx_scan_bwd) behind autograd
        mix = out_mix if r_out > 1 else None
        if return_scores:
            return ops.kmd2_scan_train(q, k, v, g, beta_e, beta_w, mix, scores=True)
        return ops.kmd2_scan_train(q, k, v, g, beta_e, beta_w, mix), None
    mix = out_mix if r_out > 1 else None
    if return_scores:
        y, sc = ops.kmd2_scan(q, k, v, g, beta_e, beta_w, mix, scores=True)
        return y, sc.detach()
    return ops.kmd2_scan(q, k, v, g, beta_e, beta_w, mix), None


def _scan_impl(q, k, v, g, beta_e, beta_w, out_mix=None):
    y, _ = _scan_core(q, k, v, g, beta_e, beta_w, out_mix, return_scores=False)
    return y


def _scan_with_update_norm_impl(q, k, v, g, beta_e, beta_w, out_mix=None):
    return _scan_core(q, k, v, g, beta_e, beta_w, out_mix, return_scores=True)


def scan(q, k, v, g, beta_e, beta_w, out_mix=None):
    """Chunk-parallel KMD-2 scan replacement (gdn3/kmd2_fast_scan.py:281)."""
    return _scan_impl(q, k, v, g, beta_e, beta_w, out_mix)


def scan_with_update_norm(q, k, v, g, beta_e, beta_w, out_mix=None):
    """Scan plus per-token update-norm scores (gdn3/kmd2_fast_scan.py:282)."""
    return _scan_with_update_norm_impl(q, k, v, g, beta_e, beta_w, out_mix)
