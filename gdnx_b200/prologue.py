"""Host-side parameters of the fused scan prologue.

The lane RoPE and braided decay are computed INSIDE the CUDA kernels; this
module only derives the per-lane constants the reference bakes into its
tables, following ``GDN3LinearAttn._lane_rope_factors``
(gdn3/gdn3_upgrade.py:342-376) and the braided-decay constants
(gdn3/gdn3_upgrade.py:127-129, 80).
"""
from __future__ import annotations

from dataclasses import dataclass

LANE_ROPE_FRACTIONS = (0.50, 0.25, 0.50, 0.50)
LANE_ROPE_SCALES = (1.0, 0.3, 0.5, 0.2)
BRAID_RATES = (0.05, 0.02, 0.005, 0.001)
DECAY_CLAMP = 0.999


@dataclass(frozen=True)
class LaneRope:
    """Per-lane partial-RoPE constants: pair count, position scale and the
    exponent denominator of ``inv_freq_i = 1 / 10000^(i / den)``.
    ``pairs = 0`` means the lane is not rotated."""
    pairs: tuple
    scale: tuple
    den: tuple
    pos0: int = 0


def lane_rope(M: int, K_dim: int, K_model: int | None = None, rotary_factor: float = 0.25,
              pos0: int = 0) -> LaneRope:
    """Constants for lanes ``0..M-1`` exactly as the reference's module builds them.

    * scale != 1: ``den = max(1, int(K_model*0.25)//2 - 1)``;
    * scale == 1: ``den = max(1, pairs-1)``; if ``pairs`` exceeds the module's
      cached table width ``int(K_model*rotary_factor)//2`` the reference uses
      cos = 1, sin = 0 (no rotation), encoded as ``pairs = 0``.
    """
    K_model = K_dim if K_model is None else K_model
    if M > 4:
        raise ValueError("lane RoPE is defined for at most 4 lanes")
    pairs, scale, den = [], [], []
    for m in range(M):
        frac, sc = LANE_ROPE_FRACTIONS[m], LANE_ROPE_SCALES[m]
        d = int(K_dim * frac // 2)
        dn = 1.0
        if d >= 1:
            if sc != 1.0:
                dn = float(max(1, int(K_model * 0.25) // 2 - 1))
            else:
                width = len(range(0, int(K_model * rotary_factor) // 2))
                if d > width:
                    d = 0
                else:
                    dn = float(max(1, d - 1))
        pairs.append(max(d, 0))
        scale.append(sc)
        den.append(dn)
    while len(pairs) < 4:
        pairs.append(0); scale.append(1.0); den.append(1.0)
    return LaneRope(tuple(pairs), tuple(scale), tuple(den), pos0)
