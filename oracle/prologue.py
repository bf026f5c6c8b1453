"""CPU restatement of the GDN3 scan prologue (test infrastructure only).

* ``braided_decay``   -- gdn3/gdn3_upgrade.py:809-822
* ``lane_rope_table`` -- gdn3/gdn3_upgrade.py:342-376 (``_lane_rope_factors``)
* ``apply_lane_rope`` -- gdn3/gdn3_upgrade.py:378-401 (``_apply_partial_rope``)
"""
from __future__ import annotations

import torch

LANE_ROPE_FRACTIONS = (0.50, 0.25, 0.50, 0.50)   # gdn3/gdn3_upgrade.py:181
LANE_ROPE_SCALES = (1.0, 0.3, 0.5, 0.2)          # gdn3/gdn3_upgrade.py:182
BRAID_RATES = (0.05, 0.02, 0.005, 0.001)         # gdn3/gdn3_upgrade.py:127-128


def braided_decay(decay_proj, rates=BRAID_RATES, clamp=0.999):
    """gamma = clamp(mean_tau exp(-min(softplus(x), 5) * tau), max=clamp).

    decay_proj [..., 4] -> [...].  gdn3/gdn3_upgrade.py:812-822.
    """
    g_raw = torch.nn.functional.softplus(decay_proj).clamp(max=5.0)
    r = torch.tensor(rates, dtype=decay_proj.dtype)
    return torch.exp(-g_raw * r).mean(dim=-1).clamp(max=clamp)


def lane_rope_params(m_idx: int, K_dim: int, K_model: int, rotary_factor: float = 0.25):
    """(d_pairs, inv_freq [d_pairs] fp32, scale, identity) for lane ``m_idx``.

    Follows the branches of ``_lane_rope_factors`` (gdn3/gdn3_upgrade.py:342-376):
    * scale != 1: denominator ``max(1, int(K*0.25)//2 - 1)``;
    * scale == 1: denominator ``max(1, d_pairs-1)``, but when ``d_pairs``
      exceeds the module's cached table width ``int(K*rotary_factor)//2``
      the reference returns cos=1, sin=0 (no rotation) -- ``identity=True``.
    """
    frac = LANE_ROPE_FRACTIONS[m_idx]
    scale = LANE_ROPE_SCALES[m_idx]
    d_pairs = int(K_dim * frac // 2)
    if d_pairs < 1:
        return 0, None, scale, True
    ar = torch.arange(0, d_pairs, dtype=torch.float32)
    if scale != 1.0:
        inv_freq = 1.0 / (10000.0 ** (ar / max(1, int(K_model * 0.25) // 2 - 1)))
        return d_pairs, inv_freq, scale, False
    table_width = len(range(0, int(K_model * rotary_factor) // 2))
    if d_pairs > table_width:
        return d_pairs, None, scale, True
    inv_freq = 1.0 / (10000.0 ** (ar / max(1, d_pairs - 1)))
    return d_pairs, inv_freq, scale, False


def lane_rope_table(m_idx, T, K_dim, K_model, rotary_factor=0.25, pos0: int = 0):
    """(cos [T,d_pairs], sin [T,d_pairs]) or (None, None).  Angles are
    ``(t * scale) * inv_freq`` with ``t`` the position (0-based in the call, plus
    ``pos0`` for a continued sequence)."""
    d_pairs, inv_freq, scale, identity = lane_rope_params(m_idx, K_dim, K_model, rotary_factor)
    if d_pairs < 1:
        return None, None
    if identity:
        return torch.ones(T, d_pairs), torch.zeros(T, d_pairs)
    pos = torch.arange(pos0, pos0 + T, dtype=torch.float32)
    ang = (pos * scale)[:, None] * inv_freq[None, :]
    return torch.cos(ang), torch.sin(ang)


def apply_lane_rope(x, K_model=None, rotary_factor=0.25, pos0: int = 0):
    """Lane-specific partial RoPE on ``x [B,T,H,M,K]``.  gdn3/gdn3_upgrade.py:378-401.

    Note the reference's second-half formula uses the already-rotated first
    half (gdn3/gdn3_upgrade.py:397-398 write through a view), so the map is
    ``x1' = x1 c - x2 s``; ``x2' = x1' s + x2 c`` -- not a plane rotation.
    """
    B, T, H, M, K = x.shape
    K_model = K if K_model is None else K_model
    out = x.clone()
    for m in range(M):
        cos_t, sin_t = lane_rope_table(m, T, K, K_model, rotary_factor, pos0)
        if cos_t is None:
            continue
        d = cos_t.shape[1]
        lane = out[:, :, :, m, :]
        x1 = lane[..., :d]
        x2 = lane[..., d:2 * d]
        c = cos_t.to(x.dtype)[None, :, None, :]
        s = sin_t.to(x.dtype)[None, :, None, :]
        # The reference assigns the first half in place and then reads the
        # (aliased) first half again for the second: x2' = x1' sin + x2 cos
        # with x1' already rotated.  Mirrored here on purpose.
        n1 = x1 * c - x2 * s
        lane[..., :d] = n1
        lane[..., d:2 * d] = lane[..., :d] * s + x2 * c
        out[:, :, :, m, :] = lane
    return out
