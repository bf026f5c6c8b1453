"""CPU restatement of the GDN3 scan prologue (test infrastructure only).

* ``braided_decay``   -- gdn3/gdn3_upgrade.py:809-822
* ``lane_rope_table`` -- gdn3/gdn3_upgrade.py:342-376 (``_lane_rope_factors``)
* ``apply_lane_rope`` -- gdn3/gdn3_upgrade.py:378-401 (``_apply_partial_rope``)
* ``projection_prologue`` -- gdn3/gdn3_upgrade.py:752-807 and :201-250 (conv, coproduct blend, gates)
"""
from __future__ import annotations

import math

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


def projection_prologue(qkv, conv_w, H, K, coprod=None, mix=None, b_proj=None, proj_a=None, w_proj=None,
                        proj_b=None):
    """GDN3 projection prologue after the GEMMs, restated op for op from
    gdn3/gdn3_upgrade.py:752-807 (causal depthwise conv, split, gates) and
    :201-250 (coproduct factors -> outer-product sum / sqrt(C), blend).
    Returns ((q, k, v) [B,T,H,K], (b_gates, w_gates))."""
    import torch.nn.functional as F
    B, T = qkv.shape[:2]
    ck = conv_w.shape[-1]
    qkv_padded = F.pad(qkv.transpose(1, 2), (ck - 1, 0))
    qkv_conv = F.conv1d(qkv_padded, conv_w, groups=3 * H * K).transpose(1, 2)
    qkv_conv = qkv_conv.reshape(B, T, H, 3, K)
    q, k, v = qkv_conv[:, :, :, 0], qkv_conv[:, :, :, 1], qkv_conv[:, :, :, 2]
    if coprod is not None:
        q_a, q_b, k_a, k_b, v_a, v_b = coprod
        mix_qk, mix_v, str_qk, str_v = mix
        C = q_a.shape[3]
        sq = math.sqrt(C)
        cp = lambda a_, b_: (torch.einsum('bthci,bthcj->bthcij', a_, b_).sum(dim=3) / sq).reshape(B, T, H, -1)
        q_c, k_c, v_c = cp(q_a, q_b), cp(k_a, k_b), cp(v_a, v_b)
        aqk = torch.sigmoid(mix_qk).view(1, 1, H, 1)
        av = torch.sigmoid(mix_v).view(1, 1, H, 1)
        sqk = str_qk.view(1, 1, H, 1)
        sv = str_v.view(1, 1, H, 1)
        q = (1 - aqk) * q + aqk * sqk * q_c
        k = (1 - aqk) * k + aqk * sqk * k_c
        v = (1 - av) * v + av * sv * v_c
    bg = wg = None
    if b_proj is not None:
        M = b_proj.shape[3]
        bg = torch.sigmoid(b_proj + proj_a.unsqueeze(3).expand(-1, -1, -1, M).unsqueeze(-1) * 0.1)
    if w_proj is not None:
        M = w_proj.shape[3]
        wg = torch.sigmoid(w_proj + proj_b.unsqueeze(3).expand(-1, -1, -1, M).unsqueeze(-1) * 0.1)
    return (q, k, v), (bg, wg)


def kmd2_prologue(mixed, conv_w, b, a, theta, dt_bias, A_log, decay_chan, bw_off, q_slot_scale=None,
                  *, H, dk=128, dv=128, r_out=1, conv_k=4):
    """Restates ``KMD2NativeAttn.forward`` between its input GEMMs and ``_scan``
    (gdn3/kmd2_native.py:140-172) op for op on the GEMM outputs.  Returns the ``_scan``
    arguments ``(qs [B,T,H,r_out,dk], k, v, g, beta_e, beta_w)``."""
    import torch.nn.functional as F
    B, T = mixed.shape[:2]
    key_dim, value_dim = H * dk, H * dv
    x = mixed.transpose(1, 2)
    x = F.silu(F.conv1d(x, conv_w, padding=conv_k - 1, groups=x.shape[1])[:, :, :T]).transpose(1, 2)
    query, key, value = torch.split(x, [key_dim, key_dim, value_dim], dim=-1)
    q = F.normalize(query.reshape(B, T, H, dk).float(), dim=-1, eps=1e-6)
    k = F.normalize(key.reshape(B, T, H, dk).float(), dim=-1, eps=1e-6)
    v = value.reshape(B, T, H, dv).float()
    q = q * (dk ** -0.5)
    b = b.float()
    a = a.float()
    beta_e = torch.sigmoid(b)
    beta_w = torch.sigmoid(b + bw_off)
    g_head = -A_log.float().exp() * F.softplus(a + dt_bias.float())
    g = (g_head.unsqueeze(-1) + decay_chan).exp()
    g = g.clamp(max=1.0)
    th = F.softplus(theta).view(B, T, H, dk // 2).float()
    Th = th.cumsum(dim=1)
    cos, sin = Th.cos(), Th.sin()

    def rope(zz, c, s):
        z1, z2 = zz[..., :dk // 2], zz[..., dk // 2:]
        return torch.cat([z1 * c - z2 * s, z1 * s + z2 * c], dim=-1)
    k = rope(k, cos, sin)
    qs = q.unsqueeze(3) * (1.0 + q_slot_scale)[None, None] if r_out > 1 else q.unsqueeze(3)
    qs = rope(qs, cos.unsqueeze(-2), sin.unsqueeze(-2))
    return qs, k, v, g, beta_e, beta_w
