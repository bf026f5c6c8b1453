"""CPU restatements of the reference recurrences (test infrastructure only).

Every function here mirrors a reference function op for op so that, on the
same CPU inputs, its outputs are bit-identical to the reference's (checked by
``tests/test_oracle_golden.py`` against fixtures the reference produced).  The
only additions are the ones the reference lacks: final-state outputs, an
externally supplied compaction sketch ``G``, and an optional canonical sign
for the singular vectors (off by default).

Conventions
-----------
* chains ``N = B*H*M`` are ordered (b, h, m) with m fastest, as the reference
  flattens them (``gdn3/_reference_recurrence.py:47-50``).
* GDN3 state: ``A [N,R,a_v,a_k]``, ``Bk [N,R,b_v,b_k]``, ``U [N,V,P]``,
  ``Vb [N,K,P]``, slot pointer ``p``; the operator it represents is
  ``S = sum_r A_r (x) B_r + U Vb^T`` (V x K).
* dense state: ``S [N,V,K]`` (row v, key column k), i.e. ``y = S q``.
* KMD-2 state: ``S [N,dk,dv]`` as in ``research/kernel_ab/ref_scan.py:36``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


# --------------------------------------------------------------------------
# GDN3 helpers (gdn3/gdn3_upgrade.py:626-719)
# --------------------------------------------------------------------------

@dataclass
class KronDims:
    a_v: int = 16
    a_k: int = 16
    b_v: int = 8
    b_k: int = 8


def kron_read_vec(A, Bk, U, Vb, x, dims: KronDims):
    """``S x`` for the Kronecker + residual state.  gdn3/gdn3_upgrade.py:626-639."""
    N = x.shape[0]
    X = x.reshape(N, dims.a_k, dims.b_k)
    AX = torch.einsum('nrvk,nkb->nrvb', A, X)
    AXB = torch.einsum('nrvb,nrwb->nrvw', AX, Bk)
    y = AXB.sum(1).reshape(N, dims.a_v * dims.b_v)
    coeff = torch.einsum('nkp,nk->np', Vb, x)
    y = y + torch.einsum('nvp,np->nv', U, coeff)
    return y


def stable_alpha(c, eps: float = 1e-6):
    """alpha(c) = (1 - e^-c)/c with a Taylor branch.  gdn3/gdn3_upgrade.py:641-648."""
    small = c.abs() < eps
    safe = torch.where(small, torch.ones_like(c), c)
    exact = -torch.expm1(-safe) / safe
    series = 1.0 - c / 2.0 + c * c / 6.0
    return torch.where(small, series, exact)


def sketch_matrix(N: int, n: int, q: int, dtype=torch.float32):
    """Gaussian sketch exactly as the reference draws it on a CPU device.

    gdn3/gdn3_upgrade.py:679-682 draws ``randn(N, n, q)`` from a fresh
    ``torch.Generator(device).manual_seed(1234)`` on every call, so every
    compaction of a run sees the same ``G``.
    """
    gen = torch.Generator(device='cpu').manual_seed(1234)
    return torch.randn(N, n, q, dtype=dtype, generator=gen)


def canonical_sign(Us, Vs, R: int):
    """Flip each rank-r pair so the largest-|.| entry of ``Vs[:, :, r]`` is > 0.

    Singular vectors are defined up to a joint sign; the reference inherits
    LAPACK's choice.  The device kernel fixes this rule, and the oracle can
    apply the same rule (``canon_signs=True``) so per-call factors compare.
    """
    Us = Us.clone()
    Vs = Vs.clone()
    for r in range(R):
        idx = Vs[:, :, r].abs().argmax(dim=1)
        s = torch.sign(Vs[:, :, r].gather(1, idx[:, None]))[:, 0]
        s = torch.where(s == 0, torch.ones_like(s), s)
        Us[:, :, r] *= s[:, None]
        Vs[:, :, r] *= s[:, None]
    return Us, Vs


def rearranged_matrix(A, Bk, U, Vb, dims: KronDims):
    """R_mat = sum_r vec(A_r) vec(B_r)^T + rearrange(U Vb^T).  gdn3/gdn3_upgrade.py:662-671."""
    N, R = A.shape[0], A.shape[1]
    vecA = A.reshape(N, R, dims.a_v * dims.a_k)
    vecB = Bk.reshape(N, R, dims.b_v * dims.b_k)
    R_mat = torch.einsum('nra,nrb->nab', vecA, vecB)
    S_res = torch.einsum('nvp,nkp->nvk', U, Vb)
    S_res = (S_res.reshape(N, dims.a_v, dims.b_v, dims.a_k, dims.b_k)
             .permute(0, 1, 3, 2, 4)
             .reshape(N, dims.a_v * dims.a_k, dims.b_v * dims.b_k))
    return R_mat + S_res


def compact_call(A, Bk, U, Vb, dims: KronDims, slow_decay: float = 0.97,
                 G: Optional[torch.Tensor] = None, canon_signs: bool = False,
                 return_factors: bool = False):
    """One compaction.  Restates ``_compact_vec`` (gdn3/gdn3_upgrade.py:650-719).

    Returns ``(A_new, B_new, U, Vb, err)``; with ``return_factors`` also the
    un-blended ``(A_svd, B_svd, S)``.
    """
    N, R = A.shape[0], A.shape[1]
    A_old = A.clone()
    Bk_old = Bk.clone()
    R_mat = rearranged_matrix(A, Bk, U, Vb, dims)
    total_energy = (R_mat ** 2).sum()
    m, n = R_mat.shape[-2], R_mat.shape[-1]
    q = min(R + 4, m, n)
    if G is None:
        G = sketch_matrix(N, n, q, R_mat.dtype)
    Y = R_mat @ G
    for _ in range(2):
        Y = R_mat @ (R_mat.transpose(-2, -1) @ Y)
    Q, _ = torch.linalg.qr(Y)
    Bm = Q.transpose(-2, -1) @ R_mat
    Ub, Ss, Vh = torch.linalg.svd(Bm, full_matrices=False)
    Us = Q @ Ub
    Vs = Vh.transpose(-2, -1)
    if canon_signs:
        Us, Vs = canonical_sign(Us, Vs, R)
    kept = (Ss[:, :R] ** 2).sum()
    err = (total_energy - kept).clamp(min=0.0)
    A_svd = torch.zeros_like(A)
    B_svd = torch.zeros_like(Bk)
    for r in range(R):
        A_svd[:, r] = (Us[:, :, r] * Ss[:, r:r + 1]).reshape(N, dims.a_v, dims.a_k)
        B_svd[:, r] = Vs[:, :, r].reshape(N, dims.b_v, dims.b_k)
    A_new = slow_decay * A_old + (1 - slow_decay) * A_svd
    B_new = slow_decay * Bk_old + (1 - slow_decay) * B_svd
    if return_factors:
        return A_new, B_new, U, Vb, err, (A_svd, B_svd, Ss[:, :R])
    return A_new, B_new, U, Vb, err


def compact_sketch_call(A, Bk, U, Vb, dims: KronDims, slow_decay: float = 0.97,
                        G: Optional[torch.Tensor] = None):
    """One compaction in the reference's ``compact_mode`` "sketch" / "sketch_noqr"
    (the two are the same code): restates ``_compact_fast``'s sketch branch
    (gdn3/gdn3_upgrade.py:565-596).  ``G`` is ``[N, n, R]`` (the reference draws it
    with ``R`` columns, seed 1234).  Returns ``(A_new, B_new, U, Vb, err)`` with
    ``err`` = 0 like the reference.
    """
    N, R = A.shape[0], A.shape[1]
    R_mat = rearranged_matrix(A, Bk, U, Vb, dims)
    n = R_mat.shape[-1]
    if G is None:
        G = sketch_matrix(N, n, R, R_mat.dtype)
    Y = R_mat @ G
    q_scale = Y.square().sum(1).sqrt().clamp_min(1e-12)
    Q = Y / q_scale[:, None, :]
    Bm = Q.transpose(-2, -1) @ R_mat
    b_scale = Bm.square().sum(-1).sqrt().clamp_min(1e-12)
    A_svd = (Q * b_scale[:, None, :]).permute(0, 2, 1).reshape(N, R, dims.a_v, dims.a_k)
    B_svd = (Bm / b_scale[:, :, None]).reshape(N, R, dims.b_v, dims.b_k)
    A_new = slow_decay * A + (1 - slow_decay) * A_svd
    B_new = slow_decay * Bk + (1 - slow_decay) * B_svd
    return A_new, B_new, U, Vb, torch.zeros((), dtype=R_mat.dtype)


# --------------------------------------------------------------------------
# GDN3 Kronecker-residual scan (gdn3/_reference_recurrence.py:33-94)
# --------------------------------------------------------------------------

@dataclass
class KRState:
    A: torch.Tensor
    Bk: torch.Tensor
    U: torch.Tensor
    Vb: torch.Tensor
    p: int
    err: torch.Tensor


def gdn3_kr_scan(q, k, v, bg, wg, dec, *, R: int = 4, P: int = 16,
                 dims: KronDims = KronDims(), slow_decay: float = 0.97,
                 G: Optional[torch.Tensor] = None, canon_signs: bool = False,
                 state: Optional[KRState] = None, dtype=torch.float32, compact_mode: str = 'svd'):
    """Frozen GDN3-KR token loop returning ``(Y [B,T,H,M,V], KRState)``.

    Mirrors ``reference_recurrent_state`` (gdn3/_reference_recurrence.py:33-94)
    op for op.  ``state`` (optional) continues from a previous call instead of
    the zero state, which is what a decode step needs.  ``compact_mode`` "sketch"
    (or "sketch_noqr") compacts with :func:`compact_sketch_call` instead, the
    reference layer's ``GDN3_COMPACT_MODE`` choice (gdn3/gdn3_upgrade.py:81,579).
    """
    if compact_mode not in ('svd', 'sketch', 'sketch_noqr'):
        raise ValueError(f'unknown compact_mode {compact_mode!r}')
    B, T, H, M, K = q.shape
    V = v.shape[-1]
    N = B * H * M

    def _flat(x, d):
        return x.permute(1, 0, 2, 3, 4).reshape(T, N, d).to(dtype)
    qf = _flat(q, K); kf = _flat(k, K); vf = _flat(v, V)
    bgf = _flat(bg, K); wgf = _flat(wg, V)
    decf = dec.permute(1, 0, 2, 3).reshape(T, N).to(dtype)

    if state is None:
        A = torch.zeros(N, R, dims.a_v, dims.a_k, dtype=dtype)
        Bk = torch.zeros(N, R, dims.b_v, dims.b_k, dtype=dtype)
        U = torch.zeros(N, V, P, dtype=dtype)
        Vb = torch.zeros(N, K, P, dtype=dtype)
        p = 0
        comp_err = torch.zeros((), dtype=dtype)
    else:
        A, Bk, U, Vb, p = state.A, state.Bk, state.U, state.Vb, state.p
        comp_err = state.err
    outs = []
    for t in range(T):
        gamma = decf[t].clamp(0.0, 1.0)
        A = A * gamma.view(N, 1, 1, 1)
        Bk = Bk * gamma.view(N, 1, 1, 1)
        Vb = Vb * gamma.view(N, 1, 1)
        k_t, q_t = kf[t], qf[t]
        h = bgf[t] * k_t
        u = wgf[t] * vf[t]
        s_h = kron_read_vec(A, Bk, U, Vb, h, dims)
        r = u - s_h
        c = (k_t * h).sum(-1)
        alpha = stable_alpha(c)
        s_q = kron_read_vec(A, Bk, U, Vb, q_t, dims)
        kq = (k_t * q_t).sum(-1)
        y = s_q + (alpha * kq).unsqueeze(-1) * r
        outs.append(y)
        new_u = alpha.unsqueeze(-1) * r
        U = torch.cat([U[:, :, :p], new_u.unsqueeze(-1), U[:, :, p + 1:]], dim=2)
        Vb = torch.cat([Vb[:, :, :p], k_t.unsqueeze(-1), Vb[:, :, p + 1:]], dim=2)
        p += 1
        if p >= P:
            with torch.no_grad():
                if compact_mode == 'svd':
                    A, Bk, U, Vb, err = compact_call(A, Bk, U, Vb, dims, slow_decay,
                                                     G=G, canon_signs=canon_signs)
                else:
                    A, Bk, U, Vb, err = compact_sketch_call(A, Bk, U, Vb, dims, slow_decay, G=G)
            comp_err = comp_err + err
            p = 0
    Y = torch.stack(outs, 0).reshape(T, B, H, M, V).permute(1, 0, 2, 3, 4).contiguous()
    return Y, KRState(A, Bk, U, Vb, p, comp_err)


# --------------------------------------------------------------------------
# Dense special case (compaction off): S is V x K
# --------------------------------------------------------------------------

def dense_scan(q, k, v, bg, wg, dec, S0: Optional[torch.Tensor] = None,
               dtype=torch.float32):
    """GDN3 recurrence with the residual never compacted (P >= T).

    With A = 0 the operator ``U Vb^T`` is a dense V x K matrix S and the loop of
    gdn3/_reference_recurrence.py:60-84 becomes, per chain and token,
    ``S <- g S``; ``r = w*v - S (b*k)``; ``a = alpha(k.(b*k))``;
    ``y = S q + a (k.q) r``; ``S <- S + a r k^T``.

    Inputs as ``gdn3_kr_scan`` (``bg``/``wg`` may be [...,1] to broadcast).
    Returns ``(Y [B,T,H,M,V], S [N,V,K])``.
    """
    B, T, H, M, K = q.shape
    V = v.shape[-1]
    N = B * H * M

    def _flat(x):
        d = x.shape[-1]
        return x.permute(1, 0, 2, 3, 4).reshape(T, N, d).to(dtype)
    qf, kf, vf, bgf, wgf = map(_flat, (q, k, v, bg, wg))
    decf = dec.permute(1, 0, 2, 3).reshape(T, N).to(dtype)
    S = torch.zeros(N, V, K, dtype=dtype) if S0 is None else S0.to(dtype).clone()
    outs = []
    for t in range(T):
        gamma = decf[t].clamp(0.0, 1.0)
        S = S * gamma.view(N, 1, 1)
        k_t, q_t = kf[t], qf[t]
        h = bgf[t] * k_t
        u = wgf[t] * vf[t]
        s_h = torch.bmm(S, h.unsqueeze(-1)).squeeze(-1)
        r = u - s_h
        alpha = stable_alpha((k_t * h).sum(-1))
        s_q = torch.bmm(S, q_t.unsqueeze(-1)).squeeze(-1)
        kq = (k_t * q_t).sum(-1)
        outs.append(s_q + (alpha * kq).unsqueeze(-1) * r)
        S = S + (alpha.unsqueeze(-1) * r).unsqueeze(-1) * k_t.unsqueeze(1)
    Y = torch.stack(outs, 0).reshape(T, B, H, M, V).permute(1, 0, 2, 3, 4).contiguous()
    return Y, S


# --------------------------------------------------------------------------
# KMD-2 (research/kernel_ab/ref_scan.py:24-48, exact_cache.py:1231-1295)
# --------------------------------------------------------------------------

def kmd2_scan(q, k, v, g, beta_e, beta_w, out_mix=None, S0=None,
              dtype=torch.float32):
    """KMD-2 frozen loop.  Returns ``(y [B,T,H,dv], scores [B,T,H], S [N,dk,dv])``.

    ``y`` follows ``research/kernel_ab/ref_scan.py:36-48`` op for op; the
    scores are ``|k| * |beta_w v - beta_e k^T S|`` as in
    ``research/kmd2_ablation/exact_cache.py:1283-1292``.
    """
    B, T, H, r_out, dk = q.shape
    dv = v.shape[-1]
    N = B * H

    def flat(x, *tail):
        return x.permute(1, 0, 2, *range(3, x.dim())).reshape(T, N, *tail).to(dtype)
    q_ = flat(q, r_out, dk); k_ = flat(k, dk); v_ = flat(v, dv)
    g_ = flat(g, dk); be_ = flat(beta_e); bw_ = flat(beta_w)
    if r_out > 1:
        mixw = out_mix[None].expand(B, -1, -1).reshape(N, 1, r_out).to(dtype)
    S = torch.zeros(N, dk, dv, dtype=dtype) if S0 is None else S0.to(dtype).clone()
    outs, scores = [], []
    for t in range(T):
        S = S * g_[t].unsqueeze(-1)
        kt = k_[t]
        kv_mem = torch.bmm(kt.unsqueeze(1), S).squeeze(1)
        upd = bw_[t].unsqueeze(-1) * v_[t] - be_[t].unsqueeze(-1) * kv_mem
        S = S - torch.bmm(kt.unsqueeze(2), (be_[t].unsqueeze(-1) * kv_mem).unsqueeze(1))
        S = S + torch.bmm(kt.unsqueeze(2), (bw_[t].unsqueeze(-1) * v_[t]).unsqueeze(1))
        yt = torch.bmm(q_[t], S)
        yt = (yt * mixw.transpose(1, 2)).sum(1) if r_out > 1 else yt.squeeze(1)
        outs.append(yt)
        scores.append(torch.linalg.vector_norm(kt, dim=-1) * torch.linalg.vector_norm(upd, dim=-1))
    y = torch.stack(outs, 0).reshape(T, B, H, dv).permute(1, 0, 2, 3)
    sc = torch.stack(scores, 0).reshape(T, B, H).permute(1, 0, 2)
    return y, sc, S


# --------------------------------------------------------------------------
# Decode step (one iteration of the loop bodies above from a supplied state)
# --------------------------------------------------------------------------

def dense_decode_step(S, q, k, v, bg, wg, gamma):
    """One GDN3 dense step.  S [N,V,K]; q,k,bg [N,K]; v,wg [N,V]; gamma [N].

    The loop body of gdn3/_reference_recurrence.py:61-84 with A = 0.
    Returns ``(y [N,V], S_new)``; S is not modified.
    """
    gamma = gamma.clamp(0.0, 1.0)
    S = S * gamma.view(-1, 1, 1)
    h = bg * k
    u = wg * v
    s_h = torch.bmm(S, h.unsqueeze(-1)).squeeze(-1)
    r = u - s_h
    alpha = stable_alpha((k * h).sum(-1))
    s_q = torch.bmm(S, q.unsqueeze(-1)).squeeze(-1)
    y = s_q + (alpha * (k * q).sum(-1)).unsqueeze(-1) * r
    S = S + (alpha.unsqueeze(-1) * r).unsqueeze(-1) * k.unsqueeze(1)
    return y, S
