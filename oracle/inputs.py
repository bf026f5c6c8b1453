"""Seeded synthetic inputs for the five BASELINE configurations (test infrastructure).

Draw order (one CPU ``torch.Generator`` seeded per config) is fixed:
``q, k, v, beta_raw, g_raw`` -- so that fixtures, tests and the benchmark see
identical data.  Distributions:

* q, k ~ N(0,1) per head, then L2-normalised over the head dim (lane shared)
* v ~ N(0,1)
* beta = sigmoid(N(0,1)) per (b, t, h, lane)
* log-decay g = -softplus(N(0,1)) * tau_lane, tau = (0.05, 0.02, 0.005, 0.001)
"""
from __future__ import annotations

import torch

TAUS = (0.05, 0.02, 0.005, 0.001)


def scan_inputs(B, T, H, M, K, V, seed, dtype=torch.float32):
    """Returns dict(q, k [B,T,H,K], v [B,T,H,V], beta [B,T,H,M], logg [B,T,H,M])
    in ``dtype`` (values rounded to ``dtype`` then kept as that dtype)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=g)
    k = torch.randn(B, T, H, K, generator=g)
    v = torch.randn(B, T, H, V, generator=g)
    beta = torch.sigmoid(torch.randn(B, T, H, M, generator=g))
    graw = torch.randn(B, T, H, M, generator=g)
    q = torch.nn.functional.normalize(q, dim=-1)
    k = torch.nn.functional.normalize(k, dim=-1)
    tau = torch.tensor(TAUS[:M], dtype=torch.float32)
    logg = -torch.nn.functional.softplus(graw) * tau
    out = dict(q=q, k=k, v=v, beta=beta, logg=logg)
    return {n: t.to(dtype) for n, t in out.items()}


def parity_inputs(B, T, H, M, K, V, seed, scale=0.1):
    """The reference parity-gate recipe (tests/test_chunk_parity.py:39-55) on a
    CPU generator: per-lane q,k,v ~ 0.1 N(0,1); gates sigmoid(5 * 0.1 N(0,1));
    decay U[0.9, 0.99).  Returns [q, k, v, bg, wg, dec] in the [B,T,H,M,*] layout."""
    g = torch.Generator().manual_seed(seed)
    rnd = lambda *s: torch.randn(*s, generator=g) * scale
    q = rnd(B, T, H, M, K); k = rnd(B, T, H, M, K); v = rnd(B, T, H, M, V)
    bg = torch.sigmoid(rnd(B, T, H, M, K) * 5)
    wg = torch.sigmoid(rnd(B, T, H, M, V) * 5)
    dec = 0.9 + 0.09 * torch.rand(B, T, H, M, generator=g)
    return [q, k, v, bg, wg, dec]


def realistic_logg(shape, seed):
    """Real-model-like decays ``g = exp(-softplus(1.2 N(0,1) - 0.6))`` as used
    by research/kernel_ab/bench_scan.py:51; returned as log-decay."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    return -torch.nn.functional.softplus(1.2 * x - 0.6)


def expand_lanes(inp, M):
    """Lane-replicated GDN3 tensors (the reference layout ``[B,T,H,M,*]``):
    ``q,k,v`` expanded over lanes; ``b = w = beta`` broadcast; ``dec = exp(logg)``.
    """
    q, k, v, beta, logg = (inp[n].float() for n in ('q', 'k', 'v', 'beta', 'logg'))
    K = q.shape[-1]
    V = v.shape[-1]
    qx = q.unsqueeze(3).expand(-1, -1, -1, M, -1)
    kx = k.unsqueeze(3).expand(-1, -1, -1, M, -1)
    vx = v.unsqueeze(3).expand(-1, -1, -1, M, -1)
    bg = beta.unsqueeze(-1).expand(-1, -1, -1, -1, K)
    wg = beta.unsqueeze(-1).expand(-1, -1, -1, -1, V)
    dec = torch.exp(logg)
    return qx, kx, vx, bg, wg, dec


CONFIGS = {
    0: dict(B=2, T=256, H=4, M=4, K=64, V=64, seed=0, dtype=torch.float32),
    1: dict(B=8, T=4096, H=16, M=4, K=128, V=128, seed=1, dtype=torch.bfloat16),
    2: dict(B=1, T=65536, H=16, M=4, K=128, V=128, seed=2, dtype=torch.bfloat16),
    4: dict(B=64, T=8192, H=16, M=4, K=128, V=128, seed=4, dtype=torch.bfloat16),
}
DECODE_CONFIG = dict(layers=24, B=256, H=16, M=4, K=128, V=128, seed=3, state_std=0.02)
