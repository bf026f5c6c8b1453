"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Usage (needs the reference source tree; it is not needed afterwards):

    python tests/golden/make_golden.py /path/to/GDNX

The script imports the reference's own modules unchanged and records, for
seeded inputs, what they return:

* ``gdn3_frozen.pt``   -- ``gdn3._reference_recurrence.reference_recurrent_state``
  (dense P >= T and compacting P = 16 cases, the parity recipe of
  ``tests/test_chunk_parity.py:39-55`` at T = 64 and the T = 48 tail), plus the
  reference's own chunked ``GDN3LinearAttn._gdn3_recurrent_state`` on the same
  inputs (its fidelity floor).
* ``gdn3_config0.pt``  -- config 0 (B=2,T=256,H=4,M=4,d=64, fp32, seed 0) through
  the frozen loop with P = T (dense) -- every 4th token and the last one.
* ``kmd2.pt``          -- ``research/kernel_ab/ref_scan.scan`` and
  ``research/kmd2_ablation/exact_cache.reference_scan_with_scores``.
* ``compaction.pt``    -- one ``GDN3LinearAttn._compact_vec`` call.
* ``compaction_sketch.pt`` -- one ``GDN3LinearAttn._compact_fast`` call with
  ``compact_mode`` "sketch" and one with "sketch_noqr" (CPU layer, so its sketch
  comes from the CPU generator, seed 1234).
* ``gdn3_kr_p256.pt``  -- the frozen loop at config 2's compaction period
  (P = 256, R = 4, A 16x16 (x) B 8x8, d = 128, one head of four lanes, bf16-rounded
  config-2 inputs, T = 1024: four compactions) -- every 8th token and the last
  one, plus the relative L2 distance of the
  reference's own chunked ``_gdn3_recurrent_state`` from it (its floor).
* ``kmd2_prologue.pt`` -- ``KMD2NativeAttn.forward`` (random parameters, r_out 4 and 1) with its
  ``_scan`` replaced by a recorder: the GEMM outputs it starts from and the ``_scan`` arguments
  the reference hands over (conv + SiLU, normalisation, gates, decays, cumulative rotation); and
  the whole forward's output with the reference's own scan, with the parameters and input.
* ``epilogue.pt``      -- the GDN3 output epilogue (``forward`` lines 842-856 restated
  by calling the same torch ops on a module's ``norm`` parameter, set to random
  values) and ``Qwen3_5RMSNormGated`` from transformers on random inputs.
* ``proj_prologue.pt`` -- the projection prologue of ``GDN3LinearAttn.forward``: the
  reference's conv module and ``_generate_coproduct_channels`` on seeded weights,
  and the gate activations (lines 797-807), with their post-GEMM inputs.
* ``prologue.pt``      -- braided decay (``forward`` lines 809-822 restated by
  calling the same torch ops on the module's buffers) and ``_apply_partial_rope``.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))


def _layer(K, V, P, dims=(16, 16, 8, 8), rotary_factor=None):
    from gdn3.gdn3_upgrade import GDN3LinearAttn
    cfg = types.SimpleNamespace(hidden_size=64, linear_num_key_heads=2,
                                linear_key_head_dim=K, linear_value_head_dim=V,
                                linear_conv_kernel_dim=4)
    if rotary_factor is not None:
        cfg.partial_rotary_factor = rotary_factor
    L = GDN3LinearAttn(cfg)
    L.P = P
    L.residual_rank = P
    L.a_v, L.a_k, L.b_v, L.b_k = dims
    return L


def make_gdn3_frozen():
    from gdn3._reference_recurrence import reference_recurrent_state
    from oracle.inputs import scan_inputs, expand_lanes, parity_inputs
    cases = {}
    # (a) config-0 distribution, small, dense (P >= T) and compacting (P = 16)
    inp = scan_inputs(1, 80, 2, 4, 64, 64, seed=10)
    ins = [t.contiguous() for t in expand_lanes(inp, 4)]
    for P in (80, 16):
        L = _layer(64, 64, P, dims=(8, 8, 8, 8))
        with torch.no_grad():
            Y = reference_recurrent_state(L, *ins)
            Yc = L._gdn3_recurrent_state(*ins)
        # inputs stored lane-shared; expand_lanes() rebuilds the reference layout
        cases[f'cfg0dist_P{P}'] = dict(inputs_compact=inp, P=P, dims=(8, 8, 8, 8), Y=Y, Y_chunked=Yc)
    # (b) the reference parity recipe at d = 128, T = 64 and the T = 48 tail
    for (B, T, seed) in ((1, 64, 0), (2, 48, 0)):
        ins = parity_inputs(B, T, 1, 4, 128, 128, seed)
        L = _layer(128, 128, 16)
        with torch.no_grad():
            Y = reference_recurrent_state(L, *ins)
            Yc = L._gdn3_recurrent_state(*ins)
        # inputs are regenerated from the seed; the checksum guards the generator
        cases[f'parity_B{B}_T{T}'] = dict(shape=(B, T, 1, 4, 128, 128), seed=seed,
                                          input_sums=[t.double().sum() for t in ins],
                                          P=16, dims=(16, 16, 8, 8), Y=Y, Y_chunked=Yc)
    torch.save(cases, HERE / 'gdn3_frozen.pt')


def make_gdn3_config0():
    from gdn3._reference_recurrence import reference_recurrent_state
    from oracle.inputs import scan_inputs, expand_lanes, CONFIGS
    c = CONFIGS[0]
    inp = scan_inputs(c['B'], c['T'], c['H'], c['M'], c['K'], c['V'], c['seed'])
    ins = [t.contiguous() for t in expand_lanes(inp, c['M'])]
    L = _layer(64, 64, c['T'], dims=(8, 8, 8, 8))
    with torch.no_grad():
        Y = reference_recurrent_state(L, *ins)
    keep = list(range(0, c['T'], 4)) + [c['T'] - 1]
    torch.save(dict(t_index=torch.tensor(keep), Y=Y[:, keep].clone(),
                    Y_sum=Y.double().sum(), Y_sq=Y.double().square().sum()),
               HERE / 'gdn3_config0.pt')


def make_kmd2():
    sys.path.insert(0, str(Path(REF) / 'research' / 'kernel_ab'))
    import ref_scan
    from research.kmd2_ablation.exact_cache import reference_scan_with_scores
    g = torch.Generator().manual_seed(77)
    out = {}
    B, T, H, dk, dv = 2, 40, 2, 32, 32
    for r_out in (1, 4):
        q = torch.randn(B, T, H, r_out, dk, generator=g) * dk ** -0.5
        k = torch.nn.functional.normalize(torch.randn(B, T, H, dk, generator=g), dim=-1)
        v = torch.randn(B, T, H, dv, generator=g)
        gd = torch.exp(-torch.nn.functional.softplus(1.2 * torch.randn(B, T, H, dk, generator=g) - 0.6))
        be = torch.sigmoid(torch.randn(B, T, H, generator=g))
        bw = torch.sigmoid(torch.randn(B, T, H, generator=g))
        mix = torch.randn(H, r_out, generator=g) if r_out > 1 else None
        y = ref_scan.scan(q, k, v, gd, be, bw, mix)
        y2, sc = reference_scan_with_scores(q, k, v, gd, be, bw, mix)
        out[f'r{r_out}'] = dict(inputs=[q, k, v, gd, be, bw, mix], y=y, y_scored=y2, scores=sc)
    # known-answer cases of tests/ablation/test_exact_cache_math.py:563-596
    q = torch.tensor([[[[[3.0]]]]], dtype=torch.float64)
    k = torch.tensor([[[[2.0]]]], dtype=torch.float64)
    v = torch.tensor([[[[5.0]]]], dtype=torch.float64)
    d = torch.tensor([[[[0.25]]]], dtype=torch.float64)
    be = torch.tensor([[[0.7]]], dtype=torch.float64)
    bw = torch.tensor([[[0.4]]], dtype=torch.float64)
    y, sc = reference_scan_with_scores(q, k, v, d, be, bw)
    out['kat'] = dict(inputs=[q, k, v, d, be, bw, None], y=y, scores=sc)
    torch.save(out, HERE / 'kmd2.pt')


def make_kr_p256():
    from gdn3._reference_recurrence import reference_recurrent_state
    from oracle.inputs import scan_inputs, expand_lanes
    B, T, H, M, K = 1, 1024, 1, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=2, dtype=torch.bfloat16)
    ins = [t.contiguous() for t in expand_lanes(inp, M)]
    L = _layer(K, K, 256)
    with torch.no_grad():
        Y = reference_recurrent_state(L, *ins)
        Yc = L._gdn3_recurrent_state(*ins)
    keep = list(range(0, T, 8)) + [T - 1]
    floor = ((Yc - Y).double().norm() / Y.double().norm()).item()
    torch.save(dict(shape=(B, T, H, M, K), seed=2, P=256, dims=(16, 16, 8, 8), t_index=torch.tensor(keep),
                    Y=Y[:, keep].clone(), Y_sum=Y.double().sum(), Y_sq=Y.double().square().sum(),
                    chunked_floor=floor),
               HERE / 'gdn3_kr_p256.pt')


def make_compaction():
    g = torch.Generator().manual_seed(5)
    N, R, V, K, P = 6, 4, 128, 128, 16
    L = _layer(K, V, P)
    A = torch.randn(N, R, 16, 16, generator=g) * 0.1
    Bk = torch.randn(N, R, 8, 8, generator=g) * 0.1
    U = torch.randn(N, V, P, generator=g) * 0.3
    Vb = torch.randn(N, K, P, generator=g) * 0.3
    with torch.no_grad():
        An, Bn, Uo, Vo, err = L._compact_vec(A, Bk, U, Vb, L.slow_decay)
    torch.save(dict(inputs=[A, Bk, U, Vb], A_new=An, B_new=Bn, err=err,
                    slow_decay=L.slow_decay), HERE / 'compaction.pt')


def make_compaction_sketch():
    g = torch.Generator().manual_seed(6)
    N, R, V, K, P = 6, 4, 128, 128, 32
    L = _layer(K, V, P)
    A = torch.randn(N, R, 16, 16, generator=g) * 0.1
    Bk = torch.randn(N, R, 8, 8, generator=g) * 0.1
    U = torch.randn(N, V, P, generator=g) * 0.2
    Vb = torch.randn(N, K, P, generator=g) * 0.2
    out = {}
    for mode in ('sketch', 'sketch_noqr'):
        L.compact_mode = mode
        with torch.no_grad():
            An, Bn, Uo, Vo, err = L._compact_fast(A, Bk, U, Vb)
        out[mode] = dict(A_new=An, B_new=Bn, err=err)
    torch.save(dict(inputs=[A, Bk, U, Vb], slow_decay=L.slow_decay, **out), HERE / 'compaction_sketch.pt')


def make_kmd2_prologue():
    import importlib
    out = {}
    for r_out in (4, 1):
        os.environ['GDN3_KMD2_ROUT'] = str(r_out)
        import gdn3.kmd2_native as KN
        importlib.reload(KN)
        cfg = types.SimpleNamespace(hidden_size=32, linear_num_value_heads=2, linear_key_head_dim=128,
                                    linear_value_head_dim=128, linear_num_key_heads=2, linear_conv_kernel_dim=4,
                                    rms_norm_eps=1e-6)
        L = KN.KMD2NativeAttn(cfg)
        g = torch.Generator().manual_seed(20 + r_out)
        with torch.no_grad():
            for name, prm in L.named_parameters():
                scale = {'rot_proj.bias': 0.5, 'A_log': 0.5, 'dt_bias': 1.0, 'decay_chan': 0.3, 'bw_off': 1.0,
                         'q_slot_scale': 0.2, 'conv1d.weight': 0.4}.get(name, 0.15)
                prm.copy_(torch.randn(prm.shape, generator=g) * scale)
            L.rot_proj.bias.sub_(1.0)  # softplus about 0.3 rad per token: the rotation turns visibly
        rec = {}

        def recorder(q, k, v, gd, be, bw):
            rec.update(q=q.detach().clone(), k=k.detach().clone(), v=v.detach().clone(), g=gd.detach().clone(),
                       beta_e=be.detach().clone(), beta_w=bw.detach().clone())
            return torch.zeros(k.shape[0], k.shape[1], k.shape[2], v.shape[-1])

        L._scan = recorder
        x = torch.randn(2, 24, 32, generator=g)
        with torch.no_grad():
            L(x)
            gemm = dict(mixed=L.in_proj_qkv(x), b=L.in_proj_b(x), a=L.in_proj_a(x), theta=L.rot_proj(x))
        prm = dict(conv_w=L.conv1d.weight.detach().clone(), dt_bias=L.dt_bias.detach().clone(),
                   A_log=L.A_log.detach().clone(), decay_chan=L.decay_chan.detach().clone(),
                   bw_off=L.bw_off.detach().clone(),
                   q_slot_scale=L.q_slot_scale.detach().clone() if r_out > 1 else None)
        # the whole forward with the reference's own token-loop scan, for the fused-forward drop-in
        L2 = KN.KMD2NativeAttn(cfg)
        L2.load_state_dict(L.state_dict())
        with torch.no_grad():
            y_fwd = L2(x)
        out[f'r{r_out}'] = dict(H=2, r_out=r_out, gemm=gemm, params=prm, scan_args=rec, x=x,
                                state_dict={k_: v_.detach().clone() for k_, v_ in L2.state_dict().items()},
                                forward=y_fwd, eps=cfg.rms_norm_eps)
    os.environ.pop('GDN3_KMD2_ROUT', None)
    torch.save(out, HERE / 'kmd2_prologue.pt')


def make_epilogue():
    import torch.nn.functional as F
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNormGated
    g = torch.Generator().manual_seed(13)
    L = _layer(128, 128, 16)
    with torch.no_grad():
        L.norm.copy_(1.0 + 0.1 * torch.randn(128, generator=g))
    y = torch.randn(2, 9, 2, 4, 128, generator=g)
    logits = torch.randn(2, 9, 2, 4, generator=g)
    V = 128
    router_weights = F.softmax(logits, dim=-1)
    routed = (router_weights.unsqueeze(-1) * y).sum(dim=3)
    routed_normed = F.normalize(routed, p=2, dim=-1, eps=1e-6) * torch.sqrt(torch.tensor(float(V)))
    out = routed_normed * L.norm
    nm = Qwen3_5RMSNormGated(128, eps=1e-6)
    with torch.no_grad():
        nm.weight.copy_(1.0 + 0.1 * torch.randn(128, generator=g))
    yk = torch.randn(2, 9, 2, 128, generator=g)
    z = torch.randn(2, 9, 2, 128, generator=g)
    with torch.no_grad():
        ok = nm(yk, z)
    torch.save(dict(y=y, logits=logits, norm=L.norm.detach().clone(), out=out.detach(),
                    y_kmd2=yk, z=z, weight=nm.weight.detach().clone(), out_kmd2=ok), HERE / 'epilogue.pt')


def make_projection_prologue():
    """Inputs after the layer's GEMMs and the outputs of the reference's own conv module,
    ``_generate_coproduct_channels`` and gate formula (gdn3/gdn3_upgrade.py:747-807)."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(21)
    L = _layer(128, 128, 16)
    H, K, M, D = L.H, L.K, L.M, L.D
    with torch.no_grad():
        L.in_proj_qkv.copy_(torch.randn(L.in_proj_qkv.shape, generator=g) * 0.05)
        L.conv1d.weight.copy_(torch.randn(L.conv1d.weight.shape, generator=g) * 0.5)
        L.coprod_mix_qk.copy_(torch.randn(H, generator=g))
        L.coprod_mix_v.copy_(torch.randn(H, generator=g))
        L.coprod_strength_qk.copy_(1 + 0.2 * torch.randn(H, generator=g))
        L.coprod_strength_v.copy_(1 + 0.2 * torch.randn(H, generator=g))
        for w in (L.W_q_a, L.W_q_b, L.W_k_a, L.W_k_b, L.W_v_a, L.W_v_b):
            w.copy_(torch.randn(w.shape, generator=g) * 0.3)
        B, T = 2, 11
        x = torch.randn(B, T, D, generator=g)
        qkv = F.linear(x, L.in_proj_qkv)
        qkv_padded = F.pad(qkv.transpose(1, 2), (L.conv_kernel_size - 1, 0))
        qkv_conv = L.conv1d(qkv_padded).transpose(1, 2).reshape(B, T, H, 3, K)
        q, k, v_raw = qkv_conv[:, :, :, 0, :], qkv_conv[:, :, :, 1, :], qkv_conv[:, :, :, 2, :]
        qo, ko, vo = L._generate_coproduct_channels(q, k, v_raw, x)
        fac = {}
        for nm, w in (("q_a", L.W_q_a), ("q_b", L.W_q_b), ("k_a", L.W_k_a), ("k_b", L.W_k_b),
                      ("v_a", L.W_v_a), ("v_b", L.W_v_b)):
            fac[nm] = F.linear(x.float(), w.float().reshape(-1, D)).view(B, T, H, w.shape[1], w.shape[2])
        b_proj = torch.randn(B, T, H, M, K, generator=g)
        w_proj = torch.randn(B, T, H, M, K, generator=g)
        proj_a = torch.randn(B, T, H, generator=g)
        proj_b = torch.randn(B, T, H, generator=g)
        pa = proj_a.unsqueeze(3).expand(-1, -1, -1, M).unsqueeze(-1).expand(-1, -1, -1, -1, K)
        pb = proj_b.unsqueeze(3).expand(-1, -1, -1, M).unsqueeze(-1).expand(-1, -1, -1, -1, K)
        bg = torch.sigmoid(b_proj + pa * 0.1)
        wg = torch.sigmoid(w_proj + pb * 0.1)
    torch.save(dict(H=H, K=K, M=M, qkv=qkv, conv_w=L.conv1d.weight.detach().clone(), factors=fac,
                    mix=[L.coprod_mix_qk.detach().clone(), L.coprod_mix_v.detach().clone(),
                         L.coprod_strength_qk.detach().clone(), L.coprod_strength_v.detach().clone()],
                    b_proj=b_proj, w_proj=w_proj, proj_a=proj_a, proj_b=proj_b,
                    q=qo, k=ko, v=vo, b_gates=bg, w_gates=wg), HERE / 'proj_prologue.pt')


def make_prologue():
    g = torch.Generator().manual_seed(9)
    out = {}
    for rf in (0.25, 0.5):
        L = _layer(128, 128, 16, rotary_factor=rf)
        x = torch.randn(1, 33, 1, 4, 128, generator=g)
        out[f'rope_rf{rf}'] = dict(x=x, y=L._apply_partial_rope(x, 33))
    L = _layer(128, 128, 16)
    dp = torch.randn(1, 33, 2, 4, 4, generator=g) * 3
    g_raw = torch.nn.functional.softplus(dp).clamp(max=5.0)
    rates = L.base_decay_rates.view(1, 1, 1, 1, 4)
    dec = torch.exp(-g_raw * rates).mean(dim=-1).clamp(max=L.decay_clamp)
    out['braid'] = dict(decay_proj=dp, decay=dec, clamp=L.decay_clamp)
    torch.save(out, HERE / 'prologue.pt')


if __name__ == '__main__':
    REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('GDNX_REFERENCE')
    if not REF:
        raise SystemExit('usage: make_golden.py /path/to/reference')
    sys.path.insert(0, REF)
    torch.manual_seed(0)
    makers = dict(gdn3_frozen=make_gdn3_frozen, gdn3_config0=make_gdn3_config0, kmd2=make_kmd2,
                  compaction=make_compaction, compaction_sketch=make_compaction_sketch, prologue=make_prologue, gdn3_kr_p256=make_kr_p256,
                  epilogue=make_epilogue, proj_prologue=make_projection_prologue,
                  kmd2_prologue=make_kmd2_prologue)
    only = sys.argv[2:]  # optional fixture names; default: all
    for name, fn in makers.items():
        if not only or name in only:
            fn()
    for f in sorted(HERE.glob('*.pt')):
        print(f.name, f.stat().st_size)
