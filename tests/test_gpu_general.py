"""The general two-pass tensor-core scan (``wyg_*`` kernels) on the input forms the
reference modules pass: GDN3 vector erase/write gates and per-lane rotated
features (``GDN3LinearAttn.forward``, gdn3/gdn3_upgrade.py:785-830), and KMD-2
per-channel decay, query slots mixed by ``out_mix`` and update-norm scores
(``KMD2NativeAttn.forward`` -> ``kmd2_fast_scan.scan``, gdn3/kmd2_native.py:150-172).

Against the fp32 oracle on the same inputs.  The tensor-core operands are bf16,
so the bar is the bf16 one (relative L2 2e-2) -- tighter than the gate of the
reference's own chunked fast scan it replaces (forward relMSE 2e-3, i.e. relative
L2 4.5e-2; research/kernel_ab/bench_scan.py:24-25).
"""
import pytest
import torch

from gdnx_b200 import ops
from gdnx_b200.prologue import lane_rope
from oracle import recurrence as R
from oracle import prologue as PR
from oracle.inputs import parity_inputs, realistic_logg, scan_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL16 = 2e-2


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def gpu(*ts):
    return [t.to(DEV) for t in ts]


def _gdn3_module_inputs(B, T, H, M, seed, rf=0.5):
    """GDN3LinearAttn-like inputs: rotated per-lane q/k (L2-normalised heads),
    vector gates sigmoid(N(0,1)), braided-range decays in (0.78, 0.999)."""
    g = torch.Generator().manual_seed(seed)
    K = 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1)
    v = torch.randn(B, T, H, K, generator=g)
    qx = PR.apply_lane_rope(q.unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, rf)
    kx = PR.apply_lane_rope(k.unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, rf)
    vx = v.unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous()
    bg = torch.sigmoid(torch.randn(B, T, H, M, K, generator=g))
    wg = torch.sigmoid(torch.randn(B, T, H, M, K, generator=g))
    dec = 0.78 + 0.219 * torch.rand(B, T, H, M, generator=g)
    return [qx, kx, vx, bg, wg, dec]


@pytest.mark.parametrize("T", [1, 64, 100, 256])
def test_gdn3_vector_gates_bf16(T):
    ins = _gdn3_module_inputs(2, T, 2, 4, seed=300 + T)
    ins = [t.to(torch.bfloat16) for t in ins[:5]] + [ins[5]]
    Yo, So = R.dense_scan(*[t.float() for t in ins])
    y, S = ops.gdn3_scan(*gpu(*ins), return_state=True, out_dtype=torch.float32)
    assert rel(y, Yo) < TOL16 and rel(S, So) < TOL16


def test_gdn3_vector_gates_fp32_forced_onto_tensor_cores_and_auto_stays_exact():
    ins = _gdn3_module_inputs(1, 192, 2, 4, seed=311)
    Yo, So = R.dense_scan(*ins)
    y, S = ops.gdn3_scan(*gpu(*ins), return_state=True, algo="chunked")
    e_tc = rel(y, Yo)
    assert e_tc < TOL16 and rel(S, So) < TOL16
    y2, S2 = ops.gdn3_scan(*gpu(*ins), return_state=True)  # fp32 GDN3: exact recurrence
    assert rel(y2, Yo) < 2e-3 and rel(S2, So) < 2e-3


def test_gdn3_reference_parity_recipe_bf16_and_state_continuation():
    ins = parity_inputs(2, 160, 1, 4, 128, 128, seed=312)
    bf = [t.to(torch.bfloat16) for t in ins[:5]] + [ins[5]]
    f = [t.float() for t in bf[:5]] + [bf[5]]
    Yo, So = R.dense_scan(*f)
    a, b = slice(0, 70), slice(70, 160)
    y1, S1 = ops.gdn3_scan(*gpu(*[t[:, a] for t in bf]), return_state=True, out_dtype=torch.float32)
    y2, S2 = ops.gdn3_scan(*gpu(*[t[:, b] for t in bf]), state=S1, return_state=True, out_dtype=torch.float32)
    assert rel(torch.cat([y1, y2], 1), Yo) < TOL16 and rel(S2, So) < TOL16


def test_general_path_agrees_with_scalar_gate_path():
    """Vector gates that repeat one value per token take the general kernels; the same
    values as scalar gates take the scalar-gate two-pass kernels: same results."""
    inp = scan_inputs(2, 200, 2, 4, 128, 128, seed=313, dtype=torch.bfloat16)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    rope = lane_rope(4, 128, 128, 0.5)
    y1, S1 = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", rope=rope, return_state=True,
                           out_dtype=torch.float32)
    bvec = beta.unsqueeze(-1).expand(-1, -1, -1, -1, 128).contiguous()
    y2, S2 = ops.gdn3_scan(q, k, v, bvec, bvec, logg, decay_kind="log", rope=rope, return_state=True,
                           out_dtype=torch.float32)
    f = {n: t.float() for n, t in inp.items()}
    qx = PR.apply_lane_rope(f["q"].unsqueeze(3).expand(-1, -1, -1, 4, -1).contiguous(), 128, 0.5)
    kx = PR.apply_lane_rope(f["k"].unsqueeze(3).expand(-1, -1, -1, 4, -1).contiguous(), 128, 0.5)
    vx = f["v"].unsqueeze(3).expand(-1, -1, -1, 4, -1)
    Yo, So = R.dense_scan(qx, kx, vx, f["beta"].unsqueeze(-1), f["beta"].unsqueeze(-1), torch.exp(f["logg"]))
    assert rel(y2, Yo) < TOL16 and rel(S2, So) < TOL16
    assert rel(y2, y1) < TOL16 and rel(S2, S1) < TOL16


def test_gdn3_braided_decay_and_vector_gates():
    ins = _gdn3_module_inputs(1, 130, 2, 4, seed=314)
    g = torch.Generator().manual_seed(315)
    dp = torch.randn(1, 130, 2, 4, 4, generator=g) * 3
    dec = PR.braided_decay(dp)
    bf = [t.to(torch.bfloat16) for t in ins[:5]]
    Yo, So = R.dense_scan(*[t.float() for t in bf], dec)
    y, S = ops.gdn3_scan(*gpu(*bf), dp.to(DEV), decay_kind="braided", return_state=True, out_dtype=torch.float32)
    assert rel(y, Yo) < TOL16 and rel(S, So) < TOL16


def _kmd2_inputs(B, T, H, r_out, seed, realistic=True, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    dk = 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, r_out, dk, generator=g), dim=-1) * dk ** -0.5
    k = torch.nn.functional.normalize(torch.randn(B, T, H, dk, generator=g), dim=-1)
    v = torch.randn(B, T, H, dk, generator=g)
    if realistic:
        gd = torch.exp(-torch.nn.functional.softplus(1.2 * torch.randn(B, T, H, dk, generator=g) - 0.6))
    else:
        gd = torch.exp(-torch.rand(B, T, H, dk, generator=g) * 0.05)
    be = torch.sigmoid(torch.randn(B, T, H, generator=g))
    bw = torch.sigmoid(torch.randn(B, T, H, generator=g))
    mix = torch.randn(H, r_out, generator=g) if r_out > 1 else None
    return [t.to(dtype) for t in (q, k, v)] + [gd, be, bw], mix


@pytest.mark.parametrize("r_out,T,realistic", [(1, 256, True), (4, 200, True), (4, 129, False)])
def test_kmd2_per_channel_decay_slots_and_scores(r_out, T, realistic):
    (q, k, v, gd, be, bw), mix = _kmd2_inputs(2, T, 3, r_out, seed=320 + T, realistic=realistic)
    yo, so, _ = R.kmd2_scan(q, k, v, gd, be, bw, mix)
    args = gpu(q, k, v, gd, be, bw)
    mixg = mix.to(DEV) if mix is not None else None
    y, sc = ops.kmd2_scan(*args, mixg, scores=True)
    assert rel(y, yo) < TOL16 and rel(sc, so) < TOL16
    y2 = ops.kmd2_scan(*args, mixg)
    assert rel(y2, y) < 1e-6


def test_kmd2_fast_scan_dropin_runs_the_tensor_core_kernels_with_state():
    from gdnx_b200 import kmd2_fast_scan
    (q, k, v, gd, be, bw), mix = _kmd2_inputs(1, 300, 2, 4, seed=330)
    yo, so, So = R.kmd2_scan(q, k, v, gd, be, bw, mix)
    args = gpu(q, k, v, gd, be, bw)
    y = kmd2_fast_scan.scan(*args, mix.to(DEV))
    y2, sc = kmd2_fast_scan.scan_with_update_norm(*args, mix.to(DEV))
    assert rel(y, yo) < TOL16 and rel(y2, yo) < TOL16 and rel(sc, so) < TOL16
    _, S = ops.kmd2_scan(*args, mix.to(DEV), return_state=True)
    assert rel(S, So.transpose(1, 2)) < TOL16


def test_kmd2_strong_per_channel_decay_inside_the_domain():
    """Per-token decays down to 0.006 (a 16-token block spans up to 2^-118)."""
    (q, k, v, gd, be, bw), _ = _kmd2_inputs(1, 192, 2, 1, seed=331)
    g = torch.Generator().manual_seed(332)
    gd = torch.exp(-5.1 * torch.rand(gd.shape, generator=g))
    yo, so, _ = R.kmd2_scan(q, k, v, gd, be, bw)
    y, sc = ops.kmd2_scan(*gpu(q, k, v, gd, be, bw), scores=True)
    assert rel(y, yo) < TOL16 and rel(sc, so) < TOL16


def test_kmd2_bf16_inputs():
    (q, k, v, gd, be, bw), mix = _kmd2_inputs(2, 256, 2, 4, seed=333, dtype=torch.bfloat16)
    yo, so, _ = R.kmd2_scan(q.float(), k.float(), v.float(), gd, be, bw, mix)
    y = ops.kmd2_scan(*gpu(q, k, v, gd, be, bw), mix.to(DEV))
    assert rel(y, yo) < TOL16


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.key for e in prof.key_averages()}


def test_module_input_forms_launch_the_tensor_core_kernels():
    """What the KMD-2 fast-scan drop-in and a bf16 GDN3 layer pass reaches wyg_*, not the
    token-recurrent kernel."""
    from gdnx_b200 import kmd2_fast_scan
    (q, k, v, gd, be, bw), mix = _kmd2_inputs(1, 128, 2, 4, seed=340)
    args = gpu(q, k, v, gd, be, bw)
    names = _kernel_names(lambda: kmd2_fast_scan.scan_with_update_norm(*args, mix.to(DEV)))
    assert any("wyg_chain_kernel" in n for n in names) and any("wyg_prep_kernel" in n for n in names), names
    assert not any("recurrent_scan_kernel" in n for n in names), names
    ins = _gdn3_module_inputs(1, 128, 2, 4, seed=341)
    bf = gpu(*[t.to(torch.bfloat16) for t in ins[:5]] + [ins[5]])
    names = _kernel_names(lambda: ops.gdn3_scan(*bf))
    assert any("wyg_chain_kernel" in n for n in names), names
    assert not any("recurrent_scan_kernel" in n for n in names), names


def test_long_call_runs_in_slabs_with_bounded_workspace():
    """64 chains x 16,384 tokens needs 1.2 GB of records at once: the call runs as two
    slabs carrying the state, its workspace stays near 1 GiB, and it matches the exact
    recurrence (per-lane bf16 inputs, vector gates, scores-free GDN3)."""
    B, T, H, M, K = 1, 16384, 16, 4, 128
    g = torch.Generator(device=DEV).manual_seed(350)
    bf = torch.bfloat16
    q = torch.nn.functional.normalize(torch.randn(B, T, H, M, K, device=DEV, generator=g), dim=-1).to(bf)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, M, K, device=DEV, generator=g), dim=-1).to(bf)
    v = torch.randn(B, T, H, M, K, device=DEV, generator=g).to(bf)
    bg = torch.sigmoid(torch.randn(B, T, H, M, K, device=DEV, generator=g)).to(bf)
    wg = torch.sigmoid(torch.randn(B, T, H, M, K, device=DEV, generator=g)).to(bf)
    dec = 0.9 + 0.099 * torch.rand(B, T, H, M, device=DEV, generator=g)
    from gdnx_b200 import _lib as L
    import ctypes as C
    a = L.ScanArgs()
    a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, M, K, K
    a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_GDN3, L.GDNX_ALGO_AUTO, 1, 64
    a.q, a.k, a.v = ops._view(q, True), ops._view(k, True), ops._view(v, True)
    a.gate_e, a.gate_w, a.decay = ops._view(bg, True), ops._view(wg, True), ops._view(dec.unsqueeze(-1), True)
    need = L.load().gdnx_scan_workspace_bytes(C.byref(a))
    assert need < (1 << 30) + (64 << 20)
    y, S = ops.gdn3_scan(q, k, v, bg, wg, dec, return_state=True, out_dtype=torch.float32)
    y2, S2 = ops.gdn3_scan(q, k, v, bg, wg, dec, return_state=True, out_dtype=torch.float32, algo="recurrent")
    assert rel(y, y2) < TOL16 and rel(S, S2) < TOL16
