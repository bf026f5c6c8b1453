"""GPU parity of the CUDA kernels (through the C ABI) against the CPU oracle and
the reference-generated golden fixtures.

Tolerances (relative L2, as the north star states): 2e-3 for fp32 I/O,
2e-2 for bf16 I/O; compaction factors 1e-3 relative Frobenius per call.
"""
from pathlib import Path

import pytest
import torch

from gdnx_b200 import ops
from gdnx_b200.prologue import lane_rope
from oracle import recurrence as R
from oracle import prologue as PR
from oracle.inputs import expand_lanes, parity_inputs, realistic_logg, scan_inputs, CONFIGS

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
DEV = "cuda:0"
TOL32, TOL16 = 2e-3, 2e-2


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def gpu(*ts):
    return [t.to(DEV) for t in ts]


# ----------------------------------------------------------------- dense GDN3 --

def _dense_case(B, T, H, M, K, seed, dtype=torch.float32, rope_rf=None):
    inp = scan_inputs(B, T, H, M, K, K, seed, dtype)
    rope = lane_rope(M, K, K, rope_rf) if rope_rf is not None else None
    qf, kf = inp["q"].float(), inp["k"].float()
    qx = qf.unsqueeze(3).expand(-1, -1, -1, M, -1)
    kx = kf.unsqueeze(3).expand(-1, -1, -1, M, -1)
    if rope_rf is not None:
        qx = PR.apply_lane_rope(qx.contiguous(), K, rope_rf)
        kx = PR.apply_lane_rope(kx.contiguous(), K, rope_rf)
    vx = inp["v"].float().unsqueeze(3).expand(-1, -1, -1, M, -1)
    beta = inp["beta"].float()
    bg = beta.unsqueeze(-1).expand(-1, -1, -1, -1, K)
    wg = beta.unsqueeze(-1).expand(-1, -1, -1, -1, K)
    dec = torch.exp(inp["logg"].float())
    Yo, So = R.dense_scan(qx, kx, vx, bg, wg, dec)
    return inp, rope, Yo, So


@pytest.mark.parametrize("algo", ["recurrent", "auto"])
def test_config0_dense_fp32_vs_oracle_and_reference(algo):
    c = CONFIGS[0]
    inp, _, Yo, So = _dense_case(c["B"], c["T"], c["H"], c["M"], c["K"], c["seed"])
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    y, S = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", return_state=True, algo=algo)
    assert rel(y, Yo) < TOL32 and rel(S, So) < TOL32
    gold = torch.load(GOLD / "gdn3_config0.pt")
    assert rel(y.cpu()[:, gold["t_index"]], gold["Y"]) < TOL32


def test_golden_frozen_dense_case_vector_gates():
    c = torch.load(GOLD / "gdn3_frozen.pt", weights_only=False)["cfg0dist_P80"]
    ins = [t.contiguous() for t in expand_lanes(c["inputs_compact"], 4)]
    y = ops.gdn3_scan(*gpu(*ins), algo="recurrent")
    assert rel(y, c["Y"]) < TOL32


def test_parity_recipe_vector_gates_per_lane_inputs():
    ins = parity_inputs(2, 48, 2, 4, 128, 128, seed=3)
    Yo, So = R.dense_scan(*ins)
    y, S = ops.gdn3_scan(*gpu(*ins), return_state=True)
    assert rel(y, Yo) < TOL32 and rel(S, So) < TOL32


@pytest.mark.parametrize("T", [1, 17, 64, 65])
def test_ragged_lengths_and_state_continuation(T):
    inp, _, Yo, So = _dense_case(1, T, 2, 4, 64, seed=11)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    y, S = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", return_state=True)
    assert rel(y, Yo) < TOL32 and rel(S, So) < TOL32
    if T > 1:
        t1 = T // 2
        y1, S1 = ops.gdn3_scan(q[:, :t1], k[:, :t1], v[:, :t1], beta[:, :t1], beta[:, :t1], logg[:, :t1],
                               decay_kind="log", return_state=True)
        y2, S2 = ops.gdn3_scan(q[:, t1:], k[:, t1:], v[:, t1:], beta[:, t1:], beta[:, t1:], logg[:, t1:],
                               decay_kind="log", state=S1, return_state=True)
        assert rel(torch.cat([y1, y2], 1), Yo) < TOL32 and rel(S2, So) < TOL32


def test_empty_inputs_are_a_no_op():
    z = torch.zeros(0, 8, 1, 64, device=DEV)
    g = torch.zeros(0, 8, 1, 4, device=DEV)
    y = ops.gdn3_scan(z, z, z, g, g, g)
    assert y.shape == (0, 8, 1, 4, 64)


def test_bf16_rope_config1_shape_slice():
    """Config-1 distributions and lane RoPE (first 64 dims on lane 0), bf16 I/O."""
    inp, rope, Yo, So = _dense_case(1, 256, 2, 4, 128, seed=1, dtype=torch.bfloat16, rope_rf=0.5)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    for algo in ("recurrent", "auto"):
        y, S = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", rope=rope, return_state=True,
                             algo=algo)
        assert y.dtype == torch.bfloat16
        assert rel(y.float(), Yo) < TOL16 and rel(S, So) < TOL16, algo


def test_realistic_decay_dense():
    inp = scan_inputs(1, 200, 2, 4, 128, 128, seed=5)
    inp["logg"] = realistic_logg(inp["logg"].shape, seed=6)
    ins = expand_lanes(inp, 4)
    Yo, So = R.dense_scan(*ins)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    y, S = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", return_state=True)
    assert rel(y, Yo) < TOL32 and rel(S, So) < TOL32


def test_braided_decay_prologue():
    g = torch.Generator().manual_seed(21)
    inp = scan_inputs(1, 40, 2, 4, 64, 64, seed=8)
    dp = torch.randn(1, 40, 2, 4, 4, generator=g) * 3
    dec = PR.braided_decay(dp)
    qx, kx, vx, bg, wg, _ = expand_lanes(inp, 4)
    Yo, _ = R.dense_scan(qx, kx, vx, bg, wg, dec)
    q, k, v, beta, dpg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], dp)
    y = ops.gdn3_scan(q, k, v, beta, beta, dpg, decay_kind="braided")
    assert rel(y, Yo) < TOL32


# ----------------------------------------------------------------- KMD-2 --

@pytest.mark.parametrize("case", ["r1", "r4"])
def test_kmd2_golden_with_scores(case):
    c = torch.load(GOLD / "kmd2.pt", weights_only=False)[case]
    q, k, v, g, be, bw, mix = c["inputs"]
    args = gpu(q, k, v, g, be, bw) + ([mix.to(DEV)] if mix is not None else [None])
    y, sc, S = ops.kmd2_scan(*args, scores=True, return_state=True)
    _, _, So = R.kmd2_scan(q, k, v, g, be, bw, mix)
    assert rel(y, c["y"]) < TOL32
    assert rel(sc, c["scores"]) < TOL32
    assert rel(S, So.transpose(1, 2)) < TOL32


def test_kmd2_known_answer():
    q = torch.tensor([[[[[3.0]]]]]); k = torch.tensor([[[[2.0]]]]); v = torch.tensor([[[[5.0]]]])
    d = torch.tensor([[[[0.25]]]]); be = torch.tensor([[[0.7]]]); bw = torch.tensor([[[0.4]]])
    # K = V = 1 is below the kernels' smallest head size: embed in 32 with zero padding
    pad = lambda x: torch.nn.functional.pad(x, (0, 31))
    y, sc = ops.kmd2_scan(*gpu(pad(q), pad(k), pad(v), torch.nn.functional.pad(d, (0, 31), value=1.0), be, bw),
                          scores=True)
    assert abs(y[0, 0, 0, 0].item() - 12.0) < 1e-5
    assert abs(sc.item() - 4.0) < 1e-5


# ----------------------------------------------------------------- decode --

@pytest.mark.parametrize("bf16", [False, True])
def test_decode_step_gdn3(bf16):
    g = torch.Generator().manual_seed(31)
    B, H, M, K = 4, 2, 4, 128
    S0 = torch.randn(B * H * M, K, K, generator=g) * 0.02
    inp = scan_inputs(B, 1, H, M, K, K, seed=32, dtype=torch.bfloat16 if bf16 else torch.float32)
    q, k, v = (inp[n][:, 0].float() for n in ("q", "k", "v"))
    beta, logg = inp["beta"][:, 0].float(), inp["logg"][:, 0].float()
    N = B * H * M
    ex = lambda x: x.unsqueeze(2).expand(-1, -1, M, -1).reshape(N, -1)
    yo, So = R.dense_decode_step(S0, ex(q), ex(k), ex(v), beta.reshape(N, 1), beta.reshape(N, 1),
                                 torch.exp(logg).reshape(N))
    S = S0.to(DEV).contiguous()
    qg, kg, vg = (inp[n][:, 0].to(DEV) for n in ("q", "k", "v"))
    y = ops.decode_step(S, qg, kg, vg, inp["beta"][:, 0].to(DEV), inp["beta"][:, 0].to(DEV),
                        inp["logg"][:, 0].to(DEV), decay_kind="log")
    tol = TOL16 if bf16 else TOL32
    assert rel(y.float().reshape(N, K), yo) < tol and rel(S, So) < TOL32


def test_decode_step_kmd2_per_channel_decay_and_slots():
    c = torch.load(GOLD / "kmd2.pt", weights_only=False)["r4"]
    q, k, v, g, be, bw, mix = c["inputs"]
    # run the oracle for 5 tokens, then one decode step from its state
    y_ref, _, S5 = R.kmd2_scan(q[:, :5], k[:, :5], v[:, :5], g[:, :5], be[:, :5], bw[:, :5], mix)
    y6, _, S6 = R.kmd2_scan(q[:, 5:6], k[:, 5:6], v[:, 5:6], g[:, 5:6], be[:, 5:6], bw[:, 5:6], mix, S0=S5)
    # K = V = 32 takes the generic recurrent path inside gdnx_decode_step
    S = S5.transpose(1, 2).contiguous().to(DEV)
    y = ops.decode_step(S, *gpu(q[:, 5], k[:, 5], v[:, 5], be[:, 5], bw[:, 5], g[:, 5]), mode="kmd2",
                        out_mix=mix.to(DEV))
    assert rel(y, y6[:, 0]) < TOL32 and rel(S, S6.transpose(1, 2)) < TOL32


# ----------------------------------------------------------------- compaction --

def test_compaction_per_call_factors():
    c = torch.load(GOLD / "compaction.pt", weights_only=False)
    A, Bk, U, Vb = c["inputs"]
    N = A.shape[0]
    G = R.sketch_matrix(N, 64, 8)
    dims = R.KronDims()
    An, Bn, _, _, err, (As, Bs, Ss) = R.compact_call(A, Bk, U, Vb, dims, c["slow_decay"], G=G, canon_signs=True,
                                                   return_factors=True)
    # the un-canonicalised oracle equals the reference's own call
    An_ref, Bn_ref, _, _, _ = R.compact_call(A, Bk, U, Vb, dims, c["slow_decay"], G=G)
    assert torch.equal(An_ref, c["A_new"])
    Ag, Bg, Ug, Vg, Gg = gpu(A, Bk, U, Vb, G)
    Ag, Bg = Ag.contiguous(), Bg.contiguous()
    e = ops.compact(Ag, Bg, Ug, Vg, Gg.contiguous(), slow_decay=c["slow_decay"])
    d = c["slow_decay"]
    As_g = (Ag.cpu() - d * A) / (1 - d)
    Bs_g = (Bg.cpu() - d * Bk) / (1 - d)
    for n in range(N):
        gap = (Ss[n, :-1] - Ss[n, 1:]).abs().min() / Ss[n, 0]
        if gap < 1e-3:
            continue  # near-degenerate singular values: the factors are ill-posed
        assert rel(As_g[n], As[n]) < 1e-3, n
        assert rel(Bs_g[n], Bs[n]) < 1e-3, n
    # sign-invariant operator check for every chain
    kron = lambda A_, B_: torch.einsum("rab,rcd->acbd", A_, B_).reshape(256, 64)
    for n in range(N):
        assert rel(kron(As_g[n], Bs_g[n]), kron(As[n], Bs[n])) < 1e-3
    assert abs(e.sum().item() - err.item()) / err.item() < 1e-3


# ----------------------------------------------------------------- GDN3-KR --

@pytest.mark.parametrize("case", ["parity_B1_T64", "parity_B2_T48", "cfg0dist_P16"])
def test_kr_scan_vs_oracle_and_reference(case):
    c = torch.load(GOLD / "gdn3_frozen.pt", weights_only=False)[case]
    if "inputs_compact" in c:
        ins = [t.contiguous() for t in expand_lanes(c["inputs_compact"], 4)]
    else:
        ins = parity_inputs(*c["shape"], c["seed"])
    B, T, H, M, K = ins[0].shape
    N, P = B * H * M, c["P"]
    dims = c["dims"]
    n = dims[2] * dims[3]
    G = R.sketch_matrix(N, n, 8)
    Yo, st = R.gdn3_kr_scan(*ins, R=4, P=P, dims=R.KronDims(*dims), G=G, canon_signs=True)
    state = ops.KRState.zeros(N, 4, P, dims, K, K, DEV)
    y = ops.gdn3_kr_scan(*gpu(*ins), state, G.to(DEV), P=P, dims=dims)
    assert rel(y, Yo) < TOL32
    assert rel(y, c["Y"]) < TOL32          # the reference itself (LAPACK signs)
    assert int(state.slot[0]) == st.p
    assert rel(state.U, st.U) < TOL32 and rel(state.Vb, st.Vb) < TOL32
    assert rel(torch.einsum("nrab,nrcd->nacbd", state.A.cpu(), state.Bk.cpu()),
               torch.einsum("nrab,nrcd->nacbd", st.A, st.Bk)) < 1e-2


def test_kr_scan_chunked_calls_equal_one_call():
    ins = parity_inputs(1, 80, 1, 4, 128, 128, seed=4)
    N, P, dims = 4, 16, (16, 16, 8, 8)
    G = R.sketch_matrix(N, 64, 8).to(DEV)
    s1 = ops.KRState.zeros(N, 4, P, dims, 128, 128, DEV)
    y1 = ops.gdn3_kr_scan(*gpu(*ins), s1, G, P=P)
    s2 = ops.KRState.zeros(N, 4, P, dims, 128, 128, DEV)
    parts = [ops.gdn3_kr_scan(*gpu(*[t[:, a:b] for t in ins]), s2, G, P=P) for a, b in ((0, 23), (23, 80))]
    assert rel(torch.cat(parts, 1), y1) < 1e-5
    assert rel(s2.U, s1.U) < 1e-5 and rel(s2.A, s1.A) < 1e-4


def test_kr_scan_one_cta_and_cluster_paths_agree():
    """80 chains (more CTA pairs than SMs: one CTA per chain) against the same chains run
    16 at a time (a two-CTA cluster per chain)."""
    B, T, P, dims = 20, 48, 16, (16, 16, 8, 8)
    ins = parity_inputs(B, T, 1, 4, 128, 128, seed=9)
    N = B * 4
    G = R.sketch_matrix(N, 64, 8).to(DEV)
    s_all = ops.KRState.zeros(N, 4, P, dims, 128, 128, DEV)
    y_all = ops.gdn3_kr_scan(*gpu(*ins), s_all, G, P=P)
    ys, us = [], []
    for b0 in range(0, B, 4):
        st = ops.KRState.zeros(16, 4, P, dims, 128, 128, DEV)
        ys.append(ops.gdn3_kr_scan(*gpu(*[t[b0:b0 + 4] for t in ins]), st, G[4 * b0:4 * b0 + 16], P=P))
        us.append(st.U)
    assert rel(torch.cat(ys, 0), y_all) < 1e-4
    assert rel(torch.cat(us, 0), s_all.U) < 1e-4


# ----------------------------------------------------------------- chunked tensor-core path --

@pytest.mark.parametrize("T,rope_rf", [(64, None), (1, None), (100, 0.5), (256, 0.5), (130, 0.25)])
def test_chunked_vs_oracle(T, rope_rf):
    inp, rope, Yo, So = _dense_case(2, T, 2, 4, 128, seed=40 + T, dtype=torch.bfloat16, rope_rf=rope_rf)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    y, S = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", rope=rope, return_state=True,
                         algo="chunked")
    assert rel(y.float(), Yo) < TOL16 and rel(S, So) < TOL16


def test_chunked_state_continuation_and_fp32_out():
    inp, _, Yo, So = _dense_case(1, 192, 2, 4, 128, seed=50, dtype=torch.bfloat16)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    a = lambda x, s: x[:, s]
    s1, s2 = slice(0, 70), slice(70, 192)
    y1, S1 = ops.gdn3_scan(a(q, s1), a(k, s1), a(v, s1), a(beta, s1), a(beta, s1), a(logg, s1), decay_kind="log",
                           return_state=True, algo="chunked", out_dtype=torch.float32)
    y2, S2 = ops.gdn3_scan(a(q, s2), a(k, s2), a(v, s2), a(beta, s2), a(beta, s2), a(logg, s2), decay_kind="log",
                           state=S1, return_state=True, algo="chunked", out_dtype=torch.float32)
    assert y1.dtype == torch.float32
    assert rel(torch.cat([y1, y2], 1), Yo) < TOL16 and rel(S2, So) < TOL16


def test_chunked_realistic_decay():
    inp = scan_inputs(1, 256, 2, 4, 128, 128, seed=51, dtype=torch.bfloat16)
    inp["logg"] = realistic_logg(inp["logg"].shape, seed=52).to(torch.bfloat16)
    Yo, So = R.dense_scan(*expand_lanes(inp, 4))
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    y, S = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", return_state=True, algo="chunked")
    assert rel(y.float(), Yo) < TOL16 and rel(S, So) < TOL16


def test_chunked_agrees_with_recurrent_on_config1_slice():
    """Both CUDA paths on the same bf16 inputs (B=8 slice of config 1, T=512)."""
    inp = scan_inputs(8, 512, 16, 4, 128, 128, seed=1, dtype=torch.bfloat16)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    rope = lane_rope(4, 128, 128, 0.5)
    yc, Sc = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", rope=rope, return_state=True,
                           algo="chunked", out_dtype=torch.float32)
    yr, Sr = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", rope=rope, return_state=True,
                           algo="recurrent", out_dtype=torch.float32)
    assert rel(yc, yr) < TOL16 and rel(Sc, Sr) < TOL16


def test_chunked_kmd2_scalar_decay():
    g = torch.Generator().manual_seed(53)
    B, T, H, dk = 2, 150, 3, 128
    q = (torch.nn.functional.normalize(torch.randn(B, T, H, 1, dk, generator=g), dim=-1) * dk ** -0.5)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, dk, generator=g), dim=-1)
    v = torch.randn(B, T, H, dk, generator=g)
    gd = torch.exp(-torch.nn.functional.softplus(1.2 * torch.randn(B, T, H, generator=g) - 0.6))
    be = torch.sigmoid(torch.randn(B, T, H, generator=g))
    bw = torch.sigmoid(torch.randn(B, T, H, generator=g))
    q, k, v = (x.to(torch.bfloat16).float() for x in (q, k, v))
    y_ref, _, S_ref = R.kmd2_scan(q, k, v, gd[..., None].expand(-1, -1, -1, dk), be, bw)
    bf = lambda x: x.to(torch.bfloat16).to(DEV)
    y, S = ops.kmd2_scan(bf(q), bf(k), bf(v), gd.to(DEV), be.to(DEV), bw.to(DEV), return_state=True, algo="chunked")
    assert rel(y, y_ref) < TOL16 and rel(S, S_ref.transpose(1, 2)) < TOL16


def test_kmd2_scores_request_takes_a_path_that_writes_them():
    """Scalar-decay KMD-2 with scores must not route to the chunked kernel (which has no scores)."""
    g = torch.Generator().manual_seed(54)
    B, T, H, dk = 1, 70, 2, 128
    q = torch.randn(B, T, H, 1, dk, generator=g) * dk ** -0.5
    k = torch.nn.functional.normalize(torch.randn(B, T, H, dk, generator=g), dim=-1)
    v = torch.randn(B, T, H, dk, generator=g)
    gd = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, H, generator=g)))
    be = torch.sigmoid(torch.randn(B, T, H, generator=g))
    bw = torch.sigmoid(torch.randn(B, T, H, generator=g))
    q, k, v = (x.to(torch.bfloat16).float() for x in (q, k, v))
    _, sc_ref, _ = R.kmd2_scan(q, k, v, gd[..., None].expand(-1, -1, -1, dk), be, bw)
    bf = lambda x: x.to(torch.bfloat16).to(DEV)
    _, sc = ops.kmd2_scan(bf(q), bf(k), bf(v), gd.to(DEV), be.to(DEV), bw.to(DEV), scores=True)
    assert rel(sc, sc_ref) < TOL16


def test_decode_step_many_chains_per_cta():
    """More chains than SMs: every persistent CTA cycles its three state stages."""
    g = torch.Generator().manual_seed(33)
    B, H, M, K = 64, 4, 4, 128
    N = B * H * M
    S0 = torch.randn(N, K, K, generator=g) * 0.02
    inp = scan_inputs(B, 1, H, M, K, K, seed=34, dtype=torch.bfloat16)
    q, k, v = (inp[n][:, 0].float() for n in ("q", "k", "v"))
    beta, logg = inp["beta"][:, 0].float(), inp["logg"][:, 0].float()
    ex = lambda x: x.unsqueeze(2).expand(-1, -1, M, -1).reshape(N, -1)
    yo, So = R.dense_decode_step(S0, ex(q), ex(k), ex(v), beta.reshape(N, 1), beta.reshape(N, 1),
                                 torch.exp(logg).reshape(N))
    S = S0.to(DEV).contiguous()
    y = ops.decode_step(S, *(inp[n][:, 0].to(DEV) for n in ("q", "k", "v")), inp["beta"][:, 0].to(DEV),
                        inp["beta"][:, 0].to(DEV), inp["logg"][:, 0].to(DEV), decay_kind="log")
    y2 = ops.decode_step(S, *(inp[n][:, 0].to(DEV) for n in ("q", "k", "v")), inp["beta"][:, 0].to(DEV),
                         inp["beta"][:, 0].to(DEV), inp["logg"][:, 0].to(DEV), decay_kind="log")
    yo2, So2 = R.dense_decode_step(So, ex(q), ex(k), ex(v), beta.reshape(N, 1), beta.reshape(N, 1),
                                   torch.exp(logg).reshape(N))
    assert rel(y.float().reshape(N, K), yo) < TOL16 and rel(y2.float().reshape(N, K), yo2) < TOL16
    assert rel(S, So2) < TOL32


@pytest.mark.parametrize("pos0", [0, 4096])
def test_decode_step_with_lane_rope(pos0):
    g = torch.Generator().manual_seed(35)
    B, H, M, K = 8, 4, 4, 128
    N = B * H * M
    S0 = torch.randn(N, K, K, generator=g) * 0.02
    inp = scan_inputs(B, 1, H, M, K, K, seed=36, dtype=torch.bfloat16)
    rf = 0.5
    qx = PR.apply_lane_rope(inp["q"].float().unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, rf, pos0=pos0)
    kx = PR.apply_lane_rope(inp["k"].float().unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, rf, pos0=pos0)
    v = inp["v"][:, 0].float().unsqueeze(2).expand(-1, -1, M, -1).reshape(N, K)
    beta, logg = inp["beta"][:, 0].float(), inp["logg"][:, 0].float()
    yo, So = R.dense_decode_step(S0, qx[:, 0].reshape(N, K), kx[:, 0].reshape(N, K), v, beta.reshape(N, 1),
                                 beta.reshape(N, 1), torch.exp(logg).reshape(N))
    S = S0.to(DEV).contiguous()
    rope = lane_rope(M, K, K, rf, pos0=pos0)
    y = ops.decode_step(S, *(inp[n][:, 0].to(DEV) for n in ("q", "k", "v")), inp["beta"][:, 0].to(DEV),
                        inp["beta"][:, 0].to(DEV), inp["logg"][:, 0].to(DEV), decay_kind="log", rope=rope)
    assert rel(y.float().reshape(N, K), yo) < TOL16 and rel(S, So) < TOL32


# ----------------------------------------------------------------- drop-in modules --

@pytest.mark.parametrize("case,P", [("parity_B1_T64", 16), ("parity_B2_T48", 16), ("cfg0dist_P80", 80),
                                     ("cfg0dist_P80", 128)])
def test_gdn3_dropin_matches_reference_outputs(case, P):
    import types
    from gdnx_b200.gdn3_upgrade import patch_layer
    c = torch.load(GOLD / "gdn3_frozen.pt", weights_only=False)[case]
    ins = ([t.contiguous() for t in expand_lanes(c["inputs_compact"], 4)] if "inputs_compact" in c
           else parity_inputs(*c["shape"], c["seed"]))
    a_v, a_k, b_v, b_k = c["dims"]
    layer = types.SimpleNamespace(R=4, P=P, a_v=a_v, a_k=a_k, b_v=b_v, b_k=b_k, slow_decay=0.97, compact_mode="svd")
    patch_layer(layer)
    y = layer._gdn3_recurrent_state(*gpu(*ins))
    assert y.dtype == torch.float32 and y.shape == c["Y"].shape
    assert rel(y, c["Y"]) < TOL32   # P >= T: no compaction reaches the outputs


@pytest.mark.parametrize("case", ["r1", "r4"])
def test_kmd2_fast_scan_dropin(case):
    from gdnx_b200 import kmd2_fast_scan
    c = torch.load(GOLD / "kmd2.pt", weights_only=False)[case]
    q, k, v, g, be, bw, mix = c["inputs"]
    args = gpu(q, k, v, g, be, bw)
    mixg = mix.to(DEV) if mix is not None else None
    y = kmd2_fast_scan.scan(*args, mixg)
    y2, sc = kmd2_fast_scan.scan_with_update_norm(*args, mixg)
    assert rel(y, c["y"]) < TOL32 and rel(y2, c["y"]) < TOL32 and rel(sc, c["scores"]) < TOL32


def test_kr_scan_with_lane_rope_and_log_decay():
    inp = scan_inputs(1, 40, 2, 4, 128, 128, seed=71)
    M, K, rf, P = 4, 128, 0.5, 16
    qx = PR.apply_lane_rope(inp["q"].unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, rf)
    kx = PR.apply_lane_rope(inp["k"].unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, rf)
    vx = inp["v"].unsqueeze(3).expand(-1, -1, -1, M, -1)
    bg = inp["beta"].unsqueeze(-1).expand(-1, -1, -1, -1, K)
    N = 1 * 2 * M
    G = R.sketch_matrix(N, 64, 8)
    Yo, st = R.gdn3_kr_scan(qx, kx, vx, bg, bg, torch.exp(inp["logg"]), R=4, P=P, G=G, canon_signs=True)
    state = ops.KRState.zeros(N, 4, P, (16, 16, 8, 8), K, K, DEV)
    q, k, v, beta, logg = gpu(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
    y = ops.gdn3_kr_scan(q, k, v, beta, beta, logg, state, G.to(DEV), P=P, decay_kind="log",
                         rope=lane_rope(M, K, K, rf))
    assert rel(y, Yo) < TOL32 and rel(state.U, st.U) < TOL32
