"""Pin the CPU oracle to outputs the reference itself produced (tests/golden)."""
from pathlib import Path

import pytest
import torch

from oracle import recurrence as R
from oracle import prologue as PR
from oracle.inputs import expand_lanes, parity_inputs, scan_inputs, CONFIGS

GOLD = Path(__file__).parent / "golden"


def _load(name):
    return torch.load(GOLD / name, weights_only=False)


def rel_l2(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("case", ["cfg0dist_P80", "cfg0dist_P16", "parity_B1_T64", "parity_B2_T48"])
def test_gdn3_frozen_loop_bit_exact(case):
    c = _load("gdn3_frozen.pt")[case]
    if "inputs_compact" in c:
        ins = [t.contiguous() for t in expand_lanes(c["inputs_compact"], 4)]
    else:
        ins = parity_inputs(*c["shape"], c["seed"])
        for t, s in zip(ins, c["input_sums"]):
            assert t.double().sum() == s
    Y, st = R.gdn3_kr_scan(*ins, R=4, P=c["P"], dims=R.KronDims(*c["dims"]))
    assert torch.equal(Y, c["Y"]), rel_l2(Y, c["Y"])
    T = ins[0].shape[1]
    assert st.p == T % c["P"]
    # the reference's own chunked path sits within its fidelity floor of the frozen loop
    assert rel_l2(c["Y_chunked"], c["Y"]) < 2e-3


def test_gdn3_config0_dense_bit_exact_and_dense_form():
    c = _load("gdn3_config0.pt")
    cfg = CONFIGS[0]
    inp = scan_inputs(cfg["B"], cfg["T"], cfg["H"], cfg["M"], cfg["K"], cfg["V"], cfg["seed"])
    ins = [t.contiguous() for t in expand_lanes(inp, cfg["M"])]
    Y, st = R.gdn3_kr_scan(*ins, R=4, P=cfg["T"], dims=R.KronDims(8, 8, 8, 8))
    assert torch.equal(Y[:, c["t_index"]], c["Y"])
    assert Y.double().sum() == c["Y_sum"]
    # dense restatement (S = U Vb^T, compaction off) agrees to fp32 rounding
    Yd, S = R.dense_scan(*ins)
    assert rel_l2(Yd, Y) < 1e-5
    S_kr = torch.einsum("nvp,nkp->nvk", st.U, st.Vb)
    assert rel_l2(S, S_kr) < 1e-5


def test_gdn3_kr_loop_at_config2_period_bit_exact():
    """P = 256 (config 2's compaction period), four compactions, bf16-rounded inputs."""
    c = _load("gdn3_kr_p256.pt")
    B, T, H, M, K = c["shape"]
    inp = scan_inputs(B, T, H, M, K, K, seed=c["seed"], dtype=torch.bfloat16)
    ins = [t.contiguous() for t in expand_lanes(inp, M)]
    Y, st = R.gdn3_kr_scan(*ins, R=4, P=c["P"], dims=R.KronDims(*c["dims"]))
    assert torch.equal(Y[:, c["t_index"]], c["Y"])
    assert Y.double().sum() == c["Y_sum"]
    assert st.p == T % c["P"]
    assert c["chunked_floor"] < 2e-3


@pytest.mark.parametrize("case", ["r1", "r4"])
def test_kmd2_loop_bit_exact(case):
    c = _load("kmd2.pt")[case]
    q, k, v, g, be, bw, mix = c["inputs"]
    y, sc, S = R.kmd2_scan(q, k, v, g, be, bw, mix)
    assert torch.equal(y, c["y"])
    torch.testing.assert_close(y, c["y_scored"], atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(sc, c["scores"], atol=1e-6, rtol=1e-5)


def test_kmd2_known_answer():
    c = _load("kmd2.pt")["kat"]
    q, k, v, g, be, bw, _ = c["inputs"]
    y, sc, S = R.kmd2_scan(q, k, v, g, be, bw, None, dtype=torch.float64)
    assert y.item() == 12.0 and c["y"].item() == 12.0
    assert sc.item() == pytest.approx(4.0) and c["scores"].item() == pytest.approx(4.0)


def test_kmd2_equals_gdn3_dense_with_folded_lanes():
    """KMD-2 with scalar decay and beta_e = beta_w = alpha*beta is the GDN3 dense scan."""
    inp = scan_inputs(1, 40, 2, 4, 32, 32, seed=3)
    ins = expand_lanes(inp, 4)
    Yg, _ = R.dense_scan(*ins)
    B, T, H, M = inp["beta"].shape
    k = inp["k"].unsqueeze(3).expand(-1, -1, -1, M, -1).reshape(B, T, H * M, -1)
    q = inp["q"].unsqueeze(3).expand(-1, -1, -1, M, -1).reshape(B, T, H * M, 1, -1)
    v = inp["v"].unsqueeze(3).expand(-1, -1, -1, M, -1).reshape(B, T, H * M, -1)
    beta = inp["beta"].reshape(B, T, H * M)
    c = beta * (k * k).sum(-1)
    be = R.stable_alpha(c) * beta
    g = torch.exp(inp["logg"]).reshape(B, T, H * M, 1).expand(-1, -1, -1, k.shape[-1])
    y, _, _ = R.kmd2_scan(q, k, v, g, be, be)
    assert rel_l2(y, Yg.reshape(B, T, H * M, -1)) < 1e-5


def test_compaction_bit_exact():
    c = _load("compaction.pt")
    A, Bk, U, Vb = c["inputs"]
    An, Bn, _, _, err = R.compact_call(A, Bk, U, Vb, R.KronDims(), c["slow_decay"])
    assert torch.equal(An, c["A_new"]) and torch.equal(Bn, c["B_new"])
    assert torch.equal(err, c["err"])


@pytest.mark.parametrize("mode", ["sketch", "sketch_noqr"])
def test_compaction_sketch_mode_bit_exact(mode):
    c = _load("compaction_sketch.pt")
    A, Bk, U, Vb = c["inputs"]
    An, Bn, _, _, err = R.compact_sketch_call(A, Bk, U, Vb, R.KronDims(), c["slow_decay"])
    assert torch.equal(An, c[mode]["A_new"]) and torch.equal(Bn, c[mode]["B_new"])
    assert float(err) == 0.0 and float(c[mode]["err"]) == 0.0


@pytest.mark.parametrize("rf", [0.25, 0.5])
def test_lane_rope_bit_exact(rf):
    c = _load("prologue.pt")[f"rope_rf{rf}"]
    assert torch.equal(PR.apply_lane_rope(c["x"], 128, rf), c["y"])


def test_braided_decay_bit_exact():
    c = _load("prologue.pt")["braid"]
    assert torch.equal(PR.braided_decay(c["decay_proj"], clamp=c["clamp"]), c["decay"])


def test_epilogues_bit_exact():
    from oracle import epilogue as E
    c = _load("epilogue.pt")
    assert torch.equal(E.lane_route(c["y"], c["logits"], c["norm"]), c["out"])
    torch.testing.assert_close(E.rms_norm_gated(c["y_kmd2"], c["z"], c["weight"]), c["out_kmd2"], rtol=0, atol=0)


def test_projection_prologue_matches_reference():
    c = _load("proj_prologue.pt")
    f = c["factors"]
    (q, k, v), (bg, wg) = PR.projection_prologue(c["qkv"], c["conv_w"], c["H"], c["K"],
                                                 coprod=[f[n] for n in ("q_a", "q_b", "k_a", "k_b", "v_a", "v_b")],
                                                 mix=c["mix"], b_proj=c["b_proj"], proj_a=c["proj_a"],
                                                 w_proj=c["w_proj"], proj_b=c["proj_b"])
    for a, b in ((q, c["q"]), (k, c["k"]), (v, c["v"]), (bg, c["b_gates"]), (wg, c["w_gates"])):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", ["r4", "r1"])
def test_kmd2_prologue_bit_exact(case):
    """The KMD-2 prologue restatement equals the arguments the reference's forward hands its _scan."""
    c = _load("kmd2_prologue.pt")[case]
    gm, pr, sa = c["gemm"], c["params"], c["scan_args"]
    out = PR.kmd2_prologue(gm["mixed"], pr["conv_w"], gm["b"], gm["a"], gm["theta"], pr["dt_bias"], pr["A_log"],
                           pr["decay_chan"], pr["bw_off"], pr["q_slot_scale"], H=c["H"], r_out=c["r_out"])
    for o, n in zip(out, ["q", "k", "v", "g", "beta_e", "beta_w"]):
        assert torch.equal(o, sa[n]), n
