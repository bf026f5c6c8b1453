"""The GDN3 projection prologue kernel (``gdnx_gdn3_prologue``) against the reference's
own conv module / coproduct blend / gate activations (fixture), and the whole layer
core (prologue -> scan with in-kernel lane RoPE and braided decay -> lane routing)
against the oracle chain."""
from pathlib import Path

import pytest
import torch

from gdnx_b200 import ops
from oracle import epilogue as E
from oracle import prologue as PR
from oracle import recurrence as R

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
DEV = "cuda:0"


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _fixture():
    c = torch.load(GOLD / "proj_prologue.pt", weights_only=False)
    f = c["factors"]
    fac = [f[n].to(DEV) for n in ("q_a", "q_b", "k_a", "k_b", "v_a", "v_b")]
    return c, fac


def test_prologue_matches_reference_fixture():
    c, fac = _fixture()
    (q, k, v), (bg, wg) = ops.gdn3_prologue(c["qkv"].to(DEV), c["conv_w"].to(DEV), H=c["H"], K=c["K"], M=c["M"],
                                            coprod=fac, mix=[m.to(DEV) for m in c["mix"]],
                                            b_proj=c["b_proj"].to(DEV), proj_a=c["proj_a"].to(DEV),
                                            w_proj=c["w_proj"].to(DEV), proj_b=c["proj_b"].to(DEV))
    for a, b in ((q, c["q"]), (k, c["k"]), (v, c["v"]), (bg, c["b_gates"]), (wg, c["w_gates"])):
        assert rel(a, b) < 1e-5


def test_layer_core_chain_bf16():
    """prologue (bf16 out) -> general scan (vector gates, lane RoPE, braided decay) -> routing."""
    from gdnx_b200.prologue import lane_rope
    c, fac = _fixture()
    H, K, M = c["H"], c["K"], c["M"]
    B, T = c["qkv"].shape[:2]
    g = torch.Generator().manual_seed(3)
    dp = torch.randn(B, T, H, M, 4, generator=g)
    logits = torch.randn(B, T, H, M, generator=g)
    norm = 1 + 0.1 * torch.randn(K, generator=g)
    (q, k, v), (bg, wg) = ops.gdn3_prologue(c["qkv"].to(DEV), c["conv_w"].to(DEV), H=H, K=K, M=M, coprod=fac,
                                            mix=[m.to(DEV) for m in c["mix"]], b_proj=c["b_proj"].to(DEV),
                                            proj_a=c["proj_a"].to(DEV), w_proj=c["w_proj"].to(DEV),
                                            proj_b=c["proj_b"].to(DEV), out_dtype=torch.bfloat16)
    y = ops.gdn3_scan(q, k, v, bg, wg, dp.to(DEV), decay_kind="braided", rope=lane_rope(M, K, K, 0.5),
                      out_dtype=torch.float32)
    out = ops.lane_route(y, logits.to(DEV), norm.to(DEV))
    # oracle chain on the same bf16-rounded prologue outputs
    qf, kf, vf, bgf, wgf = (t.float().cpu() for t in (q, k, v, bg, wg))
    qx = PR.apply_lane_rope(qf.unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, 0.5)
    kx = PR.apply_lane_rope(kf.unsqueeze(3).expand(-1, -1, -1, M, -1).contiguous(), K, 0.5)
    vx = vf.unsqueeze(3).expand(-1, -1, -1, M, -1)
    Yo, _ = R.dense_scan(qx, kx, vx, bgf, wgf, PR.braided_decay(dp))
    assert rel(y, Yo) < 2e-2
    assert rel(out, E.lane_route(Yo, logits, norm)) < 2e-2
    # and the prologue outputs themselves against the fixture at bf16 rounding
    assert rel(q, c["q"]) < 1e-2 and rel(bg, c["b_gates"]) < 1e-2


def _kmd2_prologue_dev(c):
    gm, pr = c["gemm"], c["params"]
    dv = lambda t: t.to(DEV) if t is not None else None
    return ops.kmd2_prologue(dv(gm["mixed"]), dv(pr["conv_w"]), dv(gm["b"]), dv(gm["a"]), dv(gm["theta"]), H=c["H"],
                             dt_bias=dv(pr["dt_bias"]), A_log=dv(pr["A_log"]), decay_chan=dv(pr["decay_chan"]),
                             bw_off=dv(pr["bw_off"]), q_slot_scale=dv(pr["q_slot_scale"]), r_out=c["r_out"])


@pytest.mark.parametrize("case", ["r4", "r1"])
def test_kmd2_prologue_matches_reference_scan_arguments(case):
    """gdnx_kmd2_prologue from the GEMM outputs against the _scan arguments recorded from the
    reference's own KMD2NativeAttn.forward (fp32; the cumulative rotation reaches ~7 rad)."""
    c = torch.load(GOLD / "kmd2_prologue.pt", weights_only=False)[case]
    out = _kmd2_prologue_dev(c)
    for o, n in zip(out, ["q", "k", "v", "g", "beta_e", "beta_w"]):
        assert rel(o, c["scan_args"][n]) < 1e-5, n


def test_kmd2_prologue_then_scan_matches_the_oracle_chain():
    c = torch.load(GOLD / "kmd2_prologue.pt", weights_only=False)["r4"]
    mix = torch.randn(c["H"], 4, generator=torch.Generator().manual_seed(3))
    q, k, v, g, be, bw = _kmd2_prologue_dev(c)
    y = ops.kmd2_scan(q, k, v, g, be, bw, mix.to(DEV))
    sa = c["scan_args"]
    yo, _, _ = R.kmd2_scan(sa["q"], sa["k"], sa["v"], sa["g"], sa["beta_e"], sa["beta_w"], mix)
    assert rel(y, yo) < 2e-2  # the KMD-2 scan runs on bf16 tensor-core operands


class _KMD2Layer(torch.nn.Module):
    """A module with KMD2NativeAttn's attribute names and shapes, filled from a state dict."""

    def __init__(self, sd, H, r_out, eps):
        super().__init__()
        lin = lambda w, bias=None: torch.nn.Linear(w.shape[1], w.shape[0], bias=bias is not None)
        self.H, self.dk, self.dv, self.r_out = H, 128, 128, r_out
        self.in_proj_qkv = lin(sd["in_proj_qkv.weight"])
        self.in_proj_z = lin(sd["in_proj_z.weight"])
        self.in_proj_b = lin(sd["in_proj_b.weight"])
        self.in_proj_a = lin(sd["in_proj_a.weight"])
        self.rot_proj = lin(sd["rot_proj.weight"], sd["rot_proj.bias"])
        self.out_proj = lin(sd["out_proj.weight"])
        self.conv1d = torch.nn.Conv1d(sd["conv1d.weight"].shape[0], sd["conv1d.weight"].shape[0],
                                      sd["conv1d.weight"].shape[-1], groups=sd["conv1d.weight"].shape[0], bias=False)
        self.norm = torch.nn.Module()
        self.norm.weight = torch.nn.Parameter(sd["norm.weight"].clone())
        self.norm.variance_epsilon = eps
        for n in ("dt_bias", "A_log", "decay_chan", "bw_off") + (("q_slot_scale", "out_mix") if r_out > 1 else ()):
            setattr(self, n, torch.nn.Parameter(sd[n].clone()))
        own = dict(self.named_parameters())
        with torch.no_grad():
            for n, t in sd.items():
                if n in own:
                    own[n].copy_(t)


@pytest.mark.parametrize("case", ["r4", "r1"])
def test_kmd2_fused_forward_matches_reference_forward(case):
    """gdnx_b200.kmd2_native.kmd2_forward (GEMMs in torch, prologue + scan + gated norm here)
    against the reference module's whole forward with its own token-loop scan."""
    from gdnx_b200.kmd2_native import patch_layer
    c = torch.load(GOLD / "kmd2_prologue.pt", weights_only=False)[case]
    layer = patch_layer(_KMD2Layer(c["state_dict"], c["H"], c["r_out"], c["eps"]).to(DEV))
    with torch.no_grad():
        out = layer(c["x"].to(DEV))
    assert out.shape == c["forward"].shape
    assert rel(out, c["forward"]) < 2e-2  # the scan runs on bf16 tensor-core operands
    with pytest.raises(RuntimeError):
        layer(c["x"].to(DEV))  # autograd enabled with trainable parameters: inference only
