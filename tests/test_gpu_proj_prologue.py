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
