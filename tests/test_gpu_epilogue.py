"""The output epilogues (``gdnx_epilogue``): GDN3 lane routing + head norm and the
KMD-2 gated RMS norm, against the reference-generated fixture and the oracle."""
from pathlib import Path

import pytest
import torch

from gdnx_b200 import ops
from oracle import epilogue as E

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
DEV = "cuda:0"


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def test_lane_route_matches_reference_fixture():
    c = torch.load(GOLD / "epilogue.pt", weights_only=False)
    out = ops.lane_route(c["y"].to(DEV), c["logits"].to(DEV), c["norm"].to(DEV))
    assert out.shape == c["out"].shape and rel(out, c["out"]) < 1e-6


def test_rms_norm_gated_matches_reference_fixture():
    c = torch.load(GOLD / "epilogue.pt", weights_only=False)
    out = ops.rms_norm_gated(c["y_kmd2"].to(DEV), c["z"].to(DEV), c["weight"].to(DEV))
    assert rel(out, c["out_kmd2"]) < 1e-6


def test_lane_route_bf16_strided_scan_output():
    g = torch.Generator().manual_seed(5)
    y = torch.randn(3, 40, 4, 4, 128, generator=g).to(torch.bfloat16)
    logits = torch.randn(3, 40, 4, 4, generator=g).to(torch.bfloat16)
    norm = 1 + 0.1 * torch.randn(128, generator=g)
    ref = E.lane_route(y.float(), logits.float(), norm)
    yd = y.to(DEV)[:, 5:]  # a strided view
    out = ops.lane_route(yd, logits.to(DEV)[:, 5:], norm.to(DEV))
    assert out.dtype == torch.bfloat16 and rel(out.float(), ref[:, 5:]) < 1e-2
    out32 = ops.lane_route(yd, logits.to(DEV)[:, 5:], norm.to(DEV), out_dtype=torch.float32)
    assert rel(out32, ref[:, 5:]) < 1e-5


def test_scan_then_route_equals_oracle_chain():
    from gdnx_b200.prologue import lane_rope
    from oracle import recurrence as R
    from oracle import prologue as PR
    from oracle.inputs import scan_inputs
    inp = scan_inputs(1, 96, 2, 4, 128, 128, seed=17, dtype=torch.bfloat16)
    g = {n: t.to(DEV) for n, t in inp.items()}
    y = ops.gdn3_scan(g["q"], g["k"], g["v"], g["beta"], g["beta"], g["logg"], decay_kind="log",
                      rope=lane_rope(4, 128, 128, 0.5))
    gen = torch.Generator().manual_seed(18)
    logits = torch.randn(1, 96, 2, 4, generator=gen)
    norm = 1 + 0.1 * torch.randn(128, generator=gen)
    out = ops.lane_route(y, logits.to(DEV), norm.to(DEV), out_dtype=torch.float32)
    f = {n: t.float() for n, t in inp.items()}
    qx = PR.apply_lane_rope(f["q"].unsqueeze(3).expand(-1, -1, -1, 4, -1).contiguous(), 128, 0.5)
    kx = PR.apply_lane_rope(f["k"].unsqueeze(3).expand(-1, -1, -1, 4, -1).contiguous(), 128, 0.5)
    vx = f["v"].unsqueeze(3).expand(-1, -1, -1, 4, -1)
    Yo, _ = R.dense_scan(qx, kx, vx, f["beta"].unsqueeze(-1), f["beta"].unsqueeze(-1), torch.exp(f["logg"]))
    assert rel(out, E.lane_route(Yo, logits, norm)) < 2e-2


@pytest.mark.parametrize("M", [1, 3, 8])
def test_lane_route_lane_counts(M):
    g = torch.Generator().manual_seed(6 + M)
    y = torch.randn(2, 11, 3, M, 128, generator=g)
    logits = torch.randn(2, 11, 3, M, generator=g)
    norm = 1 + 0.1 * torch.randn(128, generator=g)
    out = ops.lane_route(y.to(DEV), logits.to(DEV), norm.to(DEV))
    assert rel(out, E.lane_route(y, logits, norm)) < 1e-5


@pytest.mark.parametrize("M,dtype", [(4, torch.bfloat16), (2, torch.float32)])
def test_lane_route_with_output_gate(M, dtype):
    """The layer's output gate fused into the routing (H*V == D: no _agg_proj), the gate
    given as the [B,T,H*V] projection output."""
    g = torch.Generator().manual_seed(40 + M)
    B, T, H, V = 2, 13, 3, 128
    y = torch.randn(B, T, H, M, V, generator=g).to(dtype)
    logits = torch.randn(B, T, H, M, generator=g)
    norm = 1 + 0.1 * torch.randn(V, generator=g)
    z = torch.randn(B, T, H * V, generator=g).to(dtype)
    out = ops.lane_route(y.to(DEV), logits.to(DEV), norm.to(DEV), gate=z.to(DEV), out_dtype=torch.float32)
    ref = E.lane_route(y.float(), logits, norm, gate=z.float().view(B, T, H, V))
    assert rel(out, ref) < 1e-5
