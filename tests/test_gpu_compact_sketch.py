"""GPU parity of the "sketch" / "sketch_noqr" compaction mode (the reference layer's
GDN3_COMPACT_MODE, gdn3/gdn3_upgrade.py:81,579-596), through the C ABI: one
compaction against the reference's own call (golden fixture), and the KR scan and
the GDN3 drop-in against the oracle's frozen loop with the same compaction.

Tolerances (relative L2): 2e-3 for fp32 I/O, 2e-2 for bf16 inputs compared with an
oracle fed the same bf16-rounded values; per-call factors 1e-5 (fp32 arithmetic in
another summation order, no iteration).
"""
import types
from pathlib import Path

import pytest
import torch

from gdnx_b200 import ops
from oracle import recurrence as R
from oracle.inputs import expand_lanes, parity_inputs, scan_inputs

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).parent / "golden"
DEV = "cuda:0"
TOL32 = 2e-3


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def kron(A, Bk):
    return torch.einsum("nrab,nrcd->nacbd", A.detach().cpu(), Bk.detach().cpu())


@pytest.mark.parametrize("mode", ["sketch", "sketch_noqr"])
def test_compact_sketch_matches_reference_call(mode):
    c = torch.load(GOLD / "compaction_sketch.pt", weights_only=False)
    A, Bk, U, Vb = c["inputs"]
    N = A.shape[0]
    G = R.sketch_matrix(N, 64, 4).to(DEV)
    Ag, Bg = A.to(DEV).contiguous(), Bk.to(DEV).contiguous()
    err = ops.compact(Ag, Bg, U.to(DEV).contiguous(), Vb.to(DEV).contiguous(), G, slow_decay=c["slow_decay"],
                      compact_mode=mode)
    assert rel(Ag, c[mode]["A_new"]) < 1e-5 and rel(Bg, c[mode]["B_new"]) < 1e-5
    assert float(err.abs().max()) == 0.0


def test_compact_rejects_a_sketch_of_the_wrong_width():
    A = torch.zeros(2, 4, 16, 16, device=DEV)
    Bk = torch.zeros(2, 4, 8, 8, device=DEV)
    U = torch.zeros(2, 128, 16, device=DEV)
    with pytest.raises(ValueError):
        ops.compact(A, Bk, U, U.clone(), torch.zeros(2, 64, 8, device=DEV), compact_mode="sketch")


@pytest.mark.parametrize("T,P", [(80, 16), (1024, 256)])
def test_kr_scan_sketch_mode_vs_oracle(T, P):
    if P == 16:
        ins = parity_inputs(1, T, 1, 4, 128, 128, seed=12)
        tol = TOL32
    else:  # config 2's period, bf16-rounded config-2 inputs, four compactions
        inp = scan_inputs(1, T, 1, 4, 128, 128, seed=13, dtype=torch.bfloat16)
        ins = [t.float().contiguous() for t in expand_lanes(inp, 4)]
        tol = TOL32
    N, dims = 4, (16, 16, 8, 8)
    G = R.sketch_matrix(N, 64, 4)
    Yo, st = R.gdn3_kr_scan(*ins, R=4, P=P, dims=R.KronDims(*dims), G=G, compact_mode="sketch")
    state = ops.KRState.zeros(N, 4, P, dims, 128, 128, DEV)
    y = ops.gdn3_kr_scan(*[t.to(DEV) for t in ins], state, G.to(DEV), P=P, dims=dims, compact_mode="sketch")
    assert rel(y, Yo) < tol
    assert rel(state.U, st.U) < tol and rel(state.Vb, st.Vb) < tol
    assert rel(kron(state.A, state.Bk), kron(st.A, st.Bk)) < 1e-3
    assert float(state.err.abs().max()) == 0.0


@pytest.mark.parametrize("mode", ["sketch", "sketch_noqr"])
def test_gdn3_dropin_sketch_mode(mode):
    from gdnx_b200.gdn3_upgrade import patch_layer
    ins = parity_inputs(1, 64, 1, 4, 128, 128, seed=14)
    layer = types.SimpleNamespace(R=4, P=16, a_v=16, a_k=16, b_v=8, b_k=8, slow_decay=0.97, compact_mode=mode)
    patch_layer(layer)
    y = layer._gdn3_recurrent_state(*[t.to(DEV) for t in ins])
    Yo, _ = R.gdn3_kr_scan(*ins, R=4, P=16, G=R.sketch_matrix(4, 64, 4), compact_mode=mode)
    assert rel(y, Yo) < TOL32
    assert float(layer._last_comp_err) == 0.0
