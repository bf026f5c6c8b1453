"""Backward of the dense scan (``gdnx_scan_bwd``) against torch autograd through the
fp32 oracle on the same inputs: GDN3 (vector and scalar gates, gamma and log decays,
an initial state and a final-state gradient, lane-shared q/k/v) and KMD-2
(per-channel decay, query slots mixed by out_mix), through the drop-ins too.

The kernel computes in fp32 like the oracle, so gradients agree to fp32 rounding
(relative L2 1e-4) -- far inside the reference's own gate for its fast scan's
backward (gradient relMSE 1e-2, research/kernel_ab/bench_scan.py:24-25).
"""
import pytest
import torch

from gdnx_b200 import ops
from oracle import recurrence as R
from oracle.inputs import parity_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = 1e-4


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _leaf(ts, dev):
    return [t.detach().clone().to(dev).requires_grad_(True) for t in ts]


@pytest.mark.parametrize("T", [5, 64, 150])
def test_gdn3_vector_gates_grads(T):
    ins = parity_inputs(2, T, 2, 4, 128, 128, seed=400 + T, scale=0.3)
    g = torch.Generator().manual_seed(401)
    S0 = torch.randn(2 * 2 * 4, 128, 128, generator=g) * 0.05
    cpu = _leaf(ins + [S0], "cpu")
    Yo, So = R.dense_scan(*cpu[:6], S0=cpu[6])
    gy = torch.randn(Yo.shape, generator=g)
    gS = torch.randn(So.shape, generator=g) * 0.1
    (Yo * gy).sum().add_((So * gS).sum()).backward()
    dev = _leaf(ins + [S0], DEV)
    y, S = ops.gdn3_scan_train(*dev[:6], state=dev[6])
    assert rel(y, Yo) < 2e-3 and rel(S, So) < 2e-3
    (y * gy.to(DEV)).sum().add_((S * gS.to(DEV)).sum()).backward()
    for name, a, b in zip(["q", "k", "v", "b", "w", "decay", "state"], dev, cpu):
        assert rel(a.grad, b.grad) < TOL, name


def test_gdn3_scalar_gates_lane_shared_log_decay():
    g = torch.Generator().manual_seed(410)
    B, T, H, M, K = 1, 100, 2, 4, 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1)
    v = torch.randn(B, T, H, K, generator=g)
    beta = torch.sigmoid(torch.randn(B, T, H, M, generator=g))
    logg = -torch.nn.functional.softplus(torch.randn(B, T, H, M, generator=g)) * 0.05
    cpu = _leaf([q, k, v, beta, logg], "cpu")
    ex = lambda x: x.unsqueeze(3).expand(-1, -1, -1, M, -1)
    Yo, _ = R.dense_scan(ex(cpu[0]), ex(cpu[1]), ex(cpu[2]), cpu[3].unsqueeze(-1), cpu[3].unsqueeze(-1),
                         torch.exp(cpu[4]))
    gy = torch.randn(Yo.shape, generator=g)
    (Yo * gy).sum().backward()
    dev = _leaf([q, k, v, beta, logg], DEV)
    y, _ = ops.gdn3_scan_train(dev[0], dev[1], dev[2], dev[3], dev[3], dev[4], decay_kind="log")
    (y * gy.to(DEV)).sum().backward()
    for name, a, b in zip(["q", "k", "v", "beta", "logg"], dev, cpu):
        assert rel(a.grad, b.grad) < TOL, name


@pytest.mark.parametrize("r_out", [1, 4])
def test_kmd2_fast_scan_dropin_grads(r_out):
    from gdnx_b200 import kmd2_fast_scan
    g = torch.Generator().manual_seed(420 + r_out)
    B, T, H, dk = 2, 90, 2, 128
    q = torch.nn.functional.normalize(torch.randn(B, T, H, r_out, dk, generator=g), dim=-1) * dk ** -0.5
    k = torch.nn.functional.normalize(torch.randn(B, T, H, dk, generator=g), dim=-1)
    v = torch.randn(B, T, H, dk, generator=g)
    gd = torch.exp(-torch.nn.functional.softplus(1.2 * torch.randn(B, T, H, dk, generator=g) - 0.6))
    be = torch.sigmoid(torch.randn(B, T, H, generator=g))
    bw = torch.sigmoid(torch.randn(B, T, H, generator=g))
    mix = torch.randn(H, r_out, generator=g)
    base = [q, k, v, gd, be, bw] + ([mix] if r_out > 1 else [])
    cpu = _leaf(base, "cpu")
    yo, _, _ = R.kmd2_scan(*cpu[:6], cpu[6] if r_out > 1 else None)
    gy = torch.randn(yo.shape, generator=g)
    (yo * gy).sum().backward()
    dev = _leaf(base, DEV)
    y = kmd2_fast_scan.scan(*dev[:6], dev[6] if r_out > 1 else None)
    assert rel(y, yo) < 2e-2
    (y * gy.to(DEV)).sum().backward()
    for name, a, b in zip(["q", "k", "v", "g", "beta_e", "beta_w", "out_mix"], dev, cpu):
        assert rel(a.grad, b.grad) < TOL, name


def test_gdn3_dropin_trains_below_the_compaction_period():
    import types
    from gdnx_b200.gdn3_upgrade import patch_layer
    ins = parity_inputs(1, 48, 1, 4, 128, 128, seed=430, scale=0.3)
    layer = patch_layer(types.SimpleNamespace(R=4, P=64, a_v=16, a_k=16, b_v=8, b_k=8, slow_decay=0.97,
                                              compact_mode="svd"))
    cpu = _leaf(ins, "cpu")
    Yo, _ = R.dense_scan(*cpu)
    Yo.square().sum().backward()
    dev = _leaf(ins, DEV)
    y = layer._gdn3_recurrent_state(*dev)
    y.square().sum().backward()
    for name, a, b in zip(["q", "k", "v", "b", "w", "decay"], dev, cpu):
        assert rel(a.grad, b.grad) < TOL, name
