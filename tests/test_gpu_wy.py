"""GPU parity of the two-pass WY chunked scan (scan_wy.cu) on the cases its
design singles out: chunks on the exact path (total log2 decay below -60) and
on the folded path in one sequence, state rescaling over long sequences,
per-lane (non-shared) q/k/v views, and strided / fp32 outputs.

Oracle: the CPU restatement of the frozen GDN3 recurrence (dense case) on the
same bf16-rounded inputs; long sequences compare the chunked path with the
exact recurrent kernel.  Tolerance: relative L2 2e-2 (bf16 I/O).
"""
import pytest
import torch

from gdnx_b200 import ops
from gdnx_b200.prologue import lane_rope
from oracle import prologue as PR
from oracle import recurrence as R
from oracle.inputs import scan_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL16 = 2e-2


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def _oracle(q, k, v, beta, logg, rope_rf, M):
    """q, k, v: [B,T,H,(M,)D] float (bf16-rounded values); beta, logg: [B,T,H,M]."""
    K, V = k.shape[-1], v.shape[-1]
    lanes = lambda x: x if x.dim() == 5 else x.unsqueeze(3).expand(-1, -1, -1, M, -1)
    qx, kx, vx = lanes(q).contiguous(), lanes(k).contiguous(), lanes(v)
    if rope_rf is not None:
        qx = PR.apply_lane_rope(qx, K, rope_rf)
        kx = PR.apply_lane_rope(kx, K, rope_rf)
    bg = beta.unsqueeze(-1).expand(-1, -1, -1, -1, K)
    wg = beta.unsqueeze(-1).expand(-1, -1, -1, -1, V)
    return R.dense_scan(qx, kx, vx, bg, wg, torch.exp(logg))


def _bf(x):
    return x.to(torch.bfloat16)


def test_exact_and_folded_chunks_in_one_sequence():
    """Chunks alternate between strong decay (L_C far below -60: exact path, rescaled
    state) and mild decay (folded path)."""
    B, T, H, M, K = 2, 320, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=71)
    g = torch.Generator().manual_seed(72)
    strong = -(2.0 + torch.rand(B, T, H, M, generator=g) * 2.0)  # ~ -3 nats per token
    chunk = (torch.arange(T) // 64) % 2 == 1
    logg = torch.where(chunk[None, :, None, None], strong, inp["logg"])
    q, k, v, beta = (_bf(inp[n]) for n in ("q", "k", "v", "beta"))
    logg = _bf(logg)
    Yo, So = _oracle(q.float(), k.float(), v.float(), beta.float(), logg.float(), 0.5, M)
    rope = lane_rope(M, K, K, 0.5)
    y, S = ops.gdn3_scan(q.to(DEV), k.to(DEV), v.to(DEV), beta.to(DEV), beta.to(DEV), logg.to(DEV),
                         decay_kind="log", rope=rope, return_state=True, algo="chunked",
                         out_dtype=torch.float32)
    assert rel(y, Yo) < TOL16 and rel(S, So) < TOL16


def test_long_sequence_state_rescaling_vs_recurrent():
    """T = 3000 (ragged): the running state scale crosses its rescale threshold many
    times; both CUDA paths on the same bf16 inputs."""
    B, T, H, M, K = 2, 3000, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=73)
    g = torch.Generator().manual_seed(74)
    logg = -(0.05 + 0.1 * torch.rand(B, T, H, M, generator=g))  # L_C ~ -9 log2 per chunk
    q, k, v, beta = (_bf(inp[n]).to(DEV) for n in ("q", "k", "v", "beta"))
    logg = _bf(logg).to(DEV)
    rope = lane_rope(M, K, K, 0.5)
    kw = dict(decay_kind="log", rope=rope, return_state=True, out_dtype=torch.float32)
    yc, Sc = ops.gdn3_scan(q, k, v, beta, beta, logg, algo="chunked", **kw)
    yr, Sr = ops.gdn3_scan(q, k, v, beta, beta, logg, algo="recurrent", **kw)
    assert rel(yc, yr) < TOL16 and rel(Sc, Sr) < TOL16


def test_per_lane_qkv_views_and_state_in():
    """q/k/v given per lane ([B,T,H,M,D], lane stride != 0), a supplied initial state."""
    B, T, H, M, K = 1, 150, 3, 4, 128
    g = torch.Generator().manual_seed(75)
    nrm = lambda x: torch.nn.functional.normalize(x, dim=-1)
    q = _bf(nrm(torch.randn(B, T, H, M, K, generator=g)))
    k = _bf(nrm(torch.randn(B, T, H, M, K, generator=g)))
    v = _bf(torch.randn(B, T, H, M, K, generator=g))
    beta = _bf(torch.sigmoid(torch.randn(B, T, H, M, generator=g)))
    logg = _bf(-torch.nn.functional.softplus(torch.randn(B, T, H, M, generator=g)) * 0.05)
    S0 = torch.randn(B * H * M, K, K, generator=g) * 0.05
    # with a supplied state: against the exact recurrent kernel (itself checked against the oracle)
    rope = lane_rope(M, K, K, 0.25)
    kw = dict(decay_kind="log", rope=rope, return_state=True, out_dtype=torch.float32, state=S0.to(DEV))
    args = [x.to(DEV) for x in (q, k, v, beta, beta, logg)]
    yc, Sc = ops.gdn3_scan(*args, algo="chunked", **kw)
    yr, Sr = ops.gdn3_scan(*args, algo="recurrent", **kw)
    assert rel(yc, yr) < TOL16 and rel(Sc, Sr) < TOL16
    # and without the state, against the oracle
    Yo, So = _oracle(q.float(), k.float(), v.float(), beta.float(), logg.float(), 0.25, M)
    y, S = ops.gdn3_scan(*args, algo="chunked", decay_kind="log", rope=rope, return_state=True,
                         out_dtype=torch.float32)
    assert rel(y, Yo) < TOL16 and rel(S, So) < TOL16


@pytest.mark.parametrize("layout", ["bf16_strided", "fp32"])
def test_output_layouts(layout):
    """y written through TMA (bf16, 16-byte strides) or element stores (strided bf16 view, fp32)."""
    B, T, H, M, K = 2, 130, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=76)
    q, k, v, beta, logg = (_bf(inp[n]) for n in ("q", "k", "v", "beta", "logg"))
    Yo, So = _oracle(q.float(), k.float(), v.float(), beta.float(), logg.float(), 0.5, M)
    rope = lane_rope(M, K, K, 0.5)
    args = [x.to(DEV) for x in (q, k, v, beta, beta, logg)]
    if layout == "fp32":
        y = ops.gdn3_scan(*args, decay_kind="log", rope=rope, algo="chunked", out_dtype=torch.float32)
    else:
        big = torch.zeros(B, T, H, M, K + 3, dtype=torch.bfloat16, device=DEV)
        out = big[..., :K]  # row stride K + 3: not a TMA-describable view
        y = ops.gdn3_scan(*args, decay_kind="log", rope=rope, algo="chunked", out=out)
        assert big[..., K:].abs().sum().item() == 0
    assert rel(y.float(), Yo) < TOL16


def test_default_and_allocation_free_paths_agree():
    """The two-pass default and the single-pass allocation-free entry point."""
    B, T, H, M, K = 2, 200, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=77)
    args = [_bf(inp[n]).to(DEV) for n in ("q", "k", "v", "beta", "beta", "logg")]
    rope = lane_rope(M, K, K, 0.5)
    y1 = ops.gdn3_scan(*args, decay_kind="log", rope=rope, algo="chunked", out_dtype=torch.float32)
    y2 = torch.empty_like(y1)
    ops.gdn3_scan_noalloc(*args, decay_kind="log", rope=rope, out=y2)
    assert rel(y1, y2) < TOL16


def test_host_to_host_pipelined_scan_matches_device_scan():
    """ops.gdn3_scan_host (sliced, copies overlapped on three streams) == ops.gdn3_scan."""
    B, T, H, M, K = 5, 200, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=78)
    host = [_bf(inp[n]).pin_memory() for n in ("q", "k", "v", "beta", "beta", "logg")]
    rope = lane_rope(M, K, K, 0.5)
    out = torch.empty(B, T, H, M, K, dtype=torch.bfloat16).pin_memory()
    ops.gdn3_scan_host(*host, out=out, device=DEV, slices=3, decay_kind="log", rope=rope)
    torch.cuda.synchronize()
    ref = ops.gdn3_scan(*[t.to(DEV) for t in host], decay_kind="log", rope=rope)
    assert torch.equal(out, ref.cpu())


def test_device_status_word():
    """The workspace error word is clear after a normal call and reported when set."""
    B, T, H, M, K = 1, 70, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=79)
    args = [_bf(inp[n]).to(DEV) for n in ("q", "k", "v", "beta", "beta", "logg")]
    ws = torch.empty(1 << 24, dtype=torch.uint8, device=DEV)
    ops.gdn3_scan(*args, decay_kind="log", algo="chunked", workspace=ws)
    assert ops.device_status(ws) == 0
    ws[:4].view(torch.int32).fill_(3)  # GDNX_ETIMEOUT, as a kernel that gave up would leave it
    with pytest.raises(RuntimeError, match="gdnx device error"):
        ops.check_device_status(ws)
    ops.gdn3_scan(*args, decay_kind="log", algo="chunked", workspace=ws)  # every call clears it
    assert ops.device_status(ws) == 0


@pytest.mark.parametrize("kind", ["gamma", "braided"])
def test_decay_kinds_on_the_chunked_path(kind):
    """Decay given as gamma in (0, 1] or as the braided projection [.., 4], read by pass 1."""
    B, T, H, M, K = 1, 150, 2, 4, 128
    inp = scan_inputs(B, T, H, M, K, K, seed=80)
    g = torch.Generator().manual_seed(81)
    q, k, v, beta = (_bf(inp[n]) for n in ("q", "k", "v", "beta"))
    if kind == "gamma":
        dec_in = _bf(torch.exp(inp["logg"]))
        gam = dec_in.float()
    else:
        dec_in = _bf(torch.randn(B, T, H, M, 4, generator=g) * 3)
        gam = PR.braided_decay(dec_in.float())
    logg = torch.log(gam)
    Yo, So = _oracle(q.float(), k.float(), v.float(), beta.float(), logg, 0.5, M)
    rope = lane_rope(M, K, K, 0.5)
    y, S = ops.gdn3_scan(q.to(DEV), k.to(DEV), v.to(DEV), beta.to(DEV), beta.to(DEV), dec_in.to(DEV),
                         decay_kind=kind, rope=rope, return_state=True, algo="chunked", out_dtype=torch.float32)
    assert rel(y, Yo) < TOL16 and rel(S, So) < TOL16


def test_chain_pieces_overlap_is_bit_identical():
    """More chains than SMs: the library runs pass 1 of later chain pieces on a side stream
    beside pass 2 of earlier ones.  Each chain's result must not depend on that split."""
    B, T, H, M, K = 12, 96, 16, 4, 128  # 768 chains
    inp = scan_inputs(B, T, H, M, K, K, seed=82)
    args = [_bf(inp[n]).to(DEV) for n in ("q", "k", "v", "beta", "beta", "logg")]
    rope = lane_rope(M, K, K, 0.5)
    kw = dict(decay_kind="log", rope=rope, algo="chunked", return_state=True)
    y, S = ops.gdn3_scan(*args, **kw)
    for b0 in range(0, B, 2):  # 128 chains per call: one piece
        yb, Sb = ops.gdn3_scan(*[t[b0:b0 + 2] for t in args], **kw)
        assert torch.equal(yb, y[b0:b0 + 2])
        assert torch.equal(Sb, S[b0 * H * M:(b0 + 2) * H * M])
