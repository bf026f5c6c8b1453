"""The allocation-free scan entry point (``gdnx_scan_fwd_noalloc``).

It exists for callers that cannot allocate device memory when they call the
library -- runtimes that own a fixed memory pool, or code that must not let a
cudaMalloc synchronise the device.  It must give the same results as the
normal entry point, call after call, even though every call reuses one
library-owned scratch array.  This file is collected last on purpose.
"""
import pytest
import torch

from gdnx_b200 import ops
from gdnx_b200.prologue import lane_rope
from oracle.inputs import scan_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL16 = 2e-2


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("T", [200])
def test_noalloc_matches_the_allocating_entry_two_calls_in_a_row(T):
    rope = lane_rope(4, 128, 128, 0.5)
    for call, seed in enumerate((61, 62)):
        inp = scan_inputs(2, T, 2, 4, 128, 128, seed=seed, dtype=torch.bfloat16)
        q, k, v, beta, logg = (inp[n].to(DEV) for n in ("q", "k", "v", "beta", "logg"))
        y_ref, S_ref = ops.gdn3_scan(q, k, v, beta, beta, logg, decay_kind="log", rope=rope,
                                     return_state=True, algo="chunked")
        y = torch.empty_like(y_ref)
        S = torch.empty_like(S_ref)
        ops.gdn3_scan_noalloc(q, k, v, beta, beta, logg, decay_kind="log", rope=rope, out=y, state_out=S)
        torch.cuda.synchronize()
        assert rel(y.float(), y_ref.float()) < TOL16, call
        assert rel(S, S_ref) < TOL16, call
        assert ops.noalloc_status(DEV) == 0, call  # no bounded wait gave up


def test_noalloc_rejects_requests_the_chunked_kernel_cannot_take():
    from gdnx_b200._lib import GdnxError, GDNX_EUNSUPPORTED
    inp = scan_inputs(1, 16, 1, 4, 64, 64, seed=63, dtype=torch.bfloat16)  # K = 64: no chunked kernel
    q, k, v, beta, logg = (inp[n].to(DEV) for n in ("q", "k", "v", "beta", "logg"))
    y = torch.empty(1, 16, 1, 4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(GdnxError) as e:
        ops.gdn3_scan_noalloc(q, k, v, beta, beta, logg, decay_kind="log", out=y)
    assert e.value.status == GDNX_EUNSUPPORTED
