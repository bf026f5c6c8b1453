"""The lane routing fused with the all-gather of its output (``ops.lane_route_scatter``
into a ``distributed.PeerBuffer``): two ranks, one GPU each, NCCL for the handle
exchange and the completion barrier.  Each rank's routed rows must land bit-exactly
in both ranks' copies.  Skipped with fewer than two GPUs (the single-GPU runs)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(rank, B, T, H, M, V):
    g = torch.Generator().manual_seed(100 + rank)
    y = torch.randn(B, T, H, M, V, generator=g).to(torch.bfloat16)
    logits = torch.randn(B, T, H, M, generator=g)
    norm = 1 + 0.1 * torch.randn(V, generator=g)
    return y, logits, norm


def _worker(rank, world, port, shape, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from gdnx_b200 import ops
    from gdnx_b200.distributed import PeerBuffer
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        B, T, H, M, V = shape
        buf = PeerBuffer((world * B, T, H, V), torch.bfloat16, dev)
        y, logits, norm = _inputs(rank, B, T, H, M, V)
        yd, ld, nd = y.to(dev), logits.to(dev), norm.to(dev)
        off = rank * B * T * H * V
        ops.lane_route_scatter(yd, ld, buf.dest(off, B * T * H * V), (T * H * V, H * V, V), torch.bfloat16, nd)
        dist.all_reduce(torch.zeros(1, device=dev))  # every rank's scatter has completed
        torch.cuda.synchronize()
        ok = True
        for r in range(world):
            yr, lr, nr = (t.to(dev) for t in _inputs(r, B, T, H, M, V))
            ref = ops.lane_route(yr, lr, nr)
            ok &= torch.equal(buf.tensor[r * B:(r + 1) * B], ref)
        buf.close()
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_lane_route_scatter_two_ranks():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    shape = (2, 37, 3, 4, 128)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():  # this test's own child: stop it by its PID
            p.kill()
            p.join()
    results = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}
