"""Host-side multi-rank logic of gdnx_b200.distributed on CPU ranks (gloo, world size 2)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdnx_b200.distributed import shard_for, sharded_scan


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_scan(q, k, v, beta, logg):
    """Reference-recurrence restatement used as the per-rank scan on CPU ranks."""
    from oracle import recurrence as R
    M = beta.shape[3]
    qx = q.unsqueeze(3).expand(-1, -1, -1, M, -1)
    kx = k.unsqueeze(3).expand(-1, -1, -1, M, -1)
    vx = v.unsqueeze(3).expand(-1, -1, -1, M, -1)
    y, _ = R.dense_scan(qx, kx, vx, beta.unsqueeze(-1), beta.unsqueeze(-1), torch.exp(logg))
    return y


def _worker(rank, world, port, B, H, out_q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    from oracle.inputs import scan_inputs
    inp = scan_inputs(B, 12, H, 4, 16, 16, seed=5)
    try:
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the gather")
        y = sharded_scan(_cpu_scan, dict(q=inp["q"], k=inp["k"], v=inp["v"], beta=inp["beta"], logg=inp["logg"]),
                         world, rank)
        full = _cpu_scan(inp["q"], inp["k"], inp["v"], inp["beta"], inp["logg"])
        out_q.put((rank, "ok", float((y - full).abs().max())))
    except Exception as e:  # reported to the parent, never swallowed
        out_q.put((rank, "error", type(e).__name__ + ": " + str(e)[:120]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(B, H, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, B, H, q, fail_rank)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (s, v)) for r, s, v in (q.get(timeout=120) for _ in ps))
    for p in ps:
        p.join(timeout=60)
    return res


def test_shard_map():
    assert shard_for(8, 16, 2, 1).axis == "batch" and shard_for(8, 16, 2, 1).start == 4
    assert shard_for(1, 16, 8, 3).axis == "head" and (shard_for(1, 16, 8, 3).start, shard_for(1, 16, 8, 3).stop) == (6, 8)
    with pytest.raises(ValueError):
        shard_for(3, 5, 2, 0)


@pytest.mark.parametrize("B,H", [(4, 2), (1, 4)])
def test_two_rank_gather_equals_single_scan(B, H):
    res = _run(B, H)
    for r in (0, 1):
        status, val = res[r]
        assert status == "ok", val
        assert val < 1e-6


def test_rank_failure_surfaces_as_error_on_the_other_rank():
    res = _run(4, 2, fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"  # its collective cannot complete: gloo reports it instead of hanging


def _deadline_worker(rank, world, port, out_q, absent_rank):
    """Rank ``absent_rank`` never joins the gather (it stays alive, idle, until the end)."""
    import time
    from gdnx_b200.distributed import CollectiveTimeout, gather_with_deadline, init_scan_group
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    init_scan_group("gloo", timeout_s=30)
    x = torch.full((4,), float(rank))
    out = torch.empty(4 * world)
    try:
        if rank == absent_rank:
            time.sleep(6)
            out_q.put((rank, "absent", 0.0))
            return
        t0 = time.monotonic()
        try:
            gather_with_deadline(out, x, timeout_s=1.5)
            out_q.put((rank, "completed", time.monotonic() - t0))
        except CollectiveTimeout as e:
            out_q.put((rank, "timeout", time.monotonic() - t0))
    except Exception as e:
        out_q.put((rank, "error", type(e).__name__ + ": " + str(e)[:120]))


def test_gather_deadline_aborts_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_deadline_worker, args=(r, 2, port, q, 1)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (s, v)) for r, s, v in (q.get(timeout=120) for _ in ps))
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "absent"
    assert res[0][0] == "timeout", res[0]
    assert 1.4 < res[0][1] < 10.0  # gave up at its deadline, not at the group's 30 s timeout


def _deadline_ok_worker(rank, world, port, out_q):
    from gdnx_b200.distributed import gather_with_deadline, init_scan_group
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    init_scan_group("gloo", timeout_s=30)
    out = torch.empty(4 * world)
    gather_with_deadline(out, torch.full((4,), float(rank)), timeout_s=20)
    out_q.put((rank, "ok", float(out.sum())))
    dist.destroy_process_group()


def test_gather_with_deadline_completes_normally():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_deadline_ok_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=30)
    assert all(s == "ok" and v == 4.0 for _, s, v in res), res
