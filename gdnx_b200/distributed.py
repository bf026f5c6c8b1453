"""(batch x head) sharding of the scan over the GPUs of one node.

Chains (b, h, m) are independent, so a rank scans its own rows of the batch
(or, when the batch is smaller than the world, its own heads) with no
data-path communication; the only exchange is one all-gather of the outputs
after the scan: ``all_gather_into_tensor`` (NCCL over NVLink/NVSwitch on GPUs,
gloo in the CPU tests), or -- for the routed GDN3 output -- the routing kernel
itself storing its rows into every rank's copy of a :class:`PeerBuffer` over
NVLink (``ops.lane_route_scatter``).  Every rank keeps all M lanes of its
heads, so the lane-shared q/k/v reads stay local.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch


@dataclass(frozen=True)
class Shard:
    axis: str      # "batch" or "head"
    start: int
    stop: int

    def take(self, x: torch.Tensor, dim_batch: int = 0, dim_head: int = 2) -> torch.Tensor:
        d = dim_batch if self.axis == "batch" else dim_head
        return x.narrow(d, self.start, self.stop - self.start)


def shard_for(B: int, H: int, world: int, rank: int) -> Shard:
    """Whole batch rows first (B divisible by world), else heads (H divisible by world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if B % world == 0:
        n = B // world
        return Shard("batch", rank * n, (rank + 1) * n)
    if H % world == 0:
        n = H // world
        return Shard("head", rank * n, (rank + 1) * n)
    raise ValueError(f"cannot split B={B} or H={H} evenly over {world} ranks")


def sharded_scan(scan_fn: Callable, inputs: dict, world: int, rank: int, group=None,
                 gather: bool = True) -> torch.Tensor:
    """Scan this rank's shard with ``scan_fn(**shard_inputs) -> y [b,T,h,M,V]`` and
    (optionally) all-gather the full ``[B,T,H,M,V]`` output on every rank.

    ``inputs`` holds tensors with batch at dim 0 and heads at dim 2
    ([B,T,H,...]) plus non-tensor keyword arguments passed through.
    """
    import torch.distributed as dist
    B, _, H = inputs["k"].shape[:3]
    sh = shard_for(B, H, world, rank)
    local = {n: (sh.take(t) if torch.is_tensor(t) and t.dim() >= 3 else t) for n, t in inputs.items()}
    y = scan_fn(**local).contiguous()
    if not gather or world == 1:
        return y
    parts = torch.empty((world * y.shape[0],) + tuple(y.shape[1:]), dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(parts, y, group=group)  # rank r's shard at rows [r*b, (r+1)*b)
    if sh.axis == "batch":
        return parts
    # heads: [world*B, T, h, M, V] -> [B, T, world*h, M, V]
    parts = parts.reshape((world,) + tuple(y.shape))
    return parts.permute(1, 2, 0, 3, 4, 5).reshape(y.shape[0], y.shape[1], H, *y.shape[3:])


# ----------------------------------------------------------------------------
# failure handling: bounded collectives, abort on timeout
# ----------------------------------------------------------------------------

class CollectiveTimeout(RuntimeError):
    """A collective did not complete before its host-side deadline; the group was aborted."""


def init_scan_group(backend: str = "nccl", timeout_s: float = 60.0, device_id=None) -> None:
    """Initialise the default process group for sharded scans with failure handling on.

    For NCCL the communicator is created non-blocking (``TORCH_NCCL_USE_COMM_NONBLOCKING``)
    and asynchronous error handling is enabled (``TORCH_NCCL_ASYNC_ERROR_HANDLING``), so a
    collective that outlives ``timeout_s`` is aborted by the process group's watchdog
    (``ncclCommAbort``) instead of blocking the rank; :func:`gather_with_deadline` adds a
    host-side deadline per call.  Rendezvous comes from the usual ``MASTER_*`` / ``RANK`` /
    ``WORLD_SIZE`` environment.
    """
    import datetime
    import os
    import torch.distributed as dist
    if backend == "nccl":
        os.environ.setdefault("TORCH_NCCL_USE_COMM_NONBLOCKING", "1")
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    kw = {"device_id": device_id} if device_id is not None else {}
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)


def abort_group(group=None) -> None:
    """Abort ``group`` (the default group when None): NCCL communicators are aborted
    (``ncclCommAbort``), so no rank stays blocked in a collective a peer never joins.
    Falls back to destroying the group where the backend has no abort."""
    import torch.distributed as dist
    from torch.distributed import distributed_c10d as c10d
    try:
        c10d._abort_process_group(group if group is not None else c10d.GroupMember.WORLD)
    except Exception:
        try:
            dist.destroy_process_group(group)
        except Exception:
            pass


def gather_with_deadline(out: torch.Tensor, local: torch.Tensor, timeout_s: float, group=None,
                         poll_s: float = 0.01) -> torch.Tensor:
    """``all_gather_into_tensor(out, local)`` that gives up after ``timeout_s`` seconds.

    The collective is issued asynchronously and its completion polled on the host; past
    the deadline the group is aborted (:func:`abort_group`) and :class:`CollectiveTimeout`
    is raised, so a rank whose peer died or never joined learns of it instead of hanging.
    """
    import time
    import torch.distributed as dist
    work = dist.all_gather_into_tensor(out, local, group=group, async_op=True)
    deadline = time.monotonic() + timeout_s
    while not work.is_completed():
        if time.monotonic() > deadline:
            abort_group(group)
            raise CollectiveTimeout(f"all-gather did not complete within {timeout_s:.1f} s; group aborted")
        time.sleep(poll_s)
    work.wait()
    return out


class PeerBuffer:
    """One device buffer per rank of ``group`` (a node's GPUs, one process each), with
    every rank holding the addresses of all ranks' copies: the buffer is ``cudaMalloc``'d
    by the library, its CUDA IPC handle all-gathered through ``group`` and each peer's
    copy mapped into this process (plain peer mappings over NVLink).

    ``tensor`` is this rank's copy as a ``torch`` tensor of ``shape`` / ``dtype``;
    ``dest(rank_offset_elems)`` gives the device addresses of element offset ``o`` in
    every rank's copy, rank 0 first, after checking that ``extent`` elements from there
    stay inside the buffer.  ``close()`` (collective) unmaps and frees.
    """

    def __init__(self, shape, dtype, device, group=None):
        import ctypes as C
        import torch.distributed as dist
        from . import _lib as L
        self._dist, self._group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerBuffer: at most 8 ranks (one node)")
        self.shape, self.dtype, self.device = tuple(shape), dtype, torch.device(device)
        esz = torch.empty((), dtype=dtype).element_size()
        self.numel = 1
        for d in self.shape:
            self.numel *= int(d)
        self.esz = esz
        nbytes = self.numel * esz
        lib = L.load()
        self._lib = lib
        with torch.cuda.device(self.device):
            p = C.c_void_p()
            L.check(lib.gdnx_device_alloc(nbytes, C.byref(p)), "gdnx_device_alloc")
            self.base = p.value
            h = (C.c_uint8 * 64)()
            L.check(lib.gdnx_ipc_handle(C.c_void_p(self.base), h), "gdnx_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h), group=group)
            self.ptrs = []
            try:
                for r, hb in enumerate(handles):
                    if r == self.rank:
                        self.ptrs.append(self.base)
                        continue
                    q = C.c_void_p()
                    L.check(lib.gdnx_ipc_open((C.c_uint8 * 64).from_buffer_copy(hb), C.byref(q)), "gdnx_ipc_open")
                    self.ptrs.append(q.value)
            except Exception:  # undo this rank's mappings and buffer; the peers see the failure at their next collective
                for r, ptr in enumerate(self.ptrs):
                    if r != self.rank:
                        lib.gdnx_ipc_close(C.c_void_p(ptr))
                lib.gdnx_device_free(C.c_void_p(self.base))
                self.base = None
                raise

        class _Raw:  # a zero-copy byte view of the buffer for torch
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (self.base, False), "version": 2}

        self.tensor = torch.as_tensor(_Raw(), device=self.device).view(dtype).view(self.shape)

    def dest(self, offset: int, extent: int):
        """Device addresses of element ``offset`` in every rank's copy (``extent`` elements
        from there must lie inside the buffer)."""
        if offset < 0 or extent < 1 or offset + extent > self.numel:
            raise ValueError(f"PeerBuffer: elements [{offset}, {offset + extent}) outside [0, {self.numel})")
        return [p + offset * self.esz for p in self.ptrs]

    def close(self):
        """Collective: every rank's writes finish, every rank unmaps its peers' copies, and
        only then does each rank free its own."""
        if self.base is None:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            self._dist.barrier(group=self._group)
            for r, p in enumerate(self.ptrs):
                if r != self.rank:
                    self._lib.gdnx_ipc_close(p)
            torch.cuda.synchronize()
            self._dist.barrier(group=self._group)
            self.tensor = None
            self._lib.gdnx_device_free(self.base)
        self.base = None
