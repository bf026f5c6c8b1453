"""Torch-tensor front end of the C ABI (device memory and streams come from torch).

Every function validates on the host, builds the POD argument struct of
``include/gdnx.h`` from tensor pointers and strides, and enqueues the CUDA
kernel on ``torch.cuda.current_stream()``.  CPU tensors are rejected; there
is no fallback path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L
from .prologue import BRAID_RATES, DECAY_CLAMP, LaneRope

_DT = {torch.float32: L.GDNX_F32, torch.bfloat16: L.GDNX_BF16, torch.float16: L.GDNX_F16}
_DECAY = {"gamma": L.GDNX_DECAY_GAMMA, "log": L.GDNX_DECAY_LOG, "braided": L.GDNX_DECAY_BRAIDED}
_ALGO = {"auto": L.GDNX_ALGO_AUTO, "recurrent": L.GDNX_ALGO_RECURRENT, "chunked": L.GDNX_ALGO_CHUNKED}


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("gdnx_b200 kernels take CUDA tensors only (no CPU fallback)")


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _view(t: Optional[torch.Tensor], lanes: bool, slots: bool = False) -> L.View:
    """View of a [B,T,H,(M,)(S,)D] tensor.  ``lanes`` says whether a lane dim is present."""
    v = L.View()
    if t is None:
        return v
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}")
    if t.shape[-1] > 1 and t.stride(-1) != 1:
        raise ValueError("the last dim of every input must be contiguous")
    s = t.stride()
    v.ptr = t.data_ptr()
    v.dtype = _DT[t.dtype]
    v.dim = t.shape[-1]
    v.sb, v.st, v.sh = s[0], s[1], s[2]
    i = 3
    if lanes:
        v.sm = s[i]; i += 1
    if slots:
        v.ss = s[i]; i += 1
    return v


def _rope_struct(rope: Optional[LaneRope]) -> L.Rope:
    r = L.Rope()
    if rope is None:
        return r
    r.enable = 1
    for i in range(4):
        r.pairs[i] = rope.pairs[i]
        r.scale[i] = rope.scale[i]
        r.den[i] = rope.den[i]
    r.pos0 = rope.pos0
    return r


def _fill_decay(args, decay, decay_kind, braid_rates, braid_clamp):
    args.decay_kind = _DECAY[decay_kind]
    for i in range(4):
        args.braid_rates[i] = braid_rates[i]
    args.braid_clamp = braid_clamp


def _lanes_expand(x, M):
    """[B,T,H,D] (lane-shared) -> stride-0 [B,T,H,M,D] view; [B,T,H,M,D] unchanged."""
    if x.dim() == 4:
        return x.unsqueeze(3).expand(-1, -1, -1, M, -1)
    return x


def _gate(x, D):
    """[B,T,H,M] scalar gate -> [B,T,H,M,1]; [B,T,H,M,D] vector gate unchanged."""
    if x.dim() == 4:
        return x.unsqueeze(-1)
    if x.shape[-1] not in (1, D):
        raise ValueError("gate last dim must be 1 or the feature size")
    return x


# ----------------------------------------------------------------------------
# dense scan (GDN3 with compaction off; KMD-2)
# ----------------------------------------------------------------------------

def gdn3_scan(q, k, v, b_gate, w_gate, decay, *, decay_kind="gamma", rope: Optional[LaneRope] = None,
              state: Optional[torch.Tensor] = None, return_state: bool = False,
              out_dtype: Optional[torch.dtype] = None, algo: str = "auto",
              braid_rates=BRAID_RATES, braid_clamp=DECAY_CLAMP, out: Optional[torch.Tensor] = None,
              workspace: Optional[torch.Tensor] = None):
    """Dense GDN3 scan.  q, k: [B,T,H,(M,)K]; v: [B,T,H,(M,)V]; b_gate: [B,T,H,M(,K)];
    w_gate: [B,T,H,M(,V)]; decay: [B,T,H,M] (or [B,T,H,M,4] braided logits).

    Returns y [B,T,H,M,V] (and the final state [B*H*M, V, K] fp32 if asked).
    """
    B, T, H = k.shape[:3]
    M = b_gate.shape[3]
    K, V = k.shape[-1], v.shape[-1]
    _require_cuda(q, k, v, b_gate, w_gate, decay, state)
    qx, kx, vx = _lanes_expand(q, M), _lanes_expand(k, M), _lanes_expand(v, M)
    bg, wg = _gate(b_gate, K), _gate(w_gate, V)
    dec = decay if decay_kind == "braided" else decay.unsqueeze(-1)
    out_dtype = out_dtype or (torch.float32 if q.dtype == torch.float32 else q.dtype)
    y = out if out is not None else torch.empty(B, T, H, M, V, dtype=out_dtype, device=q.device)
    a = L.ScanArgs()
    a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, M, K, V
    a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_GDN3, _ALGO[algo], 1, 64
    a.q, a.k, a.v = _view(qx, True), _view(kx, True), _view(vx, True)
    a.gate_e, a.gate_w, a.decay = _view(bg, True), _view(wg, True), _view(dec, True)
    _fill_decay(a, dec, decay_kind, braid_rates, braid_clamp)
    a.rope = _rope_struct(rope)
    a.y, a.y_dtype = y.data_ptr(), _DT[y.dtype]
    a.y_sb, a.y_st, a.y_sh, a.y_sm = y.stride()[:4]
    st_out = None
    if state is not None:
        if state.dtype != torch.float32 or not state.is_contiguous() or state.shape != (B * H * M, V, K):
            raise ValueError("state must be contiguous fp32 [B*H*M, V, K]")
        a.state_in = state.data_ptr()
    if return_state:
        st_out = torch.empty(B * H * M, V, K, dtype=torch.float32, device=q.device)
        a.state_out = st_out.data_ptr()
    _run_scan(a, q.device, workspace)
    return (y, st_out) if return_state else y


# Scan workspaces owned by this module, one per (device, stream): grown on demand and
# reused, so repeated calls allocate nothing.  Calls on one stream are ordered, so
# they can share it; pass `workspace=` to manage the memory yourself.
_WORKSPACES = {}


# ----------------------------------------------------------------------------
# host-to-host scan with copy / compute overlap
# ----------------------------------------------------------------------------

_HOST_BUFS = {}
_HOST_BUF_CONFIGS = 4  # buffer configurations kept resident (least recently used dropped first)
_HOST_STREAMS = {}


def _host_pipeline_buffers(device, shapes_dtypes):
    """Two device buffer sets (double buffering) for the sliced host scan, cached by shape."""
    key = (device.index,) + tuple(shapes_dtypes)
    bufs = _HOST_BUFS.pop(key, None)
    if bufs is None:
        bufs = [[torch.empty(shp, dtype=dt, device=device) for shp, dt in shapes_dtypes] for _ in range(2)]
        while len(_HOST_BUFS) >= _HOST_BUF_CONFIGS:
            _HOST_BUFS.pop(next(iter(_HOST_BUFS)))
    _HOST_BUFS[key] = bufs  # most recently used last
    return bufs


def _host_copy_streams(device):
    """The copy-in and copy-out streams of the host scan on ``device`` (created once)."""
    ss = _HOST_STREAMS.get(device.index)
    if ss is None:
        ss = (torch.cuda.Stream(device), torch.cuda.Stream(device))
        _HOST_STREAMS[device.index] = ss
    return ss


def gdn3_scan_host(q, k, v, b_gate, w_gate, decay, *, out: torch.Tensor, device=None, slices: Optional[int] = None,
                   decay_kind="gamma", rope: Optional[LaneRope] = None, algo: str = "auto",
                   braid_rates=BRAID_RATES, braid_clamp=DECAY_CLAMP):
    """Dense GDN3 scan from host memory to host memory.

    Inputs and ``out`` are CPU tensors (pinned for asynchronous copies) shaped as for
    :func:`gdn3_scan`.  Chains never interact across batch rows, so the batch is cut
    into ``slices`` (default: one row each, at most 16); each slice's host->device
    copies, scan and device->host copy run on three CUDA streams ordered by events,
    so copies in both directions overlap the scans of neighbouring slices.  Device
    buffers are double-buffered and cached.  Returns ``out`` once the last copy has
    been enqueued on the current stream's timeline (synchronise before reading it).
    """
    device = torch.device(device) if device is not None else torch.device("cuda")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    ins = [q, k, v, b_gate, w_gate, decay]
    if any(t.is_cuda for t in ins + [out]):
        raise ValueError("gdn3_scan_host takes host tensors; use gdn3_scan for device tensors")
    B = k.shape[0]
    nsl = slices or min(B, 16)
    bounds = [(B * i) // nsl for i in range(nsl + 1)]
    rows = max(bounds[i + 1] - bounds[i] for i in range(nsl))
    shapes = [((rows,) + tuple(t.shape[1:]), t.dtype) for t in ins] + [((rows,) + tuple(out.shape[1:]), out.dtype)]
    bufs = _host_pipeline_buffers(device, shapes)
    with torch.cuda.device(device):
        main = torch.cuda.current_stream(device)
        h2d, d2h = _host_copy_streams(device)
        h2d.wait_stream(main)
        d2h.wait_stream(main)
        done_in = [torch.cuda.Event() for _ in range(nsl)]
        done_scan = [torch.cuda.Event() for _ in range(nsl)]
        done_out = [torch.cuda.Event() for _ in range(nsl)]
        for i in range(nsl):
            b0, b1 = bounds[i], bounds[i + 1]
            n = b1 - b0
            buf = bufs[i % 2]
            with torch.cuda.stream(h2d):
                if i >= 2:
                    h2d.wait_event(done_scan[i - 2])  # the scan two slices back has read this buffer set
                for d_t, h_t in zip(buf[:6], ins):
                    d_t[:n].copy_(h_t[b0:b1], non_blocking=True)
                done_in[i].record(h2d)
            main.wait_event(done_in[i])
            if i >= 2:
                main.wait_event(done_out[i - 2])  # its output buffer has been copied out
            dq, dk, dv, db, dw, dd = (t[:n] for t in buf[:6])
            gdn3_scan(dq, dk, dv, db, dw, dd, decay_kind=decay_kind, rope=rope, algo=algo,
                      braid_rates=braid_rates, braid_clamp=braid_clamp, out=buf[6][:n])
            done_scan[i].record(main)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done_scan[i])
                out[b0:b1].copy_(buf[6][:n], non_blocking=True)
                done_out[i].record(d2h)
        main.wait_event(done_out[nsl - 1])
        main.wait_stream(h2d)
    return out


def _cached_workspace(device, need):
    key = (device.index, _stream(device))
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def device_status(workspace: Optional[torch.Tensor] = None) -> int:
    """Device-side status of scans that used ``workspace`` (default: every workspace this
    module owns): the error word the kernels write when a bounded wait gives up
    (``GDNX_ETIMEOUT``; their outputs are then invalid), 0 otherwise.  Synchronises."""
    wss = [workspace] if workspace is not None else list(_WORKSPACES.values())
    for ws in wss:
        if ws is None or ws.numel() < 4:
            continue
        code = int(ws[:4].view(torch.int32).item())
        if code:
            return code
    return 0


def check_device_status(workspace: Optional[torch.Tensor] = None) -> None:
    """Raise ``RuntimeError`` if :func:`device_status` reports an error."""
    code = device_status(workspace)
    if code:
        raise RuntimeError("gdnx device error: " + L.load().gdnx_status_string(code).decode())


def _run_scan(a, device, workspace):
    lib = L.load()
    need = lib.gdnx_scan_workspace_bytes(C.byref(a))
    ws = workspace
    if need:
        if ws is None or ws.numel() * ws.element_size() < need:
            ws = _cached_workspace(device, need)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel() * ws.element_size()
    with torch.cuda.device(device):
        L.check(lib.gdnx_scan_fwd(C.byref(a), C.c_void_p(_stream(device))), "gdnx_scan_fwd")


def kmd2_scan(q, k, v, g, beta_e, beta_w, out_mix=None, *, scores: bool = False,
              state: Optional[torch.Tensor] = None, return_state: bool = False,
              out_dtype: Optional[torch.dtype] = None, algo: str = "auto"):
    """KMD-2 scan.  q [B,T,H,r,dk], k/g [B,T,H,dk] (g may be [B,T,H] scalar), v [B,T,H,dv],
    beta_e/beta_w [B,T,H], out_mix [H,r] (r > 1).  Returns y [B,T,H,dv]
    (+ scores [B,T,H] and/or final state [B*H, dv, dk] fp32)."""
    B, T, H, r_out, dk = q.shape
    dv = v.shape[-1]
    _require_cuda(q, k, v, g, beta_e, beta_w, out_mix, state)
    out_dtype = out_dtype or torch.float32
    y = torch.empty(B, T, H, 1, dv, dtype=out_dtype, device=q.device)
    sc = torch.empty(B, T, H, 1, dtype=torch.float32, device=q.device) if scores else None
    a = L.ScanArgs()
    a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, 1, dk, dv
    a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_KMD2, _ALGO[algo], r_out, 64
    a.q = _view(q, False, slots=True)
    a.k, a.v = _view(k, False), _view(v, False)
    a.gate_e, a.gate_w = _view(beta_e.unsqueeze(-1), False), _view(beta_w.unsqueeze(-1), False)
    gg = g if g.dim() == 4 else g.unsqueeze(-1)
    a.decay = _view(gg, False)
    _fill_decay(a, gg, "gamma", BRAID_RATES, DECAY_CLAMP)
    mix = None
    if r_out > 1:
        if out_mix is None:
            raise ValueError("out_mix is required when r_out > 1")
        mix = out_mix.detach().to(torch.float32).contiguous()
        a.out_mix = mix.data_ptr()
    a.y, a.y_dtype = y.data_ptr(), _DT[y.dtype]
    a.y_sb, a.y_st, a.y_sh, a.y_sm = y.stride()[:4]
    if sc is not None:
        a.scores = sc.data_ptr()
    st_out = None
    if state is not None:
        if state.dtype != torch.float32 or not state.is_contiguous() or state.shape != (B * H, dv, dk):
            raise ValueError("state must be contiguous fp32 [B*H, dv, dk]")
        a.state_in = state.data_ptr()
    if return_state:
        st_out = torch.empty(B * H, dv, dk, dtype=torch.float32, device=q.device)
        a.state_out = st_out.data_ptr()
    _run_scan(a, q.device, None)
    outs = [y[:, :, :, 0]]
    if scores:
        outs.append(sc[..., 0])
    if return_state:
        outs.append(st_out)
    return outs[0] if len(outs) == 1 else tuple(outs)


# ----------------------------------------------------------------------------
# GDN3 Kronecker-residual scan + compaction
# ----------------------------------------------------------------------------

@dataclass
class KRState:
    """Device state of the GDN3-KR recurrence (reference layouts,
    gdn3/_reference_recurrence.py:52-55) plus the slot pointer per chain."""
    A: torch.Tensor      # [N,R,a_v,a_k]
    Bk: torch.Tensor     # [N,R,b_v,b_k]
    U: torch.Tensor      # [N,V,P]
    Vb: torch.Tensor     # [N,K,P]
    slot: torch.Tensor   # [N] int32
    err: torch.Tensor    # [N] fp32 accumulated discarded energy

    @staticmethod
    def zeros(N, R, P, dims, V, K, device):
        a_v, a_k, b_v, b_k = dims
        f = dict(dtype=torch.float32, device=device)
        return KRState(torch.zeros(N, R, a_v, a_k, **f), torch.zeros(N, R, b_v, b_k, **f),
                       torch.zeros(N, V, P, **f), torch.zeros(N, K, P, **f),
                       torch.zeros(N, dtype=torch.int32, device=device), torch.zeros(N, **f))


_COMPACT_MODES = {"svd": L.GDNX_COMPACT_SVD, "sketch": L.GDNX_COMPACT_SKETCH, "sketch_noqr": L.GDNX_COMPACT_SKETCH}


def sketch_width(R: int, dims, compact_mode: str = "svd") -> int:
    """Columns of the compaction sketch G: min(R + 4, a_v a_k, b_v b_k) for the SVD
    (gdn3/gdn3_upgrade.py:599), R for "sketch" / "sketch_noqr" (:580)."""
    if compact_mode not in _COMPACT_MODES:
        raise ValueError(f"unknown compact_mode {compact_mode!r} (svd, sketch, sketch_noqr)")
    a_v, a_k, b_v, b_k = dims
    return R if compact_mode != "svd" else min(R + 4, a_v * a_k, b_v * b_k)


def _check_sketch(sketch, N, R, dims, compact_mode):
    want = (N, dims[2] * dims[3], sketch_width(R, dims, compact_mode))
    if tuple(sketch.shape) != want:
        raise ValueError(f"sketch must be {list(want)} for compact_mode={compact_mode!r}, got {list(sketch.shape)}")


def gdn3_kr_scan(q, k, v, b_gate, w_gate, decay, state: KRState, sketch: torch.Tensor, *,
                 P: int, R: int = 4, dims=(16, 16, 8, 8), slow_decay: float = 0.97,
                 decay_kind: str = "gamma", rope: Optional[LaneRope] = None,
                 out_dtype: Optional[torch.dtype] = None, braid_rates=BRAID_RATES,
                 braid_clamp=DECAY_CLAMP, compact_mode: str = "svd"):
    """GDN3-KR scan continuing ``state`` in place.  Shapes as ``gdn3_scan``;
    ``sketch`` is the compaction sketch G [N, b_v*b_k, sketch_width(R, dims, compact_mode)]
    (fp32).  ``compact_mode`` is the reference layer's ``GDN3_COMPACT_MODE``."""
    B, T, H = k.shape[:3]
    M = b_gate.shape[3]
    K, V = k.shape[-1], v.shape[-1]
    N = B * H * M
    _require_cuda(q, k, v, b_gate, w_gate, decay, sketch)
    _check_sketch(sketch, N, R, dims, compact_mode)
    for t in (state.A, state.Bk, state.U, state.Vb, state.err, sketch):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("KR state and sketch must be contiguous fp32")
    if state.U.shape != (N, V, P) or state.Vb.shape != (N, K, P):
        raise ValueError("state U/Vb shapes do not match [N,V,P]/[N,K,P]")
    qx, kx, vx = _lanes_expand(q, M), _lanes_expand(k, M), _lanes_expand(v, M)
    bg, wg = _gate(b_gate, K), _gate(w_gate, V)
    dec = decay if decay_kind == "braided" else decay.unsqueeze(-1)
    out_dtype = out_dtype or (torch.float32 if q.dtype == torch.float32 else q.dtype)
    y = torch.empty(B, T, H, M, V, dtype=out_dtype, device=q.device)
    ka = L.KrScanArgs()
    a = ka.base
    a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, M, K, V
    a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_GDN3, L.GDNX_ALGO_RECURRENT, 1, 64
    a.q, a.k, a.v = _view(qx, True), _view(kx, True), _view(vx, True)
    a.gate_e, a.gate_w, a.decay = _view(bg, True), _view(wg, True), _view(dec, True)
    _fill_decay(a, dec, decay_kind, braid_rates, braid_clamp)
    a.rope = _rope_struct(rope)
    a.y, a.y_dtype = y.data_ptr(), _DT[y.dtype]
    a.y_sb, a.y_st, a.y_sh, a.y_sm = y.stride()[:4]
    ka.R, ka.P = R, P
    ka.a_v, ka.a_k, ka.b_v, ka.b_k = dims
    ka.slow_decay = slow_decay
    ka.sketch = sketch.data_ptr()
    ka.A, ka.Bk, ka.U, ka.Vb = (state.A.data_ptr(), state.Bk.data_ptr(), state.U.data_ptr(),
                                state.Vb.data_ptr())
    ka.slot, ka.comp_err = state.slot.data_ptr(), state.err.data_ptr()
    ka.compact_mode = _COMPACT_MODES[compact_mode]
    lib = L.load()
    with torch.cuda.device(q.device):
        L.check(lib.gdnx_kr_scan_fwd(C.byref(ka), C.c_void_p(_stream(q.device))), "gdnx_kr_scan_fwd")
    return y


def compact(A, Bk, U, Vb, sketch, *, dims=(16, 16, 8, 8), slow_decay: float = 0.97, compact_mode: str = "svd"):
    """One compaction per chain, in place on A and Bk; returns per-chain discarded energy [N]
    (zeros in the sketch modes, like the reference)."""
    _require_cuda(A, Bk, U, Vb, sketch)
    N, R = A.shape[:2]
    _check_sketch(sketch, N, R, dims, compact_mode)
    V, P = U.shape[1:]
    K = Vb.shape[1]
    for t in (A, Bk, U, Vb, sketch):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("compaction operands must be contiguous fp32")
    err = torch.empty(N, dtype=torch.float32, device=A.device)
    ca = L.CompactArgs()
    ca.N, ca.R, ca.P, ca.V, ca.K = N, R, P, V, K
    ca.a_v, ca.a_k, ca.b_v, ca.b_k = dims
    ca.slow_decay = slow_decay
    ca.sketch, ca.A, ca.Bk, ca.U, ca.Vb, ca.err = (sketch.data_ptr(), A.data_ptr(), Bk.data_ptr(),
                                                  U.data_ptr(), Vb.data_ptr(), err.data_ptr())
    ca.compact_mode = _COMPACT_MODES[compact_mode]
    lib = L.load()
    with torch.cuda.device(A.device):
        L.check(lib.gdnx_compact(C.byref(ca), C.c_void_p(_stream(A.device))), "gdnx_compact")
    return err


# ----------------------------------------------------------------------------
# decode step
# ----------------------------------------------------------------------------

def decode_step(S, q, k, v, b_gate, w_gate, decay, *, mode: str = "gdn3", decay_kind: str = "gamma",
                rope: Optional[LaneRope] = None, out_mix=None, out: Optional[torch.Tensor] = None,
                out_dtype: Optional[torch.dtype] = None):
    """One token for every chain, updating the dense state S [N, V, K] in place.

    GDN3 (N = B*H*M): q, k [B,H,(M,)K]; v [B,H,(M,)V]; b_gate [B,H,M(,K)];
    w_gate [B,H,M(,V)]; decay [B,H,M]; returns y [B,H,M,V].
    KMD-2 (N = B*H): q [B,H,r,K]; k [B,H,K]; v [B,H,V]; beta_e/beta_w [B,H];
    decay [B,H,K] (per channel) or [B,H]; returns y [B,H,V].
    ``rope.pos0`` is the absolute position of the token.
    """
    _require_cuda(S, q, k, v, b_gate, w_gate, decay)
    kmd2 = mode == "kmd2"
    B, H = k.shape[:2]
    K, V = k.shape[-1], v.shape[-1]
    if kmd2:
        M, r_out = 1, q.shape[2]
        qv = q[:, None, :, None]                  # [B,1,H,1,r,K]
        kx, vx = k[:, None, :, None], v[:, None, :, None]
        bg, wg = b_gate[:, None, :, None, None], w_gate[:, None, :, None, None]
        dec = decay[:, None, :, None] if decay.dim() == 3 else decay[:, None, :, None, None]
    else:
        M, r_out = b_gate.shape[2], 1
        lane = lambda x: x if x.dim() == 4 else x.unsqueeze(2).expand(-1, -1, M, -1)
        qv, kx, vx = lane(q)[:, None], lane(k)[:, None], lane(v)[:, None]
        g1 = lambda x: (x.unsqueeze(-1) if x.dim() == 3 else x)[:, None]
        bg, wg = g1(b_gate), g1(w_gate)
        dec = decay[:, None, ..., None] if decay.dim() == 3 else decay[:, None]
    N = B * H * M
    if S.dtype != torch.float32 or not S.is_contiguous() or S.shape != (N, V, K):
        raise ValueError("S must be contiguous fp32 [N, V, K]")
    out_dtype = out_dtype or (torch.float32 if v.dtype == torch.float32 else v.dtype)
    y = out if out is not None else torch.empty(B, H, M, V, dtype=out_dtype, device=S.device)
    a = L.DecodeArgs()
    a.B, a.H, a.M, a.K, a.V = B, H, M, K, V
    a.mode = L.GDNX_MODE_KMD2 if kmd2 else L.GDNX_MODE_GDN3
    a.r_out = r_out
    a.q = _view(qv, True, slots=kmd2)
    a.k, a.v = _view(kx, True), _view(vx, True)
    a.gate_e, a.gate_w, a.decay = _view(bg, True), _view(wg, True), _view(dec, True)
    a.decay_kind = _DECAY[decay_kind]
    for i in range(4):
        a.braid_rates[i] = BRAID_RATES[i]
    a.braid_clamp = DECAY_CLAMP
    a.rope = _rope_struct(rope)
    mix = None
    if r_out > 1:
        mix = out_mix.detach().to(torch.float32).contiguous()
        a.out_mix = mix.data_ptr()
    a.S = S.data_ptr()
    a.y, a.y_dtype = y.data_ptr(), _DT[y.dtype]
    a.y_sb, a.y_sh, a.y_sm = y.stride()[:3]
    lib = L.load()
    with torch.cuda.device(S.device):
        L.check(lib.gdnx_decode_step(C.byref(a), C.c_void_p(_stream(S.device))), "gdnx_decode_step")
    return y[:, :, 0] if kmd2 else y


def gdn3_scan_noalloc(q, k, v, b_gate, w_gate, decay, *, decay_kind="gamma", rope: Optional[LaneRope] = None,
                      state: Optional[torch.Tensor] = None, out: torch.Tensor,
                      state_out: Optional[torch.Tensor] = None):
    """Dense GDN3 scan through ``gdnx_scan_fwd_noalloc``: the library allocates
    nothing and uses no caller workspace.  ``out`` ([B,T,H,M,V]) and the
    optional ``state_out`` ([B*H*M, V, K] fp32) must be provided by the caller;
    shapes otherwise as :func:`gdn3_scan` (chunked-kernel inputs only)."""
    B, T, H = k.shape[:3]
    M = b_gate.shape[3]
    K, V = k.shape[-1], v.shape[-1]
    _require_cuda(q, k, v, b_gate, w_gate, decay, state, out, state_out)
    qx, kx, vx = _lanes_expand(q, M), _lanes_expand(k, M), _lanes_expand(v, M)
    bg, wg = _gate(b_gate, K), _gate(w_gate, V)
    dec = decay if decay_kind == "braided" else decay.unsqueeze(-1)
    a = L.ScanArgs()
    a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, M, K, V
    a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_GDN3, L.GDNX_ALGO_CHUNKED, 1, 64
    a.q, a.k, a.v = _view(qx, True), _view(kx, True), _view(vx, True)
    a.gate_e, a.gate_w, a.decay = _view(bg, True), _view(wg, True), _view(dec, True)
    _fill_decay(a, dec, decay_kind, BRAID_RATES, DECAY_CLAMP)
    a.rope = _rope_struct(rope)
    a.y, a.y_dtype = out.data_ptr(), _DT[out.dtype]
    a.y_sb, a.y_st, a.y_sh, a.y_sm = out.stride()[:4]
    if state is not None:
        a.state_in = state.data_ptr()
    if state_out is not None:
        a.state_out = state_out.data_ptr()
    lib = L.load()
    with torch.cuda.device(q.device):
        L.check(lib.gdnx_scan_fwd_noalloc(C.byref(a), C.c_void_p(_stream(q.device))), "gdnx_scan_fwd_noalloc")
    return out


def noalloc_status(device=None) -> int:
    """Device error word of the allocation-free scans on ``device`` (after the current
    stream's work; synchronises it): 0, or ``GDNX_ETIMEOUT`` if a kernel gave up a
    bounded wait (its outputs are then invalid).  The next such scan clears it."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    lib = L.load()
    word = C.c_int32(0)
    with torch.cuda.device(device):
        L.check(lib.gdnx_scan_noalloc_status(C.byref(word), C.c_void_p(_stream(device))), "gdnx_scan_noalloc_status")
    return int(word.value)


# ----------------------------------------------------------------------------
# output epilogues
# ----------------------------------------------------------------------------

def lane_route(y: torch.Tensor, router_logits: torch.Tensor, norm: Optional[torch.Tensor] = None, *,
               gate: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
               out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """GDN3 lane routing and per-head norm in one pass (gdn3/gdn3_upgrade.py:842-856):
    ``softmax`` over the lanes of ``router_logits [B,T,H,M]``, the weighted lane sum of
    ``y [B,T,H,M,V]``, then ``F.normalize(., dim=-1, eps=1e-6) * sqrt(V) * norm``; with
    ``gate`` (the layer's output-gate pre-activation, ``[B,T,H*V]`` or ``[B,T,H,V]``) also
    ``* silu(gate)``, which is the layer's next step when ``H*V == D`` (no ``_agg_proj``,
    :861-871).  Returns ``[B,T,H,V]`` (``out_dtype`` defaults to ``y``'s)."""
    _require_cuda(y, router_logits, norm, gate, out)
    B, T, H, M, V = y.shape
    out = out if out is not None else torch.empty(B, T, H, V, dtype=out_dtype or y.dtype, device=y.device)
    a = L.EpilogueArgs()
    a.B, a.T, a.H, a.M, a.V = B, T, H, M, V
    a.kind = L.GDNX_EPILOGUE_LANE_ROUTE
    a.y = _view(y, True)
    a.router = _view(router_logits.unsqueeze(-1), True)
    if gate is not None:
        gate = gate.view(B, T, H, V) if gate.dim() == 3 else gate
        a.gate = _view(gate, False)
    w = None
    if norm is not None:
        w = norm.detach().to(torch.float32).contiguous()
        a.weight = w.data_ptr()
    a.out, a.out_dtype = out.data_ptr(), _DT[out.dtype]
    a.out_sb, a.out_st, a.out_sh = out.stride()[:3]
    lib = L.load()
    with torch.cuda.device(y.device):
        L.check(lib.gdnx_epilogue(C.byref(a), C.c_void_p(_stream(y.device))), "gdnx_epilogue")
    return out


def lane_route_scatter(y: torch.Tensor, router_logits: torch.Tensor, dests, out_strides, out_dtype: torch.dtype,
                       norm: Optional[torch.Tensor] = None, *, gate: Optional[torch.Tensor] = None) -> None:
    """:func:`lane_route` with the routed rows stored to every device address in ``dests``
    (this GPU's buffer and its peers', e.g. from ``distributed.PeerBuffer``): the routing
    fused with the all-gather of its output.  ``out_strides`` are the element strides
    (batch, token, head) of the destination layout; each destination must have room for
    ``[B,T,H,V]`` there.  The peers may read the rows once a cross-GPU collective issued
    after this call on the same stream has completed."""
    _require_cuda(y, router_logits, norm, gate)
    B, T, H, M, V = y.shape
    a = L.EpilogueArgs()
    a.B, a.T, a.H, a.M, a.V = B, T, H, M, V
    a.kind = L.GDNX_EPILOGUE_LANE_ROUTE
    a.y = _view(y, True)
    a.router = _view(router_logits.unsqueeze(-1), True)
    if gate is not None:
        gate = gate.view(B, T, H, V) if gate.dim() == 3 else gate
        a.gate = _view(gate, False)
    w = None
    if norm is not None:
        w = norm.detach().to(torch.float32).contiguous()
        a.weight = w.data_ptr()
    a.out_dtype = _DT[out_dtype]
    a.out_sb, a.out_st, a.out_sh = out_strides
    arr = (C.c_void_p * len(dests))(*dests)
    lib = L.load()
    with torch.cuda.device(y.device):
        L.check(lib.gdnx_epilogue_scatter(C.byref(a), arr, len(dests), C.c_void_p(_stream(y.device))),
                "gdnx_epilogue_scatter")


def rms_norm_gated(y: torch.Tensor, gate: torch.Tensor, weight: Optional[torch.Tensor] = None, *, eps: float = 1e-6,
                   out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """KMD-2 output norm (``Qwen3_5RMSNormGated`` as called at gdn3/kmd2_native.py:176):
    ``weight * y * rsqrt(mean(y^2) + eps) * silu(gate)`` over the last dim, computed in
    fp32 from ``y [B,T,H,V]`` and ``gate [B,T,H,V]``; output in ``out_dtype`` (default the
    gate's dtype)."""
    _require_cuda(y, gate, weight, out)
    B, T, H, V = y.shape
    out = out if out is not None else torch.empty(B, T, H, V, dtype=out_dtype or gate.dtype, device=y.device)
    a = L.EpilogueArgs()
    a.B, a.T, a.H, a.M, a.V = B, T, H, 1, V
    a.kind, a.eps = L.GDNX_EPILOGUE_RMS_GATED, eps
    a.y, a.gate = _view(y, False), _view(gate, False)
    w = None
    if weight is not None:
        w = weight.detach().to(torch.float32).contiguous()
        a.weight = w.data_ptr()
    a.out, a.out_dtype = out.data_ptr(), _DT[out.dtype]
    a.out_sb, a.out_st, a.out_sh = out.stride()[:3]
    lib = L.load()
    with torch.cuda.device(y.device):
        L.check(lib.gdnx_epilogue(C.byref(a), C.c_void_p(_stream(y.device))), "gdnx_epilogue")
    return out


def gdn3_prologue(qkv, conv_w, *, H: int, K: int, M: int, coprod=None, mix=None, b_proj=None, proj_a=None,
                  w_proj=None, proj_b=None, dims=(16, 16, 8, 8), out_dtype: Optional[torch.dtype] = None,
                  gate_dtype: Optional[torch.dtype] = None):
    """GDN3 projection prologue (gdn3/gdn3_upgrade.py:752-807, blend :201-250) after the layer's GEMMs.

    ``qkv [B,T,3*H*K]`` (the qkv projection), ``conv_w [3*H*K, 1, k]`` (the depthwise ``Conv1d``
    weight); ``coprod = (q_a, q_b, k_a, k_b, v_a, v_b)`` as ``[B,T,H,C,dim]`` factor projections and
    ``mix = (coprod_mix_qk, coprod_mix_v, coprod_strength_qk, coprod_strength_v)`` ([H] each), or None
    for dense features; ``b_proj [B,T,H,M,K]`` + ``proj_a [B,T,H]`` and ``w_proj [B,T,H,M,V]`` +
    ``proj_b [B,T,H]`` for the gates.  Returns ``(q, k, v)`` ``[B,T,H,K]`` (lane-shared; the scan
    applies the lane RoPE) and ``(b_gates, w_gates)`` ``[B,T,H,M,K]`` (or None)."""
    _require_cuda(qkv, conv_w, b_proj, w_proj)
    B, T = qkv.shape[:2]
    V = K
    out_dtype = out_dtype or qkv.dtype
    gate_dtype = gate_dtype or out_dtype
    dev = qkv.device
    q, k, v = (torch.empty(B, T, H, K, dtype=out_dtype, device=dev) for _ in range(3))
    a = L.PrologueArgs()
    a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, M, K, V
    a.a_k, a.b_k, a.a_v, a.b_v = dims[1], dims[3], dims[0], dims[2]
    cw = conv_w.detach().reshape(3 * H * K, -1).to(torch.float32).contiguous()
    a.conv_k = cw.shape[1]
    a.conv_w = cw.data_ptr()
    qv = L.View()
    qv.ptr, qv.dtype, qv.dim = qkv.data_ptr(), _DT[qkv.dtype], qkv.shape[-1]
    if qkv.stride(-1) != 1:
        raise ValueError("qkv must have a contiguous last dim")
    qv.sb, qv.st = qkv.stride(0), qkv.stride(1)
    a.qkv = qv
    keep = [cw]
    if coprod is not None:
        fs = [_view(f, False, slots=True) for f in coprod]
        a.q_a, a.q_b, a.k_a, a.k_b, a.v_a, a.v_b = fs
        a.C = coprod[0].shape[3]
        ms = [m.detach().to(torch.float32).contiguous() for m in mix]
        keep += ms
        a.mix_qk, a.mix_v, a.str_qk, a.str_v = (m.data_ptr() for m in ms)
    a.q_out, a.k_out, a.v_out = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.out_dtype = _DT[out_dtype]
    a.out_sb, a.out_st, a.out_sh = q.stride()[:3]
    bg = wg = None
    if b_proj is not None:
        bg = torch.empty(B, T, H, M, K, dtype=gate_dtype, device=dev)
        a.b_proj, a.proj_a = _view(b_proj, True), _view(proj_a.unsqueeze(-1), False)
        a.b_out = bg.data_ptr()
        a.gate_sb, a.gate_st, a.gate_sh, a.gate_sm = bg.stride()[:4]
    if w_proj is not None:
        wg = torch.empty(B, T, H, M, V, dtype=gate_dtype, device=dev)
        a.w_proj, a.proj_b = _view(w_proj, True), _view(proj_b.unsqueeze(-1), False)
        a.w_out = wg.data_ptr()
        a.wgate_sb, a.wgate_st, a.wgate_sh, a.wgate_sm = wg.stride()[:4]
    a.gate_dtype = _DT[gate_dtype]
    lib = L.load()
    with torch.cuda.device(dev):
        L.check(lib.gdnx_gdn3_prologue(C.byref(a), C.c_void_p(_stream(dev))), "gdnx_gdn3_prologue")
    return (q, k, v), (bg, wg)


def kmd2_prologue(mixed, conv_w, b, a, theta, *, H: int, dt_bias, A_log, decay_chan, bw_off,
                  q_slot_scale=None, r_out: int = 1, dk: int = 128, dv: int = 128):
    """KMD-2 prologue (gdn3/kmd2_native.py:140-172) from the layer's GEMM outputs to its scan inputs.

    ``mixed [B,T,2*H*dk+H*dv]`` (``in_proj_qkv`` output), ``conv_w`` (the depthwise ``Conv1d`` weight,
    ``[C,1,k]``), ``b``, ``a [B,T,H]`` (``in_proj_b`` / ``in_proj_a`` outputs), ``theta [B,T,H*dk/2]``
    (``rot_proj`` output); the module's ``dt_bias``, ``A_log``, ``decay_chan``, ``bw_off`` and, with
    ``r_out > 1``, ``q_slot_scale [H,r_out,dk]``.  Returns ``(q [B,T,H,r_out,dk], k, v, g [B,T,H,dk],
    beta_e, beta_w [B,T,H])`` in fp32 -- the arguments of ``KMD2NativeAttn._scan`` (``q`` squeezed to
    ``[B,T,H,dk]`` slots of one when ``r_out == 1`` is up to the caller)."""
    _require_cuda(mixed, conv_w, b, a, theta, dt_bias, A_log, decay_chan, bw_off, q_slot_scale)
    B, T = mixed.shape[:2]
    dev = mixed.device
    f32 = dict(dtype=torch.float32, device=dev)
    q = torch.empty(B, T, H, r_out, dk, **f32)
    k = torch.empty(B, T, H, dk, **f32)
    v = torch.empty(B, T, H, dv, **f32)
    g = torch.empty(B, T, H, dk, **f32)
    be = torch.empty(B, T, H, **f32)
    bw = torch.empty(B, T, H, **f32)
    ws = torch.empty(B, T, H, dk // 2, **f32)
    C_ = 2 * H * dk + H * dv
    cw = conv_w.detach().reshape(C_, -1).to(torch.float32).contiguous()
    params = [p.detach().to(torch.float32).contiguous() for p in (dt_bias, A_log, decay_chan, bw_off)]
    qss = q_slot_scale.detach().to(torch.float32).contiguous() if (r_out > 1 and q_slot_scale is not None) else None
    if (r_out > 1) != (qss is not None):
        raise ValueError("q_slot_scale is required exactly when r_out > 1")

    def view3(t, dim):
        if t.stride(-1) != 1 or t.shape[-1] != dim:
            raise ValueError("GEMM outputs must be [B,T,C] with a contiguous last dim")
        vw = L.View()
        vw.ptr, vw.dtype, vw.dim, vw.sb, vw.st = t.data_ptr(), _DT[t.dtype], dim, t.stride(0), t.stride(1)
        return vw

    args = L.Kmd2PrologueArgs()
    args.B, args.T, args.H, args.dk, args.dv = B, T, H, dk, dv
    args.r_out, args.conv_k = r_out, cw.shape[1]
    args.mixed, args.conv_w = view3(mixed, C_), cw.data_ptr()
    args.b, args.a, args.theta = view3(b, H), view3(a, H), view3(theta, H * dk // 2)
    args.dt_bias, args.A_log, args.decay_chan, args.bw_off = (p.data_ptr() for p in params)
    args.q_slot_scale = qss.data_ptr() if qss is not None else None
    args.q_out, args.k_out, args.v_out, args.g_out = q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr()
    args.beta_e_out, args.beta_w_out, args.theta_ws = be.data_ptr(), bw.data_ptr(), ws.data_ptr()
    lib = L.load()
    with torch.cuda.device(dev):
        L.check(lib.gdnx_kmd2_prologue(C.byref(args), C.c_void_p(_stream(dev))), "gdnx_kmd2_prologue")
    return q, k, v, g, be, bw


# ----------------------------------------------------------------------------
# backward of the dense scan (autograd)
# ----------------------------------------------------------------------------

def _scan_bwd(a, dy, dstate_out, B, T, H, M, K, V, r_out, de, dw, ddim, device):
    """Run gdnx_scan_bwd for forward arguments ``a``; returns per-chain-token gradients
    dq [B,T,H,M,r,K], dk, dv, dge [B,T,H,M,de], dgw, ddec, dstate_in, dmix (fp32)."""
    f32 = dict(dtype=torch.float32, device=device)
    dq = torch.empty(B, T, H, M, r_out, K, **f32)
    dk = torch.empty(B, T, H, M, K, **f32)
    dv = torch.empty(B, T, H, M, V, **f32)
    dge = torch.empty(B, T, H, M, de, **f32)
    dgw = torch.empty(B, T, H, M, dw, **f32)
    ddec = torch.empty(B, T, H, M, ddim, **f32)
    dst = torch.empty(B * H * M, V, K, **f32)
    dmix = torch.zeros(H, r_out, **f32) if r_out > 1 else None
    g = L.ScanBwdArgs()
    g.fwd = a
    dyc = dy.contiguous()
    g.dy = _view(dyc, True)
    dso = None
    if dstate_out is not None:
        dso = dstate_out.detach().to(torch.float32).contiguous()
        g.dstate_out = dso.data_ptr()
    g.dq, g.dk, g.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    g.dgate_e, g.dgate_w, g.ddecay = dge.data_ptr(), dgw.data_ptr(), ddec.data_ptr()
    g.dstate_in = dst.data_ptr()
    if dmix is not None:
        g.dout_mix = dmix.data_ptr()
    lib = L.load()
    need = lib.gdnx_scan_bwd_workspace_bytes(C.byref(g))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=device)
    g.workspace, g.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(device):
        L.check(lib.gdnx_scan_bwd(C.byref(g), C.c_void_p(_stream(device))), "gdnx_scan_bwd")
    return dq, dk, dv, dge, dgw, ddec, dst, dmix


def _sum_to(g, t):
    """Reduce a per-chain-token gradient to the shape of the input it belongs to (lane-shared
    or broadcast inputs take the sum), in the input's dtype."""
    if t is None:
        return None
    if g.shape != t.shape:
        if g.dim() == t.dim() + 1:  # lane dim absent in the input
            g = g.sum(dim=3)
        g = g.sum_to_size(t.shape)
    return g.to(t.dtype)


class _GDN3ScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, b_gate, w_gate, decay, state, decay_kind, algo):
        y, S = gdn3_scan(q, k, v, b_gate, w_gate, decay, decay_kind=decay_kind, state=state, return_state=True,
                         out_dtype=torch.float32, algo=algo)
        ctx.save_for_backward(q, k, v, b_gate, w_gate, decay, state)
        ctx.decay_kind = decay_kind
        return y, S

    @staticmethod
    def backward(ctx, dy, dS):
        q, k, v, b_gate, w_gate, decay, state = ctx.saved_tensors
        B, T, H = k.shape[:3]
        M = b_gate.shape[3]
        K, V = k.shape[-1], v.shape[-1]
        qx, kx, vx = _lanes_expand(q, M), _lanes_expand(k, M), _lanes_expand(v, M)
        bg, wg = _gate(b_gate, K), _gate(w_gate, V)
        dec = decay.unsqueeze(-1) if decay.dim() == 4 else decay
        a = L.ScanArgs()
        a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, M, K, V
        a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_GDN3, L.GDNX_ALGO_RECURRENT, 1, 64
        a.q, a.k, a.v = _view(qx, True), _view(kx, True), _view(vx, True)
        a.gate_e, a.gate_w, a.decay = _view(bg, True), _view(wg, True), _view(dec, True)
        _fill_decay(a, dec, ctx.decay_kind, BRAID_RATES, DECAY_CLAMP)
        if state is not None:
            a.state_in = state.data_ptr()
        if dy is None:
            dy = torch.zeros(B, T, H, M, V, device=k.device)
        dq, dk, dv, dge, dgw, ddec, dst, _ = _scan_bwd(a, dy, dS, B, T, H, M, K, V, 1, bg.shape[-1], wg.shape[-1],
                                                       dec.shape[-1], k.device)
        dq = dq[:, :, :, :, 0]
        dge = dge.reshape(bg.shape) if b_gate.dim() == 5 else dge[..., 0]
        dgw = dgw.reshape(wg.shape) if w_gate.dim() == 5 else dgw[..., 0]
        ddec = ddec.reshape(dec.shape) if decay.dim() == 5 else ddec[..., 0]
        return (_sum_to(dq, q), _sum_to(dk, k), _sum_to(dv, v), _sum_to(dge, b_gate), _sum_to(dgw, w_gate),
                _sum_to(ddec, decay), dst if state is not None else None, None, None)


class _KMD2ScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta_e, beta_w, out_mix, scores):
        outs = kmd2_scan(q, k, v, g, beta_e, beta_w, out_mix, scores=scores)
        ctx.save_for_backward(q, k, v, g, beta_e, beta_w, out_mix)
        if scores:
            y, sc = outs
            ctx.mark_non_differentiable(sc)
            return y, sc
        return outs, None

    @staticmethod
    def backward(ctx, dy, dsc):
        q, k, v, g, beta_e, beta_w, out_mix = ctx.saved_tensors
        B, T, H, r_out, dk_ = q.shape
        dv_ = v.shape[-1]
        a = L.ScanArgs()
        a.B, a.T, a.H, a.M, a.K, a.V = B, T, H, 1, dk_, dv_
        a.mode, a.algo, a.r_out, a.chunk = L.GDNX_MODE_KMD2, L.GDNX_ALGO_RECURRENT, r_out, 64
        a.q = _view(q, False, slots=True)
        a.k, a.v = _view(k, False), _view(v, False)
        a.gate_e, a.gate_w = _view(beta_e.unsqueeze(-1), False), _view(beta_w.unsqueeze(-1), False)
        gg = g if g.dim() == 4 else g.unsqueeze(-1)
        a.decay = _view(gg, False)
        _fill_decay(a, gg, "gamma", BRAID_RATES, DECAY_CLAMP)
        mix = None
        if r_out > 1:
            mix = out_mix.detach().to(torch.float32).contiguous()
            a.out_mix = mix.data_ptr()
        dyl = dy.unsqueeze(3)  # [B,T,H,1,V]
        dq, dk, dv, dge, dgw, ddec, _, dmix = _scan_bwd(a, dyl, None, B, T, H, 1, dk_, dv_, r_out, 1, 1,
                                                        gg.shape[-1], k.device)
        dq = dq[:, :, :, 0]
        ddec = ddec[:, :, :, 0] if g.dim() == 4 else ddec[:, :, :, 0, 0]
        dmix_out = dmix.to(out_mix.dtype) if (r_out > 1 and out_mix is not None) else None
        return (dq.to(q.dtype), dk[:, :, :, 0].to(k.dtype), dv[:, :, :, 0].to(v.dtype), ddec.to(g.dtype),
                dge[:, :, :, 0, 0].to(beta_e.dtype), dgw[:, :, :, 0, 0].to(beta_w.dtype), dmix_out, None)


def kmd2_scan_train(q, k, v, g, beta_e, beta_w, out_mix=None, *, scores: bool = False):
    """Differentiable KMD-2 scan (forward on the scan kernels, backward by ``gdnx_scan_bwd``).
    Shapes as :func:`kmd2_scan`.  Returns y [B,T,H,dv] (and detached scores [B,T,H] if asked)."""
    y, sc = _KMD2ScanFn.apply(q, k, v, g, beta_e, beta_w, out_mix, scores)
    return (y, sc) if scores else y


def gdn3_scan_train(q, k, v, b_gate, w_gate, decay, *, decay_kind="gamma", state=None, algo="auto"):
    """Differentiable dense GDN3 scan: forward on the scan kernels, backward by the exact fp32
    reverse-mode kernel (``gdnx_scan_bwd``).  Shapes as :func:`gdn3_scan` (no lane RoPE: rotate
    q/k before the call, as the reference module does).  Returns ``(y [B,T,H,M,V] fp32,
    final state [B*H*M, V, K])``."""
    return _GDN3ScanFn.apply(q, k, v, b_gate, w_gate, decay, state, decay_kind, algo)
