"""ctypes binding of the C ABI declared in ``include/gdnx.h``.

The structures below mirror the header field for field.  Loading fails
loudly when ``libgdnx.so`` is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgdnx.so"

GDNX_OK, GDNX_EINVAL, GDNX_ELAUNCH, GDNX_ETIMEOUT, GDNX_EUNSUPPORTED, GDNX_EWORKSPACE = range(6)
GDNX_F32, GDNX_BF16, GDNX_F16 = 0, 1, 2
GDNX_MODE_GDN3, GDNX_MODE_KMD2 = 0, 1
GDNX_DECAY_GAMMA, GDNX_DECAY_LOG, GDNX_DECAY_BRAIDED = 0, 1, 2
GDNX_ALGO_AUTO, GDNX_ALGO_RECURRENT, GDNX_ALGO_CHUNKED = 0, 1, 2
GDNX_EPILOGUE_LANE_ROUTE, GDNX_EPILOGUE_RMS_GATED = 0, 1
GDNX_COMPACT_SVD, GDNX_COMPACT_SKETCH = 0, 1

EXPORTED = ("gdnx_scan_fwd", "gdnx_scan_fwd_noalloc", "gdnx_scan_noalloc_status", "gdnx_scan_workspace_bytes", "gdnx_kr_scan_fwd", "gdnx_compact",
            "gdnx_decode_step", "gdnx_epilogue", "gdnx_gdn3_prologue", "gdnx_kmd2_prologue", "gdnx_scan_bwd", "gdnx_scan_bwd_workspace_bytes", "gdnx_status_string", "gdnx_version",
            "gdnx_epilogue_scatter", "gdnx_device_alloc", "gdnx_device_free", "gdnx_ipc_handle", "gdnx_ipc_open",
            "gdnx_ipc_close")


class View(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("dtype", C.c_int32), ("dim", C.c_int32),
                ("sb", C.c_int64), ("st", C.c_int64), ("sh", C.c_int64), ("sm", C.c_int64),
                ("ss", C.c_int64)]


class Rope(C.Structure):
    _fields_ = [("enable", C.c_int32), ("pairs", C.c_int32 * 4), ("scale", C.c_float * 4),
                ("den", C.c_float * 4), ("pos0", C.c_int64)]


class ScanArgs(C.Structure):
    _fields_ = [("B", C.c_int64), ("T", C.c_int64), ("H", C.c_int64), ("M", C.c_int64),
                ("K", C.c_int64), ("V", C.c_int64),
                ("mode", C.c_int32), ("algo", C.c_int32), ("r_out", C.c_int32), ("chunk", C.c_int32),
                ("q", View), ("k", View), ("v", View), ("gate_e", View), ("gate_w", View),
                ("decay", View), ("decay_kind", C.c_int32), ("braid_rates", C.c_float * 4),
                ("braid_clamp", C.c_float), ("rope", Rope),
                ("out_mix", C.c_void_p),
                ("y", C.c_void_p), ("y_dtype", C.c_int32),
                ("y_sb", C.c_int64), ("y_st", C.c_int64), ("y_sh", C.c_int64), ("y_sm", C.c_int64),
                ("scores", C.c_void_p),
                ("state_in", C.c_void_p), ("state_out", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class ScanBwdArgs(C.Structure):
    _fields_ = [("fwd", ScanArgs), ("dy", View), ("dstate_out", C.c_void_p),
                ("dq", C.c_void_p), ("dk", C.c_void_p), ("dv", C.c_void_p), ("dgate_e", C.c_void_p),
                ("dgate_w", C.c_void_p), ("ddecay", C.c_void_p), ("dstate_in", C.c_void_p),
                ("dout_mix", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class KrScanArgs(C.Structure):
    _fields_ = [("base", ScanArgs),
                ("R", C.c_int32), ("P", C.c_int32), ("a_v", C.c_int32), ("a_k", C.c_int32),
                ("b_v", C.c_int32), ("b_k", C.c_int32), ("slow_decay", C.c_float),
                ("sketch", C.c_void_p), ("A", C.c_void_p), ("Bk", C.c_void_p),
                ("U", C.c_void_p), ("Vb", C.c_void_p), ("slot", C.c_void_p), ("comp_err", C.c_void_p),
                ("compact_mode", C.c_int32)]


class CompactArgs(C.Structure):
    _fields_ = [("N", C.c_int64), ("R", C.c_int32), ("P", C.c_int32), ("V", C.c_int32), ("K", C.c_int32),
                ("a_v", C.c_int32), ("a_k", C.c_int32), ("b_v", C.c_int32), ("b_k", C.c_int32),
                ("slow_decay", C.c_float), ("sketch", C.c_void_p), ("A", C.c_void_p), ("Bk", C.c_void_p),
                ("U", C.c_void_p), ("Vb", C.c_void_p), ("err", C.c_void_p), ("compact_mode", C.c_int32)]


class DecodeArgs(C.Structure):
    _fields_ = [("B", C.c_int64), ("H", C.c_int64), ("M", C.c_int64), ("K", C.c_int64), ("V", C.c_int64),
                ("mode", C.c_int32), ("r_out", C.c_int32),
                ("q", View), ("k", View), ("v", View), ("gate_e", View), ("gate_w", View), ("decay", View),
                ("decay_kind", C.c_int32), ("braid_rates", C.c_float * 4), ("braid_clamp", C.c_float),
                ("rope", Rope), ("out_mix", C.c_void_p),
                ("S", C.c_void_p), ("y", C.c_void_p), ("y_dtype", C.c_int32),
                ("y_sb", C.c_int64), ("y_sh", C.c_int64), ("y_sm", C.c_int64)]


class EpilogueArgs(C.Structure):
    _fields_ = [("B", C.c_int64), ("T", C.c_int64), ("H", C.c_int64), ("M", C.c_int64), ("V", C.c_int64),
                ("kind", C.c_int32), ("eps", C.c_float),
                ("y", View), ("router", View), ("gate", View), ("weight", C.c_void_p),
                ("out", C.c_void_p), ("out_dtype", C.c_int32),
                ("out_sb", C.c_int64), ("out_st", C.c_int64), ("out_sh", C.c_int64)]


class PrologueArgs(C.Structure):
    _fields_ = [("B", C.c_int64), ("T", C.c_int64), ("H", C.c_int64), ("M", C.c_int64), ("K", C.c_int64),
                ("V", C.c_int64), ("C", C.c_int32), ("a_k", C.c_int32), ("b_k", C.c_int32), ("a_v", C.c_int32),
                ("b_v", C.c_int32), ("conv_k", C.c_int32), ("qkv", View), ("conv_w", C.c_void_p),
                ("q_a", View), ("q_b", View), ("k_a", View), ("k_b", View), ("v_a", View), ("v_b", View),
                ("mix_qk", C.c_void_p), ("mix_v", C.c_void_p), ("str_qk", C.c_void_p), ("str_v", C.c_void_p),
                ("b_proj", View), ("w_proj", View), ("proj_a", View), ("proj_b", View),
                ("q_out", C.c_void_p), ("k_out", C.c_void_p), ("v_out", C.c_void_p), ("out_dtype", C.c_int32),
                ("out_sb", C.c_int64), ("out_st", C.c_int64), ("out_sh", C.c_int64),
                ("b_out", C.c_void_p), ("w_out", C.c_void_p), ("gate_dtype", C.c_int32),
                ("gate_sb", C.c_int64), ("gate_st", C.c_int64), ("gate_sh", C.c_int64), ("gate_sm", C.c_int64),
                ("wgate_sb", C.c_int64), ("wgate_st", C.c_int64), ("wgate_sh", C.c_int64), ("wgate_sm", C.c_int64)]


class Kmd2PrologueArgs(C.Structure):
    _fields_ = [("B", C.c_int64), ("T", C.c_int64), ("H", C.c_int64), ("dk", C.c_int64), ("dv", C.c_int64),
                ("r_out", C.c_int32), ("conv_k", C.c_int32), ("mixed", View), ("conv_w", C.c_void_p),
                ("b", View), ("a", View), ("theta", View),
                ("dt_bias", C.c_void_p), ("A_log", C.c_void_p), ("decay_chan", C.c_void_p), ("bw_off", C.c_void_p),
                ("q_slot_scale", C.c_void_p),
                ("q_out", C.c_void_p), ("k_out", C.c_void_p), ("v_out", C.c_void_p), ("g_out", C.c_void_p),
                ("beta_e_out", C.c_void_p), ("beta_w_out", C.c_void_p), ("theta_ws", C.c_void_p)]


_lib = None


def load(path: Path = LIB_PATH):
    """Load ``libgdnx.so`` (once) and declare the exported signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not Path(path).exists():
        raise ImportError(f"gdnx_b200: {path} is missing -- run `python -m gdnx_b200.build` "
                          "(the CUDA library is required; there is no CPU fallback)")
    lib = C.CDLL(str(path))
    lib.gdnx_scan_fwd.argtypes = [C.POINTER(ScanArgs), C.c_void_p]
    lib.gdnx_scan_fwd.restype = C.c_int
    lib.gdnx_scan_fwd_noalloc.argtypes = [C.POINTER(ScanArgs), C.c_void_p]
    lib.gdnx_scan_fwd_noalloc.restype = C.c_int
    lib.gdnx_scan_noalloc_status.argtypes = [C.POINTER(C.c_int32), C.c_void_p]
    lib.gdnx_scan_noalloc_status.restype = C.c_int
    lib.gdnx_scan_workspace_bytes.argtypes = [C.POINTER(ScanArgs)]
    lib.gdnx_scan_workspace_bytes.restype = C.c_size_t
    lib.gdnx_kr_scan_fwd.argtypes = [C.POINTER(KrScanArgs), C.c_void_p]
    lib.gdnx_kr_scan_fwd.restype = C.c_int
    lib.gdnx_compact.argtypes = [C.POINTER(CompactArgs), C.c_void_p]
    lib.gdnx_compact.restype = C.c_int
    lib.gdnx_decode_step.argtypes = [C.POINTER(DecodeArgs), C.c_void_p]
    lib.gdnx_decode_step.restype = C.c_int
    lib.gdnx_epilogue.argtypes = [C.POINTER(EpilogueArgs), C.c_void_p]
    lib.gdnx_epilogue.restype = C.c_int
    lib.gdnx_gdn3_prologue.argtypes = [C.POINTER(PrologueArgs), C.c_void_p]
    lib.gdnx_gdn3_prologue.restype = C.c_int
    lib.gdnx_kmd2_prologue.argtypes = [C.POINTER(Kmd2PrologueArgs), C.c_void_p]
    lib.gdnx_kmd2_prologue.restype = C.c_int
    lib.gdnx_scan_bwd.argtypes = [C.POINTER(ScanBwdArgs), C.c_void_p]
    lib.gdnx_scan_bwd.restype = C.c_int
    lib.gdnx_epilogue_scatter.argtypes = [C.POINTER(EpilogueArgs), C.POINTER(C.c_void_p), C.c_int32, C.c_void_p]
    lib.gdnx_epilogue_scatter.restype = C.c_int
    lib.gdnx_device_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)]
    lib.gdnx_device_alloc.restype = C.c_int
    lib.gdnx_device_free.argtypes = [C.c_void_p]
    lib.gdnx_device_free.restype = C.c_int
    lib.gdnx_ipc_handle.argtypes = [C.c_void_p, C.c_void_p]
    lib.gdnx_ipc_handle.restype = C.c_int
    lib.gdnx_ipc_open.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
    lib.gdnx_ipc_open.restype = C.c_int
    lib.gdnx_ipc_close.argtypes = [C.c_void_p]
    lib.gdnx_ipc_close.restype = C.c_int
    lib.gdnx_scan_bwd_workspace_bytes.argtypes = [C.POINTER(ScanBwdArgs)]
    lib.gdnx_scan_bwd_workspace_bytes.restype = C.c_size_t
    lib.gdnx_status_string.argtypes = [C.c_int]
    lib.gdnx_status_string.restype = C.c_char_p
    lib.gdnx_version.argtypes = []
    lib.gdnx_version.restype = C.c_char_p
    _lib = lib
    return lib


class GdnxError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = load().gdnx_status_string(status).decode()
        super().__init__(f"{what}: {msg}")


def check(status: int, what: str):
    if status != GDNX_OK:
        raise GdnxError(status, what)
