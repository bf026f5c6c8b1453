"""CPU checks of the C-ABI boundary: the library loads, exports every symbol
``include/gdnx.h`` declares, and the ctypes mirror matches the C layout."""
import re
import subprocess
from pathlib import Path

import ctypes as C
import pytest

from gdnx_b200 import _lib as L

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "gdnx.h"


def declared_symbols():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"GDNX_API\s+[\w\s\*]+?\b(gdnx_\w+)\s*\(", txt)))


def test_header_declares_the_mirrored_symbols():
    assert declared_symbols() == sorted(L.EXPORTED)


def test_library_loads_and_exports_every_declared_symbol():
    lib = L.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(L.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (gdnx_\w+)", out))
    for s in declared_symbols():
        assert s in exported, s
        assert getattr(lib, s) is not None
    assert lib.gdnx_version().decode().startswith("gdnx-b200")
    assert "EINVAL" in lib.gdnx_status_string(L.GDNX_EINVAL).decode()


STRUCTS = {"gdnx_view": L.View, "gdnx_rope": L.Rope, "gdnx_scan_args": L.ScanArgs,
           "gdnx_kr_scan_args": L.KrScanArgs, "gdnx_compact_args": L.CompactArgs,
           "gdnx_decode_args": L.DecodeArgs, "gdnx_epilogue_args": L.EpilogueArgs,
           "gdnx_prologue_args": L.PrologueArgs, "gdnx_scan_bwd_args": L.ScanBwdArgs,
           "gdnx_kmd2_prologue_args": L.Kmd2PrologueArgs}


def test_ctypes_layout_matches_c(tmp_path):
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "gdnx.h"', 'int main(void){']
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines())
    for cname, py in STRUCTS.items():
        assert int(got[cname]) == C.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, f"{cname}.{f}"


def test_cpu_tensors_are_rejected_not_computed():
    import torch
    from gdnx_b200 import ops
    x = torch.zeros(1, 4, 1, 8)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gdn3_scan(x, x, x, torch.ones(1, 4, 1, 1), torch.ones(1, 4, 1, 1), torch.ones(1, 4, 1, 1))
