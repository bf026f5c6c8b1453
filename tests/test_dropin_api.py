"""The drop-in modules keep the reference's call signatures (checked without a GPU)."""
import ast
import inspect
from pathlib import Path

from gdnx_b200 import gdn3_upgrade, kmd2_fast_scan

WRAPPER_ARGUMENTS = ("q", "k", "v", "g", "beta_e", "beta_w", "out_mix")


def test_kmd2_fast_scan_signatures():
    tree = ast.parse(Path(kmd2_fast_scan.__file__).read_text())
    fns = {n.name: n for n in tree.body if isinstance(n, ast.FunctionDef)}
    for name in ("scan", "scan_with_update_norm", "_scan_impl", "_scan_with_update_norm_impl"):
        a = fns[name].args
        assert tuple(x.arg for x in a.args) == WRAPPER_ARGUMENTS
        assert len(a.defaults) == 1 and a.defaults[0].value is None
        assert not a.kwonlyargs and a.vararg is None and a.kwarg is None
    core = fns["_scan_core"].args
    assert tuple(x.arg for x in core.args) == WRAPPER_ARGUMENTS
    assert [x.arg for x in core.kwonlyargs] == ["return_scores"]


def test_gdn3_recurrent_state_signature():
    params = list(inspect.signature(gdn3_upgrade.gdn3_recurrent_state).parameters)
    assert params == ["layer", "q_features", "k_features", "v_features", "b_gates", "w_gates", "decay_factors"]


def test_compaction_sketch_widths():
    """Sketch columns per compact_mode: min(R+4, m, n) for the SVD (gdn3/gdn3_upgrade.py:599),
    R for "sketch" / "sketch_noqr" (:580); unknown modes are rejected."""
    import pytest
    from gdnx_b200 import ops
    assert ops.sketch_width(4, (16, 16, 8, 8), "svd") == 8
    assert ops.sketch_width(4, (2, 2, 2, 2), "svd") == 4
    assert ops.sketch_width(4, (16, 16, 8, 8), "sketch") == 4
    assert ops.sketch_width(4, (16, 16, 8, 8), "sketch_noqr") == 4
    with pytest.raises(ValueError):
        ops.sketch_width(4, (16, 16, 8, 8), "eigh")
