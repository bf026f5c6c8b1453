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
