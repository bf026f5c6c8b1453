"""Host-side prologue constants match the reference's lane-RoPE branches."""
import pytest
import torch

from gdnx_b200.prologue import lane_rope
from oracle.prologue import lane_rope_params


@pytest.mark.parametrize("K,rf", [(128, 0.25), (128, 0.5), (64, 0.25), (64, 0.5)])
def test_lane_rope_constants(K, rf):
    lr = lane_rope(4, K, K, rf)
    for m in range(4):
        d, inv, scale, ident = lane_rope_params(m, K, K, rf)
        if ident or d < 1:
            assert lr.pairs[m] == 0
            continue
        assert lr.pairs[m] == d and lr.scale[m] == scale
        ar = torch.arange(d, dtype=torch.float32)
        mine = 1.0 / (10000.0 ** (ar / lr.den[m]))
        assert torch.equal(mine, inv)
