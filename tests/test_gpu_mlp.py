"""Standalone FullyFusedMLP inference (BASELINE configs[3] shape: widths
16-128, depths 2/4/8, 16 outputs, fp16 inputs ~ N(0,1)) against the oracle:
tight (2e-3) against the fp16-operand emulation, 1e-2 against fp32 math."""
import numpy as np
import pytest

import oracle as o

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("W,H", [(16, 2), (32, 4), (64, 8), (128, 2), (128, 8)])
def test_mlp_forward_matches_oracle(W, H):
    import torch
    import tmnn_b200 as t
    net = t.FullyFusedMLP(W, W, H, 16, seed=7)
    w = net.weights()
    x = torch.randn(3000, W, device="cuda").half()
    y = net.forward(x).cpu().numpy()
    xf = x.float().cpu().numpy()
    s = o.make_spec(L=W, F=1, W=W, H=H, O=16)
    ref32 = o.mlp_forward(s, w, xf)
    s.fp16_operands = 1
    ref16 = o.mlp_forward(s, w, xf)
    scale = np.abs(ref32).max()
    assert np.abs(y - ref16).max() <= 2e-3 * scale
    assert np.abs(y - ref32).max() <= 1e-2 * scale
    net.close()


def test_mlp_rejects_bad_shapes():
    import tmnn_b200 as t
    with pytest.raises(ValueError):
        t.FullyFusedMLP(24, 64, 2, 16)
    with pytest.raises(ValueError):
        t.FullyFusedMLP(64, 48, 2, 16)
