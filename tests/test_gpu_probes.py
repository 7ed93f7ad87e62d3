"""In-kernel training probes (enable_probes; ProbeResult of
include/tiny-metal-nn/common.h:78-94, emitted by
mlp_kernel_emitter.cpp:903-945, :2879-3155, aggregated by
training_step_execution.cpp:1326-1369) against the same statistics computed
in numpy from the oracle's encoding and the MLP weights.

With probes on, training runs the fp32 reference-order kernels (the
reference switches to its scalar kernel).  Through backward_accumulate the
output gradient is given, so every probed quantity has a closed form:
act_max[l] = max |h_l|, grad_l2[l] = sum |dL/d pre_l|^2 over the batch,
output_abs_max = max |y|, output_min = min(0, min y) for one output (0 for
several: the reference never writes it there), hash_grad_l2 = 0.
"""
import numpy as np
import pytest

import oracle as o
from _util import cuda_trainer, oracle_spec

pytestmark = pytest.mark.gpu

CASES = [dict(L=4, F=2, log2T=12, d=3, W=32, H=2, O=1, loss=0),
         dict(L=6, F=2, log2T=13, d=3, W=64, H=3, O=3, loss=0)]


def mlp_stats(kw, hw, mw, pos, dout):
    s = oracle_spec(**kw, grad="F32")
    x = o.encode(s, hw, pos).astype(np.float64)
    W, H, O, In = kw["W"], kw["H"], kw["O"], kw["L"] * kw["F"]
    off, Ws, bs = 0, [], []
    for k in range(H):
        fin = In if k == 0 else W
        Ws.append(mw[off:off + fin * W].reshape(fin, W).astype(np.float64))
        off += fin * W
        bs.append(mw[off:off + W].astype(np.float64))
        off += W
    Wo = mw[off:off + W * O].reshape(W, O).astype(np.float64)
    bo = mw[off + W * O:off + W * O + O].astype(np.float64)
    hs, h = [], x
    for k in range(H):
        h = np.maximum(h @ Ws[k] + bs[k], 0.0)
        hs.append(h)
    y = h @ Wo + bo
    dp = [None] * H
    g = (dout.astype(np.float64) @ Wo.T) * (hs[H - 1] > 0)
    dp[H - 1] = g
    for k in range(H - 1, 0, -1):
        g = (g @ Ws[k].T) * (hs[k - 1] > 0)
        dp[k - 1] = g
    return {"act_max": [float(np.abs(a).max()) for a in hs],
            "grad_l2": [float((a * a).sum()) for a in dp],
            "output_abs_max": float(np.abs(y).max()),
            "output_min": float(min(0.0, y.min())) if O == 1 else 0.0}


@pytest.mark.parametrize("kw", CASES)
def test_probes_match_closed_form(kw):
    tr = cuda_trainer(**kw, family="Auto", grad="F32", batch=4096,
                      cfg_extra={"enable_probes": 1})
    assert tr.plan()["family"] == "SafeDebug"
    assert tr.last_probe() is None          # no pass yet
    rng = np.random.default_rng(3)
    pos = rng.uniform(-1, 1, (4096, 3)).astype(np.float32)
    dout = rng.normal(size=(4096, kw["O"])).astype(np.float32) / 4096
    hw, mw = tr.weights()
    tr.zero_gradients()
    tr.backward_accumulate(pos, dout)
    p = tr.last_probe()
    want = mlp_stats(kw, hw, mw, pos, dout)
    assert p["num_hidden_layers"] == kw["H"]
    assert not p["has_nan_forward"] and not p["has_nan_backward"]
    assert p["hash_grad_l2"] == 0.0
    np.testing.assert_allclose(p["act_max"], want["act_max"], rtol=1e-4)
    np.testing.assert_allclose(p["grad_l2"], want["grad_l2"], rtol=1e-3)
    assert abs(p["output_abs_max"] - want["output_abs_max"]) <= 1e-4 * want["output_abs_max"]
    assert abs(p["output_min"] - want["output_min"]) <= 1e-4 * max(abs(want["output_min"]), 1e-6)
    # a training step reports its own pass
    tgt = rng.normal(size=(4096, kw["O"])).astype(np.float32)
    tr.training_step(pos, tgt)
    p2 = tr.last_probe()
    assert p2 is not None and min(p2["act_max"]) > 0 and min(p2["grad_l2"]) > 0
    tr.close()


def test_probes_off_returns_none():
    tr = cuda_trainer(**CASES[0], family="Auto", grad="F32", batch=1024)
    pos = np.random.default_rng(0).uniform(-1, 1, (1024, 3)).astype(np.float32)
    tr.training_step(pos, np.zeros((1024, 1), np.float32))
    assert tr.last_probe() is None
    tr.close()
