"""Analytic input-gradient evaluation (Trainer::evaluate_with_gradient,
trainer.h:378-386; EvalGradient kernel mlp_kernel_emitter.cpp:1716-2090)
through the C ABI, against the CPU oracle and the reference's own kernel
output (tests/golden).  The CUDA kernel evaluates in fp32 in the reference's
operation order (no fused multiply-add), so against the oracle with the same
resolution table it is bit-exact; against the reference golden, whose
resolutions come from BASE*pow(SCALE, l), it agrees to fp32 round-off."""
import os

import numpy as np
import pytest

import oracle as o
from _util import batch, cuda_trainer, oracle_spec, spec_kwargs_from_tuple
from golden.make_golden import case_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

CASES = [
    dict(L=8, F=2, log2T=14, d=3, W=64, H=1),
    dict(L=8, F=1, log2T=12, d=3, W=32, H=2),
    dict(L=4, F=4, log2T=12, d=3, W=16, H=3),
    dict(L=8, F=2, log2T=14, d=4, W=64, H=2, base=8.0, scale=1.5),
    dict(L=4, F=2, log2T=10, d=3, W=256, H=2),  # width above the register path
]


def _weights(tr, rng):
    table = rng.uniform(-0.5, 0.5, tr.hash_count).astype(np.float32)
    mlp = rng.uniform(-0.3, 0.3, tr.mlp_count).astype(np.float32)
    tr.set_initial_weights(table, mlp)
    return table, mlp


@pytest.mark.parametrize("family", ["SafeDebug", "FullyFused"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "d{d}F{F}W{W}H{H}".format(**c))
def test_eval_gradient_bit_exact_vs_oracle(case, family):
    if family == "FullyFused" and case["W"] not in (64, 128):
        pytest.skip("the FullyFused training kernel is built for W in {64, 128}")
    tr = cuda_trainer(family=family, **case)
    rng = np.random.default_rng(3)
    table, mlp = _weights(tr, rng)
    pos, _ = batch(3001, case["d"], 1, seed=5,
                   lo=0.0 if case["d"] == 4 else -1.0)
    val, grad = tr.evaluate_with_gradient(pos)
    ov, og = o.eval_gradient(oracle_spec(**case), table, mlp, pos)
    assert val.shape == (3001, 1) and grad.shape == (3001, case["d"])
    assert np.array_equal(val[:, 0], ov)
    assert np.array_equal(grad, og)
    # the value is the field itself: evaluate() within fp32 round-off of the
    # lerp-form interpolation (SafeDebug evaluates in fp32)
    if family == "SafeDebug":
        ev = tr.inference(pos)
        assert np.abs(ev[:, 0] - ov).max() <= 1e-5 * max(1.0, np.abs(ov).max())
    tr.close()


@pytest.mark.parametrize("tag", ["ka", "sdf", "f1", "f4", "h3", "d4o1"])
def test_eval_gradient_matches_reference_golden(tag):
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    kw = spec_kwargs_from_tuple(sp)
    tr = cuda_trainer(**kw)
    table, mlp, pos, _, _ = case_inputs(tag, sp)
    tr.set_initial_weights(table, mlp)
    val, grad = tr.evaluate_with_gradient(pos)
    ref = g["evalgrad"]
    vs = max(1.0, np.abs(ref[:, 0]).max())
    gs = max(1.0, np.abs(ref[:, 1:4]).max())
    assert np.abs(val[:, 0] - ref[:, 0]).max() <= 1e-5 * vs
    # points on a cell face under one of the two resolution rules may land in
    # the neighbouring cell; allow a handful, bound the rest tightly
    err = np.abs(grad[:, :3] - ref[:, 1:4]).max(axis=1)
    assert (err > 1e-4 * gs).sum() <= 2
    tr.close()


def test_eval_gradient_device_tensors_and_edges():
    import torch
    kw = dict(L=8, F=2, log2T=12, d=3, W=32, H=1)
    tr = cuda_trainer(**kw)
    rng = np.random.default_rng(9)
    table, mlp = _weights(tr, rng)
    pos, _ = batch(1000, 3, 1, seed=2)
    hv, hg = tr.evaluate_with_gradient(pos)
    dv, dg = tr.evaluate_with_gradient(torch.from_numpy(pos).cuda())
    assert np.array_equal(dv.cpu().numpy(), hv)
    assert np.array_equal(dg.cpu().numpy(), hg)
    v0, g0 = tr.evaluate_with_gradient(np.zeros((0, 3), np.float32))
    assert v0.shape == (0, 1) and g0.shape == (0, 3)
    tr.close()
    multi = cuda_trainer(L=4, F=2, log2T=10, d=3, W=16, H=1, O=3)
    with pytest.raises(ValueError, match="exactly one output"):
        multi.evaluate_with_gradient(pos)
    multi.close()


def test_eval_gradient_full_size_sdf_config():
    """BASELINE's 3D SDF shape (L=16, T=2^19, W=64, H=1) at 2^18 points after
    a few training steps: bit-exact against the oracle."""
    kw = dict(L=16, F=2, log2T=19, d=3, W=64, H=1, O=1, loss=1, base=16.0,
              scale=1.447)
    tr = cuda_trainer(family="FullyFused", grad="F32", **kw)
    pos, tgt = batch(1 << 18, 3, 1, seed=4)
    for _ in range(5):
        tr.training_step(pos, tgt)
    table, mlp = tr.weights()
    val, grad = tr.evaluate_with_gradient(pos)
    ov, og = o.eval_gradient(oracle_spec(**kw), table, mlp, pos)
    assert np.array_equal(val[:, 0], ov)
    assert np.array_equal(grad, og)
    assert np.isfinite(grad).all() and np.abs(grad).max() > 0
    tr.close()
