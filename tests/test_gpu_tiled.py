"""Tiled family (level-major encode -> tcgen05 MLP -> level-major scatter)
against the CPU oracle and against the FullyFused family.

The Tiled family computes the same per-point arithmetic as the FullyFused
kernel (same fp32 interpolation order, same fp16 rounding of the features,
same tensor-core MLP, same float/fixed-point scatter of d_feature * weight),
only split into three launches with the hash-grid work mapped level by level.
So:
  * encoded features and fixed-point hash gradients are bit-identical to the
    FullyFused family's (integer sums are order independent);
  * float gradients agree with the fp16-emulating oracle at 2e-3 and with the
    fp32 oracle at the contract's 1e-2, outputs at 1e-2.
"""
import numpy as np
import pytest

import oracle as o
from _util import batch, cuda_trainer, oracle_spec

pytestmark = pytest.mark.gpu

CASES = [
    dict(L=16, F=2, log2T=14, d=3, W=64, H=1, O=1, loss=1),
    dict(L=16, F=2, log2T=12, d=4, W=64, H=2, O=4, loss=0, base=8.0, scale=1.5),
    dict(L=16, F=1, log2T=12, d=3, W=64, H=1, O=1, loss=2, huber=0.1),
    dict(L=4, F=4, log2T=12, d=3, W=64, H=3, O=2, loss=0),
    dict(L=8, F=2, log2T=12, d=3, W=128, H=1, O=16, loss=0),
    dict(L=4, F=4, log2T=12, d=4, W=64, H=2, O=3, loss=3, base=8.0, scale=1.5),
]


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def pair(kw, table="F32", grad="F32", morton=False, seed=0, N=3000):
    """A Tiled and a FullyFused trainer with the same random weights."""
    a = cuda_trainer(**kw, family="Tiled", table=table, grad=grad, morton=morton)
    b = cuda_trainer(**kw, family="FullyFused", table=table, grad=grad, morton=morton)
    assert a.plan()["family"] == "Tiled" and b.plan()["family"] == "FullyFused"
    rng = np.random.default_rng(seed)
    hw = rng.uniform(-0.5, 0.5, a.hash_count).astype(np.float32)
    _, mw = a.weights()
    a.set_initial_weights(hw, mw)
    b.set_initial_weights(hw, mw)
    lo = 0.0 if kw.get("d", 3) == 4 else -1.0
    pos, tgt = batch(N, kw.get("d", 3), kw["O"], seed=seed + 1, lo=lo)
    if kw["loss"] == 3:
        tgt = np.abs(tgt) + 0.1
    return a, b, hw, mw, pos, tgt


def emulated(kw, n, grad="F32"):
    s = oracle_spec(**kw, grad=grad)
    s.fp16_operands = 1
    s.dscale = o.pow2_scale(n)
    return s


@pytest.mark.parametrize("kw", CASES)
def test_tiled_features_and_fixed_point_gradients_equal_fused(kw):
    a, b, hw, mw, pos, tgt = pair(kw, grad="Fixed16")
    la = a.forward_backward(pos, tgt)
    lb = b.forward_backward(pos, tgt)
    assert np.array_equal(a.read_buffer(3), b.read_buffer(3))      # int32
    assert np.array_equal(a.read_buffer(21), b.read_buffer(21))    # touched
    assert rel(a.read_buffer(4), b.read_buffer(4)) <= 1e-5
    assert abs(la - lb) <= 1e-5 * abs(lb)
    # inference: the Tiled family runs the pipelined MLP kernel, which adds
    # the bias inside the MMA; a last-bit difference of a pre-activation can
    # flip the fp16 rounding of a hidden activation (2^-11 relative)
    ya, yb = a.inference(pos), b.inference(pos)
    assert np.abs(ya - yb).max() <= 2e-3 * max(np.abs(yb).max(), 1e-3)
    a.close()
    b.close()


@pytest.mark.parametrize("kw", CASES)
def test_tiled_gradients_match_oracle(kw):
    a, b, hw, mw, pos, tgt = pair(kw)
    b.close()
    lsum = a.forward_backward(pos, tgt)
    le, ge, _ = o.fwd_bwd(emulated(kw, len(pos)), hw, mw, pos, tgt)
    assert abs(lsum - le) <= 1e-3 * abs(le)
    assert rel(a.read_buffer(3), ge["hash_float"]) <= 2e-3
    assert rel(a.read_buffer(4), ge["mlp"]) <= 2e-3
    assert np.array_equal(a.read_buffer(21), ge["touched"])
    out = a.inference(pos)
    ref = o.forward(oracle_spec(**kw), hw, mw, pos)
    assert np.abs(out - ref).max() <= 1e-2 * max(np.abs(ref).max(), 1e-3)
    a.close()


def test_tiled_fp16_table_and_external_gradient():
    kw = CASES[1]
    a, b, hw, mw, pos, _ = pair(kw, table="F16", N=2000)
    b.close()
    hw16 = hw.astype(np.float16).astype(np.float32)
    d_out = (np.random.default_rng(5).normal(size=(2000, kw["O"])) * 1e-3).astype(np.float32)
    a.zero_gradients()
    a.backward_accumulate(pos, d_out)
    _, g, _ = o.fwd_bwd(emulated(kw, 2000), hw16, mw, pos, None, d_out=d_out)
    assert rel(a.read_buffer(3), g["hash_float"]) <= 2e-3
    assert rel(a.read_buffer(4), g["mlp"]) <= 2e-3
    a.close()


@pytest.mark.parametrize("N", [0, 1, 255, 257, 5000])
def test_tiled_ragged_batches(N):
    kw = dict(L=8, F=2, log2T=12, d=3, W=64, H=2, O=2, loss=0)
    a, b, hw, mw, pos, tgt = pair(kw, N=N, morton=True)
    la = a.forward_backward(pos, tgt)
    lb = b.forward_backward(pos, tgt)
    assert abs(la - lb) <= 1e-5 * max(abs(lb), 1e-12)
    if N:
        assert rel(a.read_buffer(3), b.read_buffer(3)) <= 1e-5
    assert a.inference(pos).shape == (N, 2)
    a.close()
    b.close()


def test_auto_selects_tiled_when_tables_take_a_quarter_of_l2():
    big = cuda_trainer(L=16, F=2, log2T=22, d=4, W=64, H=2, O=4, loss=0,
                       base=8.0, scale=1.5, family="Auto", table="F16",
                       grad="F32")
    assert big.plan()["family"] == "Tiled", big.plan()
    big.close()
    mid = cuda_trainer(L=16, F=2, log2T=19, d=3, W=64, H=1, O=1, loss=1,
                       family="Auto", table="F16", grad="F32")
    assert mid.plan()["family"] == "Tiled", mid.plan()
    mid.close()
    small = cuda_trainer(L=16, F=2, log2T=15, d=3, W=64, H=2, O=3, loss=0,
                         scale=1.5, family="Auto", table="F32", grad="F32")
    assert small.plan()["family"] == "FullyFused", small.plan()
    small.close()
