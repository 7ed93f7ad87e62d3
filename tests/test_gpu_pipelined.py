"""The pipelined training-step API (enqueue / finalize over two step lanes)
against the synchronous training_step: same batches, same seeds, same
kernels, so the losses agree to float-reduction order and the weights move
the same way; and the API's refusals (nothing pending, a third pending step,
a synchronous step while steps are pending, recovery modes)."""
import numpy as np
import pytest

from _util import batch, cuda_trainer

pytestmark = pytest.mark.gpu

KW = dict(L=16, F=2, log2T=14, d=3, W=64, H=1, O=1, loss=1)


def cos(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("family", ["FullyFused", "Tiled"])
def test_enqueue_finalize_matches_training_step(family):
    a = cuda_trainer(**KW, family=family, grad="F32", table="F16")
    b = cuda_trainer(**KW, family=family, grad="F32", table="F16")
    h0, m0 = a.weights()
    batches = [batch(8192, 3, 1, seed=s) for s in range(6)]
    la = [a.training_step(p, t) for p, t in batches]
    lb = []
    b.training_step_enqueue(*batches[0])
    for p, t in batches[1:]:
        b.training_step_enqueue(p, t)
        lb.append(b.training_step_finalize())
    lb.append(b.training_step_finalize())
    assert np.allclose(la, lb, rtol=1e-4)
    assert b.step() == a.step() == 6
    ha, ma = a.weights()
    hb, mb = b.weights()
    assert cos(ha - h0, hb - h0) >= 0.999
    assert cos(ma - m0, mb - m0) >= 0.999
    a.close()
    b.close()


def test_enqueue_device_inputs_and_refusals():
    import torch
    import tmnn_b200 as t
    tr = cuda_trainer(**KW, family="FullyFused", grad="F32")
    p, g = batch(4096, 3, 1, seed=1)
    with pytest.raises(ValueError):
        tr.training_step_finalize()                      # nothing pending
    tr.training_step_enqueue(torch.from_numpy(p).cuda(), torch.from_numpy(g).cuda())
    tr.training_step_enqueue(p, g)
    with pytest.raises(ValueError):
        tr.training_step_enqueue(p, g)                   # two already pending
    with pytest.raises(ValueError):
        tr.training_step(p, g)                           # steps pending
    l1 = tr.training_step_finalize()
    l2 = tr.training_step_finalize()
    assert np.isfinite(l1) and np.isfinite(l2)
    tr.training_step(p, g)                               # usable again
    tr.close()
    from tmnn_b200 import _abi
    rec = cuda_trainer(**KW, family="FullyFused", grad="F32",
                       cfg_extra={"bad_step_recovery": _abi.BAD_STEP["Skip"]})
    with pytest.raises(ValueError):
        rec.training_step_enqueue(p, g)
    rec.close()
