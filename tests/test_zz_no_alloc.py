"""The no-allocation forward/backward entry point, through the C ABI.

tmnn_cuda_forward_backward_noalloc serves callers that must not allocate
device memory when they run a step (a framework that owns the memory pool, a
fixed serving footprint, a real-time loop that cannot stall in the
allocator).  Its scratch lives in a fixed array inside the library.  These
tests check it against the ordinary tmnn_cuda_forward_backward on the same
device-resident batch, twice in a row (the array keeps the previous call's
contents, so the second call shows nothing stale leaks through), and that an
oversized batch is refused.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from _util import cuda_trainer

pytestmark = pytest.mark.gpu


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _ordinary(tr, pos, tgt):
    from tmnn_b200 import _abi
    out = C.c_double()
    tr.zero_gradients()
    st = _abi.lib.tmnn_cuda_forward_backward(
        tr._handle(), C.c_void_p(pos.data_ptr()), C.c_void_p(tgt.data_ptr()),
        pos.shape[0], _abi.PTR_DEVICE, C.byref(out))
    assert st == 0, _abi.last_error()
    return out.value, tr.read_buffer(3), tr.read_buffer(4)


def _noalloc(tr, pos, tgt):
    from tmnn_b200 import _abi
    out = C.c_double()
    tr.zero_gradients()
    st = _abi.lib.tmnn_cuda_forward_backward_noalloc(
        tr._handle(), C.c_void_p(pos.data_ptr()), C.c_void_p(tgt.data_ptr()),
        pos.shape[0], C.byref(out))
    assert st == 0, _abi.last_error()
    return out.value, tr.read_buffer(3), tr.read_buffer(4)


@pytest.mark.parametrize("family", ["SafeDebug", "FullyFused"])
def test_noalloc_matches_ordinary_twice(family):
    kw = dict(L=8, F=2, log2T=12, W=64, H=2, O=2, loss=0)
    tr = cuda_trainer(**kw, family=family, grad="Fixed16", morton=True)
    rng = np.random.default_rng(7)
    batches = [(_dev(rng.uniform(-1, 1, (n, 3)).astype(np.float32)),
                _dev(rng.normal(size=(n, 2)).astype(np.float32)))
               for n in (5000, 3001)]
    for pos, tgt in batches:  # two calls in a row, different sizes
        la, ha, ma = _ordinary(tr, pos, tgt)
        lb, hb, mb = _noalloc(tr, pos, tgt)
        # same sort, same kernels: hash gradients (integer sums) agree exactly
        # and MLP gradients (float atomics in any order) to fp32 round-off
        assert np.array_equal(ha, hb)
        assert np.abs(ma - mb).max() <= 1e-5 * max(np.abs(ma).max(), 1e-30)
        assert abs(la - lb) <= 1e-6 * abs(la)
    tr.close()


def test_noalloc_rejects_oversized_batch():
    from tmnn_b200 import _abi
    tr = cuda_trainer(L=4, F=2, log2T=10, W=16, H=1, O=1)
    pos = _dev(np.zeros((65537, 3), np.float32))
    tgt = _dev(np.zeros((65537, 1), np.float32))
    st = _abi.lib.tmnn_cuda_forward_backward_noalloc(
        tr._handle(), C.c_void_p(pos.data_ptr()), C.c_void_p(tgt.data_ptr()),
        65537, None)
    assert st == _abi.ERR_INVALID_ARGUMENT
    assert "65536" in _abi.last_error()
    tr.close()
