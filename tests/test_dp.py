"""Data parallelism.

CPU (gloo, world size 2): the design of the data-parallel step -- every rank
runs forward/backward on its shard with dL/dy scaled by the GLOBAL batch,
the gradients (int32 fixed point, so the sum is exact) and the touched maps
(max = OR) are all-reduced, and every rank applies the same Adam -- checked
with the CPU oracle: the two ranks end bit-identical to one process that
trains on the concatenated batch.

GPU (2 devices): the library's own NCCL path, tmnn_cuda_dp_init + training
steps on two GPUs, against one GPU on the concatenated batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


KW = dict(L=4, F=2, log2T=10, W=16, H=1, O=1, loss=0)
# the tensor-core family needs levels x features to be a multiple of 16
KW_FUSED = dict(L=8, F=2, log2T=10, W=64, H=1, O=1, loss=0)


def _data(steps=3, n=512):
    rng = np.random.default_rng(21)
    out = []
    for _ in range(steps):
        pos = rng.uniform(-1, 1, (2 * n, 3)).astype(np.float32)
        tgt = (np.linalg.norm(pos, axis=1, keepdims=True) - 0.5).astype(np.float32)
        out.append((pos, tgt))
    return out


def _gloo_rank(rank, world, port, q, steps):
    import sys
    for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
        sys.path.insert(0, p)
    import oracle as o
    from _util import oracle_spec
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    s = oracle_spec(**KW)
    hw, mw = o.init_weights(s, seed=5)
    w = np.concatenate([hw, mw])
    m, v = np.zeros_like(w), np.zeros_like(w)
    for step, (pos, tgt) in enumerate(_data(steps)):
        n = pos.shape[0] // world
        sl = slice(rank * n, (rank + 1) * n)
        g = o.zero_grads(s)
        o.fwd_bwd(s, w[:hw.size].copy(), w[hw.size:].copy(), pos[sl], tgt[sl],
                  inv_count=pos.shape[0], grads=g)
        for key, op in (("hash_fixed", dist.ReduceOp.SUM),
                        ("mlp", dist.ReduceOp.SUM),
                        ("touched", dist.ReduceOp.MAX)):
            t = torch.from_numpy(g[key].astype(np.int32 if key == "touched" else g[key].dtype))
            dist.all_reduce(t, op=op)
            g[key] = t.numpy().astype(g[key].dtype)
        o.adam(s, w, m, v, g, step)
    q.put((rank, w))
    dist.destroy_process_group()


@pytest.mark.parametrize("steps", [1, 3])
def test_dp_design_matches_single_process_gloo(steps):
    """One step: bit-exact (integer gradient sums are order independent).
    Later steps: the MLP's float gradient sums differ in order between the
    shard sums and one sum, so the comparison is to fp32 round-off."""
    import oracle as o
    from _util import oracle_spec
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q, steps)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    s = oracle_spec(**KW)
    hw, mw = o.init_weights(s, seed=5)
    w = np.concatenate([hw, mw])
    m, v = np.zeros_like(w), np.zeros_like(w)
    for step, (pos, tgt) in enumerate(_data(steps)):
        g = o.zero_grads(s)
        o.fwd_bwd(s, w[:hw.size].copy(), w[hw.size:].copy(), pos, tgt, grads=g)
        o.adam(s, w, m, v, g, step)
    assert np.array_equal(res[0], res[1])            # replicas agree
    if steps == 1:
        assert np.array_equal(res[0][:hw.size], w[:hw.size])   # exact hash part
    assert np.allclose(res[0][:hw.size], w[:hw.size], rtol=0, atol=1e-6)
    assert np.allclose(res[0][hw.size:], w[hw.size:], rtol=1e-4, atol=1e-6)


def _gpu_rank(rank, world, port, q, family, grad, extra=None):
    import sys
    for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tiny-metal-nn_b200"),
              os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    # the test tables are small (one bucket by default): split them in four
    # so the Tiled runs take the bucketed, pipelined exchange
    os.environ["TMNN_DP_BUCKETS"] = "4"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import tmnn_b200 as t
    from _util import cuda_trainer
    kw = KW_FUSED if family != "SafeDebug" else KW
    tr = cuda_trainer(**kw, family=family, grad=grad, device=rank, cfg_extra=extra)
    uid = [t.dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    tr.dp_init(uid[0], rank, world)
    init = tr.weights()
    losses = []
    for pos, tgt in _data():
        n = pos.shape[0] // world
        losses.append(tr.training_step(np.ascontiguousarray(pos[rank * n:(rank + 1) * n]),
                                       np.ascontiguousarray(tgt[rank * n:(rank + 1) * n])))
    tr.dp_sync_state()  # collective; needed when the optimizer is sharded
    q.put((rank, tr.weights(), losses, init))
    tr.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("family,grad,sharded", [
    ("SafeDebug", "Fixed16", False), ("FullyFused", "F32", False),
    ("Tiled", "F32", False), ("Tiled", "Fixed16", False),
    ("Tiled", "F32", True), ("FullyFused", "Fixed16", True)])
def test_dp_nccl_two_gpus_match_one(family, grad, sharded):
    """N ranks (4 when the box has them: the sharded optimizer; else 2: the
    allreduce) on slices of each batch against one process on the whole
    batch.  The Tiled family exchanges its gradients bucket by bucket behind
    the level-major scatter.  Float gradients sum in a different order, and
    Adam moves a slot by about lr whatever its gradient's size, so the float
    runs compare weight changes by direction (cosine); fixed-point runs
    compare values.  `sharded` forces the sharded optimizer from 2 ranks on
    (dp_replicated_optimizer = -1)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 4 if torch.cuda.device_count() >= 4 else 2  # 4: sharded optimizer
    from _util import cuda_trainer
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    extra = {"dp_replicated_optimizer": -1} if sharded else None
    procs = [ctx.Process(target=_gpu_rank, args=(r, world, port, q, family, grad, extra))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, wts, losses, init = q.get(timeout=120)
        res[r] = (wts, losses, init)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = cuda_trainer(**(KW_FUSED if family != "SafeDebug" else KW),
                       family=family, grad=grad)
    ref_losses = [ref.training_step(p, t) for p, t in _data()]
    (h0, m0), l0, _ = res[0]
    (h1, m1), _, _ = res[1]
    hr, mr = ref.weights()
    assert np.array_equal(h0, h1) and np.array_equal(m0, m1)
    assert np.allclose(l0, ref_losses, rtol=1e-3)
    if grad == "Fixed16":
        assert np.allclose(h0, hr, rtol=0, atol=1e-5)
        assert np.allclose(m0, mr, rtol=1e-3, atol=1e-5)
    else:
        hi, mi = res[0][2]
        def cos(a, b):
            a, b = a.astype(np.float64), b.astype(np.float64)
            return a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300)
        assert cos(h0 - hi, hr - hi) >= 0.999
        assert cos(m0 - mi, mr - mi) >= 0.999
    ref.close()


def _peer_rank(rank, world, port, q, grad):
    import sys
    for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tiny-metal-nn_b200"),
              os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["TMNN_DP_BUCKETS"] = "4"
    os.environ["TMNN_DP_P2P"] = "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import tmnn_b200 as t
    from _util import cuda_trainer
    tr = cuda_trainer(**KW_FUSED, family="Tiled", grad=grad, table="F16",
                      device=rank, cfg_extra={"dp_replicated_optimizer": -1})
    uid = [t.dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    tr.dp_init(uid[0], rank, world)
    init = tr.weights()
    losses = []
    for pos, tgt in _data():
        n = pos.shape[0] // world
        losses.append(tr.training_step(np.ascontiguousarray(pos[rank * n:(rank + 1) * n]),
                                       np.ascontiguousarray(tgt[rank * n:(rank + 1) * n])))
    reason = tr.plan()["reason"]
    tr.dp_sync_state()
    q.put((rank, tr.weights(), losses, init, reason))
    tr.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("grad", ["F32", "F16"])
def test_dp_peer_exchange_matches_one_process(grad):
    """The sharded update over NVLink peer memory (TMNN_DP_P2P=1: per
    bucket, the owner sums the ranks' partial gradients with peer loads,
    runs Adam and stores the fp16 table into every rank) against one process
    on the whole batch, with the tolerances of the NCCL sharded path."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = min(4, torch.cuda.device_count())
    from _util import cuda_trainer
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_peer_rank, args=(r, world, port, q, grad))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, wts, losses, init, reason = q.get(timeout=120)
        res[r] = (wts, losses, init, reason)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][3].startswith("peer-memory"), res[0][3]
    ref = cuda_trainer(**KW_FUSED, family="Tiled", grad=grad, table="F16")
    ref_losses = [ref.training_step(p, t) for p, t in _data()]
    (h0, m0), l0, (hi, mi), _ = res[0]
    for r in range(1, world):
        assert np.array_equal(h0, res[r][0][0]) and np.array_equal(m0, res[r][0][1])
    hr, mr = ref.weights()
    assert np.allclose(l0, ref_losses, rtol=1e-3 if grad == "F32" else 2e-3)

    def cos(a, b):
        a, b = a.astype(np.float64), b.astype(np.float64)
        return a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300)
    tol = 0.999 if grad == "F32" else 0.99
    assert cos(h0 - hi, hr - hi) >= tol
    assert cos(m0 - mi, mr - mi) >= tol
    ref.close()


def _retry_rank(rank, world, port, q):
    import sys
    for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tiny-metal-nn_b200"),
              os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import tmnn_b200 as t
    tr = _retry_trainer(rank)
    uid = [t.dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    tr.dp_init(uid[0], rank, world)
    init = tr.weights()
    pos, tgt = _data(steps=1)[0]
    n = pos.shape[0] // world
    loss = tr.training_step(np.ascontiguousarray(pos[rank * n:(rank + 1) * n]),
                            np.ascontiguousarray(tgt[rank * n:(rank + 1) * n]))
    action = tr.last_numerics()["recovery_action"]
    tr.dp_sync_state()
    q.put((rank, tr.weights(), loss, action, init))
    tr.close()
    dist.destroy_process_group()


def _retry_trainer(device):
    """FullyFused trainer whose table holds values above the fp16 range: the
    tensor-core step overflows, the fp32 SafeDebug retry does not."""
    from _util import cuda_trainer
    from tmnn_b200 import _abi
    tr = cuda_trainer(**KW_FUSED, family="FullyFused", grad="F32", device=device,
                      cfg_extra={"dp_replicated_optimizer": -1,
                                 "bad_step_recovery":
                                     _abi.BAD_STEP["FallbackAndRetryWithSafeFamily"]})
    hw, mw = tr.weights()
    tr.set_initial_weights(np.full_like(hw, 6.0e4), np.abs(mw) + 0.05)
    return tr


@pytest.mark.gpu
def test_dp_sharded_safe_family_retry_matches_one_process():
    """FallbackAndRetryWithSafeFamily under the sharded optimizer: the fp32
    master outside a rank's shard is out of date after a sharded step, and
    the SafeDebug retry reads it, so the runtime gathers it first.  Two ranks
    (sharding forced) against one process on the whole batch."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_retry_rank, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, wts, loss, action, init = q.get(timeout=120)
        res[r] = (wts, loss, action, init)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = _retry_trainer(0)
    pos, tgt = _data(steps=1)[0]
    lr = ref.training_step(pos, tgt)
    assert ref.last_numerics()["recovery_action"] == "RetriedWithSafeFamily"
    hr, mr = ref.weights()
    ref.close()
    (h0, m0), l0, a0, (hi, mi) = res[0]
    (h1, m1), _, a1, _ = res[1]
    assert a0 == a1 == "RetriedWithSafeFamily"
    assert np.array_equal(h0, h1) and np.array_equal(m0, m1)
    assert np.isfinite(h0).all() and np.isfinite(m0).all()
    assert abs(l0 - lr) <= 1e-3 * abs(lr)

    def cos(a, b):
        a, b = a.astype(np.float64), b.astype(np.float64)
        return a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300)
    assert cos(h0 - hi, hr - hi) >= 0.999
    assert cos(m0 - mi, mr - mi) >= 0.999


NERF_KW = dict(n_levels=8, n_features_per_level=2, log2_hashmap_size=14,
               base_resolution=16.0, per_level_scale=1.382)


def _nerf_rank(rank, world, port, q):
    import sys
    for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tiny-metal-nn_b200"),
              os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle as o
    import tmnn_b200 as t
    nf = t.NerfField(family="FullyFused", device=rank, **NERF_KW)
    uid = [t.dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    nf.dp_init(uid[0], rank, world)
    c0 = nf.color_weights()
    losses = []
    for s in range(3):
        pos, d, rgb, sig = o.nerf_batch(4096, 40 + s)
        n = pos.shape[0] // world
        sl = slice(rank * n, (rank + 1) * n)
        losses.append(nf.training_step(*(np.ascontiguousarray(a[sl])
                                          for a in (pos, d, rgb, sig))))
    nf.density.dp_sync_state()
    q.put((rank, losses, c0, nf.color_weights(), nf.density.weights()))
    nf.close()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_dp_nerf_two_gpus_match_one():
    """The NeRF field trained data parallel (each rank a slice of every
    batch) against one process on the whole batch: losses within 1e-3,
    colour and density weight changes aligned."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import oracle as o
    import tmnn_b200 as t
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nerf_rank, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, losses, c0, c1, dw = q.get(timeout=120)
        res[r] = (losses, c0, c1, dw)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = t.NerfField(family="FullyFused", **NERF_KW)
    h0, m0 = ref.density.weights()
    lr = [ref.training_step(*o.nerf_batch(4096, 40 + s)) for s in range(3)]
    cr = ref.color_weights()
    hr, mr = ref.density.weights()
    ref.close()
    (l0, c0, c1, (h1, m1)), (_, _, c1b, (h1b, m1b)) = res[0], res[1]
    assert np.array_equal(c1, c1b) and np.array_equal(h1, h1b)
    assert np.allclose(l0, lr, rtol=1e-3)

    def cos(a, b):
        a, b = a.astype(np.float64), b.astype(np.float64)
        return a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300)
    assert cos(c1 - c0, cr - c0) >= 0.999
    assert cos(h1 - h0, hr - h0) >= 0.999
    assert cos(m1 - m0, mr - m0) >= 0.999
