"""Parity of the CUDA path (through the C ABI) with the CPU oracle and with
the reference's own outputs (tests/golden).  Tolerances, per the contract:
hash indices and grid cells bit-exact; fp32 encoding within 1e-5 relative;
MLP outputs and gradients within 1e-2 relative for fp16 tensor-core math
(FullyFused), and at fp32 round-off for the reference-order fp32 kernels
(SafeDebug), where fixed-point hash gradients are compared bit for bit."""
import os

import numpy as np
import pytest

import oracle as o
from _util import batch, cuda_trainer, oracle_spec, spec_kwargs_from_tuple
from golden.make_golden import TAGS, case_inputs

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_known_answer_034():
    """test_default_trainer.cpp:2260-2336 through the C ABI."""
    import tmnn_b200 as t
    cfg = {"encoding": {"n_levels": 2, "n_features_per_level": 2,
                        "log2_hashmap_size": 10, "base_resolution": 4.0,
                        "per_level_scale": 2.0},
           "network": {"n_neurons": 8, "n_hidden_layers": 1}}
    with t.Trainer.from_config(cfg, n_input=3, n_output=1) as tr:
        assert tr.mlp_count == 49
        tr.set_initial_weights(np.full(tr.hash_count, 0.5, np.float32),
                               np.full(tr.mlp_count, 0.1, np.float32))
        out = tr.inference(np.array([[0.5, 0.5, 0.5]], np.float32))
        assert abs(float(out[0, 0]) - 0.34) < 1e-4


@pytest.mark.parametrize("dims", [dict(d=3, F=2), dict(d=3, F=1), dict(d=3, F=4),
                                  dict(d=4, F=2)])
def test_encoding_indices_bit_exact(dims):
    kw = dict(L=8, log2T=12, W=16, H=1, O=1, base=16.0, scale=1.447, **dims)
    tr = cuda_trainer(**kw)
    s = oracle_spec(**kw)
    rng = np.random.default_rng(11)
    table = rng.uniform(-1, 1, tr.hash_count).astype(np.float32)
    tr.set_initial_weights(table, None)
    pos = rng.uniform(-1, 1, (777, kw["d"])).astype(np.float32)
    pos[:5] = [[0.0] * kw["d"], [1.0] * kw["d"], [-1.0] * kw["d"],
               [0.5] * kw["d"], [-0.999999] * kw["d"]]
    feat, idx, cells = tr.debug_encode(pos)
    f2, i2, c2 = o.encode(s, table, pos, with_indices=True)
    assert np.array_equal(idx, i2)
    assert np.array_equal(cells, c2)
    assert np.abs(feat - f2).max() <= 1e-5 * np.abs(f2).max()
    assert np.array_equal(feat, f2)  # same operation order: exact
    tr.close()


@pytest.mark.parametrize("tag", TAGS)
def test_safedebug_gradients_match_reference_golden(tag):
    """CUDA fp32 kernels vs the reference's own scalar train kernel output.
    For tags whose per-level scale is exactly representable in powers
    (2.0, 1.5 at these level counts) the reference's pow() resolutions equal
    the iterative table, so fixed-point hash gradients match bit for bit."""
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    kw = spec_kwargs_from_tuple(sp)
    table, mlp, pos, tgt, d_out = case_inputs(tag, sp)
    tr = cuda_trainer(**kw, morton=False)
    tr.set_initial_weights(table, mlp)
    lsum = tr.forward_backward(pos, tgt)
    gh = tr.read_buffer(3)
    gm = tr.read_buffer(4)
    ref_hash = np.zeros(table.size, np.int32)
    ref_hash[g["train_hash_idx"]] = g["train_hash_val"]
    res_pow = o.level_resolutions(oracle_spec(**kw, res_mode=1))
    res_it = o.level_resolutions(oracle_spec(**kw, res_mode=0))
    if np.array_equal(res_pow, res_it):
        assert np.array_equal(gh, ref_hash)
    else:  # ulp differences of resolution: compare with the oracle instead
        _, og, _ = o.fwd_bwd(oracle_spec(**kw), table, mlp, pos, tgt)
        assert np.array_equal(gh, og["hash_fixed"])
    sc = np.abs(g["train_mlp"]).max()
    assert np.abs(gm - g["train_mlp"]).max() <= 1e-5 * sc
    assert abs(lsum - float(g["train_loss_sum"])) <= 1e-5 * abs(lsum)
    tr.close()


@pytest.mark.parametrize("tag", ["sdf", "img", "d4"])
def test_external_grad_matches_reference_golden(tag):
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    kw = spec_kwargs_from_tuple(sp)
    table, mlp, pos, tgt, d_out = case_inputs(tag, sp)
    tr = cuda_trainer(**kw, morton=False)
    tr.set_initial_weights(table, mlp)
    tr.zero_gradients()
    tr.backward_accumulate(pos, d_out)
    gh = tr.read_buffer(3)
    _, og, _ = o.fwd_bwd(oracle_spec(**kw), table, mlp, pos, None, d_out=d_out)
    assert np.array_equal(gh, og["hash_fixed"])
    assert np.abs(tr.read_buffer(4) - og["mlp"]).max() <= 1e-5 * np.abs(og["mlp"]).max()
    tr.close()


@pytest.mark.parametrize("tag", TAGS)
def test_eval_matches_reference_golden(tag):
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    kw = spec_kwargs_from_tuple(sp)
    table, mlp, pos, _, _ = case_inputs(tag, sp)
    tr = cuda_trainer(**kw)
    tr.set_initial_weights(table, mlp)
    out = tr.inference(pos)
    assert np.abs(out - g["eval"]).max() <= 1e-6 * max(1.0, np.abs(out).max())
    tr.close()


def test_weight_init_matches_oracle():
    kw = dict(L=4, F=2, log2T=12, W=32, H=2, O=3)
    tr = cuda_trainer(**kw, seed=0xDEADBEEF)
    hw, mw = tr.weights()
    h2, m2 = o.init_weights(oracle_spec(**kw), seed=0xDEADBEEF)
    assert np.array_equal(hw, h2)
    assert np.array_equal(mw, m2)
    tr.close()


@pytest.mark.parametrize("grad", ["Fixed16", "F32"])
def test_one_step_matches_oracle(grad):
    """training_step = Morton sort + fwd/bwd + sparse Adam: the hash weights
    after one step are bit-exact in fixed-point mode (integer gradient sums
    are order independent); MLP weights and the loss to fp32 round-off."""
    kw = dict(L=8, F=2, log2T=12, W=32, H=2, O=1, loss=0)
    tr = cuda_trainer(**kw, grad=grad)
    hw, mw = tr.weights()
    pos, tgt = batch(1000, 3, 1, seed=5)
    loss = tr.training_step(pos, tgt)
    ot = o.OracleTrainer(oracle_spec(**kw, grad=grad), hw, mw)
    ol = ot.training_step(pos, tgt)
    h1, m1 = tr.weights()
    assert abs(loss - ol) <= 1e-5 * abs(ol)
    if grad == "Fixed16":
        assert np.array_equal(h1, ot.hash_w)
    else:
        assert np.allclose(h1, ot.hash_w, rtol=0, atol=2e-6)
    assert np.allclose(m1, ot.mlp_w, rtol=1e-4, atol=1e-5)
    m_gpu = tr.read_buffer(8)
    assert np.allclose(m_gpu[:tr.hash_count], ot.m[:tr.hash_count], rtol=1e-5,
                       atol=1e-9)
    tr.close()


def test_training_curve_matches_oracle():
    kw = dict(L=8, F=2, log2T=12, W=32, H=2, O=1, loss=1)
    tr = cuda_trainer(**kw)
    hw, mw = tr.weights()
    ot = o.OracleTrainer(oracle_spec(**kw), hw, mw)
    for s in range(20):
        pos, tgt = batch(512, 3, 1, seed=100 + s)
        tgt = (np.linalg.norm(pos, axis=1, keepdims=True) - 0.5).astype(np.float32)
        a, b = tr.training_step(pos, tgt), ot.training_step(pos, tgt)
        assert abs(a - b) <= 2e-3 * abs(b), (s, a, b)
    tr.close()


def test_optimizer_blob_continuity():
    """test_default_trainer.cpp:2523-2584: export -> reset -> import keeps
    training continuous (< 1e-5 relative)."""
    kw = dict(L=8, F=2, log2T=12, W=32, H=1, O=1)
    pos, tgt = batch(256, 3, 1, seed=9)
    a = cuda_trainer(**kw)
    b = cuda_trainer(**kw)
    for _ in range(5):
        a.training_step(pos, tgt)
        b.training_step(pos, tgt)
    step, blob = a.export_optimizer_state()
    assert step == 5 and len(blob) == 16 + 8 * (a.hash_count + a.mlp_count)
    a.reset_optimizer()
    assert a.step() == 0
    a.import_optimizer_state(step, blob)
    assert a.step() == 5
    la, lb = a.training_step(pos, tgt), b.training_step(pos, tgt)
    assert abs(la - lb) <= 1e-5 * abs(lb)
    with pytest.raises(ValueError):
        a.import_optimizer_state(5, blob + b"\0")
    with pytest.raises(ValueError):
        a.import_optimizer_state(5, blob[:-4])
    a.close()
    b.close()


@pytest.mark.parametrize("N", [0, 1, 127, 128, 129, 1000])
def test_ragged_and_empty_batches(N):
    kw = dict(L=4, F=2, log2T=10, W=16, H=1, O=2)
    tr = cuda_trainer(**kw)
    hw, mw = tr.weights()
    pos, tgt = batch(N, 3, 2, seed=N)
    ot = o.OracleTrainer(oracle_spec(**kw), hw, mw)
    la, lb = tr.training_step(pos, tgt), ot.training_step(pos, tgt)
    assert tr.step() == 1
    assert abs(la - lb) <= 1e-5 * max(abs(lb), 1e-12)
    out = tr.inference(pos)
    assert out.shape == (N, 2)
    assert np.allclose(out, ot.evaluate(pos), rtol=1e-5, atol=1e-6)
    tr.close()


def test_split_path_matches_fused_path():
    """SplitPathMatchesFusedPath (test_default_trainer.cpp:1296): forward +
    external dL/dy + accumulate + adam_step equals training_step."""
    kw = dict(L=4, F=2, log2T=10, W=16, H=1, O=1)
    pos, tgt = batch(300, 3, 1, seed=4)
    a = cuda_trainer(**kw, morton=False)
    b = cuda_trainer(**kw, morton=False)
    a.training_step(pos, tgt)
    y = b.forward_for_training(pos)
    b.zero_gradients()
    inv_n = np.float32(1.0) / np.float32(300)
    b.backward_accumulate(pos, ((np.float32(2.0) * (y - tgt)) * inv_n).astype(np.float32))
    b.adam_step()
    ha, ma = a.weights()
    hb, mb = b.weights()
    assert np.array_equal(ha, hb)
    assert np.allclose(ma, mb, rtol=1e-5, atol=1e-7)
    a.close()
    b.close()


def test_errors_and_guards():
    import tmnn_b200 as t
    with pytest.raises(t.ConfigError):
        t.Trainer.from_config({"encoding": {"n_levels": 0}}, n_input=3, n_output=1)
    with pytest.raises(t.ConfigError):
        t.Trainer.from_config({"network": {"activation": "Tanh"}}, n_input=3,
                              n_output=1)
    tr = cuda_trainer(L=2, F=2, log2T=10, W=8, H=1, O=1)
    with pytest.raises(t.DTypeError):
        tr.training_step(np.zeros((4, 3), np.float64), np.zeros((4, 1), np.float32))
    with pytest.raises(ValueError):
        tr.training_step(np.zeros((4, 3), np.float32), np.zeros((5, 1), np.float32))
    tr.close()
    with pytest.raises(t.ClosedError):
        tr.step()


@pytest.mark.parametrize("d", [3, 4])
@pytest.mark.parametrize("key_bits", [0, 12, 8, 20])
def test_morton_order_matches_stable_sort_of_reference_codes(d, key_bits):
    """Device Morton permutation (morton_sort.h:60-110 codes): a stable sort
    on the top key_bits of the code (counting sort for <= 12 bits, CUB radix
    sort otherwise) equals numpy's stable argsort of the oracle's codes."""
    kw = dict(L=4, F=2, log2T=10, d=d, W=64, H=1, O=1)
    tr = cuda_trainer(**kw)
    rng = np.random.default_rng(d * 100 + key_bits)
    n = 70001
    pos = rng.uniform(-1.05, 1.05, (n, d)).astype(np.float32)
    pos[:1000] = pos[1000:2000]  # duplicate codes exercise stability
    perm = tr.debug_morton_order(pos, key_bits)
    f = o.lib.tmo_morton4 if d == 4 else o.lib.tmo_morton3
    codes = np.array([f(*map(float, p)) for p in pos], np.uint64)
    end = 32 if d == 4 else 30
    shift = end - key_bits if 0 < key_bits < end else 0
    want = np.argsort(codes >> np.uint64(shift), kind="stable")
    assert np.array_equal(perm, want.astype(np.uint32))
    tr.close()
