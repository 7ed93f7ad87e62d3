"""Pins the CPU oracle (oracle/tmnn_oracle.c) to the reference itself.

Sources of truth, in order of strength:
  * tests/golden/ref_*.npz: outputs of the reference's own generated MSL
    kernels (scalar train / external-grad / eval), its static Adam and Philox
    MSL, and its host Morton code, compiled here by oracle/ref_build.py and
    dumped by tests/golden/make_golden.py;
  * the reference's known answers (tests/unit/tmnn/test_default_trainer.cpp,
    test_kernel_generation.cpp, test_training_step_execution.cpp,
    test_tmnn_core.cpp);
  * published Philox-4x32-10 known-answer vectors (Random123, SC'11).
"""
import os

import numpy as np
import pytest

import oracle as o
from golden.make_golden import SIMD_TAGS, TAGS, case_inputs

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def spec_from(sp, res_mode=1, grad_mode=o.GRAD_FIXED16):
    L, F, log2T, d, W, H, O, loss, base, scale, huber = sp
    return o.make_spec(L=int(L), F=int(F), log2T=int(log2T), d=int(d),
                       W=int(W), H=int(H), O=int(O), loss=int(loss),
                       base=float(base), scale=float(scale),
                       huber_delta=float(huber), res_mode=res_mode,
                       grad_mode=grad_mode)


def test_known_answer_forward_034():
    # test_default_trainer.cpp:2260-2336: L=2 F=2 T=2^10 base 4 scale 2,
    # W=8 H=1 O=1, table = 0.5, MLP = 0.1, pos (0.5,0.5,0.5) -> 0.34.
    s = o.make_spec(L=2, F=2, log2T=10, base=4, scale=2, W=8, H=1, O=1)
    assert o.mlp_weight_count(s) == 49
    h = np.full(o.hash_grid_size(s), 0.5, np.float32)
    m = np.full(o.mlp_weight_count(s), 0.1, np.float32)
    out = o.forward(s, h, m, np.array([[0.5, 0.5, 0.5]], np.float32))
    assert abs(out[0, 0] - 0.34) < 1e-4


def test_mlp_weight_count_formula():
    # test_kernel_generation.cpp:39-45: 2112 + 4160 + 65
    s = o.make_spec(L=16, F=2, W=64, H=2, O=1)
    assert o.mlp_weight_count(s) == 2112 + 4160 + 65


def test_philox_known_answers():
    kat = [
        ([0, 0, 0, 0], [0, 0], [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
        ([0xffffffff] * 4, [0xffffffff] * 2,
         [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
        ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344],
         [0xa4093822, 0x299f31d0], [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
    ]
    for ctr, key, want in kat:
        assert list(o.philox(ctr, key)) == want


def test_adam_bias_corrections_and_count_split():
    # adam_params.h:33-52; test_training_step_execution.cpp:62-88
    hs = 1 << 24
    assert (int(np.float32(hs & 0xFFFF)) | (int(np.float32(hs >> 16)) << 16)) == hs
    bc1, bc2 = o.bias_corrections(0.9, 0.99, 0)
    assert bc1 == np.float32(1) - np.float32(0.9)
    assert np.isclose(bc2, 0.01, rtol=1e-5)


@pytest.mark.parametrize("tag", TAGS)
def test_train_kernel_matches_reference_golden(tag):
    """Scalar train kernel of the reference vs the oracle (pow resolutions as
    that kernel uses): int32 fixed-point hash gradients bit-exact; MLP
    gradients (summed by float atomics in the reference) within 1e-5; loss."""
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    s = spec_from(sp)
    table, mlp, pos, tgt, d_out = case_inputs(tag, sp)
    lsum, grads, _ = o.fwd_bwd(s, table, mlp, pos, tgt)
    ref_hash = np.zeros(table.size, np.int32)
    ref_hash[g["train_hash_idx"]] = g["train_hash_val"]
    assert np.array_equal(grads["hash_fixed"], ref_hash)
    scale = np.abs(g["train_mlp"]).max()
    assert np.abs(grads["mlp"] - g["train_mlp"]).max() <= 1e-5 * scale
    assert abs(lsum - float(g["train_loss_sum"])) <= 1e-5 * abs(lsum)
    # touched slots: the reference marks them only in the float2 scatter
    # (3D, F == 2); its scalar int-atomic scatter emits no mask (see the
    # defect note in the oracle) so there the reference mask stays empty.
    ref_touched = np.unpackbits(g["train_mask"].view(np.uint8),
                                bitorder="little")[:o.tracked_slots(s)]
    if s.F == 2 and s.d == 3:
        assert np.array_equal(ref_touched, grads["touched"])
    else:
        assert ref_touched.sum() == 0 and grads["touched"].sum() > 0


def output_layer(sp):
    """Slice of the MLP buffer holding the output layer (weights, bias)."""
    L, F, _, _, W, H, O = (int(x) for x in sp[:7])
    n = L * F * W + W + (H - 1) * (W * W + W)
    return slice(n, n + W * O + O)


@pytest.mark.parametrize("tag", SIMD_TAGS)
def test_simd_train_kernel_matches_reference_golden(tag):
    """The reference's default training kernel for one-output shapes, the
    simdgroup-matrix variant (mlp_kernel_emitter.cpp:2104-2718: scalar
    encode with iterative resolutions, 8-row simdgroup tiles for the MLP and
    the W0 gradient, scatter with pow resolutions), against the oracle with
    pow resolutions: int32 hash gradients bit-exact, loss and the hidden
    layers' gradients to 1e-5.  The output layer is left out: in that kernel
    the 8 lanes of a batch add their contributions to the same threadgroup
    words without atomics (mlp_kernel_emitter.cpp:2418, :2422), a data race
    (on the GPU's lockstep lanes one write survives), so its value there is
    not a function of the inputs; the scalar kernel's test above pins the
    oracle's output layer."""
    g = np.load(os.path.join(GOLDEN, f"ref_simd_{tag}.npz"))
    sp = tuple(g["spec"])
    s = spec_from(sp)
    table, mlp, pos, tgt, _ = case_inputs(tag, sp)
    lsum, grads, _ = o.fwd_bwd(s, table, mlp, pos, tgt)
    ref_hash = np.zeros(table.size, np.int32)
    ref_hash[g["hash_idx"]] = g["hash_val"]
    assert np.array_equal(grads["hash_fixed"], ref_hash)
    assert abs(lsum - float(g["loss_sum"])) <= 1e-5 * abs(lsum)
    keep = np.ones(mlp.size, bool)
    keep[output_layer(sp)] = False
    scale = np.abs(g["mlp"][keep]).max()
    assert np.abs(grads["mlp"][keep] - g["mlp"][keep]).max() <= 1e-5 * scale
    ref_touched = np.unpackbits(g["mask"].view(np.uint8),
                                bitorder="little")[:o.tracked_slots(s)]
    if s.F == 2 and s.d == 3:
        assert np.array_equal(ref_touched, grads["touched"])


def test_simd_train_kernel_at_benchmark_shape(ref):
    """The same pin at the benchmarked sdf3d shape (16 levels x 2, 2^19
    table, 64 wide), against the live reference build."""
    tag = "bench_sdf3d"
    if not ref.has_simd_train(tag):
        pytest.skip("no SIMD train kernel built for " + tag)
    sp = ref.spec_tuple(tag)
    table, mlp, pos, tgt, _ = case_inputs(tag, sp, seed=7)
    r = ref.train_simd(tag, sp, table, mlp, pos, tgt)
    lsum, grads, _ = o.fwd_bwd(spec_from(sp), table, mlp, pos, tgt)
    assert np.array_equal(r["grad_hash"], grads["hash_fixed"])
    assert abs(float(r["loss_partials"].sum()) - lsum) <= 1e-5 * abs(lsum)


@pytest.mark.parametrize("tag", ["bench_sdf3d", "bench_image"])
def test_concurrent_threadgroups_match_sequential(ref, tag):
    """The reference arm runs several emulated threadgroups at once, each
    lane on its own copy of the kernel's threadgroup arrays; its fixed-point
    hash gradients, touched mask and loss partials equal the one-at-a-time
    run, and the float MLP gradients differ only by summation order."""
    sp = ref.spec_tuple(tag)
    table, mlp, pos, tgt, _ = case_inputs(tag, sp, seed=5)
    a = ref.train(tag, sp, table, mlp, pos, tgt)
    b = ref.train_lanes(tag, sp, table, mlp, pos, tgt, lanes=4)
    assert np.array_equal(a["grad_hash"], b["grad_hash"])
    assert np.array_equal(a["mask"], b["mask"])
    assert np.array_equal(a["loss_partials"], b["loss_partials"])
    scale = max(1e-30, float(np.abs(a["grad_mlp"]).max()))
    assert np.abs(a["grad_mlp"] - b["grad_mlp"]).max() <= 1e-5 * scale


@pytest.mark.parametrize("tag", TAGS)
def test_external_grad_kernel_matches_reference_golden(tag):
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    s = spec_from(sp)
    table, mlp, pos, tgt, d_out = case_inputs(tag, sp)
    _, grads, _ = o.fwd_bwd(s, table, mlp, pos, None, d_out=d_out)
    ref_hash = np.zeros(table.size, np.int32)
    ref_hash[g["ext_hash_idx"]] = g["ext_hash_val"]
    assert np.array_equal(grads["hash_fixed"], ref_hash)
    scale = np.abs(g["ext_mlp"]).max()
    assert np.abs(grads["mlp"] - g["ext_mlp"]).max() <= 1e-5 * scale


@pytest.mark.parametrize("tag", TAGS)
def test_eval_kernel_matches_reference_golden(tag):
    """Reference eval kernel (iterative resolution) vs oracle forward: the
    vec4 fast path of the reference groups the output dot product in fours,
    so the comparison is at 1e-6 relative, not bit-exact."""
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    s = spec_from(sp, res_mode=0)
    table, mlp, pos, _, _ = case_inputs(tag, sp)
    out = o.forward(s, table, mlp, pos)
    assert np.abs(out - g["eval"]).max() <= 1e-6 * max(1.0, np.abs(out).max())


EVALGRAD_TAGS = ("ka", "sdf", "f1", "f4", "h3", "d4o1")


@pytest.mark.parametrize("tag", EVALGRAD_TAGS)
def test_eval_gradient_kernel_matches_reference_golden(tag):
    """Reference EvalGradient kernel (mlp_kernel_emitter.cpp:1716-2090, scalar
    path, resolution BASE*pow(SCALE, l)) vs the oracle: bit-exact.  The
    kernel writes [value, d/dx, d/dy, d/dz]; in 4D the d/dw component is not
    written, so only the first three are compared."""
    g = np.load(os.path.join(GOLDEN, f"ref_{tag}.npz"))
    sp = tuple(g["spec"])
    table, mlp, pos, _, _ = case_inputs(tag, sp)
    out, grad = o.eval_gradient(spec_from(sp, res_mode=1), table, mlp, pos)
    ref = g["evalgrad"]
    assert np.array_equal(out, ref[:, 0])
    assert np.array_equal(grad[:, :3], ref[:, 1:4])


def test_eval_gradient_matches_finite_differences():
    """d(value)/d(pos) agrees with central differences of the oracle's own
    value (known-answer style rule of test_default_trainer.cpp:2338-2412),
    away from cell boundaries."""
    sp = (4, 2, 10, 3, 16, 2, 1, 0, 4.0, 1.5, 1.0)
    s = spec_from(sp, res_mode=0)
    table, mlp, pos, _, _ = case_inputs("fd", sp, seed=7)
    pos = pos[:64].astype(np.float64)
    _, grad = o.eval_gradient(s, table, mlp, pos.astype(np.float32))
    h = 1e-3
    ok = 0
    for i in range(pos.shape[0]):
        for a in range(3):
            pp, pm = pos[i].copy(), pos[i].copy()
            pp[a] += h
            pm[a] -= h
            vp, _ = o.eval_gradient(s, table, mlp, pp[None].astype(np.float32))
            vm, _ = o.eval_gradient(s, table, mlp, pm[None].astype(np.float32))
            fd = (float(vp[0]) - float(vm[0])) / (2 * h)
            if abs(fd - grad[i, a]) <= 2e-2 * max(1.0, abs(fd)):
                ok += 1
    # points whose +-h stencil crosses a cell face of some level or a ReLU
    # kink do not follow the local derivative; they are a small minority
    assert ok >= 0.9 * pos.shape[0] * 3


def test_static_kernels_match_reference_golden():
    g = np.load(os.path.join(GOLDEN, "ref_static.npz"))
    assert np.array_equal(o.init_uniform(1027, -0.25, 0.75, 0xDEADBEEF12345678, 17),
                          g["uniform"])
    assert np.allclose(o.init_normal(1027, 0.1, 2.0, 42, 5), g["normal"],
                       rtol=1e-5, atol=1e-5)
    assert [o.lib.tmo_morton3(*p) for p in g["p3"]] == list(g["morton3"])
    assert [o.lib.tmo_morton4(*p) for p in g["p4"]] == list(g["morton4"])


def _adam_case(g, sparse_pairs=None):
    hs = g["adam_gh"].size
    s = o.make_spec(L=1, F=2, log2T=11, W=1, H=1, O=1)  # 4096 hash floats
    assert o.hash_grid_size(s) == hs
    p = g["adam_params"]
    w, m, v = g["adam_w"].copy(), g["adam_m"].copy(), g["adam_v"].copy()
    touched = np.zeros(hs // 2, np.uint8)
    if sparse_pairs is not None:
        touched[sparse_pairs] = 1
    grads = {"hash_fixed": g["adam_gh"].copy(), "mlp": g["adam_gm"].copy(),
             "touched": touched}
    # the golden MLP section has 97 weights; the oracle's Adam is size-agnostic
    o.adam(s, w, m, v, grads, step=6, lr_hash=float(p[0]), lr_mlp=float(p[1]),
           beta1=float(p[2]), beta2=float(p[3]), eps=float(p[4]),
           l1=float(p[7]), l2=float(p[8]), sparse=sparse_pairs is not None)
    return w, m, v, hs


def test_adam_matches_reference_golden():
    g = np.load(os.path.join(GOLDEN, "ref_static.npz"))
    w, m, v, hs = _adam_case(g)  # unified (dense) kernel
    assert np.array_equal(w, g["unified_w"])
    assert np.array_equal(m, g["unified_m"])
    assert np.array_equal(v, g["unified_v"])
    w, m, v, hs = _adam_case(g, g["touched_pairs"])  # sparse hash + dense MLP
    assert np.array_equal(w[:hs], g["sparse_w"])
    assert np.array_equal(m[:hs], g["sparse_m"])
    assert np.array_equal(w[hs:], g["dense_w"])
    assert np.array_equal(v[hs:], g["dense_v"])


def test_reference_h3_backward_defect_documented(ref):
    """The reference's scalar train kernel reuses h0/h1 in place (mlp_kernel_
    emitter.cpp:2962-2970, :3098-3113): for num_hidden_layers >= 3 layer 2
    overwrites layer 0's activations, so layer 1's weight gradient is formed
    from the wrong buffer.  The oracle back-propagates correctly; this test
    records that the two differ there, and that the oracle's gradient agrees
    with a finite difference."""
    sp = ref.spec_tuple("h3")
    s = spec_from(sp, grad_mode=o.GRAD_FLOAT)
    table, mlp, pos, tgt, _ = case_inputs("h3", sp)
    pos, tgt = pos[:8], tgt[:8]
    r = ref.train("h3", sp, table, mlp, pos, tgt)
    _, grads, _ = o.fwd_bwd(s, table, mlp, pos, tgt)
    assert not np.allclose(r["grad_mlp"], grads["mlp"], rtol=1e-3)
    m64 = mlp.astype(np.float64)
    def loss_at(mv):
        out = o.forward(spec_from(sp, res_mode=1), table, mv.astype(np.float32), pos)
        return float(((out.astype(np.float64) - tgt) ** 2).mean())
    k = 2 * 4 * 8 + 8 + 5  # an entry of W1 (layer 1 weights)
    eps = 1e-3
    mp, mm = m64.copy(), m64.copy()
    mp[k] += eps
    mm[k] -= eps
    fd = (loss_at(mp) - loss_at(mm)) / (2 * eps)
    assert abs(fd - grads["mlp"][k]) <= 2e-3 * max(1e-3, abs(fd))


def test_oracle_matches_live_reference(ref):
    """Same comparison as the golden tests on fresh seeds, against the live
    reference build (only where oracle/_ref exists)."""
    for tag in ("sdf", "img", "d4"):
        sp = ref.spec_tuple(tag)
        table, mlp, pos, tgt, _ = case_inputs(tag, sp, seed=99)
        r = ref.train(tag, sp, table, mlp, pos, tgt)
        _, grads, _ = o.fwd_bwd(spec_from(sp), table, mlp, pos, tgt)
        assert np.array_equal(r["grad_hash"], grads["hash_fixed"])


def test_morton_sort_matches_reference(ref):
    rng = np.random.default_rng(3)
    pos = rng.uniform(-1, 1, (2000, 3)).astype(np.float32)
    tgt = rng.normal(size=(2000, 1)).astype(np.float32)
    rp, rt = ref.morton_sort(pos, tgt)
    perm = o.morton_order(pos)
    codes = np.array([o.lib.tmo_morton3(*p) for p in pos[perm]])
    assert np.all(np.diff(codes.astype(np.int64)) >= 0)
    # same codes in the same order; within a run of equal codes the
    # reference's std::sort order is unspecified, compare as multisets
    rc = np.array([ref.morton3(*p) for p in rp])
    assert np.array_equal(rc, codes)
    assert np.array_equal(np.sort(rp.view(np.uint32).ravel()),
                          np.sort(pos[perm].view(np.uint32).ravel()))


def test_spec_limits_match_reference(ref):
    cases = [(16, 2, 19, 3, 64, 1, 1), (16, 2, 9, 3, 64, 1, 1),
             (16, 3, 19, 3, 64, 1, 1), (33, 2, 19, 3, 64, 1, 1),
             (16, 2, 19, 5, 64, 1, 1), (16, 2, 19, 3, 513, 1, 1),
             (16, 2, 19, 3, 64, 9, 1), (16, 2, 25, 4, 64, 2, 4)]
    for c in cases:
        ok, _ = ref.validate(*c)
        L, F, log2T, d, W, H, O = c
        mine = (1 <= L <= 32 and F in (1, 2, 4) and 10 <= log2T <= 24 and
                d in (3, 4) and 0 < W <= 512 and 1 <= H <= 8)
        assert ok == mine, c
        assert ref.mlp_weight_count(L * F, W, H, O) == o.mlp_weight_count(
            o.make_spec(L=L, F=F, W=W, H=H, O=O))
