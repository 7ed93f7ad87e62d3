#!/usr/bin/env python3
"""Generate tests/golden/ref_*.npz from the reference itself (oracle/_ref: the
reference's generated MSL kernels and host code compiled here).

The fixtures let the parity tests pin the oracle and the CUDA path on machines
where the reference sources are absent.  Inputs are regenerated from the
seeds below (numpy PCG64), so each fixture stores only the reference's
outputs.  Run: python tests/golden/make_golden.py [simd]
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import ref_oracle  # noqa: E402

N_POINTS = 300
TAGS = ("ka", "sdf", "img", "d4", "f1", "f4", "cos")
# specs for which the reference's compiler realises the simdgroup-matrix
# training kernel (one output, one or two hidden layers)
SIMD_TAGS = ("sdf", "f4")
# single-output specs whose EvalGradient kernel output is also stored
EVALGRAD_ONLY = ("d4o1", "h3")


def case_inputs(tag, sp, seed=1):
    L, F, log2T, d, W, H, O = (int(x) for x in sp[:7])
    rng = np.random.default_rng(seed)
    T = 1 << log2T
    table = rng.uniform(-0.5, 0.5, L * T * F).astype(np.float32)
    In = L * F
    n_mlp = In * W + W + (H - 1) * (W * W + W) + W * O + O
    mlp = rng.uniform(-0.3, 0.3, n_mlp).astype(np.float32)
    lo = 0.0 if d == 4 else -1.0
    pos = rng.uniform(lo, 1.0, (N_POINTS, d)).astype(np.float32)
    tgt = rng.normal(size=(N_POINTS, O)).astype(np.float32)
    d_out = (rng.normal(size=(N_POINTS, O)) * 1e-3).astype(np.float32)
    return table, mlp, pos, tgt, d_out


def simd_main():
    """ref_simd_<tag>.npz: the simdgroup-matrix training kernel (the
    reference's default for these shapes) on the same inputs as ref_<tag>."""
    for tag in SIMD_TAGS:
        sp = ref_oracle.spec_tuple(tag)
        table, mlp, pos, tgt, _ = case_inputs(tag, sp)
        tr = ref_oracle.train_simd(tag, sp, table, mlp, pos, tgt)
        nz = np.nonzero(tr["grad_hash"])[0].astype(np.uint32)
        np.savez_compressed(
            os.path.join(HERE, f"ref_simd_{tag}.npz"),
            spec=np.array(sp, np.float64), hash_idx=nz,
            hash_val=tr["grad_hash"][nz], mlp=tr["grad_mlp"],
            loss_sum=np.float64(tr["loss_partials"].sum()), mask=tr["mask"])


def main():
    simd_main()
    for tag in TAGS:
        sp = ref_oracle.spec_tuple(tag)
        table, mlp, pos, tgt, d_out = case_inputs(tag, sp)
        tr = ref_oracle.train(tag, sp, table, mlp, pos, tgt)
        ex = ref_oracle.train(tag, sp, table, mlp, pos, tgt, d_out=d_out)
        ev = ref_oracle.evaluate(tag, sp, table, mlp, pos)
        extra = {}
        if int(sp[6]) == 1:
            extra["evalgrad"] = ref_oracle.eval_gradient(tag, sp, table, mlp, pos)
        nz = np.nonzero(tr["grad_hash"])[0].astype(np.uint32)
        nze = np.nonzero(ex["grad_hash"])[0].astype(np.uint32)
        np.savez_compressed(
            os.path.join(HERE, f"ref_{tag}.npz"), spec=np.array(sp, np.float64),
            train_hash_idx=nz, train_hash_val=tr["grad_hash"][nz],
            train_mlp=tr["grad_mlp"], train_loss_sum=np.float64(tr["loss_partials"].sum()),
            train_mask=tr["mask"], ext_hash_idx=nze,
            ext_hash_val=ex["grad_hash"][nze], ext_mlp=ex["grad_mlp"], eval=ev,
            **extra)
    for tag in EVALGRAD_ONLY:
        sp = ref_oracle.spec_tuple(tag)
        table, mlp, pos, _, _ = case_inputs(tag, sp)
        np.savez_compressed(
            os.path.join(HERE, f"ref_{tag}.npz"), spec=np.array(sp, np.float64),
            evalgrad=ref_oracle.eval_gradient(tag, sp, table, mlp, pos))
    # Philox init, Morton codes, Adam: small vectors
    rng = np.random.default_rng(5)
    uni = ref_oracle.init_uniform(1027, -0.25, 0.75, 0xDEADBEEF12345678, 17)
    nor = ref_oracle.init_normal(1027, 0.1, 2.0, 42, 5)
    p3 = rng.uniform(-1.2, 1.2, (512, 3)).astype(np.float32)
    p4 = rng.uniform(-1.2, 1.2, (512, 4)).astype(np.float32)
    m3 = np.array([ref_oracle.morton3(*p) for p in p3], np.uint32)
    m4 = np.array([ref_oracle.morton4(*p) for p in p4], np.uint32)
    hs, ms = 4096, 97
    w = rng.normal(size=hs + ms).astype(np.float32)
    gh = rng.integers(-300000, 300000, hs).astype(np.int32)
    gm = (rng.normal(size=ms) * 1e-2).astype(np.float32)
    m = (rng.normal(size=hs + ms) * 1e-3).astype(np.float32)
    v = np.abs(rng.normal(size=hs + ms) * 1e-5).astype(np.float32)
    params = ref_oracle.adam_params(1e-2, 1e-3, 0.9, 0.99, 1e-15, 0.0, 1e-4,
                                    hs, ms, 6)
    wu, mu, vu = w.copy(), m.copy(), v.copy()
    ghu = np.concatenate([gh, np.zeros(ms, np.int32)])
    ref_oracle.adam_unified(wu, ghu, gm, mu, vu, params)
    touched_pairs = np.nonzero(rng.random(hs // 2) < 0.4)[0].astype(np.uint32)
    idx = (touched_pairs * 2).astype(np.uint32)
    wh, mh, vh = w[:hs].copy(), m[:hs].copy(), v[:hs].copy()
    ref_oracle.adam_sparse(wh, gh.copy(), mh, vh, params, idx)
    wd, md, vd = w[hs:].copy(), m[hs:].copy(), v[hs:].copy()
    ref_oracle.adam_dense(wd, gm.copy(), md, vd, params)
    np.savez_compressed(
        os.path.join(HERE, "ref_static.npz"), uniform=uni, normal=nor, p3=p3,
        p4=p4, morton3=m3, morton4=m4, adam_w=w, adam_gh=gh, adam_gm=gm,
        adam_m=m, adam_v=v, adam_params=params, unified_w=wu, unified_m=mu,
        unified_v=vu, touched_pairs=touched_pairs, sparse_w=wh, sparse_m=mh,
        sparse_v=vh, dense_w=wd, dense_m=md, dense_v=vd)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    # "simd": write only the SIMD-kernel fixtures
    simd_main() if sys.argv[1:] == ["simd"] else main()
