"""CPU checks of the NeRF-field restatement (oracle/oracle.py OracleNerf):
the SH basis is orthonormal on the sphere and has the closed-form values at
the poles; the plain-MLP backward matches finite differences; a few oracle
training steps reduce the loss.  The reference has no NeRF network, so these
pin the restatement to the mathematics, not to reference outputs."""
import numpy as np

import oracle as o


def test_sh_orthonormal_and_pole_values():
    rng = np.random.default_rng(0)
    d = rng.normal(size=(100000, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    Y = o.sh4(d.astype(np.float32)).astype(np.float64)
    gram = 4 * np.pi * (Y.T @ Y) / d.shape[0]
    assert np.abs(gram - np.eye(16)).max() < 0.03
    z = o.sh4(np.array([[0.0, 0.0, 1.0]], np.float32))[0]
    # Y_0^0 = 1/(2 sqrt(pi)), Y_1^0 = sqrt(3/(4 pi)), Y_2^0 = sqrt(5/pi)/2,
    # Y_3^0 = sqrt(7/pi)/2 at the pole; every m != 0 term vanishes there
    expect = {0: 0.5 / np.sqrt(np.pi), 2: np.sqrt(3 / (4 * np.pi)),
              6: 0.5 * np.sqrt(5 / np.pi), 12: 0.5 * np.sqrt(7 / np.pi)}
    for k in range(16):
        assert abs(z[k] - expect.get(k, 0.0)) < 1e-6, k


def test_mlp_train_matches_finite_differences():
    s = o.color_spec(W=64, H=2)
    rng = np.random.default_rng(1)
    n_w = o.mlp_weight_count(s)
    w = rng.uniform(-0.3, 0.3, n_w).astype(np.float32)
    x = rng.normal(size=(8, 32)).astype(np.float32)
    t = rng.random((8, 3)).astype(np.float32)
    g = np.zeros(n_w, np.float32)
    loss, dx = o.mlp_train(s, w, x, t, 8, 1, g)

    def f(wv, xv):
        gg = np.zeros(n_w, np.float32)
        return o.mlp_train(s, wv, xv, t, 8, 1, gg)[0] / 8.0

    h = 1e-3
    ok = 0
    ks = rng.choice(n_w, 16, replace=False)
    for k in ks:
        wp, wm = w.copy(), w.copy()
        wp[k] += h
        wm[k] -= h
        fd = (f(wp, x) - f(wm, x)) / (wp[k] - wm[k])
        ok += abs(fd - g[k]) <= 2e-2 * max(1e-2, abs(fd))
    # a stencil that crosses a ReLU kink does not follow the local slope
    assert ok >= len(ks) - 2
    xp, xm = x.copy(), x.copy()
    xp[3, 20] += h
    xm[3, 20] -= h
    fd = (f(w, xp) - f(w, xm)) / (xp[3, 20] - xm[3, 20])
    assert abs(fd - dx[3, 20]) <= 2e-2 * max(1e-2, abs(fd))


def test_oracle_nerf_loss_decreases():
    sd = o.make_spec(L=8, F=2, log2T=12, d=3, W=64, H=1, O=16,
                     scale=1.382, grad_mode=o.GRAD_FLOAT)
    rng = np.random.default_rng(2)
    table = rng.uniform(-1e-4, 1e-4, o.hash_grid_size(sd)).astype(np.float32)
    dmlp = rng.uniform(-0.2, 0.2, o.mlp_weight_count(sd)).astype(np.float32)
    cmlp = rng.uniform(-0.2, 0.2, o.mlp_weight_count(o.color_spec())).astype(np.float32)
    nerf = o.OracleNerf(sd, table, dmlp, cmlp)
    losses = []
    for i in range(30):
        pos, d, rgb, sig = o.nerf_batch(512, 100 + i)
        losses.append(nerf.training_step(pos, d, rgb, sig))
    assert np.mean(losses[-5:]) < 0.7 * np.mean(losses[:5])
