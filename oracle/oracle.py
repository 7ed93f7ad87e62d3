"""ctypes binding of the CPU oracle (oracle/libtmnn_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, as the checker.  The product never
imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libtmnn_oracle.so")

LOSS = {"L2": 0, "L1": 1, "Huber": 2, "Cosine": 3}
GRAD_FIXED16, GRAD_FLOAT = 0, 1


class Spec(C.Structure):
    _fields_ = [("L", C.c_int32), ("F", C.c_int32), ("log2T", C.c_int32),
                ("d", C.c_int32), ("W", C.c_int32), ("H", C.c_int32),
                ("O", C.c_int32), ("loss", C.c_int32), ("base", C.c_float),
                ("scale", C.c_float), ("huber_delta", C.c_float),
                ("active_levels", C.c_int32), ("grad_mode", C.c_int32),
                ("res_mode", C.c_int32), ("fp16_operands", C.c_int32),
                ("dscale", C.c_float)]


class AdamCfg(C.Structure):
    _fields_ = [("lr_hash", C.c_float), ("lr_mlp", C.c_float),
                ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("l1_hash", C.c_float), ("l2_mlp", C.c_float),
                ("grad_clip", C.c_float), ("weight_decay", C.c_float),
                ("step", C.c_uint32), ("sparse_hash", C.c_int32),
                ("entry_width", C.c_int32)]


class InitCfg(C.Structure):
    _fields_ = [("hash_zero", C.c_int32), ("hash_range", C.c_float),
                ("mlp_mode", C.c_int32), ("gain", C.c_float),
                ("mlp_uniform_range", C.c_float),
                ("mlp_normal_stddev", C.c_float), ("seed", C.c_uint64)]


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    if not os.path.exists(_LIB_PATH):
        build()
    lib = C.CDLL(_LIB_PATH)
    P = C.c_void_p
    sp = C.POINTER(Spec)
    lib.tmo_round6.restype = C.c_float
    lib.tmo_round6.argtypes = [C.c_float]
    lib.tmo_level_resolutions.argtypes = [sp, P]
    lib.tmo_hash_grid_size.restype = C.c_uint64
    lib.tmo_hash_grid_size.argtypes = [sp]
    lib.tmo_mlp_weight_count.restype = C.c_int64
    lib.tmo_mlp_weight_count.argtypes = [sp]
    lib.tmo_hash3.restype = C.c_uint32
    lib.tmo_hash3.argtypes = [C.c_int32] * 3 + [C.c_uint32]
    lib.tmo_hash4.restype = C.c_uint32
    lib.tmo_hash4.argtypes = [C.c_int32] * 4 + [C.c_uint32]
    lib.tmo_encode.argtypes = [sp, P, P, C.c_int64, P, P, P]
    lib.tmo_forward.argtypes = [sp, P, P, P, C.c_int64, P]
    lib.tmo_mlp_forward.argtypes = [sp, P, P, C.c_int64, P]
    lib.tmo_eval_gradient.argtypes = [sp, P, P, P, C.c_int64, P, P]
    lib.tmo_mlp_train.restype = C.c_double
    lib.tmo_mlp_train.argtypes = [sp, P, P, P, C.c_int64, C.c_int64, C.c_int,
                                  P, P]
    lib.tmo_sh4.argtypes = [C.c_float, C.c_float, C.c_float, P]
    lib.tmo_fwd_bwd.restype = C.c_double
    lib.tmo_fwd_bwd.argtypes = [sp, P, P, P, P, P, C.c_int64, C.c_int64, P, P,
                                P, P, P]
    lib.tmo_fwd_bwd_par.restype = C.c_double
    lib.tmo_fwd_bwd_par.argtypes = [sp, P, P, P, P, C.c_int64, C.c_int64, P,
                                    P, P, P, C.c_int]
    lib.tmo_adam_bias_corrections.argtypes = [C.c_float, C.c_float, C.c_uint32,
                                              P, P]
    lib.tmo_adam.argtypes = [C.POINTER(AdamCfg), P, P, P, C.c_uint64,
                             C.c_uint64, P, P, P, P, C.c_int]
    lib.tmo_philox4x32_10.argtypes = [P, P, P]
    lib.tmo_init_uniform.argtypes = [P, C.c_uint64, C.c_float, C.c_float,
                                     C.c_uint64, C.c_uint32]
    lib.tmo_init_normal.argtypes = [P, C.c_uint64, C.c_float, C.c_float,
                                    C.c_uint64, C.c_uint32]
    lib.tmo_init_weights.argtypes = [sp, C.POINTER(InitCfg), P, P]
    lib.tmo_morton3.restype = C.c_uint32
    lib.tmo_morton3.argtypes = [C.c_float] * 3
    lib.tmo_morton4.restype = C.c_uint32
    lib.tmo_morton4.argtypes = [C.c_float] * 4
    lib.tmo_morton_order.argtypes = [P, C.c_int64, C.c_int, P]
    return lib


lib = _load()


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def make_spec(L=16, F=2, log2T=19, d=3, W=64, H=1, O=1, loss="L2",
              base=16.0, scale=1.447, huber_delta=1.0, active_levels=0,
              grad_mode=GRAD_FIXED16, res_mode=0, fp16_operands=0, dscale=0.0):
    return Spec(L, F, log2T, d, W, H, O, LOSS[loss] if isinstance(loss, str)
                else loss, base, scale, huber_delta, active_levels, grad_mode,
                res_mode, fp16_operands, dscale)


def pow2_scale(n):
    """The fused kernel's dL/dy scale for a batch of n: 2^(e-1) where
    n = m * 2^e with m in [0.5, 1) (frexp)."""
    import math
    return math.ldexp(1.0, math.frexp(float(max(n, 1)))[1] - 1)


def hash_grid_size(s):
    return int(lib.tmo_hash_grid_size(C.byref(s)))


def mlp_weight_count(s):
    return int(lib.tmo_mlp_weight_count(C.byref(s)))


def level_resolutions(s):
    r = np.zeros(s.L, np.float32)
    lib.tmo_level_resolutions(C.byref(s), _p(r))
    return r


def encode(s, table, pos, with_indices=False):
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    feat = np.zeros((N, s.L * s.F), np.float32)
    idx = np.zeros((N, s.L, 1 << s.d), np.uint32) if with_indices else None
    cells = np.zeros((N, s.L, s.d), np.int32) if with_indices else None
    lib.tmo_encode(C.byref(s), _p(table), _p(pos), N, _p(feat), _p(idx),
                   _p(cells))
    return (feat, idx, cells) if with_indices else feat


def forward(s, table, mlp, pos):
    pos = np.ascontiguousarray(pos, np.float32)
    out = np.zeros((pos.shape[0], s.O), np.float32)
    lib.tmo_forward(C.byref(s), _p(table), _p(mlp), _p(pos), pos.shape[0],
                    _p(out))
    return out


def mlp_forward(s, mlp, x):
    """Plain MLP on features x [N x L*F] (use L = n_input, F = 1)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros((x.shape[0], s.O), np.float32)
    lib.tmo_mlp_forward(C.byref(s), _p(mlp), _p(x), x.shape[0], _p(out))
    return out


def eval_gradient(s, table, mlp, pos):
    """Field value [N] and d(value)/d(pos) [N x d] of a single-output net."""
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    out = np.zeros(N, np.float32)
    grad = np.zeros((N, s.d), np.float32)
    lib.tmo_eval_gradient(C.byref(s), _p(np.ascontiguousarray(table, np.float32)),
                          _p(np.ascontiguousarray(mlp, np.float32)), _p(pos), N,
                          _p(out), _p(grad))
    return out, grad


def tracked_slots(s):
    n = hash_grid_size(s)
    return n // 2 if s.F == 2 else n


def fwd_bwd(s, table, mlp, pos, tgt=None, d_out=None, inv_count=0,
            grads=None, want_out=False):
    """Returns (loss_sum, grads dict, outputs or None).  grads accumulates."""
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    if grads is None:
        grads = zero_grads(s)
    out = np.zeros((N, s.O), np.float32) if want_out else None
    tgt = None if tgt is None else np.ascontiguousarray(tgt, np.float32)
    d_out = None if d_out is None else np.ascontiguousarray(d_out, np.float32)
    loss = lib.tmo_fwd_bwd(C.byref(s), _p(table), _p(mlp), _p(pos), _p(tgt),
                           _p(d_out), N, inv_count, _p(grads["mlp"]),
                           _p(grads.get("hash_fixed")),
                           _p(grads.get("hash_float")), _p(grads["touched"]),
                           _p(out))
    return loss, grads, out


def fwd_bwd_par(s, table, mlp, pos, tgt, grads, nthreads=0, inv_count=0):
    pos = np.ascontiguousarray(pos, np.float32)
    return lib.tmo_fwd_bwd_par(C.byref(s), _p(table), _p(mlp), _p(pos),
                               _p(np.ascontiguousarray(tgt, np.float32)),
                               pos.shape[0], inv_count, _p(grads["mlp"]),
                               _p(grads.get("hash_fixed")),
                               _p(grads.get("hash_float")),
                               _p(grads["touched"]), nthreads)


def zero_grads(s):
    g = {"mlp": np.zeros(mlp_weight_count(s), np.float32),
         "touched": np.zeros(tracked_slots(s), np.uint8)}
    if s.grad_mode == GRAD_FIXED16:
        g["hash_fixed"] = np.zeros(hash_grid_size(s), np.int32)
    else:
        g["hash_float"] = np.zeros(hash_grid_size(s), np.float32)
    return g


def bias_corrections(beta1, beta2, step):
    a, b = C.c_float(), C.c_float()
    lib.tmo_adam_bias_corrections(beta1, beta2, step, C.byref(a), C.byref(b))
    return a.value, b.value


def adam(s, w, m, v, grads, step, lr_hash=1e-2, lr_mlp=1e-3, beta1=0.9,
         beta2=0.99, eps=1e-15, l1=0.0, l2=0.0, clip=0.0, wd=0.0,
         sparse=None, nthreads=0):
    """In-place Adam on flat [hash | mlp] arrays.  sparse defaults to the
    reference rule: sparse hash update iff l1 == 0."""
    if sparse is None:
        sparse = l1 == 0.0
    cfg = AdamCfg(lr_hash, lr_mlp, beta1, beta2, eps, l1, l2, clip, wd, step,
                  1 if sparse else 0, 2 if s.F == 2 else 1)
    hc = hash_grid_size(s)
    lib.tmo_adam(C.byref(cfg), _p(w), _p(m), _p(v), hc, w.size - hc,
                 _p(grads.get("hash_fixed")), _p(grads.get("hash_float")),
                 _p(grads["mlp"]), _p(grads["touched"]), nthreads)


def philox(ctr, key):
    c = np.asarray(ctr, np.uint32)
    k = np.asarray(key, np.uint32)
    out = np.zeros(4, np.uint32)
    lib.tmo_philox4x32_10(_p(c), _p(k), _p(out))
    return out


def init_uniform(count, low, high, seed, counter_base=0):
    out = np.zeros(count, np.float32)
    lib.tmo_init_uniform(_p(out), count, low, high, seed, counter_base)
    return out


def init_normal(count, mean, std, seed, counter_base=0):
    out = np.zeros(count, np.float32)
    lib.tmo_init_normal(_p(out), count, mean, std, seed, counter_base)
    return out


MLP_INIT = {"KaimingUniform": 0, "KaimingNormal": 1, "XavierUniform": 2,
            "XavierNormal": 3, "Uniform": 4, "Normal": 5, "Zero": 6}


def init_weights(s, seed=42, hash_range=1e-4, hash_zero=False,
                 mlp_mode="KaimingUniform", gain=float(np.float32(np.sqrt(2))),
                 mlp_uniform_range=1e-2, mlp_normal_stddev=1e-2):
    h = np.zeros(hash_grid_size(s), np.float32)
    m = np.zeros(mlp_weight_count(s), np.float32)
    cfg = InitCfg(1 if hash_zero else 0, hash_range, MLP_INIT[mlp_mode], gain,
                  mlp_uniform_range, mlp_normal_stddev, seed)
    lib.tmo_init_weights(C.byref(s), C.byref(cfg), _p(h), _p(m))
    return h, m


def morton_order(pos):
    pos = np.ascontiguousarray(pos, np.float32)
    perm = np.zeros(pos.shape[0], np.uint32)
    lib.tmo_morton_order(_p(pos), pos.shape[0], pos.shape[1], _p(perm))
    return perm


class OracleTrainer:
    """The reference's fused training step restated on the CPU:
    Morton sort -> fwd/bwd (+scatter) -> loss = sum/N -> Adam (sparse hash
    unless l1>0) -> zero grads (default_trainer.cpp:883-1045)."""

    def __init__(self, s, hash_w, mlp_w, lr_hash=1e-2, lr_mlp=1e-3,
                 beta1=0.9, beta2=0.99, eps=1e-15, l1=0.0, l2=0.0,
                 morton=True, nthreads=1, table_fp16=False):
        self.s = s
        # table_fp16: the encode reads an fp16 copy of the table (the
        # FullyFused family's gather copy with table_dtype F16), rounded to
        # nearest-even from the fp32 master after every update; Adam still
        # updates the fp32 master
        self.table_fp16 = table_fp16
        self.w = np.concatenate([hash_w, mlp_w]).astype(np.float32)
        self.m = np.zeros_like(self.w)
        self.v = np.zeros_like(self.w)
        self.hc = hash_w.size
        self.step = 0
        self.opt = dict(lr_hash=lr_hash, lr_mlp=lr_mlp, beta1=beta1,
                        beta2=beta2, eps=eps, l1=l1, l2=l2)
        self.morton = morton
        self.nthreads = nthreads

    @property
    def hash_w(self):
        return self.w[:self.hc]

    @property
    def mlp_w(self):
        return self.w[self.hc:]

    def training_step(self, pos, tgt):
        pos = np.ascontiguousarray(pos, np.float32)
        tgt = np.ascontiguousarray(tgt, np.float32).reshape(pos.shape[0],
                                                             self.s.O)
        if self.morton and pos.shape[0] > 1:
            perm = morton_order(pos)
            pos, tgt = pos[perm], tgt[perm]
        g = zero_grads(self.s)
        table, mlp = self.w[:self.hc].copy(), self.w[self.hc:].copy()
        if self.table_fp16:
            table = table.astype(np.float16).astype(np.float32)
        if self.s.fp16_operands:
            # the tensor-core kernel's dL/dy scale follows the batch size
            self.s.dscale = pow2_scale(max(pos.shape[0], 1))
        if self.nthreads == 1:
            loss, g, _ = fwd_bwd(self.s, table, mlp, pos, tgt, grads=g)
        else:
            loss = fwd_bwd_par(self.s, table, mlp, pos, tgt, g, self.nthreads)
        adam(self.s, self.w, self.m, self.v, g, self.step,
             nthreads=self.nthreads, **self.opt)
        self.step += 1
        if pos.shape[0] == 0:
            return 0.0
        return float(np.float32(loss) / np.float32(pos.shape[0]))

    def evaluate(self, pos):
        return forward(self.s, self.w[:self.hc], self.w[self.hc:], pos)


# ------------------------------------------------------------ NeRF field

def sh4(dirs):
    """Real SH (16 coefficients) of unit directions [N x 3]."""
    dirs = np.ascontiguousarray(dirs, np.float32)
    out = np.zeros((dirs.shape[0], 16), np.float32)
    for i in range(dirs.shape[0]):
        lib.tmo_sh4(float(dirs[i, 0]), float(dirs[i, 1]), float(dirs[i, 2]),
                    out[i].ctypes.data_as(C.c_void_p))
    return out


def mlp_train(s, mlp, x, tgt, inv_count, out_act, grad_mlp):
    """(loss_sum, dx) of a plain-MLP training pass; grad_mlp accumulates."""
    x = np.ascontiguousarray(x, np.float32)
    tgt = np.ascontiguousarray(tgt, np.float32)
    dx = np.zeros_like(x)
    loss = lib.tmo_mlp_train(C.byref(s), _p(np.ascontiguousarray(mlp, np.float32)),
                             _p(x), _p(tgt), x.shape[0], inv_count, out_act,
                             _p(grad_mlp), _p(dx))
    return loss, dx


def color_spec(W=64, H=2):
    """The colour network as a plain MLP: 32 inputs (SH 16 | geometry 15 |
    pad 1), sigmoid RGB, L2."""
    return make_spec(L=32, F=1, log2T=1, d=3, W=W, H=H, O=3, loss="L2",
                     grad_mode=GRAD_FLOAT)


def _color_input(dirs, dens):
    x = np.zeros((dirs.shape[0], 32), np.float32)
    x[:, :16] = sh4(dirs)
    x[:, 16:31] = dens[:, 1:16]
    return x


class OracleNerf:
    """CPU restatement of the NeRF-style field step (density HashGrid+MLP ->
    16 outputs, sigma = exp(out0); colour MLP on [SH(dir) | out 1..15 | 0]
    -> sigmoid RGB; loss sum_c (rgb-rgb_t)^2 + (sigma-sigma_t)^2 averaged;
    Adam on both).  Parity unpinned: the reference has no such network."""

    def __init__(self, sd, table, dmlp, cmlp, color_W=64, color_H=2, lr=1e-2):
        self.sd = sd
        self.sc = color_spec(color_W, color_H)
        self.w = np.concatenate([table, dmlp]).astype(np.float32)
        self.m = np.zeros_like(self.w)
        self.v = np.zeros_like(self.w)
        self.hc = table.size
        self.cw = np.array(cmlp, np.float32)
        self.cm = np.zeros_like(self.cw)
        self.cv = np.zeros_like(self.cw)
        self.lr = lr
        self.step = 0

    def inference(self, pos, dirs):
        dens = forward(self.sd, self.w[:self.hc], self.w[self.hc:], pos)
        z = mlp_forward(self.sc, self.cw, _color_input(dirs, dens))
        return 1.0 / (1.0 + np.exp(-z)), np.exp(dens[:, 0])

    def training_step(self, pos, dirs, rgb, sigma):
        N = pos.shape[0]
        table, dmlp = self.w[:self.hc].copy(), self.w[self.hc:].copy()
        dens = forward(self.sd, table, dmlp, pos)
        gc = np.zeros_like(self.cw)
        lc, dx = mlp_train(self.sc, self.cw, _color_input(dirs, dens), rgb, N,
                           1, gc)
        s = np.exp(dens[:, 0].astype(np.float32))
        r = (s - sigma).astype(np.float32)
        dy = np.zeros((N, 16), np.float32)
        dy[:, 0] = (np.float32(2.0) * r) * s * np.float32(1.0 / N)
        dy[:, 1:16] = dx[:, 16:31]
        ld = float(np.sum(r.astype(np.float64) ** 2))
        cfg = AdamCfg(self.lr, self.lr, 0.9, 0.99, 1e-15, 0.0, 0.0, 0.0, 0.0,
                      self.step, 0, 1)
        lib.tmo_adam(C.byref(cfg), _p(self.cw), _p(self.cm), _p(self.cv), 0,
                     self.cw.size, None, None, _p(gc), None, 1)
        _, g, _ = fwd_bwd(self.sd, table, dmlp, pos, None, d_out=dy)
        adam(self.sd, self.w, self.m, self.v, g, self.step, lr_hash=self.lr,
             lr_mlp=self.lr)
        self.step += 1
        return (lc + ld) / N


def nerf_batch(n, seed):
    """Seeded NeRF samples: positions U[0,1)^3, unit directions (normalised
    Gaussians), smooth targets: RGB = sigmoid of 8 random sinusoids of the
    position per channel plus a linear term in the direction; density =
    4 sigmoid(sum of 8 sinusoids)."""
    rng = np.random.default_rng(seed)
    pos = rng.random((n, 3), dtype=np.float32)
    d = rng.normal(size=(n, 3)).astype(np.float32)
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    fr = np.random.default_rng(1234)
    k = fr.normal(size=(4, 8, 3)) * 4.0
    ph = fr.uniform(0, 2 * np.pi, (4, 8))
    a = fr.normal(size=(4, 8)) * 0.5
    dirw = fr.normal(size=(3, 3)) * 0.3
    f = np.einsum("nd,ckd->nck", pos.astype(np.float64), k) + ph[None]
    f = (np.sin(f) * a[None]).sum(-1)  # [n, 4]
    rgb = 1.0 / (1.0 + np.exp(-(f[:, :3] + d.astype(np.float64) @ dirw)))
    sigma = 4.0 / (1.0 + np.exp(-f[:, 3]))
    return pos, d, rgb.astype(np.float32), sigma.astype(np.float32)
