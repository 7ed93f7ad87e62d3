"""ctypes access to oracle/_ref: the reference's own code compiled here
(its generated MSL kernels run as C++ through oracle/ref/metal_shim.h, and its
host helpers).  TEST INFRASTRUCTURE ONLY: used to pin the CPU restatement and
as the reference arm of bench.py.  Build with oracle/ref_build.py.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

P = C.c_void_p


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def available(tag="host"):
    return os.path.exists(os.path.join(REF_DIR, f"libtmnn_ref_{tag}.so"))


_cache = {}


def _lib(tag):
    if tag not in _cache:
        _cache[tag] = C.CDLL(os.path.join(REF_DIR, f"libtmnn_ref_{tag}.so"))
    return _cache[tag]


def spec_tuple(tag):
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "tmnn_ref_build", os.path.join(HERE, "ref_build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.SPECS[tag]


def _config(L, F, log2T, base, scale, W, H, N, mlp):
    return np.concatenate([np.array([L, F, log2T, base, scale, W, H, N],
                                    np.float32), mlp]).astype(np.float32)


def train(tag, sp, table, mlp, pos, tgt, d_out=None, active_levels=0):
    """Runs the reference's scalar train kernel (or its ExternalGrad twin when
    d_out is given).  Returns dict(loss_partials, grad_hash[int32],
    grad_mlp, mask_words, summary_words)."""
    L, F, log2T, d, W, H, O = sp[:7]
    lib = _lib(tag)
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    tgt = np.ascontiguousarray(tgt, np.float32) if tgt is not None else \
        np.zeros((N, O), np.float32)
    cfg = _config(L, F, log2T, sp[8], sp[9], W, H, N, mlp)
    gh = np.zeros(table.size, np.int32)
    gm = np.zeros(mlp.size, np.float32)
    tgs = (N + 127) // 128
    lp = np.zeros(max(tgs, 1), np.float32)
    tp = np.array([N, 0, 1.0, active_levels if active_levels > 0 else L, 0, 0,
                   0, 0], np.float32)
    slots = table.size // 2 if F == 2 else table.size
    mask = np.zeros((slots + 31) // 32, np.uint32)
    summ = np.zeros((slots + 2047) // 2048 + 1, np.uint32)
    table = np.ascontiguousarray(table, np.float32)
    mlp = np.ascontiguousarray(mlp, np.float32)
    if d_out is None:
        lib.tmnn_ref_train(_p(pos), _p(tgt), _p(cfg), _p(table), _p(gh),
                           _p(gm), _p(lp), _p(tp), _p(mask), _p(summ),
                           _p(mlp), C.c_uint32(N))
    else:
        d_out = np.ascontiguousarray(d_out, np.float32)
        lib.tmnn_ref_extgrad(_p(pos), _p(tgt), _p(cfg), _p(table), _p(gh),
                             _p(gm), _p(lp), _p(tp), _p(d_out), _p(mask),
                             _p(summ), _p(mlp), C.c_uint32(N))
    return dict(loss_partials=lp, grad_hash=gh, grad_mlp=gm, mask=mask,
                summary=summ)


def has_simd_train(tag):
    """Whether the reference's compiler realises the simdgroup-matrix
    training kernel for spec `tag` (then its default training kernel)."""
    return available(tag) and hasattr(_lib(tag), "tmnn_ref_train_simd")


def train_simd(tag, sp, table, mlp, pos, tgt, active_levels=0):
    """Runs the reference's simdgroup-matrix train kernel (threadgroups of
    32 threads over 64 points, 8-row simdgroup tiles).  Same outputs as
    train()."""
    L, F, log2T, d, W, H, O = sp[:7]
    lib = _lib(tag)
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    tgt = np.ascontiguousarray(tgt, np.float32)
    cfg = _config(L, F, log2T, sp[8], sp[9], W, H, N, mlp)
    gh = np.zeros(table.size, np.int32)
    gm = np.zeros(mlp.size, np.float32)
    lib.tmnn_ref_train_simd_points_per_tg.restype = C.c_uint32
    per = lib.tmnn_ref_train_simd_points_per_tg()
    tgs = (N + per - 1) // per
    lp = np.zeros(max(tgs, 1), np.float32)
    tp = np.array([N, 0, 1.0, active_levels if active_levels > 0 else L, 0, 0,
                   0, 0], np.float32)
    slots = table.size // 2 if F == 2 else table.size
    mask = np.zeros((slots + 31) // 32, np.uint32)
    summ = np.zeros((slots + 2047) // 2048 + 1, np.uint32)
    table = np.ascontiguousarray(table, np.float32)
    mlp = np.ascontiguousarray(mlp, np.float32)
    lib.tmnn_ref_train_simd(_p(pos), _p(tgt), _p(cfg), _p(table), _p(gh),
                            _p(gm), _p(lp), _p(tp), _p(mask), _p(summ),
                            _p(mlp), C.c_uint32(N))
    return dict(loss_partials=lp, grad_hash=gh, grad_mlp=gm, mask=mask,
                summary=summ)


def train_lanes(tag, sp, table, mlp, pos, tgt, lanes=8):
    """Runs the reference's scalar training kernel for a bench_* spec with up
    to `lanes` emulated threadgroups at once.  Same outputs as train(); the
    float MLP-gradient sums may differ in order."""
    L, F, log2T, d, W, H, O = sp[:7]
    lib = _lib(tag)
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    tgt = np.ascontiguousarray(tgt, np.float32)
    cfg = _config(L, F, log2T, sp[8], sp[9], W, H, N, mlp)
    gh = np.zeros(table.size, np.int32)
    gm = np.zeros(mlp.size, np.float32)
    tgs = (N + 127) // 128
    lp = np.zeros(max(tgs, 1), np.float32)
    tp = np.array([N, 0, 1.0, L, 0, 0, 0, 0], np.float32)
    slots = table.size // 2 if F == 2 else table.size
    mask = np.zeros((slots + 31) // 32, np.uint32)
    summ = np.zeros((slots + 2047) // 2048 + 1, np.uint32)
    table = np.ascontiguousarray(table, np.float32)
    mlp = np.ascontiguousarray(mlp, np.float32)
    lib.tmnn_ref_train_lanes(_p(pos), _p(tgt), _p(cfg), _p(table), _p(gh),
                             _p(gm), _p(lp), _p(tp), _p(mask), _p(summ),
                             _p(mlp), C.c_uint32(N), C.c_uint32(lanes))
    return dict(loss_partials=lp, grad_hash=gh, grad_mlp=gm, mask=mask,
                summary=summ)


def train_lanes_max(tag):
    """How many threadgroups train_lanes can run at once."""
    lib = _lib(tag)
    lib.tmnn_ref_train_lanes_max.restype = C.c_uint32
    return int(lib.tmnn_ref_train_lanes_max())


def mask_to_touched(mask, slots):
    bits = np.unpackbits(mask.view(np.uint8), bitorder="little")
    return bits[:slots].astype(np.uint8)


def evaluate(tag, sp, table, mlp, pos):
    L, F, log2T, d, W, H, O = sp[:7]
    lib = _lib(tag)
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    cfg = _config(L, F, log2T, sp[8], sp[9], W, H, N, mlp)
    out = np.zeros((N, O), np.float32)
    lib.tmnn_ref_eval(_p(pos), _p(out), _p(cfg),
                      _p(np.ascontiguousarray(table, np.float32)),
                      _p(np.ascontiguousarray(mlp, np.float32)),
                      C.c_uint32(N))
    return out


def eval_gradient(tag, sp, table, mlp, pos):
    """The reference's EvalGradient kernel: returns its raw [N x 4] output
    (value, then d/dx, d/dy, d/dz -- in 4D the fourth component is not
    written by the kernel)."""
    L, F, log2T, d, W, H, O = sp[:7]
    lib = _lib(tag)
    pos = np.ascontiguousarray(pos, np.float32)
    N = pos.shape[0]
    cfg = _config(L, F, log2T, sp[8], sp[9], W, H, N, mlp)
    out = np.zeros((N, 4), np.float32)
    lib.tmnn_ref_eval_gradient(_p(pos), _p(out), _p(cfg),
                               _p(np.ascontiguousarray(table, np.float32)),
                               _p(np.ascontiguousarray(mlp, np.float32)),
                               C.c_uint32(N))
    return out


def adam_params(lr_enc, lr_net, b1, b2, eps, l1, l2, hash_size, mlp_count,
                step, clip=0.0, wd=0.0):
    lib = _lib("host")
    out = np.zeros(13, np.float32)
    f = C.c_float
    lib.tmnn_ref_adam_params(_p(out), f(lr_enc), f(lr_net), f(b1), f(b2),
                             f(eps), f(l1), f(l2), C.c_uint32(hash_size),
                             C.c_uint32(mlp_count), C.c_uint32(step), f(clip),
                             f(wd))
    return out


def adam_unified(w, gh, gm, m, v, params):
    lib = _lib("static")
    lib.tmnn_ref_adam_unified(_p(w), _p(gh), _p(gm), _p(m), _p(v), _p(params),
                              C.c_uint32(w.size))


def adam_sparse(w, gh, m, v, params, idx):
    lib = _lib("static")
    lib.tmnn_ref_adam_sparse(_p(w), _p(gh), _p(m), _p(v), _p(params),
                             _p(idx), C.c_uint32(idx.size))


def adam_dense(w, g, m, v, params):
    lib = _lib("static")
    lib.tmnn_ref_adam_dense(_p(w), _p(g), _p(m), _p(v), _p(params),
                            C.c_uint32(w.size))


def init_uniform(count, low, high, seed, counter_base=0):
    out = np.zeros(count, np.float32)
    _lib("static").tmnn_ref_init_uniform(
        _p(out), C.c_uint32(seed & 0xFFFFFFFF), C.c_uint32(seed >> 32),
        C.c_uint32(counter_base), C.c_uint32(count), C.c_float(low),
        C.c_float(high))
    return out


def init_normal(count, mean, std, seed, counter_base=0):
    out = np.zeros(count, np.float32)
    _lib("static").tmnn_ref_init_normal(
        _p(out), C.c_uint32(seed & 0xFFFFFFFF), C.c_uint32(seed >> 32),
        C.c_uint32(counter_base), C.c_uint32(count), C.c_float(mean),
        C.c_float(std))
    return out


def morton3(x, y, z):
    f = _lib("host").tmnn_ref_morton3
    f.restype = C.c_uint32
    return f(C.c_float(x), C.c_float(y), C.c_float(z))


def morton4(x, y, z, w):
    f = _lib("host").tmnn_ref_morton4
    f.restype = C.c_uint32
    return f(C.c_float(x), C.c_float(y), C.c_float(z), C.c_float(w))


def morton_sort(pos, tgt):
    pos = np.ascontiguousarray(pos, np.float32)
    tgt = np.ascontiguousarray(tgt, np.float32).reshape(pos.shape[0], -1)
    po = np.zeros_like(pos)
    to = np.zeros_like(tgt)
    _lib("host").tmnn_ref_morton_sort(_p(pos), _p(tgt), C.c_int(pos.shape[0]),
                                      C.c_int(pos.shape[1]),
                                      C.c_int(tgt.shape[1]), _p(po), _p(to))
    return po, to


def mlp_weight_count(In, W, H, O):
    return _lib("host").tmnn_ref_mlp_weight_count(In, W, H, O)


def validate(L, F, log2T, d, W, H, O, loss=0, huber=1.0):
    buf = C.create_string_buffer(256)
    rc = _lib("host").tmnn_ref_validate(L, F, log2T, d, W, H, O, loss,
                                        C.c_float(huber), buf, 256)
    return rc == 0, buf.value.decode()
