"""Helpers shared by the parity tests: build matching CUDA trainers and
oracle specs from one description."""
import numpy as np

import oracle as o

LOSS_NAMES = {0: "L2", 1: "L1", 2: "Huber", 3: "Cosine"}


def cuda_trainer(L=16, F=2, log2T=19, d=3, W=64, H=1, O=1, loss=0, base=16.0,
                 scale=1.447, huber=1.0, family="SafeDebug", grad="Fixed16",
                 table="F32", morton=True, seed=42, lr_enc=1e-2, lr_net=1e-3,
                 l1=0.0, l2=0.0, batch=1024, sparse=None, device=0,
                 cfg_extra=None):
    import tmnn_b200 as t
    from tmnn_b200 import _abi
    spec = _abi.Spec(L, F, log2T, d, base, scale, W, H, O, loss, huber,
                     _abi.DTYPE_F16 if table == "F16" else _abi.DTYPE_F32)
    cfg = _abi.TrainCfg()
    t.lib.tmnn_cuda_default_train_cfg(cfg)
    cfg.family = _abi.FAMILY[family]
    cfg.hash_grad_format = {"Fixed16": _abi.GRAD_FIXED16, "F32": _abi.GRAD_F32,
                            "F16": _abi.GRAD_F16}[grad]
    cfg.morton_sort = 1 if morton else 0
    cfg.seed = seed
    cfg.lr_encoding = lr_enc
    cfg.lr_network = lr_net
    cfg.l1_reg = l1
    cfg.l2_reg = l2
    cfg.batch_size = batch
    if sparse is not None:
        cfg.sparse_hash_adam = 1 if sparse else 0
    for k, v in (cfg_extra or {}).items():
        setattr(cfg, k, v)
    return t.Trainer.from_spec(spec, cfg, device=device)


def oracle_spec(L=16, F=2, log2T=19, d=3, W=64, H=1, O=1, loss=0, base=16.0,
                scale=1.447, huber=1.0, grad="Fixed16", res_mode=0, **_):
    return o.make_spec(L=L, F=F, log2T=log2T, d=d, W=W, H=H, O=O, loss=loss,
                       base=base, scale=scale, huber_delta=huber,
                       grad_mode=o.GRAD_FIXED16 if grad == "Fixed16" else o.GRAD_FLOAT,
                       res_mode=res_mode)


def spec_kwargs_from_tuple(sp):
    L, F, log2T, d, W, H, O, loss, base, scale, huber = sp
    return dict(L=int(L), F=int(F), log2T=int(log2T), d=int(d), W=int(W),
                H=int(H), O=int(O), loss=int(loss), base=float(base),
                scale=float(scale), huber=float(huber))


def batch(N, d, O, seed=0, lo=-1.0):
    rng = np.random.default_rng(seed)
    pos = rng.uniform(lo, 1.0, (N, d)).astype(np.float32)
    tgt = rng.normal(size=(N, O)).astype(np.float32)
    return pos, tgt
