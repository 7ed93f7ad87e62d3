"""tmnn_b200 -- Python front end of the B200 hot-path library (libtmnn_cuda.so).

Mirrors the reference's Python binding `tiny_metal_nn`
(src/python/tmnn_pybind.cpp:254-600, tiny_metal_nn/__init__.py):
``Trainer.from_config(config, n_input=..., n_output=...)``, ``training_step``,
``inference``, ``step``, ``close`` / context manager, and the typed errors
ClosedError, ConcurrentTrainingStepError, ConfigError (a ValueError) and
DTypeError (a TypeError).  It adds the rest of ITrainerRuntime
(include/tiny-metal-nn/trainer.h:136-219): the split / accumulation API,
optimizer-state export/import, weight access, the network plan and
data-parallel initialisation.

Arrays may be float32 C-contiguous numpy arrays (host, copied) or CUDA
torch tensors (device pointers, zero copy).  Every call goes through the
C ABI in include/tmnn_cuda.h; nothing here computes.
"""
from __future__ import annotations

import ctypes as C
import json
import threading

import numpy as np

from . import _abi
from ._abi import lib

__version__ = "0.1.0"
__all__ = ["Trainer", "ClosedError", "ConcurrentTrainingStepError",
           "ConfigError", "DTypeError", "TmnnError", "dp_unique_id", "NerfField",
           "__version__"]


class TmnnError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


class ClosedError(RuntimeError):
    pass


class ConcurrentTrainingStepError(RuntimeError):
    pass


class ConfigError(ValueError):
    pass


class DTypeError(TypeError):
    pass


def _check(status, what=""):
    if status == _abi.OK:
        return
    msg = _abi.last_error()
    if what:
        msg = f"{what}: {msg}"
    if status == _abi.ERR_CONCURRENT_CALL:
        raise ConcurrentTrainingStepError(msg)
    if status == _abi.ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise TmnnError(status, msg)


def _is_cuda_tensor(x):
    return type(x).__module__.startswith("torch") and getattr(x, "is_cuda", False)


def _arg(x, name, width):
    """(pointer, rows, flags, keepalive) for an input array."""
    if x is None:
        return None, 0, 0, None
    if _is_cuda_tensor(x):
        import torch
        if x.dtype != torch.float32:
            raise DTypeError(f"{name} must be float32")
        if not x.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if x.dim() != 2 or x.shape[1] != width:
            raise ValueError(f"{name} must be 2D (batch_size, {width})")
        return C.c_void_p(x.data_ptr()), x.shape[0], _abi.PTR_DEVICE, x
    if not isinstance(x, np.ndarray):
        x = np.asarray(x)
    if x.dtype != np.float32:
        raise DTypeError(f"{name} must be float32, got {x.dtype}")
    if not x.flags["C_CONTIGUOUS"]:
        raise ValueError(f"{name} must be C-contiguous")
    if x.ndim != 2 or x.shape[1] != width:
        raise ValueError(f"{name} must be 2D (batch_size, {width})")
    return x.ctypes.data_as(C.c_void_p), x.shape[0], 0, x


class FullyFusedMLP:
    """Standalone FullyFusedMLP inference on fp16 device inputs."""

    def __init__(self, n_input, width, hidden_layers, n_output, seed=42,
                 device=0):
        h = C.c_void_p()
        st = lib.tmnn_cuda_mlp_create(device, n_input, width, hidden_layers,
                                      n_output, seed, C.byref(h))
        if st != _abi.OK:
            raise ValueError(lib.tmnn_cuda_mlp_last_error().decode())
        self._h = h
        self.n_input, self.n_output = n_input, n_output
        self.count = (n_input * width + width +
                      (hidden_layers - 1) * (width * width + width) +
                      width * n_output + n_output)

    def weights(self):
        out = np.empty(self.count, np.float32)
        _check_mlp(lib.tmnn_cuda_mlp_weights(self._h, None,
                                             out.ctypes.data_as(C.c_void_p),
                                             self.count))
        return out

    def set_weights(self, w):
        w = np.ascontiguousarray(w, np.float32)
        _check_mlp(lib.tmnn_cuda_mlp_weights(self._h, w.ctypes.data_as(C.c_void_p),
                                             None, w.size))

    def forward(self, x_f16, out=None):
        """x_f16: CUDA torch.float16 [n, n_input]; returns fp32 [n, n_output]."""
        import torch
        assert x_f16.is_cuda and x_f16.dtype == torch.float16 and x_f16.is_contiguous()
        n = x_f16.shape[0]
        if out is None:
            out = torch.empty((n, self.n_output), dtype=torch.float32,
                              device=x_f16.device)
        _check_mlp(lib.tmnn_cuda_mlp_forward(self._h, C.c_void_p(x_f16.data_ptr()),
                                             C.c_void_p(out.data_ptr()), n))
        return out

    def stream(self):
        s = C.c_void_p()
        _check_mlp(lib.tmnn_cuda_mlp_stream(self._h, C.byref(s)))
        return s.value

    def close(self):
        if self._h is not None:
            lib.tmnn_cuda_mlp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check_mlp(st):
    if st != _abi.OK:
        raise TmnnError(st, lib.tmnn_cuda_mlp_last_error().decode())


class NerfField:
    """NeRF-style field: HashGrid density network (16 outputs, sigma =
    exp(out0)) + colour network on [SH4(dir) | geometry out 1..15] with
    sigmoid RGB, trained jointly (include/tmnn_cuda.h, tmnn_cuda_nerf_*)."""

    def __init__(self, n_levels=16, n_features_per_level=2,
                 log2_hashmap_size=19, base_resolution=16.0,
                 per_level_scale=1.382, density_width=64,
                 density_hidden_layers=1, color_width=64,
                 color_hidden_layers=2, lr=1e-2, seed=42, family="Auto",
                 table_dtype="F32", device=0):
        cfg = _abi.NerfCfg()
        cfg.density = _abi.Spec(n_levels, n_features_per_level,
                                log2_hashmap_size, 3, base_resolution,
                                per_level_scale, density_width,
                                density_hidden_layers, 16, 0, 1.0,
                                _abi.DTYPE_F16 if table_dtype == "F16"
                                else _abi.DTYPE_F32)
        cfg.lr = lr
        cfg.color_width = color_width
        cfg.color_hidden_layers = color_hidden_layers
        cfg.family = _abi.FAMILY[family]
        cfg.seed = seed
        h = C.c_void_p()
        st = lib.tmnn_cuda_nerf_create(device, C.byref(cfg), C.byref(h))
        if st != _abi.OK:
            msg = lib.tmnn_cuda_nerf_last_error().decode()
            if st == _abi.ERR_INVALID_ARGUMENT:
                raise ValueError(msg)
            raise TmnnError(st, msg)
        self._h = h
        self.color_count = (32 * color_width + color_width +
                            (color_hidden_layers - 1) *
                            (color_width * color_width + color_width) +
                            color_width * 3 + 3)
        d = C.c_void_p()
        _check_nerf(lib.tmnn_cuda_nerf_density(h, C.byref(d)))
        self.density = Trainer(d, 3, 16)
        self.density._borrowed = True

    def color_weights(self):
        out = np.empty(self.color_count, np.float32)
        _check_nerf(lib.tmnn_cuda_nerf_color_weights(
            self._h, None, out.ctypes.data_as(C.c_void_p), out.size))
        return out

    def set_color_weights(self, w):
        w = np.ascontiguousarray(w, np.float32)
        _check_nerf(lib.tmnn_cuda_nerf_color_weights(
            self._h, w.ctypes.data_as(C.c_void_p), None, w.size))

    def _args(self, *arrays):
        ptrs, flags, n = [], 0, None
        for a, w in arrays:
            p, rows, f, _k = _arg(a, "input", w) if w > 1 else _arg(
                a.reshape(-1, 1) if hasattr(a, "reshape") else a, "input", 1)
            if n is None:
                n, flags = rows, f
            elif rows != n or f != flags:
                raise ValueError("arrays must match in rows and placement")
            ptrs.append(p)
        return ptrs, n, flags

    def training_step(self, pos, dirs, rgb, sigma, profile=False):
        (pp, dp, cp, sp), n, flags = self._args((pos, 3), (dirs, 3), (rgb, 3),
                                                (sigma, 1))
        if profile:
            flags |= _abi.PROFILE
        loss = C.c_float()
        _check_nerf(lib.tmnn_cuda_nerf_train_step(self._h, pp, dp, cp, sp, n,
                                                  flags, C.byref(loss)))
        return loss.value

    def inference(self, pos, dirs):
        (pp, dp), n, flags = self._args((pos, 3), (dirs, 3))
        if flags & _abi.PTR_DEVICE:
            import torch
            rgb = torch.empty((n, 3), dtype=torch.float32, device=pos.device)
            sig = torch.empty((n,), dtype=torch.float32, device=pos.device)
            rp, sp = C.c_void_p(rgb.data_ptr()), C.c_void_p(sig.data_ptr())
        else:
            rgb = np.empty((n, 3), np.float32)
            sig = np.empty((n,), np.float32)
            rp = rgb.ctypes.data_as(C.c_void_p)
            sp = sig.ctypes.data_as(C.c_void_p)
        _check_nerf(lib.tmnn_cuda_nerf_inference(self._h, pp, dp, rp, sp, n,
                                                 flags))
        return rgb, sig

    def profile(self):
        """(phase milliseconds of the last profiled step, kernel launches)."""
        ms = (C.c_float * 4)()
        n = C.c_uint64()
        _check_nerf(lib.tmnn_cuda_nerf_profile(self._h, ms, C.byref(n)))
        return {"density_forward": ms[0], "color": ms[1],
                "density_backward": ms[2], "density_adam": ms[3]}, n.value

    def stream(self):
        return self.density.stream()

    def dp_init(self, unique_id: bytes, rank: int, world: int):
        """Data-parallel training over `world` ranks (one per GPU): each rank
        passes its shard of every batch; gradients and losses are summed
        over the ranks."""
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        _check_nerf(lib.tmnn_cuda_nerf_dp_init(self._h, buf, rank, world))

    def close(self):
        if self._h is not None:
            self.density.close()
            lib.tmnn_cuda_nerf_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check_nerf(st):
    if st == _abi.OK:
        return
    msg = lib.tmnn_cuda_nerf_last_error().decode()
    if st == _abi.ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise TmnnError(st, msg)


def dp_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _check(lib.tmnn_cuda_dp_unique_id(buf), "dp_unique_id")
    return bytes(buf)


class Trainer:
    """One trainer = one CUDA context on one GPU (tmnn::Trainer)."""

    def __init__(self, handle, n_input, n_output):
        self._h = handle
        self.n_input = n_input
        self.n_output = n_output
        self._lock = threading.Lock()
        plan = self.plan()
        self.hash_count = plan["hash_grid_size"]
        self.mlp_count = plan["mlp_weight_count"]
        self.last_result = None
        self._pending = []

    # ---------------------------------------------------------- creation
    @staticmethod
    def from_config(config, *, n_input, n_output, device=0):
        """tcnn-style config dict (or JSON text); see factory_json.h."""
        text = config if isinstance(config, str) else json.dumps(config)
        h = C.c_void_p()
        st = lib.tmnn_cuda_ctx_create_from_json(device, n_input, n_output,
                                                text.encode(), C.byref(h))
        if st == _abi.ERR_INVALID_ARGUMENT:
            raise ConfigError(_abi.last_error())
        _check(st, "from_config")
        return Trainer(h, n_input, n_output)

    @staticmethod
    def from_spec(spec: _abi.Spec, cfg: _abi.TrainCfg | None = None, device=0):
        h = C.c_void_p()
        _check(lib.tmnn_cuda_ctx_create(device, C.byref(spec),
                                        C.byref(cfg) if cfg else None,
                                        C.byref(h)), "create")
        return Trainer(h, spec.spatial_dims, spec.num_outputs)

    # ---------------------------------------------------------- lifetime
    def close(self):
        if self._h is not None:
            if not getattr(self, "_borrowed", False):
                _check(lib.tmnn_cuda_ctx_destroy(self._h), "close")
            self._h = None

    def closed(self):
        return self._h is None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _handle(self):
        if self._h is None:
            raise ClosedError("trainer is closed")
        return self._h

    def _guarded(self, fn):
        if not self._lock.acquire(blocking=False):
            raise ConcurrentTrainingStepError(
                "training_step is already in progress on another thread. "
                "Trainer is single-threaded; use one Trainer per thread.")
        try:
            return fn()
        finally:
            self._lock.release()

    # ---------------------------------------------------------- training
    def training_step(self, input, target, profile=False):
        """Fused forward + backward + Adam; returns the mean loss."""
        h = self._handle()
        pp, n, f1, _k1 = _arg(input, "input", self.n_input)
        tp, nt, f2, _k2 = _arg(target, "target", self.n_output)
        if n != nt:
            raise ValueError("input and target must have matching batch_size")
        if f1 != f2:
            raise ValueError("input and target must both be host or both CUDA")
        res = _abi.StepResult()
        flags = f1 | (_abi.PROFILE if profile else 0)
        self._guarded(lambda: _check(
            lib.tmnn_cuda_train_step(h, pp, tp, n, flags, C.byref(res)),
            "training_step"))
        self.last_result = res
        return res.loss

    def training_step_enqueue(self, input, target):
        """Queue one training step without waiting for it (two may be in
        flight; the upload of one overlaps the other's kernels).  The arrays
        are kept alive, and must not be modified, until the step is
        finalized.  Pair every call with training_step_finalize()."""
        h = self._handle()
        pp, n, f1, k1 = _arg(input, "input", self.n_input)
        tp, nt, f2, k2 = _arg(target, "target", self.n_output)
        if n != nt:
            raise ValueError("input and target must have matching batch_size")
        if f1 != f2:
            raise ValueError("input and target must both be host or both CUDA")
        self._guarded(lambda: _check(
            lib.tmnn_cuda_train_step_enqueue(h, pp, tp, n, f1),
            "training_step_enqueue"))
        self._pending.append((k1, k2))

    def training_step_finalize(self):
        """Wait for the oldest enqueued step; returns its mean loss."""
        h = self._handle()
        res = _abi.StepResult()
        self._guarded(lambda: _check(
            lib.tmnn_cuda_train_step_finalize(h, C.byref(res)),
            "training_step_finalize"))
        if self._pending:
            self._pending.pop(0)
        self.last_result = res
        return res.loss

    def last_numerics(self):
        """NumericsReport of the last training step (dict), with the
        recovery action the guard took."""
        r = self.last_result
        if r is None:
            return None
        return {"finite_forward": bool(r.finite_forward),
                "finite_backward": bool(r.finite_backward),
                "finite_update": bool(r.finite_update),
                "max_abs_gradient": r.max_abs_gradient,
                "max_abs_update": r.max_abs_update,
                "grad_norm": r.grad_norm,
                "probed": bool(r.numerics_probed),
                "reported": bool(r.numerics_reported),
                "anomaly": bool(r.has_numerics_anomaly),
                "recovery_action": _abi.RECOVERY_ACTION[r.recovery_action]}

    def last_probe(self):
        """ProbeResult of the last training_step / forward_backward (dict:
        per-hidden-layer activation max and gradient sum of squares, output
        range, NaN flags), or None when enable_probes is off or no pass has
        run (TrainingStepResult.probe / read_last_split_probe)."""
        r = _abi.ProbeResult()
        st = lib.tmnn_cuda_last_probe(self._handle(), C.byref(r))
        if st != _abi.OK:
            return None
        H = r.num_hidden_layers
        return {"num_hidden_layers": H,
                "has_nan_forward": bool(r.has_nan_forward),
                "has_nan_backward": bool(r.has_nan_backward),
                "hash_grad_l2": r.hash_grad_l2,
                "act_max": list(r.act_max)[:H], "grad_l2": list(r.grad_l2)[:H],
                "output_abs_max": r.output_abs_max,
                "output_min": r.output_min}

    def numerics_stats(self):
        """Counters of the numerics guard (dict)."""
        s = _abi.NumericsStats()
        _check(lib.tmnn_cuda_get_numerics_stats(self._handle(), C.byref(s)),
               "numerics_stats")
        return {k: getattr(s, k) for k, _ in s._fields_}

    def forward_backward(self, input, target):
        """Accumulate gradients of the internal loss (no optimizer step);
        returns the summed loss of the batch."""
        h = self._handle()
        pp, n, f1, _k1 = _arg(input, "input", self.n_input)
        tp, nt, f2, _k2 = _arg(target, "target", self.n_output)
        if n != nt or f1 != f2:
            raise ValueError("input and target must match")
        out = C.c_double()
        self._guarded(lambda: _check(lib.tmnn_cuda_forward_backward(
            h, pp, tp, n, f1, C.byref(out)), "forward_backward"))
        return out.value

    def read_buffer(self, role):
        """Host copy of a runtime buffer as a numpy array."""
        _ptr, nbytes, dt = self.buffer(role)
        arr = np.empty(nbytes // [4, 2, 4, 1][dt],
                       [np.float32, np.float16, np.int32, np.uint8][dt])
        h = self._handle()
        self._guarded(lambda: _check(lib.tmnn_cuda_read_buffer(
            h, role, arr.ctypes.data_as(C.c_void_p), nbytes), "read_buffer"))
        return arr

    def forward_for_training(self, input):
        return self._forward(input, lib.tmnn_cuda_forward)

    def zero_gradients(self):
        h = self._handle()
        self._guarded(lambda: _check(lib.tmnn_cuda_zero_grads(h)))

    def backward_accumulate(self, input, d_output):
        h = self._handle()
        pp, n, f1, _k1 = _arg(input, "input", self.n_input)
        dp, nd, f2, _k2 = _arg(d_output, "d_output", self.n_output)
        if n != nd or f1 != f2:
            raise ValueError("input and d_output must match")
        self._guarded(lambda: _check(
            lib.tmnn_cuda_backward_accumulate(h, pp, dp, n, f1),
            "backward_accumulate"))

    def adam_step(self):
        h = self._handle()
        self._guarded(lambda: _check(lib.tmnn_cuda_adam_step(h), "adam_step"))

    # ---------------------------------------------------------- inference
    def _forward(self, input, fn, out=None):
        h = self._handle()
        pp, n, flags, _k = _arg(input, "input", self.n_input)
        if flags & _abi.PTR_DEVICE:
            import torch
            if out is None:
                out = torch.empty((n, self.n_output), dtype=torch.float32,
                                  device=input.device)
            optr = C.c_void_p(out.data_ptr())
        else:
            out = np.empty((n, self.n_output), np.float32) if out is None else out
            optr = out.ctypes.data_as(C.c_void_p)
        self._guarded(lambda: _check(fn(h, pp, optr, n, flags), "inference"))
        return out

    def inference(self, input, out=None):
        return self._forward(input, lib.tmnn_cuda_evaluate, out)

    evaluate = inference

    def evaluate_with_gradient(self, input, out=None, gradients=None):
        """(values [N, 1], gradients [N, n_input]) of a single-output field:
        the value and d(value)/d(position) (Trainer::evaluate_with_gradient,
        trainer.h:378-386).  Host arrays or CUDA tensors, like inference()."""
        h = self._handle()
        pp, n, flags, _k = _arg(input, "input", self.n_input)
        if flags & _abi.PTR_DEVICE:
            import torch
            if out is None:
                out = torch.empty((n, self.n_output), dtype=torch.float32,
                                  device=input.device)
            if gradients is None:
                gradients = torch.empty((n, self.n_input), dtype=torch.float32,
                                        device=input.device)
            optr = C.c_void_p(out.data_ptr())
            gptr = C.c_void_p(gradients.data_ptr())
        else:
            if out is None:
                out = np.empty((n, self.n_output), np.float32)
            if gradients is None:
                gradients = np.empty((n, self.n_input), np.float32)
            optr = out.ctypes.data_as(C.c_void_p)
            gptr = gradients.ctypes.data_as(C.c_void_p)
        self._guarded(lambda: _check(lib.tmnn_cuda_evaluate_with_gradient(
            h, pp, optr, gptr, n, flags), "evaluate_with_gradient"))
        return out, gradients

    inference_with_gradient = evaluate_with_gradient

    def debug_morton_order(self, input, key_bits=0):
        """Device Morton permutation of a host batch (parity instrument)."""
        h = self._handle()
        pp, n, flags, _k = _arg(input, "input", self.n_input)
        if flags:
            raise ValueError("debug_morton_order takes host arrays")
        perm = np.zeros(n, np.uint32)
        self._guarded(lambda: _check(lib.tmnn_cuda_debug_morton_order(
            h, pp, n, key_bits, perm.ctypes.data_as(C.c_void_p)),
            "debug_morton_order"))
        return perm

    def debug_encode(self, input):
        """(features, corner_index, cells) of the encoding (host arrays)."""
        h = self._handle()
        pp, n, flags, _k = _arg(input, "input", self.n_input)
        if flags:
            raise ValueError("debug_encode takes host arrays")
        plan = self.plan()
        L, F, d = plan["n_levels"], plan["n_features_per_level"], self.n_input
        feat = np.zeros((n, L * F), np.float32)
        idx = np.zeros((n, L, 1 << d), np.uint32)
        cells = np.zeros((n, L, d), np.int32)
        self._guarded(lambda: _check(lib.tmnn_cuda_debug_encode(
            h, pp, n, feat.ctypes.data_as(C.c_void_p),
            idx.ctypes.data_as(C.c_void_p), cells.ctypes.data_as(C.c_void_p)),
            "debug_encode"))
        return feat, idx, cells

    # ---------------------------------------------------------- state
    def is_gpu_available(self):
        """True while the trainer holds its CUDA device (the reference's
        Trainer.is_gpu_available, src/python/tmnn_pybind.cpp:337-342)."""
        self._handle()
        return True

    def step(self):
        s = C.c_uint32()
        _check(lib.tmnn_cuda_get_step(self._handle(), C.byref(s)))
        return s.value

    def set_initial_weights(self, hash_weights=None, mlp_weights=None):
        h = self._handle()
        hw = None if hash_weights is None else np.ascontiguousarray(hash_weights, np.float32)
        mw = None if mlp_weights is None else np.ascontiguousarray(mlp_weights, np.float32)
        self._guarded(lambda: _check(lib.tmnn_cuda_set_initial_weights(
            h, None if hw is None else hw.ctypes.data_as(C.c_void_p),
            0 if hw is None else hw.size,
            None if mw is None else mw.ctypes.data_as(C.c_void_p),
            0 if mw is None else mw.size), "set_initial_weights"))

    def weights(self):
        """(hash, mlp) host copies of the live fp32 weights."""
        h = self._handle()
        hw = np.empty(self.hash_count, np.float32)
        mw = np.empty(self.mlp_count, np.float32)
        self._guarded(lambda: _check(lib.tmnn_cuda_get_weights(
            h, hw.ctypes.data_as(C.c_void_p), hw.size,
            mw.ctypes.data_as(C.c_void_p), mw.size), "get_weights"))
        return hw, mw

    def export_optimizer_state(self):
        """(step, payload bytes) of OptimizerStateBlob v1."""
        h = self._handle()
        n = C.c_size_t()
        st = C.c_uint32()
        _check(lib.tmnn_cuda_export_opt_state(h, None, 0, C.byref(n), C.byref(st)))
        buf = (C.c_uint8 * n.value)()
        self._guarded(lambda: _check(lib.tmnn_cuda_export_opt_state(
            h, buf, n.value, C.byref(n), C.byref(st)), "export_optimizer_state"))
        return st.value, bytes(buf)

    def import_optimizer_state(self, step, payload: bytes):
        h = self._handle()
        buf = (C.c_uint8 * len(payload)).from_buffer_copy(payload)
        self._guarded(lambda: _check(lib.tmnn_cuda_import_opt_state(
            h, buf, len(payload), step), "import_optimizer_state"))

    def reset_optimizer(self):
        h = self._handle()
        self._guarded(lambda: _check(lib.tmnn_cuda_reset_optimizer(h)))

    def buffer(self, role):
        v = _abi.BufferView()
        _check(lib.tmnn_cuda_get_buffer(self._handle(), role, C.byref(v)),
               "buffer")
        return v.device_ptr, v.bytes, v.dtype

    def plan(self):
        p = _abi.Plan()
        _check(lib.tmnn_cuda_get_plan(self._handle(), C.byref(p)), "plan")
        return {"family": _abi.FAMILY_NAME.get(p.family, str(p.family)),
                "fallback_reason": p.fallback_reason,
                "mlp_weight_count": p.mlp_weight_count,
                "hash_grid_size": p.hash_grid_size,
                "device_bytes": p.device_bytes,
                "n_levels": p.n_levels,
                "n_features_per_level": p.n_features_per_level,
                "reason": p.reason.decode()}

    def stream(self):
        s = C.c_void_p()
        _check(lib.tmnn_cuda_get_stream(self._handle(), C.byref(s)))
        return s.value

    def synchronize(self):
        _check(lib.tmnn_cuda_synchronize(self._handle()))

    def launch_count(self):
        n = C.c_uint64()
        _check(lib.tmnn_cuda_launch_count(self._handle(), C.byref(n)))
        return n.value

    def dp_sync_state(self):
        """Collective: gather the sharded optimizer state on every rank."""
        h = self._handle()
        self._guarded(lambda: _check(lib.tmnn_cuda_dp_sync_state(h),
                                     "dp_sync_state"))

    def dp_init(self, unique_id: bytes, rank: int, world: int):
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        h = self._handle()
        self._guarded(lambda: _check(lib.tmnn_cuda_dp_init(h, buf, rank, world),
                                     "dp_init"))
