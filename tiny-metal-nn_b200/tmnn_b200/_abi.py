"""ctypes declarations of include/tmnn_cuda.h (libtmnn_cuda.so, built in-tree).

Importing this module loads the CUDA library; there is no fallback: if the
library is missing the import fails with instructions to build it.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libtmnn_cuda.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_CONCURRENT_CALL = 17

FAMILY = {"Auto": -1, "FullyFused": 0, "Tiled": 1, "SafeDebug": 2}
FAMILY_NAME = {v: k for k, v in FAMILY.items()}
PTR_DEVICE = 1
PROFILE = 2
BUF_HASH_WEIGHTS, BUF_MLP_WEIGHTS, BUF_GRAD_HASH, BUF_GRAD_MLP = 1, 2, 3, 4
BUF_FUSED_WEIGHTS, BUF_FUSED_M, BUF_FUSED_V = 7, 8, 9
BUF_HASH_GATHER, BUF_TOUCHED = 20, 21
LOSS = {"L2": 0, "L1": 1, "Huber": 2, "Cosine": 3}
GRAD_FIXED16, GRAD_F32, GRAD_F16 = 0, 1, 2
DTYPE_F32, DTYPE_F16 = 0, 1


class Spec(C.Structure):
    _fields_ = [("n_levels", C.c_int32), ("n_features_per_level", C.c_int32),
                ("log2_hashmap_size", C.c_int32), ("spatial_dims", C.c_int32),
                ("base_resolution", C.c_float), ("per_level_scale", C.c_float),
                ("hidden_dim", C.c_int32), ("num_hidden_layers", C.c_int32),
                ("num_outputs", C.c_int32), ("loss", C.c_int32),
                ("huber_delta", C.c_float), ("table_dtype", C.c_int32)]


class TrainCfg(C.Structure):
    _fields_ = [("batch_size", C.c_int32), ("lr_encoding", C.c_float),
                ("lr_network", C.c_float), ("beta1", C.c_float),
                ("beta2", C.c_float), ("epsilon", C.c_float),
                ("l1_reg", C.c_float), ("l2_reg", C.c_float),
                ("grad_clip", C.c_float), ("weight_decay", C.c_float),
                ("hash_init", C.c_int32), ("hash_init_range", C.c_float),
                ("mlp_init", C.c_int32), ("mlp_nonlinearity", C.c_int32),
                ("mlp_uniform_range", C.c_float),
                ("mlp_normal_stddev", C.c_float), ("mlp_kaiming_a", C.c_float),
                ("seed", C.c_uint64), ("family", C.c_int32),
                ("hash_grad_format", C.c_int32), ("morton_sort", C.c_int32),
                ("sparse_hash_adam", C.c_int32), ("active_levels", C.c_int32),
                ("dp_replicated_optimizer", C.c_int32),
                ("numerics_sampling_mode", C.c_int32),
                ("numerics_sample_interval", C.c_int32),
                ("bad_step_recovery", C.c_int32),
                ("morton_key_bits", C.c_int32),
                ("enable_probes", C.c_int32), ("reserved", C.c_int32)]


class StepResult(C.Structure):
    _fields_ = [("loss", C.c_float), ("step", C.c_uint32),
                ("batch_size", C.c_uint32), ("numerics_ok", C.c_int32),
                ("gpu_ms", C.c_float), ("family", C.c_int32),
                ("sort_ms", C.c_float), ("fwd_bwd_ms", C.c_float),
                ("allreduce_ms", C.c_float), ("adam_ms", C.c_float),
                ("grad_norm", C.c_float), ("finite_forward", C.c_int32),
                ("finite_backward", C.c_int32), ("finite_update", C.c_int32),
                ("max_abs_gradient", C.c_float), ("max_abs_update", C.c_float),
                ("numerics_probed", C.c_int32),
                ("numerics_reported", C.c_int32),
                ("has_numerics_anomaly", C.c_int32),
                ("recovery_action", C.c_int32)]


class NerfCfg(C.Structure):
    _fields_ = [("density", Spec), ("lr", C.c_float),
                ("color_width", C.c_uint32),
                ("color_hidden_layers", C.c_uint32), ("family", C.c_int32),
                ("seed", C.c_uint64)]


class NumericsStats(C.Structure):
    _fields_ = [("reports", C.c_uint64), ("anomalies", C.c_uint64),
                ("skipped", C.c_uint64), ("rolled_back", C.c_uint64),
                ("safe_family_recoveries", C.c_uint64),
                ("last_anomaly_step", C.c_uint32),
                ("safe_family_active", C.c_int32)]


SAMPLING = {"Sampled": 0, "Periodic": 1, "FullPerStep": 2, "Disabled": 3}
BAD_STEP = {"SignalOnly": 0, "Throw": 1, "Skip": 2, "Rollback": 3,
            "FallbackAndRetryWithSafeFamily": 4}
RECOVERY_ACTION = {0: "None", 1: "Skipped", 2: "RolledBack",
                   3: "RetriedWithSafeFamily"}


class ProbeResult(C.Structure):
    _fields_ = [("num_hidden_layers", C.c_uint32),
                ("has_nan_forward", C.c_int32), ("has_nan_backward", C.c_int32),
                ("hash_grad_l2", C.c_float), ("act_max", C.c_float * 8),
                ("grad_l2", C.c_float * 8), ("output_abs_max", C.c_float),
                ("output_min", C.c_float)]


class BufferView(C.Structure):
    _fields_ = [("device_ptr", C.c_void_p), ("bytes", C.c_size_t),
                ("dtype", C.c_int32)]


class Plan(C.Structure):
    _fields_ = [("family", C.c_int32), ("fallback_reason", C.c_int32),
                ("mlp_weight_count", C.c_uint32),
                ("hash_grid_size", C.c_uint64), ("device_bytes", C.c_uint64),
                ("n_levels", C.c_int32), ("n_features_per_level", C.c_int32),
                ("spatial_dims", C.c_int32), ("num_outputs", C.c_int32),
                ("reason", C.c_char * 128)]


# (name, restype, argtypes) for every entry point of include/tmnn_cuda.h
P = C.c_void_p
u32 = C.c_uint32
_SIGS = [
    ("tmnn_cuda_default_train_cfg", None, [C.POINTER(TrainCfg)]),
    ("tmnn_cuda_validate_spec", C.c_int, [C.POINTER(Spec)]),
    ("tmnn_cuda_ctx_create", C.c_int,
     [C.c_int, C.POINTER(Spec), C.POINTER(TrainCfg), C.POINTER(P)]),
    ("tmnn_cuda_ctx_create_from_json", C.c_int,
     [C.c_int, u32, u32, C.c_char_p, C.POINTER(P)]),
    ("tmnn_cuda_ctx_destroy", C.c_int, [P]),
    ("tmnn_cuda_set_initial_weights", C.c_int, [P, P, C.c_size_t, P, C.c_size_t]),
    ("tmnn_cuda_get_weights", C.c_int, [P, P, C.c_size_t, P, C.c_size_t]),
    ("tmnn_cuda_train_step", C.c_int, [P, P, P, u32, u32, C.POINTER(StepResult)]),
    ("tmnn_cuda_train_step_enqueue", C.c_int, [P, P, P, u32, u32]),
    ("tmnn_cuda_train_step_finalize", C.c_int, [P, C.POINTER(StepResult)]),
    ("tmnn_cuda_forward_backward", C.c_int,
     [P, P, P, u32, u32, C.POINTER(C.c_double)]),
    ("tmnn_cuda_read_buffer", C.c_int, [P, C.c_int32, P, C.c_size_t]),
    ("tmnn_cuda_forward_backward_noalloc", C.c_int,
     [P, P, P, u32, C.POINTER(C.c_double)]),
    ("tmnn_cuda_forward", C.c_int, [P, P, P, u32, u32]),
    ("tmnn_cuda_zero_grads", C.c_int, [P]),
    ("tmnn_cuda_backward_accumulate", C.c_int, [P, P, P, u32, u32]),
    ("tmnn_cuda_adam_step", C.c_int, [P]),
    ("tmnn_cuda_evaluate", C.c_int, [P, P, P, u32, u32]),
    ("tmnn_cuda_evaluate_with_gradient", C.c_int, [P, P, P, P, u32, u32]),
    ("tmnn_cuda_get_numerics_stats", C.c_int, [P, C.POINTER(NumericsStats)]),
    ("tmnn_cuda_debug_morton_order", C.c_int, [P, P, u32, C.c_int32, P]),
    ("tmnn_cuda_debug_encode", C.c_int, [P, P, u32, P, P, P]),
    ("tmnn_cuda_export_opt_state", C.c_int,
     [P, P, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(u32)]),
    ("tmnn_cuda_import_opt_state", C.c_int, [P, P, C.c_size_t, u32]),
    ("tmnn_cuda_reset_optimizer", C.c_int, [P]),
    ("tmnn_cuda_get_step", C.c_int, [P, C.POINTER(u32)]),
    ("tmnn_cuda_get_buffer", C.c_int, [P, C.c_int32, C.POINTER(BufferView)]),
    ("tmnn_cuda_last_probe", C.c_int, [P, C.POINTER(ProbeResult)]),
    ("tmnn_cuda_get_plan", C.c_int, [P, C.POINTER(Plan)]),
    ("tmnn_cuda_get_stream", C.c_int, [P, C.POINTER(P)]),
    ("tmnn_cuda_synchronize", C.c_int, [P]),
    ("tmnn_cuda_dp_unique_id", C.c_int, [P]),
    ("tmnn_cuda_dp_init", C.c_int, [P, P, C.c_int, C.c_int]),
    ("tmnn_cuda_dp_sync_state", C.c_int, [P]),
    ("tmnn_cuda_mlp_create", C.c_int,
     [C.c_int, u32, u32, u32, u32, C.c_uint64, C.POINTER(P)]),
    ("tmnn_cuda_mlp_destroy", C.c_int, [P]),
    ("tmnn_cuda_mlp_weights", C.c_int, [P, P, P, C.c_size_t]),
    ("tmnn_cuda_mlp_forward", C.c_int, [P, P, P, u32]),
    ("tmnn_cuda_mlp_stream", C.c_int, [P, C.POINTER(P)]),
    ("tmnn_cuda_mlp_last_error", C.c_char_p, []),
    ("tmnn_cuda_nerf_create", C.c_int, [C.c_int, C.POINTER(NerfCfg), C.POINTER(P)]),
    ("tmnn_cuda_nerf_destroy", C.c_int, [P]),
    ("tmnn_cuda_nerf_density", C.c_int, [P, C.POINTER(P)]),
    ("tmnn_cuda_nerf_dp_init", C.c_int, [P, P, C.c_int, C.c_int]),
    ("tmnn_cuda_nerf_color_weights", C.c_int, [P, P, P, C.c_size_t]),
    ("tmnn_cuda_nerf_train_step", C.c_int,
     [P, P, P, P, P, u32, u32, C.POINTER(C.c_float)]),
    ("tmnn_cuda_nerf_inference", C.c_int, [P, P, P, P, P, u32, u32]),
    ("tmnn_cuda_nerf_profile", C.c_int, [P, P, C.POINTER(C.c_uint64)]),
    ("tmnn_cuda_nerf_last_error", C.c_char_p, []),
    ("tmnn_cuda_last_error", C.c_char_p, []),
    ("tmnn_cuda_launch_count", C.c_int, [P, C.POINTER(C.c_uint64)]),
]
SYMBOLS = [s[0] for s in _SIGS]


def load(path: str = LIB_PATH):
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build the CUDA library first "
            "(make -C tiny-metal-nn_b200 or __graft_entry__.build()); "
            "there is no CPU fallback")
    lib = C.CDLL(path)
    for name, res, args in _SIGS:
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


lib = load()


def last_error() -> str:
    return (lib.tmnn_cuda_last_error() or b"").decode()
