"""CPU-side checks of the C ABI: the library loads, exports every entry point
include/tmnn_cuda.h declares, and validates configurations (the JSON front
end runs before any device work, so its errors surface without a GPU)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tmnn_cuda.h")
LIB = os.path.join(ROOT, "tiny-metal-nn_b200", "libtmnn_cuda.so")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(tmnn_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], check=True,
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (tmnn_cuda_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_python_binding_covers_header():
    import tmnn_b200._abi as abi
    assert sorted(abi.SYMBOLS) == declared_symbols()


def test_library_is_sm100a_only():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", LIB],
                         capture_output=True, text=True).stdout
    assert "sm_100a" in out


def test_default_config_matches_reference_defaults():
    import tmnn_b200 as t
    from tmnn_b200 import _abi
    c = _abi.TrainCfg()
    t.lib.tmnn_cuda_default_train_cfg(C.byref(c))
    # TrainerConfig (trainer.h:34-61) and WeightInitConfig (weight_init.h)
    assert c.batch_size == 1024
    assert abs(c.lr_encoding - 1e-2) < 1e-9 and abs(c.lr_network - 1e-3) < 1e-9
    assert abs(c.beta1 - 0.9) < 1e-7 and abs(c.beta2 - 0.99) < 1e-7
    assert c.seed == 42 and abs(c.hash_init_range - 1e-4) < 1e-10


@pytest.mark.parametrize("env,field,value", [
    ({"TMNN_BAD_STEP_MODE": " Skip "}, "bad_step_recovery", 2),
    ({"TMNN_BAD_STEP_MODE": "safe-family-fallback"}, "bad_step_recovery", 4),
    ({"TMNN_BAD_STEP_MODE": "strict"}, "bad_step_recovery", 1),
    ({"TMNN_NUMERICS_SAMPLING_MODE": "full-per-step"}, "numerics_sampling_mode", 2),
    ({"TMNN_NUMERICS_SAMPLING_MODE": "OFF"}, "numerics_sampling_mode", 3),
    ({"TMNN_NUMERICS_SAMPLE_INTERVAL": "0"}, "numerics_sample_interval", 1),
    ({"TMNN_NUMERICS_SAMPLE_INTERVAL": "32"}, "numerics_sample_interval", 32),
    ({}, "numerics_sample_interval", 128),
])
def test_numerics_policy_from_environment(monkeypatch, env, field, value):
    """load_runtime_policy's environment variables and spellings
    (src/tiny_metal_nn/runtime/runtime_policy.h:78-161)."""
    import tmnn_b200 as t
    from tmnn_b200 import _abi
    for k in ("TMNN_BAD_STEP_MODE", "TMNN_NUMERICS_SAMPLING_MODE",
              "TMNN_NUMERICS_SAMPLE_INTERVAL"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    c = _abi.TrainCfg()
    t.lib.tmnn_cuda_default_train_cfg(C.byref(c))
    assert getattr(c, field) == value


def _create(cfg_json, n_in=3, n_out=1):
    import tmnn_b200 as t
    h = C.c_void_p()
    st = t.lib.tmnn_cuda_ctx_create_from_json(0, n_in, n_out, cfg_json.encode(),
                                              C.byref(h))
    return st, t._abi.last_error(), h


@pytest.mark.parametrize("cfg,frag", [
    ('{"encoding": {"n_levels": 0}}', "encoding.n_levels: must be positive"),
    ('{"encoding": {"otype": "Frequency"}}', "unsupported encoding otype"),
    ('{"encoding": {"interpolation": "Nearest"}}', "only 'Linear'"),
    ('{"network": {"activation": "Tanh"}}', "only 'ReLU'"),
    ('{"network": {"otype": "TiledMLP"}}', "reserved for later"),
    ('{"loss": {"otype": "Huber", "huber_delta": -1}}', "loss.huber_delta"),
    ('{"optimizer": {"learning_rate": 0}}', "optimizer.learning_rate"),
    ('{"weight_init": {"mlp_init": "Orthogonal"}}', "allowed: KaimingUniform"),
    ('{"bogus": 1}', "config.bogus: unknown key"),
    ('{"encoding": {"n_levels": 2.5}}', "must be an integer"),
    ('{"encoding": ', "json:"),
    ('{"b200": {"bad_step_recovery": "Retry"}}', "allowed: SignalOnly, Throw"),
    ('{"b200": {"numerics_sampling_mode": "Often"}}', "allowed: Sampled"),
    ('{"b200": {"morton_key_bits": 40}}', "b200.morton_key_bits: must be in [0, 32]"),
    ('{"b200": {"hash_grad_format": "BF16"}}', "allowed: Fixed16, F32, F16"),
    ('{"b200": {"enable_probes": 2}}', "b200.enable_probes"),
])
def test_config_errors_reported_without_gpu(cfg, frag):
    st, msg, _ = _create(cfg)
    assert st == 1, (st, msg)
    assert frag in msg, msg


@pytest.mark.parametrize("b200", ['{"hash_grad_format": "F16"}',
                                  '{"enable_probes": true}'])
def test_new_b200_keys_parse_without_gpu(b200):
    """The fp16 gradient format and the probe switch parse (creation then
    fails only for want of a device)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st, msg, _ = _create('{"b200": %s}' % b200)
    assert st != 0 and "device" in msg.lower(), msg


def test_valid_config_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st, msg, h = _create('{"loss": {"otype": "L1"}, "optimizer": {"learning_rate": 0.01}}')
    assert st != 0 and "device" in msg.lower()
    assert not h.value


def test_reference_import_name():
    """`import tiny_metal_nn` gives the same front end as tmnn_b200, with the
    reference's Trainer methods (is_gpu_available included)."""
    import tiny_metal_nn
    import tmnn_b200
    assert tiny_metal_nn.Trainer is tmnn_b200.Trainer
    assert issubclass(tiny_metal_nn.ConfigError, ValueError)
    assert issubclass(tiny_metal_nn.DTypeError, TypeError)
    for name in ("from_config", "training_step", "inference", "step",
                 "close", "is_gpu_available"):
        assert hasattr(tiny_metal_nn.Trainer, name)
