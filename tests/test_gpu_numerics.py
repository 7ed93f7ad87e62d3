"""Numerics guard on the device (NumericsGuard + the sampled probes +
bad-step recovery: src/tiny_metal_nn/runtime/numerics_guard.cpp,
training_step_execution.cpp:237-456, :1080-1235) through the C ABI.

Failures are made on the host: non-finite or huge weights written with
set_initial_weights.  No test faults, traps or hangs the GPU; a bad step is
detected from values the kernels compute and read back."""
import numpy as np
import pytest

from _util import batch

pytestmark = pytest.mark.gpu

KW = dict(L=4, F=2, log2T=12, d=3, W=64, H=1, O=1)


def make(mode="Sampled", recovery="SignalOnly", family="SafeDebug", **kw):
    from tmnn_b200 import _abi
    import tmnn_b200 as t
    spec_kw = dict(KW, **kw)
    spec = _abi.Spec(spec_kw["L"], spec_kw["F"], spec_kw["log2T"], spec_kw["d"],
                     16.0, 1.447, spec_kw["W"], spec_kw["H"], spec_kw["O"], 0,
                     1.0, _abi.DTYPE_F32)
    cfg = _abi.TrainCfg()
    t.lib.tmnn_cuda_default_train_cfg(cfg)
    cfg.family = _abi.FAMILY[family]
    cfg.hash_grad_format = _abi.GRAD_FIXED16 if family == "SafeDebug" else _abi.GRAD_F32
    cfg.numerics_sampling_mode = _abi.SAMPLING[mode]
    cfg.bad_step_recovery = _abi.BAD_STEP[recovery]
    cfg.batch_size = 4096
    return t.Trainer.from_spec(spec, cfg)


def test_sampling_schedule_and_probe_values():
    """Sampled mode probes steps 0 and 1 and every 128th; the probe's max
    |g|, gradient norm and max |update| equal the same quantities computed
    from the gradients and optimizer state read back after forward_backward
    (the reference's probe_backward/update_numerics arithmetic)."""
    tr = make()
    ref = make()
    pos, tgt = batch(4096, 3, 1, seed=3)
    # reference quantities from an identical trainer: gradients of the same
    # batch before any update (fixed-point hash grads are order independent)
    ref.forward_backward(pos, tgt)
    from tmnn_b200 import _abi
    gh = ref.read_buffer(_abi.BUF_GRAD_HASH).astype(np.float64) / 65536.0
    gm = ref.read_buffer(_abi.BUF_GRAD_MLP).astype(np.float64)
    g = np.concatenate([gh, gm])
    tr.training_step(pos, tgt)
    n0 = tr.last_numerics()
    assert n0["probed"] and n0["reported"] and not n0["anomaly"]
    assert abs(n0["max_abs_gradient"] - np.abs(g).max()) <= 1e-5 * np.abs(g).max()
    assert abs(n0["grad_norm"] - np.sqrt((g * g).sum())) <= 1e-4 * np.sqrt((g * g).sum())
    # first Adam step from m = v = 0: |update| = lr * |mhat| / (sqrt(vhat)+eps)
    # = lr for every nonzero finite gradient (bias corrections cancel)
    assert abs(n0["max_abs_update"] - 1e-2) <= 1e-6
    probed = [True]
    for step in range(1, 130):
        tr.training_step(pos, tgt)
        probed.append(tr.last_numerics()["probed"])
    assert probed[:3] == [True, True, False]
    assert probed[128] and not probed[127] and not probed[129]
    assert tr.numerics_stats()["reports"] == 3
    tr.close()
    ref.close()


def _poison(tr, value=np.nan):
    hw, mw = tr.weights()
    mw = mw.copy()
    mw[-1] = value  # output bias: every point's output becomes non-finite
    tr.set_initial_weights(hw, mw)
    return hw, mw


def test_signal_only_reports_anomaly_and_applies_update():
    tr = make(mode="Disabled")
    pos, tgt = batch(2048, 3, 1, seed=4)
    tr.training_step(pos, tgt)
    assert not tr.last_numerics()["probed"]  # Disabled: no probe on a good step
    _poison(tr)
    step = tr.step()
    tr.training_step(pos, tgt)
    n = tr.last_numerics()
    # a non-finite loss forces the probe even when sampling is disabled
    assert n["anomaly"] and not n["finite_forward"] and n["probed"]
    assert not n["finite_backward"]  # NaN reaches the MLP gradients
    assert n["recovery_action"] == "None"
    st = tr.numerics_stats()
    assert st["anomalies"] == 1 and st["last_anomaly_step"] == step
    tr.close()


@pytest.mark.parametrize("recovery,action", [("Skip", "Skipped"),
                                             ("Rollback", "RolledBack")])
def test_skip_and_rollback_leave_weights_unchanged(recovery, action):
    tr = make(recovery=recovery)
    pos, tgt = batch(2048, 3, 1, seed=5)
    tr.training_step(pos, tgt)
    hw, mw = _poison(tr)
    step = tr.step()
    tr.training_step(pos, tgt)
    n = tr.last_numerics()
    assert n["anomaly"] and n["recovery_action"] == action
    h2, m2 = tr.weights()
    assert np.array_equal(h2, hw) and np.array_equal(m2, mw, equal_nan=True)
    assert tr.step() == step + 1  # the step still counts, as in the reference
    # the gradients were cleared: a healthy step afterwards is finite
    mw[-1] = 0.0
    tr.set_initial_weights(hw, mw)
    tr.training_step(pos, tgt)
    assert not tr.last_numerics()["anomaly"]
    tr.close()


def test_throw_mode_raises_and_keeps_state():
    import tmnn_b200 as t
    tr = make(recovery="Throw")
    pos, tgt = batch(2048, 3, 1, seed=6)
    tr.training_step(pos, tgt)
    hw, mw = _poison(tr)
    step = tr.step()
    with pytest.raises(t.TmnnError, match="numerics anomaly detected"):
        tr.training_step(pos, tgt)
    assert tr.step() == step
    h2, m2 = tr.weights()
    assert np.array_equal(h2, hw) and np.array_equal(m2, mw, equal_nan=True)
    tr.close()


def test_fallback_retries_with_safe_family():
    """An anomaly only the fp16 tensor-core path has (hidden activations
    above the fp16 range) is recovered by re-running the step with the fp32
    SafeDebug kernels; the family then stays SafeDebug."""
    tr = make(recovery="FallbackAndRetryWithSafeFamily", family="FullyFused",
              L=8)
    assert tr.plan()["family"] == "FullyFused"
    pos, tgt = batch(2048, 3, 1, seed=7)
    hw, mw = tr.weights()
    hw = np.full_like(hw, 6.0e4)
    mw = np.abs(mw) + 0.05
    tr.set_initial_weights(hw, mw)
    step = tr.step()
    tr.training_step(pos, tgt)
    n = tr.last_numerics()
    assert n["recovery_action"] == "RetriedWithSafeFamily"
    assert not n["anomaly"] and n["finite_forward"] and n["finite_update"]
    assert tr.last_result.family == 2  # SafeDebug
    st = tr.numerics_stats()
    assert st["safe_family_recoveries"] == 1 and st["safe_family_active"] == 1
    assert tr.step() == step + 1
    h2, m2 = tr.weights()
    assert np.isfinite(h2).all() and np.isfinite(m2).all()
    assert not np.array_equal(m2, mw)  # the retried update was applied
    # a persistent anomaly with SafeDebug already active is an error
    import tmnn_b200 as t
    _poison(tr)
    with pytest.raises(t.TmnnError, match="already active"):
        tr.training_step(pos, tgt)
    tr.close()
