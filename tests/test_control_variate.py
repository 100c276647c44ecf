"""Control-variate SGD on the CPU: the sampling of controls (bit-exact between the library's host
code and the FP64 restatement, and the reference's own unit test), the orthonormalisation and the
all-controls property of the restated step (controls = accumulation is plain SGD on the mean
gradient, crates/sejong-train/examples/control_variate_contract.rs:156-170)."""
import ctypes

import numpy as np
import pytest

from oracle import control_variate as ocv
from oracle import model as om
from oracle.corpus import synthetic_corpus
from oracle.rng import Rng


def _observations(count, n=16):
    return [np.array([j % (i + 1) for j in range(n)], dtype=np.int32) for i in range(count)]


def test_stratified_weights_cover_the_population():
    """control_variate.rs:901-933 ported: 11 observations, 5 controls over 3 strata, 2000 draws."""
    from sejong_b200.control_variate import ControlVariateConfig, control_weights
    cv = ControlVariateConfig(controls=5, rank=2, sampling="stratified", strata=3, basis_refresh=4,
                              predictor_learning_rate=0.01)
    obs = _observations(11)
    state = ctypes.c_uint64(7)
    totals = np.zeros(11)
    for _ in range(2000):
        w = control_weights(obs, cv, state)
        assert int((w > 0).sum()) == 5
        assert abs(float(w.sum()) - 1.0) < 1e-6
        totals += w.astype(np.float64) / 2000.0
    assert np.all(np.abs(totals - 1.0 / 11.0) < 0.01)


@pytest.mark.parametrize("controls,sampling,strata,count", [(5, "stratified", 3, 11), (2, "uniform", 1, 8),
                                                            (3, "stratified", 2, 7), (4, "stratified", 4, 4)])
def test_weights_equal_the_restatement(controls, sampling, strata, count):
    """Same decisions, same generator state, bit for bit, as the FP64 restatement (entropy strata,
    allocation, partial Fisher-Yates with Rng::index)."""
    from sejong_b200.control_variate import ControlVariateConfig, control_weights
    cv = ControlVariateConfig(controls=controls, rank=2, sampling=sampling, strata=strata)
    corp = synthetic_corpus(3, 20000)
    rng_data = Rng(5)
    state = ctypes.c_uint64(99)
    ref = Rng(99)
    for _ in range(20):
        obs = [np.asarray(corp.batch(rng_data, 1, 32)[0]).reshape(-1) for _ in range(count)]
        w = control_weights(obs, cv, state)
        r = ocv.control_weights(obs, controls, sampling, strata, ref)
        assert np.array_equal(w, r)
        assert state.value == ref.state


def test_orthonormalize_restatement():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((40, 6))
    q = ocv.orthonormalize(x)
    assert np.abs(q.T @ q - np.eye(6)).max() < 1e-12
    # span preserved column by column (Gram-Schmidt: q_k in span(x_0..x_k))
    for k in range(6):
        coef, *_ = np.linalg.lstsq(x[:, :k + 1], q[:, k], rcond=None)
        assert np.abs(x[:, :k + 1] @ coef - q[:, k]).max() < 1e-10
    # a repeated column falls back to the least-occupied coordinate
    y = np.concatenate([x[:, :2], x[:, :1]], axis=1)
    q = ocv.orthonormalize(y)
    assert np.abs(q.T @ q - np.eye(3)).max() < 1e-12


def test_all_controls_is_plain_sgd():
    """With every observation a control, the predictions cancel (delta = 0) and the step is SGD on
    the mean gradient of the observations, exactly."""
    c = om.small_hierarchy(width=64, layers=1, heads=2, kv_heads=1, ffn=64, local=32, local_heads=1, local_ffn=64,
                           patch=4, window=8)
    params = om.initialize(c)
    layout = [(n, np.shape(v)) for n, v in params.items()]
    corp = synthetic_corpus(2, 20000)
    rng = Rng(11)
    obs = [corp.batch(rng, 1, 32) for _ in range(3)]
    state = ocv.init_state(layout, c, 2, 123)
    new, metrics = ocv.step(params, state, c, obs, 32, lr=0.05, weight_decay=0.0, clip_enabled=False, clip_norm=1.0,
                            rank=2, controls=3, sampling="stratified", strata=2, basis_refresh=10,
                            predictor_lr=0.1, cast=None)
    assert metrics["controls"] == 3
    mean = {k: np.zeros_like(v, dtype=np.float64) for k, v in params.items()}
    for (ids, tg), w in zip(obs, metrics["weights"]):  # w = f32(1/3), as the reference's f32 weights
        _, g = om.loss_and_grads(params, c, ids, tg, 32)
        for k in mean:
            mean[k] += float(w) * g[k]
    for k in params:
        assert np.abs(new[k] - (params[k] - 0.05 * mean[k])).max() < 1e-12, k
    for bk in state.blocks:
        assert np.abs(bk.A).max() < 1e-15
