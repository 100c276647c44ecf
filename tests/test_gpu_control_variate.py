"""Control-variate SGD on the GPU against the FP64 restatement (oracle/control_variate.py).

A reduced hierarchical model, 4 observations per step, 2 stratified controls, rank 2, bases refreshed
every third step, gradient diagnostics every second.  Bars:
  * the control decisions (weights, generator states) equal the restatement's bit for bit;
  * the initial bases (normal draws of the basis generator, orthonormalised) within 1e-5;
  * per step: the loss within 1e-3; the weight update, the predictors and (after the refresh) the
    new bases within 2e-2 relative L2 over all predicted matrices together -- the bf16 path's
    gradient bar, since each is linear in the control gradients (a single 2 x 2 projection of a
    gradient is too few numbers for a per-matrix bar); the deferred coefficients (a difference of
    two predictions) and the predictor's mean squared residual within 5e-2;
  * with every observation a control the step equals the plain SGD step of the byte trainer with
    gradient accumulation within 2e-5 (crates/sejong-train/examples/control_variate_contract.rs:
    156-170);
  * a run saved after step 2 and resumed equals the uninterrupted run within 2e-5 (the contract's
    resume bar, :105-125).
"""
import numpy as np
import pytest
import torch

from oracle import control_variate as ocv
from oracle import model as om
from oracle.corpus import synthetic_corpus
from oracle.rng import Rng

pytestmark = pytest.mark.gpu

SEQ, ACC = 128, 4
LR = 0.05


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a))


def _setup(controls=2, diagnostics=2, refresh=3):
    from sejong_b200 import model as pm
    from sejong_b200.control_variate import ControlVariateConfig
    from sejong_b200.train import TrainConfig
    c = pm.small_hierarchy()
    tc = TrainConfig(sequence=SEQ, batch=1, optimizer="sgd", learning_rate=LR, min_learning_rate=LR,
                     warmup_steps=0, steps=100, weight_decay=0.0, clip_enabled=False, accumulation=ACC,
                     gradient_diagnostics_every=diagnostics, seed=123)
    cv = ControlVariateConfig(controls=controls, rank=2, sampling="stratified", strata=2, basis_refresh=refresh,
                              predictor_learning_rate=0.1)
    return c, tc, cv


def _oracle_config(c):
    h = c.hierarchy
    return om.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width, kv_heads=c.kv_heads,
                          rope_theta=c.rope_theta, norm_epsilon=c.norm_epsilon,
                          hierarchy=om.HierarchyConfig(**h.__dict__), seed=c.seed)


def _steps(n):
    corp = synthetic_corpus(5, 200000)
    rng = Rng(31)
    return [[corp.batch(rng, 1, SEQ) for _ in range(ACC)] for _ in range(n)]


def test_three_steps_match_the_restatement():
    from sejong_b200.control_variate import ControlVariateTrainer
    from sejong_b200.model import initialize, reference_layout
    c, tc, cv = _setup()
    params = initialize(c)
    tr = ControlVariateTrainer(c, tc, cv, device=0, params=params)
    oc = _oracle_config(c)
    layout = [(n, s) for n, s, _ in reference_layout(c)]
    state = ocv.init_state(layout, oc, cv.rank, tc.seed)
    assert [b.name for b in state.blocks] == [b.name for b in tr.blocks]
    for j, bk in enumerate(state.blocks):
        assert float(np.abs(tr.U[j].cpu().numpy() - bk.U).max()) < 1e-5, bk.name
        assert float(np.abs(tr.V[j].cpu().numpy() - bk.V).max()) < 1e-5, bk.name
    ref = {k: np.asarray(v, np.float64) for k, v in params.items()}
    worst = {"update": 0.0, "predictor": 0.0, "deferred": 0.0, "bases": 0.0, "mse": 0.0}
    for step, obs in enumerate(_steps(3)):
        before = tr.parameters()
        m = tr.step(obs)
        torch.cuda.synchronize()
        assert tr.tr.device_error() == 0
        ref_before = ref
        ref, rm = ocv.step(ref, state, oc, obs, SEQ, lr=LR, weight_decay=0.0, clip_enabled=False, clip_norm=1.0,
                           rank=cv.rank, controls=cv.controls, sampling=cv.sampling, strata=cv.strata,
                           basis_refresh=cv.basis_refresh, predictor_lr=cv.predictor_learning_rate,
                           diagnostics_every=tc.gradient_diagnostics_every)
        assert np.array_equal(m["weights"], rm["weights"]), step
        assert tr.sampling_rng.value == state.sampling
        assert m["basis_refreshed"] == rm["basis_refreshed"]
        assert abs(m["loss"] - rm["loss"]) < 1e-3, (step, m["loss"], rm["loss"])
        after = tr.parameters()
        upd = {k: after[k] - before[k] for k in after}
        rupd = {k: ref[k] - ref_before[k] for k in ref}
        num = sum(np.linalg.norm(upd[k] - rupd[k]) ** 2 for k in upd)
        den = sum(np.linalg.norm(rupd[k]) ** 2 for k in upd)
        r2 = cv.rank ** 2
        P = tr.P.cpu().numpy()
        pairs = {"predictor": [(P[:, j * r2:(j + 1) * r2], bk.P) for j, bk in enumerate(state.blocks)],
                 "deferred": [(tr.A[j].cpu().numpy(), bk.A) for j, bk in enumerate(state.blocks)],
                 "bases": [(tr.U[j].cpu().numpy(), bk.U) for j, bk in enumerate(state.blocks)] +
                          [(tr.V[j].cpu().numpy(), bk.V) for j, bk in enumerate(state.blocks)]}
        for key, ab in pairs.items():  # relative L2 over all predicted matrices together
            den_k = sum(float(np.linalg.norm(b) ** 2) for _, b in ab)
            if den_k > 0:
                err = (sum(float(np.linalg.norm(np.asarray(a, np.float64) - b) ** 2) for a, b in ab) / den_k) ** 0.5
                worst[key] = max(worst[key], err)
        worst["update"] = max(worst["update"], (num / den) ** 0.5)
        if m["gradient_diagnostics"]:
            worst["mse"] = max(worst["mse"], rel(m["predictor_mse"], rm["predictor_mse"]))
    tr.close()
    print("worst relative L2:", worst)
    # the deferred coefficient is lr times the difference of two predictions (all observations' mean
    # minus the weighted controls'), so their bf16-level errors enter it relative to that difference
    assert worst["update"] < 2e-2 and worst["predictor"] < 2e-2 and worst["bases"] < 2e-2, worst
    assert worst["deferred"] < 5e-2 and worst["mse"] < 5e-2, worst


def test_all_controls_equal_plain_sgd():
    from sejong_b200.control_variate import ControlVariateTrainer
    from sejong_b200.model import initialize
    from sejong_b200.train import ByteTrainer
    c, tc, cv = _setup(controls=ACC, diagnostics=0, refresh=100)
    params = initialize(c)
    obs = _steps(1)[0]
    tr = ControlVariateTrainer(c, tc, cv, device=0, params=params)
    m = tr.step(obs)
    cv_w = tr.parameters()
    tr.close()
    sgd = ByteTrainer(c, tc, device=0, params=params)
    for i, (ids, tg) in enumerate(obs):
        sgd.stage_batch(ids, tg)
        sgd.forward_backward(first=i == 0, last=i == ACC - 1)
    sgd.optimizer_step()
    torch.cuda.synchronize()
    assert abs(m["loss"] - sgd.loss()) < 1e-5
    ref_w = sgd.parameters()
    worst = max(float(np.abs(cv_w[k] - ref_w[k]).max()) for k in ref_w)
    assert worst < 2e-5, worst
    sgd.close()


def test_resume_equals_the_uninterrupted_run():
    from sejong_b200.control_variate import ControlVariateTrainer
    from sejong_b200.model import initialize
    c, tc, cv = _setup(diagnostics=0, refresh=3)
    params = initialize(c)
    steps = _steps(4)
    a = ControlVariateTrainer(c, tc, cv, device=0, params=params)
    saved = None
    for i, obs in enumerate(steps):
        a.step(obs)
        if i == 1:
            saved = a.snapshot()  # folds U A V^T into the weights first, as the reference's save does
    final_a = a.snapshot()
    a.close()
    b = ControlVariateTrainer(c, tc, cv, device=0, params=saved[0])
    b.load_state_tensors(saved[1])
    b.step_count = 2
    b.tr.opt_state[0] = 2.0
    for obs in steps[2:]:
        b.step(obs)
    final_b = b.snapshot()
    b.close()
    worst_w = max(float(np.abs(final_a[0][k] - final_b[0][k]).max()) for k in final_a[0])
    worst_s = max(float(np.abs(final_a[1][k] - final_b[1][k]).max()) for k in final_a[1])
    assert worst_w < 2e-5 and worst_s < 2e-5, (worst_w, worst_s)
