"""GPU parity of the whole training step against the FP64 oracle on identical seeds and inputs.

Bar: loss within 1e-3 absolute; every bf16-path gradient within 2e-2
relative L2 of the FP64 gradient; the optimizer update, fed the same gradients, within f32
round-off of the FP64 AdamW transition.  Gradients that are exactly zero in the reference
(input_projection: nothing is injected) must be exactly zero here too.

The FP64 oracle runs at the weights the compute path binds: every matrix cast to bf16, as the
reference casts every leaf to its compute precision each step (crates/sejong-model/src/lib.rs:
206-219) and passes the gradient of the cast straight to the f32 master (graph.rs:807-812).
What is compared is therefore the arithmetic of the bf16 path (bf16 activations, f32
accumulation), not the choice of bf16 weights itself.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import model as omodel
from oracle.corpus import synthetic_corpus
from oracle.rng import Rng

pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-3
GRAD_TOL = 2e-2


def oracle_config(c):
    h = c.hierarchy
    oh = None if h is None else omodel.HierarchyConfig(**h.__dict__)
    ox = None if c.experts is None else omodel.ExpertConfig(c.experts.count, c.experts.top_k, c.experts.ffn_width)
    return omodel.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                              kv_heads=c.kv_heads, rope_theta=c.rope_theta, norm_epsilon=c.norm_epsilon,
                              hierarchy=oh, experts=ox, seed=c.seed, init_std=c.init_std, router_std=c.router_std)


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / nb) if nb > 0 else float(np.linalg.norm(a))


def make_case(config_name, batch, seq, **overrides):
    from sejong_b200 import model as pm
    c = getattr(pm, config_name)()
    if overrides:
        c = pm.with_(c, **overrides)
    corp = synthetic_corpus(5, 200000)
    ids, targets = corp.batch(Rng(77), batch, seq)
    return c, ids, targets


def run_parity(c, ids, targets, batch, seq, optimizer="adamw"):
    from sejong_b200.model import initialize
    from sejong_b200.train import ByteTrainer, TrainConfig
    params = initialize(c)
    tc = TrainConfig(sequence=seq, batch=batch, optimizer=optimizer, warmup_steps=0, steps=100)
    tr = ByteTrainer(c, tc, device=0, params=params)
    tr.stage_batch(ids, targets)
    tr.forward_backward()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    loss = tr.loss()
    grads = tr.gradients()
    ref_loss, ref_grads = omodel.loss_and_grads(params, oracle_config(c), ids, targets, seq, cast="bf16")
    assert abs(loss - ref_loss) < LOSS_TOL, (loss, ref_loss)
    worst = {}
    for name, g in ref_grads.items():
        if np.all(g == 0):
            assert np.all(grads[name] == 0), name
            continue
        worst[name] = rel(grads[name], g)
    bad = {k: v for k, v in worst.items() if v > GRAD_TOL}
    assert not bad, f"gradients beyond {GRAD_TOL}: {bad}"
    # optimizer: same (GPU) gradients through the FP64 AdamW transition
    tr.optimizer_step()
    torch.cuda.synchronize()
    new = tr.parameters()
    otc = omodel.TrainConfig(sequence=seq, batch=batch, warmup_steps=0, steps=100)
    if optimizer == "adamw":
        ref_new, norm = omodel.adam_update(params, {k: v.astype(np.float64) for k, v in grads.items()},
                                           omodel.AdamState(), otc)
        assert abs(float(tr.hyper[4]) - norm) < 1e-5 * max(norm, 1.0)
        for k in params:
            assert float(np.max(np.abs(new[k] - ref_new[k]))) < 2e-6, k
    return loss, ref_loss, worst


def test_step_parity_small_hierarchy():
    c, ids, tg = make_case("small_hierarchy", 2, 256)
    run_parity(c, ids, tg, 2, 256)


def test_step_parity_dense_c1_shape():
    c, ids, tg = make_case("config_c1", 2, 512)
    run_parity(c, ids, tg, 2, 512)


def test_step_parity_c3_architecture_reduced_batch():
    """C3's exact architecture (window 128, 8 global layers d768 HQ12/HK4) on one 1024-byte row."""
    c, ids, tg = make_case("config_c3", 1, 1024)
    run_parity(c, ids, tg, 1, 1024)


def test_step_parity_reference_init():
    """The reference's own fan-in initialisation (global_bos = 0) through the same path."""
    c, ids, tg = make_case("small_hierarchy", 2, 128, init_std=0.0)
    run_parity(c, ids, tg, 2, 128)


def test_step_parity_moe():
    """MoE FFN on the global stage (the C5 block): top-2 of 4 SwiGLU experts, grouped GEMMs over the
    packed expert rows, router gradient through the softmax top-k."""
    from sejong_b200 import model as pm
    c, ids, tg = make_case("small_hierarchy", 2, 512, experts=pm.ExpertConfig(4, 2, 128))
    run_parity(c, ids, tg, 2, 512)


def test_graph_replay_matches_eager_and_loss_decreases():
    from sejong_b200.model import initialize, small_hierarchy
    from sejong_b200.train import ByteTrainer, TrainConfig
    c = small_hierarchy()
    corp = synthetic_corpus(5, 200000)
    rng = Rng(9)
    batches = [corp.batch(rng, 2, 256) for _ in range(6)]
    params = initialize(c)
    tc = TrainConfig(sequence=256, batch=2, learning_rate=1e-3, warmup_steps=0, steps=100)
    eager = ByteTrainer(c, tc, device=0, params=params)
    graphed = ByteTrainer(c, tc, device=0, params=params)
    graphed.stage_batch(*batches[0])
    graphed.capture()           # capture runs nothing; the first replay is step 1
    losses_e, losses_g = [], []
    for ids, tg in batches:
        eager.stage_batch(ids, tg)
        eager.step()
        losses_e.append(eager.loss())
        graphed.stage_batch(ids, tg)
        graphed.replay()
        losses_g.append(graphed.loss())
    torch.cuda.synchronize()
    np.testing.assert_allclose(losses_g, losses_e, rtol=0, atol=2e-3)
    assert rel(graphed.w.cpu().numpy(), eager.w.cpu().numpy()) < 1e-3
    assert float(eager.opt_state[0]) == 6.0 and float(graphed.opt_state[0]) == 6.0
