"""The MoE additions of this build (expert capacity, load-balancing loss) in the FP64 restatement
(oracle/model.py), no GPU: the capacity rule against a plain loop over (choice, row), and the loss's
gradient against its closed form p (f - <f, p>) * weight * E / rows, which the device kernel
sj_moe_aux applies.  With capacity unlimited and weight 0 the oracle is the reference's block."""
import math

import numpy as np
import torch

from oracle import model as om
from oracle import ops


def test_capacity_rule_matches_a_plain_loop():
    rng = np.random.default_rng(0)
    rows, k, E = 300, 2, 8
    logits = torch.tensor(rng.normal(size=(rows, E)))
    _, ids = ops.route_topk(logits, k)
    cap = math.ceil(1.25 * rows * k / E) - 20   # tight enough to drop
    got = om.apply_capacity(ids, E, cap)
    fill = [0] * E
    want = ids.clone()
    for j in range(k):
        for r in range(rows):
            e = int(ids[r, j])
            if fill[e] < cap:
                fill[e] += 1
            else:
                want[r, j] = -1
    assert torch.equal(got, want)
    assert (got == -1).any()
    for e in range(E):
        assert int((got == e).sum()) <= cap


def test_aux_gradient_closed_form():
    rng = np.random.default_rng(1)
    rows, k, E, w = 64, 2, 8, 0.01
    logits = torch.tensor(rng.normal(size=(rows, E)), requires_grad=True)
    ids = ops.route_topk(logits.detach(), k)[1]
    loss = om.aux_loss(logits, ids, E, w)
    loss.backward()
    p = torch.softmax(logits.detach(), 1)
    f = torch.nn.functional.one_hot(ids.reshape(-1), E).double().mean(0)
    want = w * E / rows * p * (f[None, :] - (p * f[None, :]).sum(1, keepdim=True))
    assert torch.allclose(logits.grad, want, atol=1e-15)
    assert abs(float(loss.detach()) - w * E * float((f * p.mean(0)).sum())) < 1e-15


def test_defaults_keep_the_reference_block():
    c = om.small_hierarchy()
    c.experts = om.ExpertConfig(4, 2, 64)
    params = om.initialize(c)
    rng = np.random.default_rng(2)
    ids = rng.integers(0, 256, size=256)
    tg = rng.integers(0, 256, size=256)
    l0, g0 = om.loss_and_grads(params, c, ids, tg, 256)
    c2 = om.with_(c, moe_capacity_factor=100.0, moe_aux_weight=0.0)
    l1, g1 = om.loss_and_grads(params, c2, ids, tg, 256)
    assert l0 == l1 and all(np.array_equal(g0[n], g1[n]) for n in g0)
    c3 = om.with_(c, moe_aux_weight=0.01)
    l2, _ = om.loss_and_grads(params, c3, ids, tg, 256)
    assert l2 > l0
