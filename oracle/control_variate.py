"""Control-variate SGD restated on the CPU in FP64 -- test infrastructure only: the checker of
sejong_b200.control_variate, never called by the product path.

Follows crates/sejong-train/src/control_variate.rs:
  * predicted_parameter (:31-40), SgdState::new (:67-121: basis generator draws, orthonormalised
    bases, zero deferred coefficients and predictors), flush (:235-246) and refresh_bases (:248-282);
  * entropy and control_weights (:289-349: entropy strata, allocation, partial Fisher-Yates);
  * augmented_feature (:375-387), correction_norm (:365-373);
  * one step of train_configured (:502-830) for the dense-gradient SGD route: corrected weights bound,
    control forward / backward, projected targets U^T G V, predictions, sketches, the clipped norm
    with the correction terms, the SGD, deferred and predictor updates, the basis refresh.
The bound corrected weight W + U A V^T is the low-rank matmul of graph.rs:244-271 folded into W
(equal in exact arithmetic); Engine::orthonormalize_columns restates hierarchy_orthogonal_column
(python/sejong_kernels/ops/hierarchy.py:346-397) and transport_coefficients
hierarchy_coefficient_transport (hierarchy.py:290-315).
"""
import math
from dataclasses import dataclass, field

import numpy as np

from . import model as om
from . import ops
from .rng import Rng

SAMPLING_MIX = 0x38B87C4D9F0A1265
BASIS_MIX = 0xA41239C507EF68BD
MASK64 = (1 << 64) - 1


def predicted_parameter(name, shape):
    return (len(shape) == 2 and name not in ("embedding", "global_bos", "input_projection")
            and not name.startswith("encoder.") and not name.endswith(".router")
            and ".experts." not in name and ".expert." not in name)


def entropy(values):
    v = np.asarray(values, dtype=np.int64).reshape(-1)
    counts = np.bincount(v, minlength=257)
    n = float(v.size)
    total = 0.0
    for c in counts:
        if c > 0:
            p = c / n
            total += -p * math.log(p)
    return total


def control_weights(inputs, controls, sampling, strata_cfg, rng):
    """control_variate.rs:305-349 with the oracle Rng."""
    count = len(inputs)
    strata = 1 if sampling == "uniform" else strata_cfg
    order = list(range(count))
    if strata > 1:
        ent = [entropy(x) for x in inputs]
        order = sorted(order, key=lambda i: (ent[i], i))
    groups = [list(order[h * count // strata:(h + 1) * count // strata]) for h in range(strata)]
    alloc = [1] * strata
    for _ in range(strata, controls):
        cands = [h for h in range(strata) if alloc[h] < len(groups[h])]
        # max by ratio, ties to the lowest stratum
        h = max(cands, key=lambda h: (len(groups[h]) / (alloc[h] + 1), -h))
        alloc[h] += 1
    weights = np.zeros(count, dtype=np.float32)
    for group, selected in zip(groups, alloc):
        weight = np.float32(len(group)) / np.float32(count * selected)
        for i in range(selected):
            j = i + rng.index(len(group) - i)
            group[i], group[j] = group[j], group[i]
            weights[group[i]] = weight
    return weights


def orthonormalize(x):
    """hierarchy_orthogonal_column for every column in order, in FP64."""
    q = np.array(x, dtype=np.float64, copy=True)
    rows, cols = q.shape
    for col in range(cols):
        def sweep():
            for _ in range(2):
                for prev in range(col):
                    q[:, col] -= np.dot(q[:, col], q[:, prev]) * q[:, prev]
        sweep()
        norm = float(np.dot(q[:, col], q[:, col]))
        if norm < 1e-20:
            occ = (q[:, :col] ** 2).sum(axis=1) if col else np.zeros(rows)
            score = 1.0 - occ
            pivot = int(np.argmax(score))  # first of the maxima
            q[:, col] = 0.0
            q[pivot, col] = 1.0
            sweep()
            norm = float(np.dot(q[:, col], q[:, col]))
        q[:, col] /= math.sqrt(norm)
    return q


def transport(h, left, right):
    """Each feature row's r x r coefficient C -> left^T C right."""
    r = left.shape[0]
    c = h.reshape(h.shape[0], r, r)
    return np.einsum("ka,fkl,lb->fab", left, c, right).reshape(h.shape)


def encode(p, c, ids, seq):
    """Model::encode (architecture.rs:330-351) in FP64: the embedding rows, and for the hierarchical
    model the encoder blocks and encoder_norm."""
    import torch
    pt = {k: torch.tensor(v, dtype=torch.float64) for k, v in p.items()}
    ids_t = torch.as_tensor(np.asarray(ids, dtype=np.int64).reshape(-1))
    x = ops.embedding(pt["embedding"], ids_t)
    h = c.hierarchy
    if h is None:
        return x.numpy()
    x = om._blocks(pt, om.local_stage(c, True), x, seq, c)
    return ops.rmsnorm(x, pt["encoder_norm"], c.norm_epsilon).numpy()


def feature(encoded, embedding, labels):
    """augmented_feature: [row means of E, of the target embedding rows, of their product, 1]."""
    e = np.asarray(encoded, dtype=np.float64)
    t = np.asarray(embedding, dtype=np.float64)[np.asarray(labels, dtype=np.int64).reshape(-1)]
    return np.concatenate([e.mean(0), t.mean(0), (e * t).mean(0), [1.0]])


@dataclass
class Block:
    name: str
    U: np.ndarray
    V: np.ndarray
    A: np.ndarray
    P: np.ndarray


@dataclass
class State:
    blocks: list
    sampling: int
    basis: int
    step: int = 0
    trace: dict = field(default_factory=dict)


def init_state(params_layout, c, rank, seed):
    """SgdState::new: per predicted matrix (reference order) a*r then b*r normal draws of
    Rng(seed ^ BASIS_MIX), each orthonormalised; A = 0, P = 0 [3 w + 1, r^2]."""
    basis = Rng(seed ^ BASIS_MIX)
    width = c.hierarchy.encoder_width if c.hierarchy is not None else c.width
    blocks = []
    for name, shape in params_layout:
        if not predicted_parameter(name, shape):
            continue
        a, b = shape
        left = basis.bulk_normal(a * rank).reshape(a, rank)
        right = basis.bulk_normal(b * rank).reshape(b, rank)
        blocks.append(Block(name, orthonormalize(left), orthonormalize(right), np.zeros((rank, rank)),
                            np.zeros((3 * width + 1, rank * rank))))
    return State(blocks, (seed ^ SAMPLING_MIX) & MASK64, basis.state)


def corrected(params, state):
    out = dict(params)
    for bk in state.blocks:
        out[bk.name] = params[bk.name] + bk.U @ bk.A @ bk.V.T
    return out


def flush(params, state):
    params = corrected(params, state)
    for bk in state.blocks:
        bk.A = np.zeros_like(bk.A)
    return params


def step(params, state, c, observations, seq, *, lr, weight_decay, clip_enabled, clip_norm, rank, controls,
         sampling, strata, basis_refresh, predictor_lr, diagnostics_every=0, cast="bf16"):
    """One control-variate SGD step (dense gradients, loss_scale 1).  `observations` is a list of
    (ids, targets); `lr` the step's learning rate.  Returns (params, metrics); `state` advances."""
    rr = rank * rank
    acc = len(observations)
    refreshed = (state.step + 1) % basis_refresh == 0
    diagnostics = diagnostics_every > 0 and (state.step + 1) % diagnostics_every == 0
    measure = clip_enabled or diagnostics
    rng = Rng(0)
    rng.state = state.sampling
    weights = control_weights([np.asarray(i).reshape(-1) for i, _ in observations], controls, sampling, strata, rng)
    state.sampling = rng.state
    bound = corrected(params, state)
    nb = len(state.blocks)
    grad = {k: np.zeros_like(v, dtype=np.float64) for k, v in params.items()}
    mean_pred = [np.zeros(rr) for _ in range(nb)]
    ctrl_pred = [np.zeros(rr) for _ in range(nb)]
    mean_target = [np.zeros(rr) for _ in range(nb)]
    pgrad = [np.zeros_like(bk.P) for bk in state.blocks]
    sketches = [None] * nb
    loss = 0.0
    gsm = rsm = mse = 0.0
    k = 0
    for (ids, targets), w in zip(observations, weights):
        w = float(w)
        feat = feature(encode(om.compute_cast(bound, cast), c, ids, seq), params["embedding"], targets)
        if w > 0:
            lo, g = om.loss_and_grads(bound, c, ids, targets, seq, cast=cast)
            loss += w * lo
            for key in grad:
                grad[key] += w * g[key]
            if diagnostics:
                sample = sum(float((g[key] ** 2).sum()) for key in g)
                gsm += w * sample
                rsm += w * sample
        for j, bk in enumerate(state.blocks):
            pred = feat @ bk.P
            mean_pred[j] += pred / acc
            if w <= 0:
                continue
            gj = g[bk.name]
            if refreshed and k < 2:
                left, right = gj @ bk.V, gj.T @ bk.U
                sketches[j] = (left, right) if k == 0 else (sketches[j][0] - left, sketches[j][1] - right)
            target = (bk.U.T @ gj @ bk.V).reshape(-1)
            if measure:
                mean_target[j] += w * target
            ctrl_pred[j] += w * pred
            resid = pred - target
            if diagnostics:
                gu, gv = bk.U.T @ bk.U, bk.V.T @ bk.V
                pm = pred.reshape(rank, rank)
                mse += w * float(resid @ resid) / rr
                rsm += w * (float((pm * (gu @ pm @ gv)).sum()) - 2.0 * float(pred @ target))
            pgrad[j] += np.outer(feat, resid) * (2.0 * w / rr)
        if w > 0:
            k += 1
    base = sum(float((grad[key] ** 2).sum()) for key in grad)
    norm2 = base
    deltas = []
    for j, bk in enumerate(state.blocks):
        d = (mean_pred[j] - ctrl_pred[j]).reshape(rank, rank)
        gu, gv = bk.U.T @ bk.U, bk.V.T @ bk.V
        if measure:
            norm2 += float((d * (gu @ d @ gv)).sum()) + 2.0 * float(mean_target[j] @ d.reshape(-1))
        deltas.append(d)
    norm = math.sqrt(max(norm2, 0.0))
    clipping = clip_norm / norm if (clip_enabled and norm > clip_norm) else 1.0
    new = {}
    for key, v in params.items():
        decay = 1.0 - lr * weight_decay if np.ndim(v) > 1 else 1.0
        new[key] = v * decay - lr * clipping * grad[key]
    for j, bk in enumerate(state.blocks):
        bk.A = bk.A * (1.0 - lr * weight_decay) - lr * clipping * deltas[j]
        bk.P = bk.P - predictor_lr * pgrad[j]
    state.step += 1
    metrics = {"loss": loss, "weights": weights, "controls": int((weights > 0).sum()), "gradient_norm":
               norm if measure else None, "basis_refreshed": refreshed, "clipping": clipping}
    if diagnostics:
        residual_mean = base
        for j, bk in enumerate(state.blocks):
            cp = ctrl_pred[j].reshape(rank, rank)
            gu, gv = bk.U.T @ bk.U, bk.V.T @ bk.V
            residual_mean += float((cp * (gu @ cp @ gv)).sum()) - 2.0 * float(mean_target[j] @ ctrl_pred[j])
        metrics.update(predictor_mse=mse, control_gradient_dispersion=max(gsm - base, 0.0),
                       control_residual_dispersion=max(rsm - residual_mean, 0.0))
    if refreshed:
        new = flush(new, state)
        eps = math.sqrt(float(np.finfo(np.float32).eps))
        for j, bk in enumerate(state.blocks):
            if sketches[j] is None:
                continue
            ls, rs = sketches[j]
            magnitude = math.sqrt(float((ls ** 2).sum()) + float((rs ** 2).sum()))
            if magnitude == 0:
                continue
            reg = magnitude * eps
            U_new = orthonormalize(ls + reg * bk.U)
            V_new = orthonormalize(rs + reg * bk.V)
            bk.P = transport(bk.P, bk.U.T @ U_new, bk.V.T @ V_new)
            bk.U, bk.V = U_new, V_new
    return new, metrics
