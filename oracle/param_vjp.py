"""Parameter VJP (low-rank factors + selected residual rows) and the compact SGD step.

Restates crates/sejong-gpu/src/parameter_vjp.rs and python/sejong_kernels/ops/parameter.py:

* `budget`, `issued_gemm`, `selects_compression`: the integer tile-cost model that decides which
  weight gradients are compressed (parameter_vjp.rs:9-13, 85-130), with the reference's tile
  constants BM16 / BN32 / BK32.
* group decision (crates/sejong-gpu/src/graph.rs:915-1005): the Matmul nodes sharing one input
  X with rows >= features form a group; the donor is the member with the widest output (the
  LAST such member, Rust `max_by_key`); members are pruned by `selects_compression` with the
  current member count until stable.
* `parameter_indices` (parameter.py:25-62): SplitMix64 from a seed drawn with one
  `rng.next_u64()` (parameter_vjp.rs:190); a partial Fisher-Yates of R donor columns, then of S
  of the NB feature blocks; Rows / Map of the selected feature rows.
* `basis_cgs2` (parameter.py:65-129): classical Gram-Schmidt, twice, of the selected donor
  columns with the small-norm cutoff EPS = gamma(rows * (4 r + 1)) of parameter_vjp.rs:226-235.
* `prepare` / `vjp` (parameter.py:131-191, parameter_vjp.rs:260-321): left = X^T Q,
  E = [Q^T ; (X - Q left^T)[:, selected rows]^T * NB/S], (right ; tail) = E dY.
* the factored gradient G = scale (left right + scatterRows(tail)) (parameter.py:204-244) and
  the compact SGD update w <- w (1 - lr wd [rank > 1]) - lr clip G with the FP64 norm of G
  (crates/sejong-train/src/control_variate.rs:720-774, parameter.py:264-291).

The basis is shared per (rows, rank) and the feature selection per width over a whole backward
pass (graph.rs:974-990), so the RNG advances once per preparation that needed either.
"""
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import model as om
from .rng import MASK64, Rng

BM, BN, BK = 16, 32, 32
F32_EPS = 2.0 ** -23


@dataclass
class VjpConfig:
    """sejong_core::ParameterVjpConfig (crates/sejong-core/src/lib.rs:444-466)."""
    rank: int = 16
    residual_fraction: float = 0.25
    block_rows: int = 32
    seed: int = 7


def _ceil_div(a, b):
    return -(-a // b)


def _next_pow2(n):
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def issued_gemm(m, n, k):
    return 2 * (_ceil_div(m, BM) * BM) * (_ceil_div(n, BN) * BN) * (_ceil_div(k, BK) * BK)


def budget(cfg, n, a, donor):
    rank = min(cfg.rank, n, a, donor)
    blocks = _ceil_div(a, cfg.block_rows)
    selected = max(min(int(np.ceil(blocks * cfg.residual_fraction)), blocks), 1)
    return rank, blocks, selected


def selects_compression(cfg, n, a, b, donor, uses):
    if n < a or uses <= 1:
        return False
    rank, blocks, selected = budget(cfg, n, a, donor)
    if selected == blocks:
        return False
    k = selected * cfg.block_rows
    padded = _ceil_div(n, BM) * BM
    last = max(rank - 1, 0)
    full, tail = last // BN, last % BN
    tiles = BN * full * (full + 1) // 2 + tail * (full + 1)
    streaming = 2 * (4 * padded * BN + padded) * tiles + 5 * padded * rank
    resident = 8 * _next_pow2(n) * _next_pow2(rank) * rank + 5 * _next_pow2(n) * rank
    qr = max(streaming, resident)
    shared = qr + issued_gemm(a, rank, n) + issued_gemm(k, n, rank)
    own = issued_gemm(rank + k, b, n) + issued_gemm(a, b, rank)
    return own * uses + shared < issued_gemm(a, b, n) * uses


def group_active(cfg, n, width, member_widths, donor_width):
    """Indices of the compressed members (graph.rs:944-965)."""
    active = set(range(len(member_widths)))
    while True:
        count = len(active)
        if count == 0:
            break
        active = {i for i in active if selects_compression(cfg, n, width, member_widths[i], donor_width, count)}
        if len(active) == count:
            break
    return active


def donor_index(member_widths):
    """Rust Iterator::max_by_key: the last member of maximal output width."""
    best = 0
    for i, w in enumerate(member_widths):
        if w >= member_widths[best]:
            best = i
    return best


def parameter_indices(seed, a, b, nb, s, r, group):
    """The reference's parameter_indices kernel: (columns[r], rows[s*group], row_map[a])."""
    rng = Rng(seed)
    cols = list(range(b))
    columns = []
    for i in range(r):
        j = i + rng.index(b - i)
        cols[i], cols[j] = cols[j], cols[i]
        columns.append(cols[i])
    blocks = list(range(nb))
    rows = []
    row_map = np.full(a, -1, dtype=np.int64)
    for i in range(s):
        j = i + rng.index(nb - i)
        blocks[i], blocks[j] = blocks[j], blocks[i]
        value = blocks[i]
        for o in range(group):
            index = value * group + o
            position = i * group + o
            rows.append(index if index < a else -1)
            if index < a:
                row_map[index] = position
    return np.asarray(columns, dtype=np.int64), np.asarray(rows, dtype=np.int64), row_map


def basis_eps(rows, rank):
    operations = rows * (4.0 * rank + 1.0)
    roundoff = operations * (F32_EPS / 2.0)
    tol = roundoff / (1.0 - roundoff) if roundoff < 1.0 else np.inf
    return float(np.float32(min(tol, np.finfo(np.float32).max)))


def basis_cgs2(y, eps):
    """CGS2 of the columns of y [N, r] with the reference's small-norm cutoff (FP64)."""
    q = np.array(y, dtype=np.float64, copy=True)
    for cur in range(q.shape[1]):
        v = q[:, cur].copy()
        original = float(v @ v)
        for _ in range(2):
            coef = q[:, :cur].T @ v
            v = v - q[:, :cur] @ coef
        mag = float(v @ v)
        q[:, cur] = v / np.sqrt(mag) if mag > eps * eps * original else 0.0
    return q


@dataclass
class Prepared:
    q: np.ndarray
    left: np.ndarray
    e: np.ndarray
    row_map: np.ndarray
    rows: np.ndarray
    columns: np.ndarray


class VjpState:
    """Per-backward-pass sharing of bases (per (rows, rank)) and feature selections (per width)."""

    def __init__(self, cfg, rng):
        self.cfg = cfg
        self.rng = rng
        self.bases = {}
        self.selections = {}
        self.draws = 0

    def prepare(self, x, donor):
        cfg = self.cfg
        n, a = x.shape
        b = donor.shape[1]
        rank, blocks, selected = budget(cfg, n, a, b)
        basis = self.bases.get((n, rank))
        selection = self.selections.get(a)
        if basis is None or selection is None:
            seed = self.rng.next_u64()
            self.draws += 1
            columns, rows, row_map = parameter_indices(
                seed, a if selection is None else 0, b if basis is None else 0, blocks if selection is None else 0,
                selected if selection is None else 0, rank if basis is None else 0, cfg.block_rows)
            if basis is None:
                q = basis_cgs2(donor[:, columns], basis_eps(n, rank))
                basis = (q, columns)
                self.bases[(n, rank)] = basis
            if selection is None:
                selection = (rows, row_map)
                self.selections[a] = selection
        q, columns = basis
        rows, row_map = selection
        inverse = float(np.float32(blocks) / np.float32(selected))
        left, e = prepare_factors(x, q, rows, inverse)
        return Prepared(q, left, e, row_map, rows, columns)


def prepare_factors(x, q, rows, inverse):
    """parameter_prepare (parameter.py:131-166): left = X^T Q and
    E = [Q^T ; (X - Q left^T)[:, rows] * inverse] (zero rows for padded entries rows[i] < 0)."""
    x = np.asarray(x, dtype=np.float64)
    q = np.asarray(q, dtype=np.float64)
    rank = q.shape[1]
    left = x.T @ q
    e = np.zeros((rank + len(rows), x.shape[0]))
    e[:rank] = q.T
    for pos, row in enumerate(rows):
        if row >= 0:
            e[rank + pos] = (x[:, row] - q @ left[row]) * inverse
    return left, e


def factored_gradient(prep, dy, scale=1.0):
    """G = scale (left right + scatterRows(tail)) with (right; tail) = E dY."""
    coeff = prep.e @ dy
    r = prep.q.shape[1]
    right, tail = coeff[:r], coeff[r:]
    g = prep.left @ right
    sel = prep.row_map >= 0
    g[sel] += tail[prep.row_map[sel]]
    return scale * g, right, tail


def vjp_gradients(params, c, ids, targets, seq, cfg, rng, cast=None, scale=1.0):
    """Loss and the per-parameter gradients of one observation with the parameter VJP.

    The forward runs in FP64 at `compute_cast(params, cast)`; input VJPs are exact (autograd);
    for every compressed Matmul node the weight gradient is the factored one.  Nodes are visited
    in reverse creation order, as the reference tape does, which fixes the RNG consumption order.
    Returns (loss, grads, info) where info lists the compressed weights and the draws.
    """
    params = om.compute_cast(params, cast)
    p = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True) for k, v in params.items()}
    records = []

    def hook(name, x, y):
        if y.requires_grad:
            y.retain_grad()
        records.append((name, x, y))

    om.MATMUL_HOOK = hook
    try:
        ids_t = torch.as_tensor(np.asarray(ids, dtype=np.int64))
        tg_t = torch.as_tensor(np.asarray(targets, dtype=np.int64))
        h = om.hidden(p, c, ids_t, seq)
        logits = om.mm(h, p, "output")
        loss = om.ops.cross_entropy(logits, tg_t).mean()
    finally:
        om.MATMUL_HOOK = None
    (loss * scale).backward()
    grads = {k: (t.grad.detach().numpy().copy() if t.grad is not None else np.zeros(t.shape))
             for k, t in p.items()}
    # group members: Matmul nodes by input tensor, weight a trainable parameter, rows >= features
    members = {}
    for idx, (name, x, y) in enumerate(records):
        if x.dim() == 2 and x.shape[0] >= x.shape[1]:
            members.setdefault(id(x), []).append(idx)
    state = VjpState(cfg, rng)
    groups = {}
    compressed = []
    for idx in reversed(range(len(records))):
        name, x, y = records[idx]
        key = id(x)
        if key not in members or idx not in members[key]:
            continue
        if key not in groups:
            mem = members[key]
            widths = [records[i][2].shape[1] for i in mem]
            donor = mem[donor_index(widths)]
            n, width = x.shape
            active = group_active(cfg, n, width, widths, records[donor][2].shape[1])
            if active:
                prep = state.prepare(x.detach().numpy(), records[donor][2].detach().numpy())
                groups[key] = (prep, {mem[i] for i in active})
            else:
                groups[key] = None
        group = groups[key]
        if group is not None and idx in group[1]:
            g, _, _ = factored_gradient(group[0], y.grad.detach().numpy())
            grads[name] = grads[name] - (x.detach().T @ y.grad.detach()).numpy() + g  # replace dense part
            compressed.append(name)
    info = {"compressed": compressed, "draws": state.draws, "selections": state.selections,
            "bases": {k: v[1] for k, v in state.bases.items()}}
    return float(loss.detach()), grads, info


def sgd_update(params, grads, tc, step):
    """Compact SGD (control_variate.rs:720-774): FP64 norm, clip, w (1 - lr wd) - lr clip G."""
    norm = float(np.sqrt(sum(float(np.sum(np.asarray(g, dtype=np.float64) ** 2)) for g in grads.values())))
    clipping = float(np.float32(tc.clip_norm / norm)) if (tc.clip_enabled and norm > tc.clip_norm) else 1.0
    lr = om.ops.lr_schedule(step, tc.learning_rate, tc.min_learning_rate, tc.warmup_steps, tc.steps)
    out = {}
    for name, w in params.items():
        decay = lr * tc.weight_decay if np.ndim(w) > 1 else 0.0
        out[name] = np.asarray(w, dtype=np.float64) * (1.0 - decay) - lr * clipping * np.asarray(grads[name])
    return out, norm
