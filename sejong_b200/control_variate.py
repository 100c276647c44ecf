"""Control-variate SGD (crates/sejong-train/src/control_variate.rs:236-877) on the byte-model step.

Each optimizer step draws `accumulation` observations.  A stratified (or uniform) sample of
`controls` of them, weighted N_h / (M m_h) per stratum (`control_weights`), runs the full forward
and backward; every observation runs the encoder and gives an augmented feature [mean encoded row,
mean target-embedding row, mean of their product, 1].  For each predicted matrix W [a, b] (every
matrix outside the embedding, the encoder, the input projection, the routers and the experts) the
trainer keeps orthonormal bases U [a, r], V [b, r], a deferred coefficient A [r, r] and a linear
predictor P [3 w + 1, r^2] of the projected gradient U^T G V from the feature.  The step
  * binds W + U A V^T as the compute weight (Model::bind_with_corrections with the low-rank matmul
    of graph.rs:244-271 folded into the bound weight),
  * applies the weighted control gradients to W with dense SGD, the control-variate correction
    delta = mean prediction - weighted control prediction to A (A <- A (1 - lr wd) - lr clip delta),
    and a least-squares step to P, with the correction's norm terms in the clipped gradient norm,
  * every `basis_refresh` steps folds U A V^T into W, and rebuilds U and V from the first two
    controls' gradient sketches (G V, G^T U, contrasted when there are two), transporting P's
    coefficients into the new bases.

Every operation runs in libsejong_b200.so: the trainer's step kernels, sj_sgemm for the f32 small
products, and the sj_cv_* kernels; the host holds the generators and the sampling decisions.
The parameter VJP is not combined with control variates here (`ControlVariateTrainer` refuses it).
"""
import ctypes
import math
import time
from dataclasses import dataclass, replace

import numpy as np
import torch

from . import _lib
from ._lib import EPI_ACCUM, EPI_STORE, SJ_F32, call
from .checkpoint import SGD_BASIS_MIX, SGD_SAMPLING_MIX
from .model import INTERLEAVE, VOCAB, reference_layout
from .train import ByteTrainer, _ptr

F32_EPS_SQRT = float(np.sqrt(np.float32(np.finfo(np.float32).eps)))


@dataclass
class ControlVariateConfig:
    """sejong_core::ControlVariateConfig (crates/sejong-core/src/lib.rs:477-507)."""
    controls: int
    rank: int
    sampling: str = "stratified"   # "uniform" | "stratified"
    strata: int = 1
    basis_refresh: int = 32
    predictor_learning_rate: float = 1e-3

    def validate(self, observations):
        if not 0 < self.controls <= observations:
            raise ValueError("control_variate.controls must be in 1..=accumulation")
        if self.rank <= 0 or self.basis_refresh <= 0:
            raise ValueError("control_variate.rank and basis_refresh must be positive")
        if not (math.isfinite(self.predictor_learning_rate) and self.predictor_learning_rate > 0):
            raise ValueError("control_variate.predictor_learning_rate must be finite and positive")
        if self.sampling not in ("uniform", "stratified"):
            raise ValueError(f"control_variate.sampling {self.sampling!r}")
        if self.sampling == "stratified" and not (0 < self.strata <= self.controls and self.strata <= observations):
            raise ValueError("stratified sampling requires 1 <= strata <= controls <= accumulation")


def predicted_parameter(name, shape):
    """predicted_parameter (control_variate.rs:31-40)."""
    return (len(shape) == 2 and name not in ("embedding", "global_bos", "input_projection")
            and not name.startswith("encoder.") and not name.endswith(".router")
            and ".experts." not in name and ".expert." not in name)


def entropy(values):
    """entropy (control_variate.rs:289-303): Shannon entropy (nats) of the byte histogram, FP64."""
    counts = np.bincount(np.asarray(values, dtype=np.int64).reshape(-1), minlength=257)
    n = float(np.asarray(values).size)
    total = 0.0
    for c in counts:  # the reference sums in bin order
        if c > 0:
            p = float(c) / n
            total += -p * math.log(p)
    return total


def control_weights(inputs, cv, rng_state, lib=None):
    """control_weights (control_variate.rs:305-349): f32 weight per observation, N_h / (M m_h) for the
    m_h observations drawn (partial Fisher-Yates with Rng::index) from each stratum h of N_h, 0 for
    the rest.  Strata are equal slices of the observations sorted by input entropy (ties by index);
    the controls beyond one per stratum go, one at a time, to the stratum with the largest N_h /
    (m_h + 1) that has observations left (ties to the lowest stratum).  `rng_state` is a
    ctypes.c_uint64 advanced in place."""
    lib = lib or _lib.load()
    count = len(inputs)
    strata = 1 if cv.sampling == "uniform" else cv.strata
    order = list(range(count))
    if strata > 1:
        ent = [entropy(x) for x in inputs]
        order.sort(key=lambda i: (ent[i], i))
    groups = [order[h * count // strata:(h + 1) * count // strata] for h in range(strata)]
    alloc = [1] * strata
    for _ in range(strata, cv.controls):
        best = None
        for h in range(strata):
            if alloc[h] >= len(groups[h]):
                continue
            ratio = len(groups[h]) / (alloc[h] + 1)
            if best is None or ratio > best[0]:
                best = (ratio, h)
        if best is None:
            raise ValueError("validated control count fits strata")
        alloc[best[1]] += 1
    weights = np.zeros(count, dtype=np.float32)
    for group, selected in zip(groups, alloc):
        weight = np.float32(len(group)) / np.float32(count * selected)
        group = list(group)
        for i in range(selected):
            j = i + int(lib.sj_rng_index(ctypes.byref(rng_state), len(group) - i))
            group[i], group[j] = group[j], group[i]
            weights[group[i]] = weight
    return weights


@dataclass
class Block:
    """A predicted reference matrix [a, b] inside fused layout entry `entry` [a, fused_cols]: its
    columns sit at `cols` (the qkv concatenation, the gate/up interleave, the padded head)."""
    name: str
    a: int
    b: int
    entry: str
    fused_cols: int
    cols: np.ndarray


def member_columns(entry, part, ref_shapes):
    """Fused-layout columns of reference matrix `part` of FlatLayout entry `entry`."""
    b = ref_shapes[part][1]
    if entry.name.endswith(".qkv"):
        q, k, _ = entry.parts
        start = {0: 0, 1: ref_shapes[q][1], 2: ref_shapes[q][1] + ref_shapes[k][1]}[entry.parts.index(part)]
        return np.arange(start, start + b, dtype=np.int32)
    if entry.name.endswith(".gate_up"):
        j = np.arange(b, dtype=np.int32)
        base = (j // INTERLEAVE) * (2 * INTERLEAVE) + j % INTERLEAVE
        return base if part == entry.parts[0] else base + INTERLEAVE
    return np.arange(b, dtype=np.int32)


class ControlVariateTrainer:
    """The control-variate SGD loop of control_variate::train_configured over a ByteTrainer."""

    def __init__(self, config, train, cv, device=None, params=None):
        if train.parameter_vjp is not None:
            raise ValueError("control-variate SGD with the parameter VJP is not supported by this build")
        if train.values:
            raise ValueError("control-variate SGD is the byte model's trainer (no value head)")
        if config.hierarchy is not None and train.sequence <= config.hierarchy.patch_size:
            raise ValueError("control-variate training sequence must exceed patch_size to observe global gradients")
        accumulation = int(train.accumulation)
        cv.validate(accumulation)
        self.cv = cv
        self.tc = replace(train, optimizer="sgd")
        self.tr = ByteTrainer(config, self.tc, device=device, params=params)
        self.c = config
        self.lib = self.tr.lib
        tr = self.tr
        dev = tr.dev
        f32 = torch.float32
        ref = reference_layout(config)
        ref_shapes = {n: s for n, s, _ in ref}
        owner = {}
        for e in tr.layout.entries.values():
            for part in e.parts:
                owner[part] = e
        r = cv.rank
        self.blocks = []
        for name, shape, _ in ref:
            if not predicted_parameter(name, shape):
                continue
            if r > min(shape):
                raise ValueError(f"predictor rank {r} exceeds matrix dimensions of {name}")
            e = owner[name]
            self.blocks.append(Block(name, shape[0], shape[1], e.name, e.shape[1],
                                     member_columns(e, name, ref_shapes)))
        if not self.blocks:
            raise ValueError("control-variate training requires a predicted matrix")
        nb, rr = len(self.blocks), r * r
        self.width = config.hierarchy.encoder_width if config.hierarchy is not None else config.width
        self.features = 3 * self.width + 1
        F = self.features
        z = lambda *s: torch.zeros(*s, dtype=f32, device=dev)  # noqa: E731
        self.U = [z(bk.a, r) for bk in self.blocks]
        self.V = [z(bk.b, r) for bk in self.blocks]
        self.Vsc = [z(bk.fused_cols, r) for bk in self.blocks]
        self.maps = [torch.from_numpy(bk.cols).to(dev) for bk in self.blocks]
        self.GU, self.GV = z(nb, r, r), z(nb, r, r)
        self.A = z(nb, r, r)
        self.P = z(F, nb * rr)
        # per step
        self.feat = z(F)
        self.pred = z(nb * rr)
        self.mean_pred, self.ctrl_pred, self.mean_target = z(nb * rr), z(nb * rr), z(nb * rr)
        self.T, self.delta = z(nb * rr), z(nb * rr)
        self.PG = z(F, nb * rr)
        self.SL = [z(bk.a, r) for bk in self.blocks]
        self.SR = [z(bk.b, r) for bk in self.blocks]
        amax = max(bk.a for bk in self.blocks)
        fmax = max(bk.fused_cols for bk in self.blocks)
        self.tmp_a = z(amax * r)
        self.tmp_f = z(fmax * r)
        self.tmp_b = z(max(bk.b for bk in self.blocks) * r)
        self.corr = z(max(bk.a * bk.fused_cols for bk in self.blocks))
        self.ov_l, self.ov_r = z(r, r), z(r, r)
        self.eye = torch.eye(r, dtype=f32, device=dev)
        self.ident = torch.arange(nb, dtype=torch.int32, device=dev)
        self.G = z(tr.layout.total)
        self.partials = torch.zeros(tr.n_partials + nb, dtype=torch.float64, device=dev)
        self.terms = torch.zeros(nb, dtype=torch.float64, device=dev)
        self.norm_partials = torch.zeros(self.lib.sj_sumsq_partials(max(tr.layout.total, F * nb * rr)),
                                         dtype=torch.float64, device=dev)
        self.emb_off = tr.layout["embedding"].offset
        self.step_count = 0
        seed = int(train.seed)
        self.sampling_rng = ctypes.c_uint64((seed ^ SGD_SAMPLING_MIX) & (2**64 - 1))
        self.basis_rng = ctypes.c_uint64((seed ^ SGD_BASIS_MIX) & (2**64 - 1))
        self._init_bases()

    # ------------------------------------------------------------------ helpers
    @property
    def s(self):
        return self.tr.stream

    def _sgemm(self, a, lda, at, b, ldb, bt, c, ldc, m, n, k, epi=EPI_STORE):
        call("sj_sgemm", a, lda, at, b, ldb, bt, c, ldc, m, n, k, epi, None, 0, None, 0, 0, self.s)

    def _add(self, x, z, y, n, alpha):
        """y = x + alpha z (f32, n elements)."""
        call("sj_add", x, z, y, n, float(alpha), SJ_F32, self.s)

    def _sumsq(self, ptr, n):
        """FP64 sum of squares of n f32 values (host value; synchronises)."""
        call("sj_grad_sumsq", ptr, n, _ptr(self.norm_partials), self.s)
        k = self.lib.sj_sumsq_partials(n)
        return float(self.norm_partials[:k].sum().item())

    def _orthonormalize(self, x, q, j, gram):
        bk_rows, r = x.shape
        call("sj_cv_orthonormalize", _ptr(x), _ptr(q), _ptr(gram), bk_rows, r, self.s)

    def _scatter_v(self, j):
        bk = self.blocks[j]
        call("sj_cv_scatter_rows", _ptr(self.V[j]), bk.b, self.cv.rank, _ptr(self.maps[j]), _ptr(self.Vsc[j]),
             bk.fused_cols, self.s)

    def _init_bases(self):
        """SgdState::new (control_variate.rs:67-121): per predicted matrix, a * r then b * r normal
        draws of the basis generator, each orthonormalised, and their Gram matrices."""
        r = self.cv.rank
        for j, bk in enumerate(self.blocks):
            for rows, dst, gram in ((bk.a, self.U[j], self.GU[j]), (bk.b, self.V[j], self.GV[j])):
                vals = np.empty(rows * r, dtype=np.float32)
                call("sj_rng_normal_fill", ctypes.byref(self.basis_rng), vals.ctypes.data, vals.size, 1.0)
                x = torch.from_numpy(vals.reshape(rows, r)).to(self.tr.dev)
                self._orthonormalize(x, dst, j, gram)
                torch.cuda.current_stream(self.tr.dev).synchronize()
            self._scatter_v(j)

    def _entries(self):
        """Predicted blocks grouped by their fused layout entry."""
        groups = {}
        for j, bk in enumerate(self.blocks):
            groups.setdefault(bk.entry, []).append(j)
        return groups

    def _correction(self, entry, members):
        """self.corr [a, fused cols] = sum over the entry's members of (U A) Vsc^T."""
        r = self.cv.rank
        e = self.tr.layout[entry]
        a, fc = e.shape
        first = True
        for j in members:
            self._sgemm(_ptr(self.U[j]), r, 0, _ptr(self.A[j]), r, 0, _ptr(self.tmp_a), r, a, r, r)
            if first:
                call("sj_zero", _ptr(self.corr), a * fc * 4, self.s)
                first = False
            self._sgemm(_ptr(self.tmp_a), r, 0, _ptr(self.Vsc[j]), r, 1, _ptr(self.corr), fc, a, fc, r, EPI_ACCUM)
        return e, a * fc

    def bind(self):
        """The compute weights of the corrected matrices: bf16(W + U A V^T)."""
        tr = self.tr
        for entry, members in self._entries().items():
            e, n = self._correction(entry, members)
            call("sj_cv_bind", _ptr(tr.w, e.offset), _ptr(self.corr), _ptr(tr.wb, e.offset), n, self.s)

    def flush(self):
        """SgdState::flush (control_variate.rs:235-246): W += U A V^T, A = 0."""
        tr = self.tr
        for entry, members in self._entries().items():
            e, n = self._correction(entry, members)
            self._add(_ptr(tr.w, e.offset), _ptr(self.corr), _ptr(tr.w, e.offset), n, 1.0)
        call("sj_zero", _ptr(self.A), self.A.numel() * 4, self.s)
        call("sj_cast", _ptr(tr.w), SJ_F32, _ptr(tr.wb), _lib.SJ_BF16, tr.layout.total, self.s)

    # ------------------------------------------------------------------ the step
    def _feature(self, enc, dtype, width):
        tr = self.tr
        call("sj_cv_feature", _ptr(enc), dtype, width, _ptr(tr.w, self.emb_off), width, _ptr(tr.targets),
             tr.rows, width, VOCAB, _ptr(self.feat), self.s)

    def step(self, observations):
        """One optimizer step over `accumulation` observations [(ids, targets), ...] (host int arrays
        of batch x sequence).  Returns the step's metrics (the fields of the reference's record)."""
        tr, cv, tc = self.tr, self.cv, self.tc
        r, nb = cv.rank, len(self.blocks)
        rr = r * r
        n_pred = nb * rr
        F = self.features
        ls = float(tc.loss_scale)
        acc = len(observations)
        if acc != int(tc.accumulation):
            raise ValueError(f"{acc} observations for accumulation {tc.accumulation}")
        refreshed = (self.step_count + 1) % cv.basis_refresh == 0
        gde = int(tc.gradient_diagnostics_every)
        diagnostics = gde > 0 and (self.step_count + 1) % gde == 0
        measure = bool(tc.clip_enabled) or diagnostics
        inputs = [np.asarray(ids).reshape(-1) for ids, _ in observations]
        weights = control_weights(inputs, cv, self.sampling_rng, self.lib)
        controls = int((weights > 0).sum())
        tr.stream = torch.cuda.current_stream(tr.dev).cuda_stream
        self.bind()
        for t in (self.G, self.mean_pred, self.ctrl_pred, self.mean_target, self.PG):
            call("sj_zero", _ptr(t), t.numel() * 4, self.s)
        losses = torch.zeros(controls, dtype=torch.float64, device=tr.dev)
        gsm = rsm = mse = 0.0
        diag_seconds = 0.0
        k = 0
        for (ids, targets), w in zip(observations, weights):
            tr.stage_batch(ids, targets)
            w = float(w)
            if w > 0:
                tr.obs_weight = w
                tr._local_forward_backward(first=True)   # g = w * loss_scale * grad of the mean CE
                losses[k:k + 1].copy_(tr.loss_sum)
                self._add(_ptr(self.G), _ptr(tr.g), _ptr(self.G), tr.layout.total, 1.0)
                enc, dt, width = ((tr.zE, _lib.SJ_BF16, self.width) if self.c.hierarchy is not None
                                  else (tr.runs["global"].x[0], SJ_F32, self.width))
            else:
                enc, dt, width = tr.encode()
            self._feature(enc, dt, width)
            self._sgemm(_ptr(self.feat), F, 0, _ptr(self.P), n_pred, 0, _ptr(self.pred), n_pred, 1, n_pred, F)
            self._add(_ptr(self.mean_pred), _ptr(self.pred), _ptr(self.mean_pred), n_pred, 1.0 / acc)
            if w <= 0:
                continue
            inv = 1.0 / (w * ls)
            for j, bk in enumerate(self.blocks):
                e = tr.layout[bk.entry]
                # tmp = G_F Vsc [a, r] (= G V);  T_j = U^T tmp
                self._sgemm(_ptr(tr.g, e.offset), bk.fused_cols, 0, _ptr(self.Vsc[j]), r, 0, _ptr(self.tmp_a), r,
                            bk.a, r, bk.fused_cols)
                self._sgemm(_ptr(self.U[j]), r, 1, _ptr(self.tmp_a), r, 0, _ptr(self.T, j * rr), r, r, r, bk.a)
                if refreshed and k < 2:
                    # sketches (control_variate.rs:676-697): G V and G^T U of the first control, minus the
                    # second's when there is one
                    sign = 1.0 if k == 0 else -1.0
                    if k == 0:
                        call("sj_zero", _ptr(self.SL[j]), self.SL[j].numel() * 4, self.s)
                        call("sj_zero", _ptr(self.SR[j]), self.SR[j].numel() * 4, self.s)
                    self._add(_ptr(self.SL[j]), _ptr(self.tmp_a), _ptr(self.SL[j]), bk.a * r, sign * inv)
                    self._sgemm(_ptr(tr.g, e.offset), bk.fused_cols, 1, _ptr(self.U[j]), r, 0, _ptr(self.tmp_f), r,
                                bk.fused_cols, r, bk.a)
                    call("sj_cv_gather_rows", _ptr(self.tmp_f), bk.fused_cols, r, _ptr(self.maps[j]),
                         _ptr(self.tmp_b), bk.b, sign * inv, self.s)
                    self._add(_ptr(self.SR[j]), _ptr(self.tmp_b), _ptr(self.SR[j]), bk.b * r, 1.0)
            # targets in gradient units: T / (w loss_scale)
            call("sj_cv_gather_rows", _ptr(self.T), nb, rr, _ptr(self.ident), _ptr(self.T), nb, inv, self.s)
            if measure:
                self._add(_ptr(self.mean_target), _ptr(self.T), _ptr(self.mean_target), n_pred, w)
            self._add(_ptr(self.ctrl_pred), _ptr(self.pred), _ptr(self.ctrl_pred), n_pred, w)
            if diagnostics:
                t_diag = time.perf_counter()
                sample = self._sumsq(_ptr(tr.g), tr.layout.total) / (w * ls) ** 2
                gsm += w * sample
                rsm += w * sample
                self._add(_ptr(self.pred), _ptr(self.T), _ptr(self.delta), n_pred, -1.0)  # residual = pred - T
                mse += w * self._sumsq(_ptr(self.delta), n_pred) / rr
                call("sj_cv_block_terms", _ptr(self.GU), _ptr(self.GV), _ptr(self.pred), _ptr(self.T),
                     _ptr(self.terms), nb, r, -2.0, 1.0, self.s)
                rsm += w * float(self.terms.sum().item())
                diag_seconds += time.perf_counter() - t_diag
            call("sj_cv_outer", _ptr(self.feat), F, _ptr(self.pred), _ptr(self.T), 1.0, n_pred, 2.0 * w / rr,
                 _ptr(self.PG), self.s)
            k += 1
        tr.obs_weight = None
        # delta = mean prediction - weighted control prediction (control_variate.rs:692-698)
        self._add(_ptr(self.mean_pred), _ptr(self.ctrl_pred), _ptr(self.delta), n_pred, -1.0)
        # the clipped norm: |G|^2 (FP64 partials) + per block <D, GU D GV> + 2 <mean target, D>, all in
        # loss-scaled units
        n0 = tr.n_partials
        call("sj_grad_sumsq", _ptr(self.G), tr.layout.total, _ptr(self.partials), self.s)
        if measure:
            call("sj_cv_block_terms", _ptr(self.GU), _ptr(self.GV), _ptr(self.delta), _ptr(self.mean_target),
                 _ptr(self.partials, n0), nb, r, 2.0, ls * ls, self.s)
        else:
            call("sj_zero", _ptr(self.partials, n0), nb * 8, self.s)
        call("sj_optim_prepare", _ptr(self.partials), n0 + nb, _ptr(tr.opt_state), _ptr(tr.hyper),
             tc.learning_rate, tc.min_learning_rate, tc.warmup_steps, tc.steps, tc.beta1, tc.beta2, tc.clip_norm,
             int(tc.clip_enabled), tc.loss_scale, self.s)
        call("sj_sgd", _ptr(tr.w), _ptr(self.G), _ptr(tr.wb), tr.layout.total, tr.layout.n_decay, _ptr(tr.hyper),
             tc.weight_decay, self.s)
        call("sj_cv_deferred_update", _ptr(self.A), _ptr(self.delta), _ptr(tr.hyper), tc.weight_decay, ls, n_pred,
             self.s)
        self._add(_ptr(self.P), _ptr(self.PG), _ptr(self.P), F * n_pred, -cv.predictor_learning_rate)
        base_norm = None
        if diagnostics:
            t_diag = time.perf_counter()
            base_norm = self._sumsq(_ptr(self.G), tr.layout.total) / (ls * ls)
            call("sj_cv_block_terms", _ptr(self.GU), _ptr(self.GV), _ptr(self.ctrl_pred), _ptr(self.mean_target),
                 _ptr(self.terms), nb, r, -2.0, 1.0, self.s)
            residual_mean = base_norm + float(self.terms.sum().item())
            diag_seconds += time.perf_counter() - t_diag
        self.step_count += 1
        if refreshed:
            self.refresh_bases()
        torch.cuda.current_stream(tr.dev).synchronize()
        loss = float(losses.sum().item())
        hyper = tr.hyper.cpu().numpy()
        out = {"loss": loss, "controls": controls, "basis_refreshed": refreshed,
               "gradient_norm": float(hyper[4]) if measure else None, "learning_rate": float(hyper[0]),
               "gradient_diagnostics": diagnostics, "weights": weights}
        if diagnostics:
            gd = max(gsm - base_norm, 0.0)
            rd = max(rsm - residual_mean, 0.0)
            out.update(predictor_mse=mse, control_gradient_dispersion=gd, control_residual_dispersion=rd,
                       diagnostic_seconds=diag_seconds,
                       residual_variance_ratio_diagnostic=(rd / gd if controls > 1 and gd > 0 else None))
        return out

    def refresh_bases(self):
        """SgdState::refresh_bases (control_variate.rs:248-282)."""
        self.flush()
        r, nb = self.cv.rank, len(self.blocks)
        rr = r * r
        P_new = self.P.clone()
        for j, bk in enumerate(self.blocks):
            mag2 = self._sumsq(_ptr(self.SL[j]), bk.a * r) + self._sumsq(_ptr(self.SR[j]), bk.b * r)
            magnitude = np.float32(math.sqrt(mag2))
            if magnitude == 0:
                continue
            reg = float(magnitude * np.float32(F32_EPS_SQRT))
            U_new = torch.empty_like(self.U[j])
            V_new = torch.empty_like(self.V[j])
            self._add(_ptr(self.SL[j]), _ptr(self.U[j]), _ptr(self.SL[j]), bk.a * r, reg)
            self._orthonormalize(self.SL[j], U_new, j, self.GU[j])
            self._add(_ptr(self.SR[j]), _ptr(self.V[j]), _ptr(self.SR[j]), bk.b * r, reg)
            self._orthonormalize(self.SR[j], V_new, j, self.GV[j])
            # U_old^T U_new and V_old^T V_new move each feature's coefficient into the new bases
            self._sgemm(_ptr(self.U[j]), r, 1, _ptr(U_new), r, 0, _ptr(self.ov_l), r, r, r, bk.a)
            self._sgemm(_ptr(self.V[j]), r, 1, _ptr(V_new), r, 0, _ptr(self.ov_r), r, r, r, bk.b)
            call("sj_cv_transport", _ptr(self.P), nb * rr, j * rr, _ptr(self.ov_l), _ptr(self.ov_r), _ptr(P_new),
                 self.features, r, self.s)
            self.U[j], self.V[j] = U_new, V_new
            self._scatter_v(j)
        torch.cuda.current_stream(self.tr.dev).synchronize()
        self.P = P_new

    # ------------------------------------------------------------------ state
    def state_tensors(self):
        """SgdState::tensors (control_variate.rs:208-233) after a flush: sgd.version, the sampling and
        basis generators, and cv.<name>.{left, right, deferred, predictor} per predicted matrix."""
        from .checkpoint import rng_words
        self.flush()
        torch.cuda.current_stream(self.tr.dev).synchronize()
        r = self.cv.rank
        rr = r * r
        out = {"sgd.version": np.array([1.0], dtype=np.float32),
               "sgd.sampling_rng": rng_words(self.sampling_rng.value),
               "sgd.basis_rng": rng_words(self.basis_rng.value)}
        P = self.P.cpu().numpy()
        for j, bk in enumerate(self.blocks):
            out[f"cv.{bk.name}.left"] = self.U[j].cpu().numpy()
            out[f"cv.{bk.name}.right"] = self.V[j].cpu().numpy()
            out[f"cv.{bk.name}.deferred"] = self.A[j].cpu().numpy()
            out[f"cv.{bk.name}.predictor"] = np.ascontiguousarray(P[:, j * rr:(j + 1) * rr])
        return out

    def load_state_tensors(self, tensors):
        """SgdState::load (control_variate.rs:122-195) for the control-variate route."""
        from .checkpoint import ArtifactError, rng_from_words
        version = tensors.get("sgd.version")
        if version is None or np.shape(version) != (1,) or float(np.asarray(version)[0]) != 1.0:
            raise ArtifactError("unsupported or missing SGD state version")
        r = self.cv.rank
        rr = r * r
        expected = 3 + 4 * len(self.blocks)
        if len(tensors) != expected:
            raise ArtifactError("SGD checkpoint tensor count differs from its configuration")
        self.sampling_rng.value = rng_from_words(tensors["sgd.sampling_rng"], "sgd.sampling_rng")
        self.basis_rng.value = rng_from_words(tensors["sgd.basis_rng"], "sgd.basis_rng")
        P = np.zeros((self.features, len(self.blocks) * rr), dtype=np.float32)
        for j, bk in enumerate(self.blocks):
            shapes = {"left": (bk.a, r), "right": (bk.b, r), "deferred": (r, r), "predictor": (self.features, rr)}
            for suffix, shape in shapes.items():
                key = f"cv.{bk.name}.{suffix}"
                if key not in tensors or tuple(np.shape(tensors[key])) != shape:
                    raise ArtifactError(f"control-variate state {key} missing or misshapen")
            self.U[j].copy_(torch.from_numpy(np.asarray(tensors[f"cv.{bk.name}.left"], np.float32)))
            self.V[j].copy_(torch.from_numpy(np.asarray(tensors[f"cv.{bk.name}.right"], np.float32)))
            self.A[j].copy_(torch.from_numpy(np.asarray(tensors[f"cv.{bk.name}.deferred"], np.float32)))
            P[:, j * rr:(j + 1) * rr] = tensors[f"cv.{bk.name}.predictor"]
            self._scatter_v(j)
            self._sgemm(_ptr(self.U[j]), r, 1, _ptr(self.U[j]), r, 0, _ptr(self.GU[j]), r, r, r, bk.a)
            self._sgemm(_ptr(self.V[j]), r, 1, _ptr(self.V[j]), r, 0, _ptr(self.GV[j]), r, r, r, bk.b)
        self.P.copy_(torch.from_numpy(P))
        torch.cuda.current_stream(self.tr.dev).synchronize()

    def parameters(self):
        """Reference-named f32 master weights (the base W, without the deferred correction)."""
        return self.tr.parameters()

    def snapshot(self):
        """What `save` (control_variate.rs:389-406) writes: the deferred correction folded into the
        weights first, then the weights and the state tensors."""
        tensors = self.state_tensors()
        return self.parameters(), tensors

    def close(self):
        self.tr.close()
