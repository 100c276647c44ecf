"""The byte-Transformer training step on one B200: an explicit schedule of fused kernels.

Replaces the reference's per-observation tape (crates/sejong-gpu/src/graph.rs:67-913)
and training loops (crates/sejong-train/src/lib.rs:387-453, AdamW;
control_variate.rs:767-799, plain SGD) for the dense and hierarchical byte models
(crates/sejong-model/src/architecture.rs:201-393).  Instead of a tape of ~1,400
small launches per step, the step is a fixed sequence of C-ABI calls
(include/sejong.h) over buffers allocated once:

  forward   embedding -> blocks [RMSNorm, QKV GEMM + RoPE epilogue, GQA attention,
            Wo GEMM + residual epilogue, RMSNorm, gate/up GEMM + SwiGLU epilogue,
            down GEMM + residual epilogue] -> (hierarchy: encoder norm, patch pool,
            global blocks, broadcast, decoder blocks) -> final norm -> head GEMM (f32
            logits) -> fused cross entropy (loss, dlogits)
  backward  the same in reverse: weight gradients as TN GEMMs accumulating into one
            flat f32 gradient buffer, input gradients as NT GEMMs, RMSNorm backward
            fused with the residual-gradient add, attention backward with the inverse
            RoPE in its dq/dk store
  update    FP64 gradient norm -> device-side clip / LR / bias correction -> one
            multi-tensor AdamW (or SGD) launch that also writes the bf16 weights the
            next forward reads.

Every activation is retained (the reference's "retain" mode); the step issues no
host synchronisation, so it can be captured in a CUDA graph (`capture`).
Precision: bf16 weights and activations, f32 accumulation, f32 gradients, master
weights and moments, FP64 loss and gradient norm.
"""
import ctypes
import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib, distributed, param_vjp
from .expert_parallel import EpContext
from ._lib import (EPI_ACCUM, EPI_RESIDUAL, EPI_ROPE, EPI_STORE, EPI_SWIGLU, SJ_BF16, SJ_F32, call)
from .model import (HEAD_DIM, NATIVE_VOCAB, VOCAB, VOCAB_PAD, FlatLayout, global_stage, initialize, local_stage,
                    reference_layout, router_pad)


@dataclass
class TrainConfig:
    """sejong_core::TrainConfig fields used by the step (crates/sejong-core/src/lib.rs:308-434)."""
    sequence: int
    batch: int
    optimizer: str = "adamw"          # "adamw" | "sgd"
    learning_rate: float = 3e-4
    min_learning_rate: float = 3e-5
    warmup_steps: int = 0
    steps: int = 10000
    beta1: float = 0.9
    beta2: float = 0.95
    epsilon: float = 1e-8
    weight_decay: float = 0.1
    clip_norm: float = 1.0
    clip_enabled: bool = True
    loss_scale: float = 1.0
    seed: int = 123
    # weight gradients through the parameter VJP (low-rank factors + selected rows), as the
    # reference's control-variate trainer does (crates/sejong-train/src/control_variate.rs)
    parameter_vjp: Optional[param_vjp.VjpConfig] = None
    # NativeValue training (crates/sejong-train/src/memory.rs:799-1065) when > 0: the number of values
    # of the categorical head; `batch` requests per step, each padded to `sequence` bytes
    values: int = 0
    # loop settings of the train CLI (TrainConfig::checkpoint_every / log_every /
    # gradient_diagnostics_every, crates/sejong-core/src/lib.rs:308-362); the step itself ignores them
    # MoE additions the reference lacks (opt-in; 0 keeps its semantics): the capacity factor of each
    # expert (capacity = ceil(factor * rows * top_k / experts), sj_route_capacity) and the weight of
    # the load-balancing loss (sj_moe_aux)
    moe_capacity_factor: float = 0.0
    moe_aux_loss_weight: float = 0.0
    # observations per optimizer step (TrainConfig::accumulation): each observation's loss and
    # gradient enter with weight 1 / accumulation (crates/sejong-train/src/lib.rs:387-415)
    accumulation: int = 1
    checkpoint_every: int = 500
    log_every: int = 10
    gradient_diagnostics_every: int = 0
    # recompute the forward of each global-stage block inside the backward from its saved input
    # instead of keeping its activations (Graph::checkpoint, crates/sejong-gpu/src/graph.rs:151-174)
    activation_checkpointing: bool = False
    # the control-variate budget (a control_variate.ControlVariateConfig) of optimizer
    # "control_variate_sgd", which control_variate.ControlVariateTrainer runs
    control_variate: Optional[object] = None


def _ptr(t, offset_elems=0):
    return t.data_ptr() + offset_elems * t.element_size()


class _StageRun:
    """Activation and gradient buffers of one stage (encoder, global or decoder)."""

    def __init__(self, stage, batch, seq, dev, ep=None, checkpoint=False):
        self.stage, self.batch, self.seq = stage, batch, seq
        n, d, f, cq = batch * seq, stage.width, stage.ffn, stage.qkv_width
        self.rows = n
        bf, f32 = torch.bfloat16, torch.float32
        e = lambda *s, dt=bf: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        # the residual stream (block inputs x[i], x[L] = stage output, and the mid-block x1) is f32;
        # GEMM operands (normalised activations, attention output, SwiGLU output) are bf16
        self.x = [e(n, d, dt=f32) for _ in range(stage.layers + 1)]
        # activation checkpointing (Graph::checkpoint, crates/sejong-gpu/src/graph.rs:151-174): only the
        # block inputs x[i] are kept; every block shares one set of activation buffers, which the
        # backward refills by running the block's forward again just before the block's backward
        self.checkpoint = bool(checkpoint)
        self.layers = []
        for i in range(stage.layers):
            if self.checkpoint and i > 0:
                self.layers.append(self.layers[0])
                continue
            self.layers.append(dict(z1=e(n, d), inv1=e(n, dt=f32), qkv=e(n, cq), o=e(n, d),
                                    lse=e(n * stage.heads, dt=f32), x1=e(n, d, dt=f32), z2=e(n, d),
                                    inv2=e(n, dt=f32), gu=e(n, 2 * f), h=e(n, f)))
        # backward workspace
        self.dx = e(n, d, dt=f32)
        self.dxb = e(n, d)
        self.dz = e(n, d, dt=f32)
        self.dh = e(n, f)
        self.dgu = e(n, 2 * f)
        self.do = e(n, d)
        self.dqkv = e(n, cq)
        self.delta = e(_lib.load().sj_attn_workspace(batch, seq, stage.heads, stage.kv_heads), dt=f32)
        self.partials = e(_lib.load().sj_rmsnorm_workspace(n, d), dt=f32)
        self.moe = stage.experts is not None
        self.ep = ep if self.moe else None
        if self.moe:  # the load-balancing loss's per-256-row partials (sj_moe_aux)
            self.aux_ws = e(max(1, _lib.load().sj_moe_aux_workspace(n, stage.experts.count)), dt=f32)
        if self.ep is not None:
            # expert-parallel MoE: this rank routes its own rows and runs its experts on every rank's
            # rows routed to them; the packed A / expert output of each layer, d_out and dA live in the
            # symmetric heap (peers write and read them), the rest is rank-local
            ex, W = stage.experts, ep.world
            local = ex.count // W
            cap = _lib.load().sj_ep_receive_capacity(n, ex.top_k, ex.count, W)
            fe, i32 = ex.ffn_width, torch.int32
            self.cap = cap
            for i, L in enumerate(self.layers):
                p = f"{stage.prefix}.{i}"
                L.update(logits=e(n, router_pad(ex.count), dt=f32), ids=e(n, ex.top_k, dt=i32),
                         gates=e(n, ex.top_k, dt=f32), group_rows=e(2 * local + 1, dt=i32), pos=e(n * ex.top_k, dt=i32),
                         gu=e(cap, 2 * fe), h=e(cap, fe))
                ep.reserve(f"{p}.counts", 4 * W * ex.count)
                ep.reserve(f"{p}.a", 2 * cap * d)
                ep.reserve(f"{p}.out", 2 * cap * d)
            ep.reserve(f"{stage.prefix}.d_out", 2 * cap * d)
            ep.reserve(f"{stage.prefix}.da", 4 * cap * d)
            self.d_gates = e(n * ex.top_k, dt=f32)
            self.dh_packed, self.dgu_packed = e(cap, fe), e(cap, 2 * fe)
            self.dlogits = e(n, router_pad(ex.count))
        elif self.moe:
            # MoE FFN (architecture.rs:229-241): routing and the expert rows packed per expert, each
            # expert's segment padded to 128 rows (sj_route_pack); kept per layer for the backward
            ex = stage.experts
            cap = _lib.load().sj_moe_capacity(n, ex.top_k, ex.count)
            fe, i32 = ex.ffn_width, torch.int32
            self.cap = cap
            for i, L in enumerate(self.layers):
                if self.checkpoint and i > 0:
                    continue  # the shared set of the first block
                L.update(logits=e(n, router_pad(ex.count), dt=f32), ids=e(n, ex.top_k, dt=i32), gates=e(n, ex.top_k, dt=f32),
                         group_rows=e(ex.count + 1, dt=i32), pos=e(n * ex.top_k, dt=i32), row_slot=e(cap, dt=i32),
                         a=e(cap, d), gu=e(cap, 2 * fe), h=e(cap, fe), out=e(cap, d))
            self.d_out, self.d_gates = e(cap, d), e(n * ex.top_k, dt=f32)
            self.dh_packed, self.dgu_packed = e(cap, fe), e(cap, 2 * fe)
            self.da = e(cap, d, dt=f32)
            self.dlogits = e(n, router_pad(ex.count))


class ByteTrainer:
    """One data-parallel replica of the byte-model training step on the current CUDA device."""

    def __init__(self, config, train, device=None, params=None, process_group=None, expert_parallel=False,
                 ep_timeout_ms=10000):
        self.c, self.tc = config, train
        self.launches = 0
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        torch.cuda.set_device(self.dev)
        self.lib = _lib.load()
        call("sj_device_init", self.dev.index)
        self.pg = process_group
        self.world = torch.distributed.get_world_size(process_group) if process_group is not None else 1
        rank = torch.distributed.get_rank(process_group) if process_group is not None else 0
        self.ep = None
        if expert_parallel:
            if config.experts is None or config.experts.count % self.world:
                raise ValueError("expert parallelism needs an MoE model whose expert count the world size divides")
            if train.parameter_vjp is not None:
                raise ValueError("expert parallelism with the parameter VJP is not supported")
            self.ep = EpContext(rank, self.world, self.dev, process_group, ep_timeout_ms)
        self.values = int(train.values)
        self.layout = FlatLayout(config, expert_shard=(rank, self.world) if self.ep else None, values=self.values)
        if params is None:
            params = initialize(config, self.lib)
            if self.values:
                from .value import initialize_value
                params.update(initialize_value(config, self.values, self.lib))
        total = self.layout.total
        f32 = torch.float32
        self.w = torch.from_numpy(self.layout.pack(params)).to(self.dev)
        self.wb = torch.empty(total, dtype=torch.bfloat16, device=self.dev)
        self.g = torch.zeros(total, dtype=f32, device=self.dev)
        self.m = torch.zeros(total, dtype=f32, device=self.dev)
        self.v = torch.zeros(total, dtype=f32, device=self.dev)
        # gradient-norm partials: [replicated range | rank-local expert range (all-reduced)]
        sb = self.layout.shared_begin
        self.n_shared_partials = self.lib.sj_sumsq_partials(total - sb)
        self.n_partials = self.n_shared_partials + (self.lib.sj_sumsq_partials(sb) if sb else 0)
        self.partials = torch.zeros(self.n_partials, dtype=torch.float64, device=self.dev)
        self.opt_state = torch.zeros(2, dtype=torch.float64, device=self.dev)
        self.hyper = torch.zeros(8, dtype=f32, device=self.dev)
        self.loss_sum = torch.zeros(1, dtype=torch.float64, device=self.dev)
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        call("sj_cast", _ptr(self.w), SJ_F32, _ptr(self.wb), SJ_BF16, total, self.stream)

        b, t = train.batch, train.sequence
        self.rows = b * t
        h = config.hierarchy
        bf = torch.bfloat16
        e = lambda *s, dt=bf: torch.empty(*s, dtype=dt, device=self.dev)  # noqa: E731
        self.ids = torch.zeros(self.rows, dtype=torch.int32, device=self.dev)
        self.targets = torch.zeros(self.rows, dtype=torch.int32, device=self.dev)
        ckpt = bool(train.activation_checkpointing)
        if ckpt and self.ep is not None:
            raise ValueError("activation checkpointing with expert parallelism is not supported")
        if h is None:
            self.runs = {"global": _StageRun(global_stage(config), b, t, self.dev, self.ep, checkpoint=ckpt)}
            top_width = config.width
        else:
            assert t % h.patch_size == 0, "sequence must be a multiple of the patch size"
            self.patches = t // h.patch_size
            self.runs = {"encoder": _StageRun(local_stage(config, True), b, t, self.dev),
                         "global": _StageRun(global_stage(config), b, self.patches, self.dev, self.ep, checkpoint=ckpt),
                         "decoder": _StageRun(local_stage(config, False), b, t, self.dev)}
            de, dg, dd = h.encoder_width, config.width, h.decoder_width
            np_ = b * self.patches
            self.zE, self.invE = e(self.rows, de), e(self.rows, dt=torch.float32)
            self.pooled = e(np_, de)
            self.zG, self.invG = e(np_, dg), e(np_, dt=torch.float32)
            self.zd = e(np_, dd)
            self.bos = e(8, dd)
            self.zD, self.invD = e(self.rows, dd), e(self.rows, dt=torch.float32)
            self.y = e(self.rows, dg, dt=torch.float32)
            # backward
            self.dE = e(self.rows, de, dt=torch.float32)
            self.dzd, self.dbos = e(np_, dd), e(8, dd)
            self.dpool = e(np_, de, dt=torch.float32)
            self.dy32 = e(self.rows, dg, dt=torch.float32)
            self.dyb = e(self.rows, dg)
            self.top_partials = e(self.lib.sj_rmsnorm_workspace(self.rows, max(dg, de, dd)), dt=torch.float32)
            top_width = dg
        self.hf, self.invF = e(self.rows, top_width), e(self.rows, dt=torch.float32)
        if self.values:  # NativeValue head: SEP row and label per request, f32 value logits
            self.sel = torch.zeros(b, dtype=torch.int32, device=self.dev)
            self.labels = torch.zeros(b, dtype=torch.int32, device=self.dev)
            self.vlogits = e(b, self.values, dt=torch.float32)
            self.vdlogits = e(b, self.values, dt=torch.float32)
            if h is not None:
                self.xin = e(self.rows, config.width)  # native embedding output, input_projection operand
        else:
            self.logits = e(self.rows, VOCAB_PAD, dt=torch.float32)
            self.dlogits = e(self.rows, VOCAB_PAD)
        self.dhead = e(self.rows, top_width, dt=torch.float32)
        self.dheadb = e(self.rows, top_width)
        if h is None:
            self.top_partials = e(self.lib.sj_rmsnorm_workspace(self.rows, top_width), dt=torch.float32)
        # RoPE (cos, sin) tables, one per distinct stage sequence length, built once
        self.rope_tables = {}
        for run in self.runs.values():
            if run.seq not in self.rope_tables:
                tab = torch.empty(run.seq * HEAD_DIM, dtype=torch.float32, device=self.dev)
                call("sj_rope_table", _ptr(tab), run.seq, HEAD_DIM, 0, float(config.rope_theta), self.stream)
                self.rope_tables[run.seq] = tab
        if self.ep is not None:
            self.ep.finalize()
        self.graph = None
        self.vjp = None
        # weight of the staged observation's loss and gradient; None = 1 / accumulation (the control-
        # variate trainer sets each control's own weight)
        self.obs_weight = None
        if train.parameter_vjp is not None:
            self._init_vjp(train.parameter_vjp)

    # kernels each entry point launches (zero fills are kernels too)
    KERNELS = {"sj_moe_aux": 2, "sj_gemm": 1, "sj_rmsnorm_fwd": 1, "sj_rmsnorm_bwd": 2, "sj_rmsnorm_bwd_ex": 2, "sj_attn_gqa_fwd": 1,
               "sj_attn_gqa_bwd": 3,
               "sj_zero": 1, "sj_param_basis": 5, "sj_param_prepare": 3}

    @classmethod
    def kernels_of(cls, name, args):
        """Kernel launches one C-ABI call makes."""
        if name == "sj_attn_gqa_bwd":
            # the banded kernel (window <= 128, one query head per kv head, a RoPE table or no
            # rotation) needs no dQ finish pass
            hq, hk, window, theta, table = args[20], args[21], args[23], args[24], args[25]
            return 2 if 0 < window <= 128 and hq == hk and (table or theta <= 0) else 3
        return cls.KERNELS.get(name, 1)

    def _call(self, name, *args):
        call(name, *args)
        self.launches += self.kernels_of(name, args)

    # ------------------------------------------------------------------ parameter pointers
    def wb_ptr(self, name):
        return _ptr(self.wb, self.layout[name].offset)

    def w_ptr(self, name):
        return _ptr(self.w, self.layout[name].offset)

    def g_ptr(self, name):
        return _ptr(self.g, self.layout[name].offset)

    # ------------------------------------------------------------------ primitives
    def _gemm(self, a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epi=EPI_STORE, aux=0, ld_aux=0,
              rope_cols=0, rope_t=0, split_k=0):
        self._call("sj_gemm", a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epi, 1.0, aux, ld_aux, rope_cols,
             rope_t, float(self.c.rope_theta) if epi == EPI_ROPE else 0.0, split_k, self.stream)

    @staticmethod
    def _dt(t):
        return SJ_F32 if t.dtype == torch.float32 else SJ_BF16

    def _norm(self, x, wname, y, inv, rows, d):
        self._call("sj_rmsnorm_fwd", _ptr(x), self._dt(x), self.w_ptr(wname), _ptr(y), _ptr(inv), rows, d,
             float(self.c.norm_epsilon), self.stream)

    def _norm_bwd(self, x, wname, inv, dz, dres, dres_b, partials, rows, d, accumulate=True):
        """dres (+)= the norm's input gradient; accumulate=False writes it (the first gradient of a
        residual stream, which then needs no zero fill)."""
        self._call("sj_rmsnorm_bwd_ex", _ptr(x), self._dt(x), self.w_ptr(wname), _ptr(inv), _ptr(dz), _ptr(dres),
             _ptr(dres_b) if dres_b is not None else 0, self.g_ptr(wname), _ptr(partials), rows, d, int(accumulate),
             self.stream)

    def _zero(self, t):
        self._call("sj_zero", _ptr(t), t.numel() * t.element_size(), self.stream)

    # ------------------------------------------------------------------ parameter VJP
    def _init_vjp(self, cfg):
        """Plan and buffers of the parameter VJP (crates/sejong-gpu/src/parameter_vjp.rs:133-321).

        The generator state lives on the device and advances there, so the step stays free of
        host round trips; bases are kept per (rows, rank) and selections per width, as the
        reference shares them within one backward pass."""
        self.vjp = param_vjp.plan(self.c, self.tc.batch, self.tc.sequence, cfg)
        dev, i32, f32 = self.dev, torch.int32, torch.float32
        # with data parallelism every rank draws its own basis and selection from its own X; the
        # sum of the ranks' factored gradients (the all-reduce) applies every rank's terms
        rank = torch.distributed.get_rank(self.pg) if self.pg is not None else 0
        seed = distributed.rank_seed(cfg.seed, rank)
        self.vjp_rng = torch.from_numpy(np.array([seed], dtype=np.uint64).view(np.int64)).to(dev)
        self.vjp_q, self.vjp_columns, self.vjp_rows, self.vjp_map = {}, {}, {}, {}
        basis_ws = left = e = coeff = 1
        for g in self.vjp.groups.values():
            donor = g.members[g.donor].width
            self.vjp_q.setdefault(g.basis_key, torch.empty(g.rows, g.rank, dtype=f32, device=dev))
            self.vjp_columns.setdefault(g.basis_key, torch.zeros(g.rank, dtype=i32, device=dev))
            self.vjp_rows.setdefault(g.features, torch.zeros(g.k, dtype=i32, device=dev))
            self.vjp_map.setdefault(g.features, torch.zeros(g.features, dtype=i32, device=dev))
            basis_ws = max(basis_ws, self.lib.sj_param_basis_workspace(g.rows, g.features, g.rank))
            left = max(left, g.features * g.rank)
            e = max(e, (g.rank + g.k) * g.rows)
            coeff = max(coeff, (g.rank + g.k) * sum(m.width for m in g.members))
        self.vjp_ws = torch.empty((basis_ws + 7) // 8, dtype=torch.float64, device=dev)
        self.vjp_left = torch.empty(left, dtype=f32, device=dev)
        self.vjp_e = torch.empty(e, dtype=torch.bfloat16, device=dev)
        self.vjp_coeff = torch.empty(coeff, dtype=f32, device=dev)

    def vjp_statistics(self):
        """The counts of the reference's VjpStatistics for one backward pass (graph.rs:915-1005):
        matrices whose gradient is factored, matrices with an exact gradient, bases computed and
        groups prepared."""
        nodes = param_vjp.matmul_nodes(self.c, self.tc.batch, self.tc.sequence)
        compressed = len(self.vjp.compressed)
        return {"compressed_matrices": compressed, "dense_matrices": len(nodes) - compressed,
                "basis_groups": sum(1 for g in self.vjp.groups.values() if g.new_basis),
                "projection_groups": len(self.vjp.groups)}

    def evaluate(self):
        """Mean cross entropy of the staged batch, forward only (benchmark.rs:71-97 `evaluate`)."""
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        self._zero(self.loss_sum)
        self._forward()
        return float(self.loss_sum.item()) * max(1, self.tc.accumulation) * self.world

    def vjp_rng_state(self):
        """The device generator state as the reference Rng's u64."""
        return int(self.vjp_rng.cpu().numpy().view(np.uint64)[0])

    def _member_layout(self, g, fused):
        """(column offset, width, interleave) of each member inside the fused weight `fused`:
        `*.qkv` holds query | key | value; `*.gate_up` interleaves gate and up in 16-column blocks."""
        if fused.endswith(".gate_up"):
            return [(0, m.width, 16) for m in g.members]
        out, col = [], 0
        for m in g.members:
            out.append((col, m.width, 0))
            col += m.width
        return out

    def _weight_grad(self, key, x, dy, gname):
        """dW += X^T dY for the fused weight `gname` (X [n, a] bf16, dY [n, width] bf16): a dense
        TN GEMM, or, for a group the plan compresses, the parameter VJP of its active members."""
        n, a = x.shape
        width = dy.shape[1]
        g = self.vjp.groups.get(key) if self.vjp is not None else None
        if g is None:
            self._gemm(_ptr(x), a, 1, _ptr(dy), width, 0, self.g_ptr(gname), width, SJ_F32, a, width, n, EPI_ACCUM)
            return
        layout = self._member_layout(g, gname)
        wname = gname
        r, k = g.rank, g.k
        cols, q = self.vjp_columns[g.basis_key], self.vjp_q[g.basis_key]
        rows, row_map = self.vjp_rows[a], self.vjp_map[a]
        if g.draw:
            donor_width = g.members[g.donor].width
            self._call("sj_param_indices", _ptr(self.vjp_rng), a if g.new_selection else 0,
                       donor_width if g.new_basis else 0, g.blocks if g.new_selection else 0,
                       g.selected if g.new_selection else 0, r if g.new_basis else 0, g.block_rows,
                       _ptr(cols), _ptr(rows), _ptr(row_map), self.stream)
        if g.new_basis:
            off, _, interleave = layout[g.donor]
            if interleave:
                assert g.donor == len(g.members) - 1, "an interleaved donor must be the second half"
            self._call("sj_param_basis", _ptr(x), a, n, a, _ptr(self.wb, self.layout[wname].offset + off), width,
                       interleave, _ptr(cols), r, param_vjp.basis_eps(n, r), _ptr(q), _ptr(self.vjp_ws), self.stream)
        self._call("sj_param_prepare", _ptr(x), a, n, a, _ptr(q), r, _ptr(rows), k, g.inverse, _ptr(self.vjp_left),
                   _ptr(self.vjp_e), self.stream)
        # (right ; tail) = E dY over all columns of the fused weight
        coeff = self.vjp_coeff[:(r + k) * width]
        self._zero(coeff)
        self._gemm(_ptr(self.vjp_e), n, 0, _ptr(dy), width, 0, _ptr(coeff), width, SJ_F32, r + k, width, n, EPI_ACCUM)
        interleaved = layout[0][2] > 0
        if interleaved:
            assert len(g.active) in (0, len(g.members)), "gate and up share one decision (equal widths)"
            spans = [(0, width, True)]
        else:
            spans = []
            for i, (off, w, _) in enumerate(layout):
                compressed = i in g.active
                if spans and spans[-1][2] == compressed and spans[-1][0] + spans[-1][1] == off:
                    spans[-1] = (spans[-1][0], spans[-1][1] + w, compressed)   # one launch per contiguous run
                else:
                    spans.append((off, w, compressed))
        for off, w, compressed in spans:
            if compressed:
                self._call("sj_param_materialize", _ptr(self.vjp_left), _ptr(coeff, off), width, _ptr(row_map), a, w,
                           r, self.g_ptr(gname) + off * 4, width, 1, self.stream)
            else:
                self._gemm(_ptr(x), a, 1, _ptr(dy, off), width, 0, self.g_ptr(gname) + off * 4, width, SJ_F32, a, w,
                           n, EPI_ACCUM)

    # ------------------------------------------------------------------ blocks
    def _block_fwd(self, run, i):
        s, a = run.stage, run.layers[i]
        n, d, f, cq, seq = run.rows, s.width, s.ffn, s.qkv_width, run.seq
        p = f"{s.prefix}.{i}"
        x, xn = run.x[i], run.x[i + 1]
        self._norm(x, f"{p}.attention_norm", a["z1"], a["inv1"], n, d)
        self._gemm(_ptr(a["z1"]), d, 0, self.wb_ptr(f"{p}.qkv"), cq, 0, _ptr(a["qkv"]), cq, SJ_BF16, n, cq, d,
                   EPI_ROPE, aux=_ptr(self.rope_tables[seq]), rope_cols=(s.heads + s.kv_heads) * HEAD_DIM,
                   rope_t=seq)
        qkv = a["qkv"]
        self._call("sj_attn_gqa_fwd", _ptr(qkv), cq, _ptr(qkv, s.heads * HEAD_DIM), cq,
             _ptr(qkv, (s.heads + s.kv_heads) * HEAD_DIM), cq, _ptr(a["o"]), d, _ptr(a["lse"]), run.batch, seq,
             s.heads, s.kv_heads, HEAD_DIM, s.window, self.stream)
        self._gemm(_ptr(a["o"]), d, 0, self.wb_ptr(f"{p}.attention_output"), d, 0, _ptr(a["x1"]), d, SJ_F32, n, d, d,
                   EPI_RESIDUAL, aux=_ptr(x), ld_aux=d)
        self._norm(a["x1"], f"{p}.ffn_norm", a["z2"], a["inv2"], n, d)
        if run.moe:
            self._moe_fwd(run, a, p, xn)
            return
        self._gemm(_ptr(a["z2"]), d, 0, self.wb_ptr(f"{p}.gate_up"), 2 * f, 0, _ptr(a["gu"]), 2 * f, SJ_BF16, n,
                   2 * f, d, EPI_SWIGLU, aux=_ptr(a["h"]), ld_aux=f)
        self._gemm(_ptr(a["h"]), f, 0, self.wb_ptr(f"{p}.down"), d, 0, _ptr(xn), d, SJ_F32, n, d, f, EPI_RESIDUAL,
                   aux=_ptr(a["x1"]), ld_aux=d)

    def _block_bwd(self, run, i):
        """run.dx / run.dxb hold dL/d(block output); on return dL/d(block input)."""
        s, a = run.stage, run.layers[i]
        n, d, f, cq, seq = run.rows, s.width, s.ffn, s.qkv_width, run.seq
        p = f"{s.prefix}.{i}"
        dx, dxb = run.dx, run.dxb
        # FFN: down, SwiGLU, gate/up
        if run.moe:
            self._moe_bwd(run, a, p)
        else:
            self._gemm(_ptr(a["h"]), f, 1, _ptr(dxb), d, 0, self.g_ptr(f"{p}.down"), d, SJ_F32, f, d, n, EPI_ACCUM)
            self._gemm(_ptr(dxb), d, 0, self.wb_ptr(f"{p}.down"), d, 1, _ptr(run.dh), f, SJ_BF16, n, f, d)
            self._call("sj_swiglu_bwd", _ptr(a["gu"]), _ptr(run.dh), _ptr(run.dgu), n, f, self.stream)
            self._weight_grad(f"{p}.z2", a["z2"], run.dgu, f"{p}.gate_up")
            self._gemm(_ptr(run.dgu), 2 * f, 0, self.wb_ptr(f"{p}.gate_up"), 2 * f, 1, _ptr(run.dz), d, SJ_F32, n, d,
                       2 * f)
        self._norm_bwd(a["x1"], f"{p}.ffn_norm", a["inv2"], run.dz, dx, dxb, run.partials, n, d)
        # attention: output projection, attention, QKV
        self._gemm(_ptr(a["o"]), d, 1, _ptr(dxb), d, 0, self.g_ptr(f"{p}.attention_output"), d, SJ_F32, d, d, n,
                   EPI_ACCUM)
        self._gemm(_ptr(dxb), d, 0, self.wb_ptr(f"{p}.attention_output"), d, 1, _ptr(run.do), d, SJ_BF16, n, d, d)
        qkv, dqkv = a["qkv"], run.dqkv
        kq, vq = s.heads * HEAD_DIM, (s.heads + s.kv_heads) * HEAD_DIM
        self._call("sj_attn_gqa_bwd", _ptr(qkv), cq, _ptr(qkv, kq), cq, _ptr(qkv, vq), cq, _ptr(a["o"]), d, _ptr(a["lse"]),
             _ptr(run.do), d, _ptr(dqkv), cq, _ptr(dqkv, kq), cq, _ptr(dqkv, vq), cq, _ptr(run.delta), run.batch,
             seq, s.heads, s.kv_heads, HEAD_DIM, s.window, float(self.c.rope_theta), _ptr(self.rope_tables[seq]),
             self.stream)
        self._weight_grad(f"{p}.z1", a["z1"], dqkv, f"{p}.qkv")
        self._gemm(_ptr(dqkv), cq, 0, self.wb_ptr(f"{p}.qkv"), cq, 1, _ptr(run.dz), d, SJ_F32, n, d, cq)
        self._norm_bwd(run.x[i], f"{p}.attention_norm", a["inv1"], run.dz, dx, dxb, run.partials, n, d)

    # ------------------------------------------------------------------ mixture of experts
    def _gemm_grouped(self, a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epi, groups, group_rows,
                      mode, b_rows=0, c_rows=0, aux=0, ld_aux=0):
        self._call("sj_gemm_grouped", a, lda, a_trans, b, ldb, b_trans, c, ldc, c_dtype, m, n, k, epi, aux, ld_aux,
                   groups, group_rows, mode, b_rows, c_rows, self.stream)

    def _moe_fwd(self, run, a, p, xn):
        """The MoE FFN of a block (architecture.rs:229-241): router logits, top-k routing, the routed
        rows packed per expert, one grouped GEMM per projection over all experts, and the gated
        combine with the residual add into the block output `xn`."""
        if run.ep is not None:
            return self._moe_fwd_ep(run, a, p, xn)
        ex = run.stage.experts
        n, d, fe, E, k, cap = run.rows, run.stage.width, ex.ffn_width, ex.count, ex.top_k, run.cap
        gp = _ptr(a["group_rows"])
        ep = router_pad(E)  # router columns (and logits) padded to 8; the padding is zero and ignored
        self._gemm(_ptr(a["z2"]), d, 0, self.wb_ptr(f"{p}.router"), ep, 0, _ptr(a["logits"]), ep, SJ_F32, n, ep, d)
        self._call("sj_route_topk", _ptr(a["logits"]), ep, n, E, k, _ptr(a["ids"]), _ptr(a["gates"]), self.stream)
        self._route_capacity(a, n, k, E)
        self._call("sj_route_pack", _ptr(a["ids"]), n, E, k, gp, _ptr(a["pos"]), _ptr(a["row_slot"]), cap, self.stream)
        self._call("sj_moe_dispatch", _ptr(a["z2"]), d, _ptr(a["row_slot"]), cap, k, d, _ptr(a["a"]), self.stream)
        self._gemm_grouped(_ptr(a["a"]), d, 0, self.wb_ptr(f"{p}.experts.0.gate_up"), 2 * fe, 0, _ptr(a["gu"]), 2 * fe,
                           SJ_BF16, cap, 2 * fe, d, EPI_SWIGLU, E, gp, 1, b_rows=d, aux=_ptr(a["h"]), ld_aux=fe)
        self._gemm_grouped(_ptr(a["h"]), fe, 0, self.wb_ptr(f"{p}.experts.0.down"), d, 0, _ptr(a["out"]), d, SJ_BF16,
                           cap, d, fe, EPI_STORE, E, gp, 1, b_rows=fe)
        self._call("sj_moe_combine", _ptr(a["out"]), _ptr(a["pos"]), _ptr(a["gates"]), _ptr(a["x1"]), _ptr(xn), n, k,
                   d, self.stream)

    def _moe_bwd(self, run, a, p):
        """Backward of _moe_fwd into run.dz (the gradient at the FFN norm's output), accumulating the
        expert and router weight gradients (graph.rs:600-624 for the routing terms)."""
        if run.ep is not None:
            return self._moe_bwd_ep(run, a, p)
        ex = run.stage.experts
        n, d, fe, E, k, cap = run.rows, run.stage.width, ex.ffn_width, ex.count, ex.top_k, run.cap
        gp = _ptr(a["group_rows"])
        gate_up, down = f"{p}.experts.0.gate_up", f"{p}.experts.0.down"
        self._call("sj_moe_combine_bwd", _ptr(a["out"]), _ptr(a["row_slot"]), _ptr(a["gates"]), _ptr(run.dx),
                   _ptr(run.d_out), _ptr(run.d_gates), cap, k, d, self.stream)
        self._gemm_grouped(_ptr(a["h"]), fe, 1, _ptr(run.d_out), d, 0, self.g_ptr(down), d, SJ_F32, fe, d, cap,
                           EPI_ACCUM, E, gp, 2, c_rows=fe)
        self._gemm_grouped(_ptr(run.d_out), d, 0, self.wb_ptr(down), d, 1, _ptr(run.dh_packed), fe, SJ_BF16, cap, fe,
                           d, EPI_STORE, E, gp, 1, b_rows=fe)
        self._call("sj_swiglu_bwd", _ptr(a["gu"]), _ptr(run.dh_packed), _ptr(run.dgu_packed), cap, fe, self.stream)
        self._gemm_grouped(_ptr(a["a"]), d, 1, _ptr(run.dgu_packed), 2 * fe, 0, self.g_ptr(gate_up), 2 * fe, SJ_F32, d,
                           2 * fe, cap, EPI_ACCUM, E, gp, 2, c_rows=d)
        self._gemm_grouped(_ptr(run.dgu_packed), 2 * fe, 0, self.wb_ptr(gate_up), 2 * fe, 1, _ptr(run.da), d, SJ_F32,
                           cap, d, 2 * fe, EPI_STORE, E, gp, 1, b_rows=d)
        self._call("sj_moe_dispatch_bwd", _ptr(run.da), _ptr(a["pos"]), _ptr(run.dz), d, n, k, d, self.stream)
        ep = router_pad(E)
        self._call("sj_route_topk_bwd", _ptr(a["logits"]), ep, _ptr(a["ids"]), _ptr(a["gates"]), _ptr(run.d_gates),
                   _ptr(run.dlogits), ep, n, E, k, self.stream)
        self._moe_aux(a, run, n, k, E)
        self._gemm(_ptr(run.dlogits), ep, 0, self.wb_ptr(f"{p}.router"), ep, 1, _ptr(run.dz), d, SJ_F32, n, d, ep,
                   EPI_ACCUM)
        self._gemm(_ptr(a["z2"]), d, 1, _ptr(run.dlogits), ep, 0, self.g_ptr(f"{p}.router"), ep, SJ_F32, d, ep, n,
                   EPI_ACCUM)

    def _route_capacity(self, a, n, k, E):
        """The expert capacity (an addition to the reference): slots beyond it leave their expert."""
        cf = float(self.tc.moe_capacity_factor)
        if cf > 0:
            self._call("sj_route_capacity", _ptr(a["ids"]), n, k, E, max(1, math.ceil(cf * n * k / E)), self.stream)

    def _moe_aux(self, a, run, n, k, E):
        """The load-balancing loss (an addition to the reference) of this rank's rows: its value joins
        the loss sum (as the mean over the ranks and observations), its gradient the router's."""
        w = float(self.tc.moe_aux_loss_weight)
        if w > 0:
            obs = self.obs_weight if self.obs_weight is not None else 1.0 / float(max(1, self.tc.accumulation))
            erp = router_pad(E)
            self._call("sj_moe_aux", _ptr(a["logits"]), erp, n, E, k, w, obs / self.world,
                       _ptr(self.loss_sum), _ptr(run.dlogits), erp, float(self.tc.loss_scale) * obs / self.world,
                       _ptr(run.aux_ws), self.stream)

    def _ep_barrier(self, ep):
        self._call("sj_ep_barrier", ep.rank, ep.world, ep.peers, ep.offset("flags"), _ptr(ep.epoch), ep.timeout_ms,
                   self.stream)

    def _moe_fwd_ep(self, run, a, p, xn):
        """_moe_fwd with the experts sharded over the ranks: the routing is local; the counts go to
        every rank, which lays out its experts' rows (sj_ep_route_pack); the rows are pushed to their
        owners, which run their experts on them; the outputs are pulled back by the combine."""
        ep, ex = run.ep, run.stage.experts
        n, d, fe, E, k, cap = run.rows, run.stage.width, ex.ffn_width, ex.count, ex.top_k, run.cap
        local = E // ep.world
        first = local * ep.rank
        gp = _ptr(a["group_rows"])
        ids, pos = _ptr(a["ids"]), _ptr(a["pos"])
        erp = router_pad(E)
        self._gemm(_ptr(a["z2"]), d, 0, self.wb_ptr(f"{p}.router"), erp, 0, _ptr(a["logits"]), erp, SJ_F32, n, erp, d)
        self._call("sj_route_topk", _ptr(a["logits"]), erp, n, E, k, ids, _ptr(a["gates"]), self.stream)
        self._route_capacity(a, n, k, E)
        self._call("sj_ep_route_pack", ids, n, E, k, ep.rank, ep.world, ep.peers, ep.offset(f"{p}.counts"),
                   ep.offset("flags"), _ptr(ep.epoch), gp, pos, cap, ep.timeout_ms, self.stream)
        self._call("sj_ep_dispatch", _ptr(a["z2"]), d, ids, pos, n, k, d, E, ep.rank, ep.world, ep.peers,
                   ep.offset(f"{p}.a"), gp, self.stream)
        self._ep_barrier(ep)
        self._gemm_grouped(ep.ptr(f"{p}.a"), d, 0, self.wb_ptr(f"{p}.experts.{first}.gate_up"), 2 * fe, 0, _ptr(a["gu"]),
                           2 * fe, SJ_BF16, cap, 2 * fe, d, EPI_SWIGLU, local, gp, 1, b_rows=d, aux=_ptr(a["h"]),
                           ld_aux=fe)
        self._gemm_grouped(_ptr(a["h"]), fe, 0, self.wb_ptr(f"{p}.experts.{first}.down"), d, 0, ep.ptr(f"{p}.out"), d,
                           SJ_BF16, cap, d, fe, EPI_STORE, local, gp, 1, b_rows=fe)
        self._ep_barrier(ep)
        self._call("sj_ep_combine", ep.peers, ep.world, ep.offset(f"{p}.out"), ids, pos, _ptr(a["gates"]),
                   _ptr(a["x1"]), _ptr(xn), n, k, d, E, self.stream)

    def _moe_bwd_ep(self, run, a, p):
        """Backward of _moe_fwd_ep: gate * dy pushed to the owners, which run the expert backward
        GEMMs on their rows; dA pulled back and summed per row; the router backward is local."""
        ep, ex = run.ep, run.stage.experts
        n, d, fe, E, k, cap = run.rows, run.stage.width, ex.ffn_width, ex.count, ex.top_k, run.cap
        local = E // ep.world
        first = local * ep.rank
        gp = _ptr(a["group_rows"])
        ids, pos = _ptr(a["ids"]), _ptr(a["pos"])
        gate_up, down = f"{p}.experts.{first}.gate_up", f"{p}.experts.{first}.down"
        d_out, da = f"{run.stage.prefix}.d_out", f"{run.stage.prefix}.da"
        self._call("sj_ep_combine_bwd", ep.peers, ep.rank, ep.world, ep.offset(f"{p}.out"), ep.offset(d_out), ids, pos,
                   _ptr(a["gates"]), _ptr(run.dx), _ptr(run.d_gates), gp, n, k, d, E, self.stream)
        self._ep_barrier(ep)
        self._gemm_grouped(_ptr(a["h"]), fe, 1, ep.ptr(d_out), d, 0, self.g_ptr(down), d, SJ_F32, fe, d, cap,
                           EPI_ACCUM, local, gp, 2, c_rows=fe)
        self._gemm_grouped(ep.ptr(d_out), d, 0, self.wb_ptr(down), d, 1, _ptr(run.dh_packed), fe, SJ_BF16, cap, fe,
                           d, EPI_STORE, local, gp, 1, b_rows=fe)
        self._call("sj_swiglu_bwd_live", _ptr(a["gu"]), _ptr(run.dh_packed), _ptr(run.dgu_packed), cap, fe,
                   gp + 4 * local, self.stream)
        self._gemm_grouped(ep.ptr(f"{p}.a"), d, 1, _ptr(run.dgu_packed), 2 * fe, 0, self.g_ptr(gate_up), 2 * fe,
                           SJ_F32, d, 2 * fe, cap, EPI_ACCUM, local, gp, 2, c_rows=d)
        self._gemm_grouped(_ptr(run.dgu_packed), 2 * fe, 0, self.wb_ptr(gate_up), 2 * fe, 1, ep.ptr(da), d, SJ_F32,
                           cap, d, 2 * fe, EPI_STORE, local, gp, 1, b_rows=d)
        self._ep_barrier(ep)
        self._call("sj_ep_dispatch_bwd", ep.peers, ep.world, ep.offset(da), ids, pos, _ptr(run.dz), d, n, k, d, E,
                   self.stream)
        erp = router_pad(E)
        self._call("sj_route_topk_bwd", _ptr(a["logits"]), erp, ids, _ptr(a["gates"]), _ptr(run.d_gates),
                   _ptr(run.dlogits), erp, n, E, k, self.stream)
        self._moe_aux(a, run, n, k, E)
        self._gemm(_ptr(run.dlogits), erp, 0, self.wb_ptr(f"{p}.router"), erp, 1, _ptr(run.dz), d, SJ_F32, n, d, erp,
                   EPI_ACCUM)
        self._gemm(_ptr(a["z2"]), d, 1, _ptr(run.dlogits), erp, 0, self.g_ptr(f"{p}.router"), erp, SJ_F32, d, erp, n,
                   EPI_ACCUM)

    def _stage_fwd(self, run):
        for i in range(run.stage.layers):
            self._block_fwd(run, i)

    def _stage_bwd(self, run):
        for _ in self._stage_bwd_gen(run):
            pass

    def _stage_bwd_gen(self, run):
        """The stage's blocks backward; yields "half" once the upper half of the blocks is done (their
        weight gradients are final: a gradient bucket of the overlapped exchange)."""
        half = run.stage.layers // 2
        for i in reversed(range(run.stage.layers)):
            if i == half - 1 and half > 0:
                yield "half"
            if run.checkpoint and i < run.stage.layers - 1:
                # Op::Checkpoint's backward (graph.rs:756-799): the block's forward again, from its saved
                # input x[i], into the shared activation buffers (it rewrites x[i+1] with the values it
                # already holds: the forward kernels are deterministic).  The last block's activations
                # are still in the buffers from the forward pass, so it is not run again.
                self._block_fwd(run, i)
            self._block_bwd(run, i)

    # ------------------------------------------------------------------ model
    def encode(self):
        """Model::encode (architecture.rs:330-351) of the staged batch: the embedding and, for the
        hierarchical model, the encoder stage and its norm.  Returns (rows buffer, dtype code, width):
        the f32 embedding rows of the dense model, the bf16 encoder output zE of the hierarchical one."""
        c, h = self.c, self.c.hierarchy
        n = self.rows
        emb, vocab = ("native_embedding", NATIVE_VOCAB) if self.values else ("embedding", VOCAB)
        if h is None:
            run = self.runs["global"]
            self._call("sj_embedding_fwd", self.wb_ptr(emb), _ptr(self.ids), _ptr(run.x[0]), SJ_F32, n,
                       c.width, vocab, self.stream)
            return run.x[0], SJ_F32, c.width
        enc = self.runs["encoder"]
        de, dg = h.encoder_width, c.width
        if self.values:  # hidden_from (architecture.rs:353-367): native embedding -> input_projection
            self._call("sj_embedding_fwd", self.wb_ptr(emb), _ptr(self.ids), _ptr(self.xin), SJ_BF16, n, dg,
                       vocab, self.stream)
            self._gemm(_ptr(self.xin), dg, 0, self.wb_ptr("input_projection"), de, 0, _ptr(enc.x[0]), de, SJ_F32,
                       n, de, dg)
        else:
            self._call("sj_embedding_fwd", self.wb_ptr(emb), _ptr(self.ids), _ptr(enc.x[0]), SJ_F32, n, de,
                       VOCAB, self.stream)
        self._stage_fwd(enc)
        self._norm(enc.x[-1], "encoder_norm", self.zE, self.invE, n, de)
        return self.zE, SJ_BF16, de

    def _forward(self):
        c, h = self.c, self.c.hierarchy
        n = self.rows
        b = self.tc.batch
        weight = self.obs_weight if self.obs_weight is not None else 1.0 / float(max(1, self.tc.accumulation))
        if h is None:
            run = self.runs["global"]
            self.encode()
            self._stage_fwd(run)
            top = run.x[-1]
            top_width = c.width
        else:
            enc, glob, dec = self.runs["encoder"], self.runs["global"], self.runs["decoder"]
            de, dg, dd, pt = h.encoder_width, c.width, h.decoder_width, h.patch_size
            np_ = b * self.patches
            self.encode()
            self._call("sj_patch_pool_fwd", _ptr(self.zE), _ptr(self.pooled), b, self.tc.sequence, de, pt, self.stream)
            self._gemm(_ptr(self.pooled), de, 0, self.wb_ptr("encoder_to_global"), dg, 0, _ptr(glob.x[0]), dg,
                       SJ_F32, np_, dg, de)
            self._stage_fwd(glob)
            self._norm(glob.x[-1], "global_norm", self.zG, self.invG, np_, dg)
            self._gemm(_ptr(self.zG), dg, 0, self.wb_ptr("global_to_decoder"), dd, 0, _ptr(self.zd), dd, SJ_BF16,
                       np_, dd, dg)
            self._gemm(self.wb_ptr("global_bos"), dg, 0, self.wb_ptr("global_to_decoder"), dd, 0, _ptr(self.bos), dd,
                       SJ_BF16, 1, dd, dg)
            self._gemm(_ptr(self.zE), de, 0, self.wb_ptr("encoder_to_decoder"), dd, 0, _ptr(dec.x[0]), dd, SJ_F32,
                       n, dd, de)
            self._call("sj_patch_broadcast_fwd", _ptr(self.zd), _ptr(self.bos), _ptr(dec.x[0]), SJ_F32, 1, b,
                       self.tc.sequence, dd, pt, self.stream)
            self._stage_fwd(dec)
            self._norm(dec.x[-1], "decoder_norm", self.zD, self.invD, n, dd)
            self._gemm(_ptr(self.zD), dd, 0, self.wb_ptr("output_projection"), dg, 0, _ptr(self.y), dg, SJ_F32, n,
                       dg, dd)
            top = self.y
            top_width = dg
        self._norm(top, "final_norm", self.hf, self.invF, n, top_width)
        if self.values:
            # value.rs:147-152: the SEP rows, cast to f32, through the f32 affine head; the loss is the
            # mean cross entropy over the requests of the global batch (seed 1 / requests)
            bt = self.tc.batch
            self._call("sj_value_head_fwd", _ptr(self.hf), top_width, n, _ptr(self.sel), bt, top_width,
                       self.w_ptr("native_value"), self.w_ptr("native_bias"), self.values, _ptr(self.labels),
                       distributed.ce_seed(bt, self.world, self.tc.loss_scale) * weight, _ptr(self.vlogits),
                       _ptr(self.vdlogits), _ptr(self.loss_sum), distributed.ce_seed(bt, self.world) * weight,
                       self.stream)
            return top, top_width
        self._gemm(_ptr(self.hf), top_width, 0, self.wb_ptr("output"), VOCAB_PAD, 0, _ptr(self.logits), VOCAB_PAD,
                   SJ_F32, n, VOCAB, top_width)
        self._call("sj_cross_entropy", _ptr(self.logits), VOCAB_PAD, _ptr(self.targets), n, VOCAB,
                   distributed.ce_seed(n, self.world, self.tc.loss_scale) * weight, 0, _ptr(self.dlogits), VOCAB_PAD,
                   _ptr(self.loss_sum), distributed.ce_seed(n, self.world) * weight, self.stream)
        return top, top_width

    def _backward(self, top, top_width):
        for _ in self._backward_gen(top, top_width):
            pass

    def _backward_gen(self, top, top_width):
        """The backward pass; yields a tag where a range of the flat gradient has become final (the
        gradient buckets of the overlapped data-parallel exchange, `grad_buckets`)."""
        c, h = self.c, self.c.hierarchy
        n, b = self.rows, self.tc.batch
        if self.values:
            # value head: dW, dbias and the SEP rows of dh (every other row of dh is zero)
            self._zero(self.dhead)
            self._call("sj_value_head_bwd", _ptr(self.hf), top_width, n, _ptr(self.sel), b, top_width,
                       self.w_ptr("native_value"), _ptr(self.vdlogits), self.values, self.g_ptr("native_value"),
                       self.g_ptr("native_bias"), _ptr(self.dhead), top_width, self.stream)
        else:
            # head: dW_out += h^T dlogits ; dh = dlogits W_out^T
            self._gemm(_ptr(self.hf), top_width, 1, _ptr(self.dlogits), VOCAB_PAD, 0, self.g_ptr("output"), VOCAB_PAD,
                       SJ_F32, top_width, VOCAB, n, EPI_ACCUM)
            self._gemm(_ptr(self.dlogits), VOCAB_PAD, 0, self.wb_ptr("output"), VOCAB_PAD, 1, _ptr(self.dhead),
                       top_width, SJ_F32, n, top_width, VOCAB)
        emb, vocab = ("native_embedding", NATIVE_VOCAB) if self.values else ("embedding", VOCAB)
        if h is None:
            run = self.runs["global"]
            self._norm_bwd(top, "final_norm", self.invF, self.dhead, run.dx, run.dxb, self.top_partials, n, c.width,
                           accumulate=False)
            for tag in self._stage_bwd_gen(run):
                yield f"global_{tag}"
            self._call("sj_embedding_bwd", _ptr(run.dx), _ptr(self.ids), self.g_ptr(emb), n, c.width, vocab,
                 self.stream)
            return
        enc, glob, dec = self.runs["encoder"], self.runs["global"], self.runs["decoder"]
        de, dg, dd, pt = h.encoder_width, c.width, h.decoder_width, h.patch_size
        np_, t = b * self.patches, self.tc.sequence
        # final norm -> output_projection
        self._norm_bwd(self.y, "final_norm", self.invF, self.dhead, self.dy32, self.dyb, self.top_partials, n, dg,
                       accumulate=False)
        self._gemm(_ptr(self.zD), dd, 1, _ptr(self.dyb), dg, 0, self.g_ptr("output_projection"), dg, SJ_F32, dd, dg,
                   n, EPI_ACCUM)
        self._gemm(_ptr(self.dyb), dg, 0, self.wb_ptr("output_projection"), dg, 1, _ptr(dec.dz), dd, SJ_F32, n, dd, dg)
        self._norm_bwd(dec.x[-1], "decoder_norm", self.invD, dec.dz, dec.dx, dec.dxb, dec.partials, n, dd,
                       accumulate=False)
        self._stage_bwd(dec)
        yield "decoder"
        # decoder input = encoder_to_decoder(zE) + broadcast(global_to_decoder(zG), bos)
        self._gemm(_ptr(self.zE), de, 1, _ptr(dec.dxb), dd, 0, self.g_ptr("encoder_to_decoder"), dd, SJ_F32, de, dd,
                   n, EPI_ACCUM)
        self._gemm(_ptr(dec.dxb), dd, 0, self.wb_ptr("encoder_to_decoder"), dd, 1, _ptr(self.dE), de, SJ_F32, n, de,
                   dd)
        self._call("sj_patch_broadcast_bwd", _ptr(dec.dx), _ptr(self.dzd), _ptr(self.dbos), b, t, dd, pt, self.stream)
        self._gemm(_ptr(self.zG), dg, 1, _ptr(self.dzd), dd, 0, self.g_ptr("global_to_decoder"), dd, SJ_F32, dg, dd,
                   np_, EPI_ACCUM)
        self._gemm(self.wb_ptr("global_bos"), dg, 1, _ptr(self.dbos), dd, 0, self.g_ptr("global_to_decoder"), dd,
                   SJ_F32, dg, dd, 1, EPI_ACCUM)
        self._gemm(_ptr(self.dbos), dd, 0, self.wb_ptr("global_to_decoder"), dd, 1, self.g_ptr("global_bos"), dg,
                   SJ_F32, 1, dg, dd, EPI_ACCUM)
        self._gemm(_ptr(self.dzd), dd, 0, self.wb_ptr("global_to_decoder"), dd, 1, _ptr(glob.dz), dg, SJ_F32, np_, dg,
                   dd)
        self._norm_bwd(glob.x[-1], "global_norm", self.invG, glob.dz, glob.dx, glob.dxb, glob.partials, np_, dg,
                       accumulate=False)
        for tag in self._stage_bwd_gen(glob):
            yield f"global_{tag}"
        yield "global"
        # encoder_to_global, patch pool
        self._gemm(_ptr(self.pooled), de, 1, _ptr(glob.dxb), dg, 0, self.g_ptr("encoder_to_global"), dg, SJ_F32, de,
                   dg, np_, EPI_ACCUM)
        self._gemm(_ptr(glob.dxb), dg, 0, self.wb_ptr("encoder_to_global"), dg, 1, _ptr(self.dpool), de, SJ_F32, np_,
                   de, dg)
        self._call("sj_patch_pool_bwd", _ptr(self.dpool), _ptr(self.dE), b, t, de, pt, self.stream)
        self._norm_bwd(enc.x[-1], "encoder_norm", self.invE, self.dE, enc.dx, enc.dxb, enc.partials, n, de,
                       accumulate=False)
        self._stage_bwd(enc)
        if self.values:  # input_projection, then the native embedding (dy32 is free again: [rows, width] f32)
            self._gemm(_ptr(self.xin), dg, 1, _ptr(enc.dxb), de, 0, self.g_ptr("input_projection"), de, SJ_F32, dg, de,
                       n, EPI_ACCUM)
            self._gemm(_ptr(enc.dxb), de, 0, self.wb_ptr("input_projection"), de, 1, _ptr(self.dy32), dg, SJ_F32, n,
                       dg, de)
            self._call("sj_embedding_bwd", _ptr(self.dy32), _ptr(self.ids), self.g_ptr(emb), n, dg, vocab, self.stream)
        else:
            self._call("sj_embedding_bwd", _ptr(enc.dx), _ptr(self.ids), self.g_ptr(emb), n, de, VOCAB, self.stream)

    # ------------------------------------------------------------------ public step API
    def _local_forward_backward(self, first=True):
        """Loss and gradients of the staged batch; `first` = False adds them to those of the previous
        observations of the same step (gradient accumulation) instead of starting from zero."""
        for _ in self._local_forward_backward_gen(first):
            pass

    def _local_forward_backward_gen(self, first=True):
        """_local_forward_backward, yielding the tags of _backward_gen (the stream may change between
        phases: each phase reads the current stream)."""
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        if first:
            self._zero(self.g)
            self._zero(self.loss_sum)
        top, width = self._forward()
        for tag in self._backward_gen(top, width):
            yield tag
            self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        sb = self.layout.shared_begin
        if sb:  # sum of squares of this rank's experts' gradients, summed over the ranks by the exchange
            self._call("sj_grad_sumsq", _ptr(self.g), sb, _ptr(self.partials, self.n_shared_partials), self.stream)

    def _exchange(self):
        """Data-parallel exchange: sum of the per-rank gradients (each seeded with 1/global rows, so
        the sum is the global-batch mean gradient) and of the loss, over NCCL."""
        if self.world > 1:
            sb = self.layout.shared_begin
            if sb:  # expert parallelism: the experts' gradients stay with their owners
                distributed.exchange(self.g[sb:], self.loss_sum, self.pg, self.partials[self.n_shared_partials:])
            else:
                distributed.exchange(self.g, self.loss_sum, self.pg)

    # ------------------------------------------------------------------ overlapped data-parallel exchange
    def overlapped_exchange(self):
        """Whether the gradient exchange runs in buckets that overlap the backward pass: data parallel,
        without expert parallelism (whose exchange covers only the replicated range) and without the
        NativeValue head (whose native embedding sits among the first-final matrices)."""
        return self.world > 1 and self.layout.shared_begin == 0 and not self.values

    def grad_buckets(self):
        """The flat gradient's buckets (`gradient_buckets`)."""
        return gradient_buckets(self.layout, self.c)

    def _bucket_reduce(self, tag, works):
        """Start the SUM all-reduce of every bucket that `tag` completes (NCCL's stream, after the work
        enqueued so far on this one); `works` collects the handles."""
        for t, b, e in self._buckets:
            if t == tag:
                works.append(torch.distributed.all_reduce(self.g[b:e], group=self.pg, async_op=True))

    def _finish_exchange(self, works):
        self._bucket_reduce(None, works)
        works.append(torch.distributed.all_reduce(self.loss_sum, group=self.pg, async_op=True))
        for w in works:
            w.wait()  # this stream waits for NCCL's (the host does not block)

    def forward_backward(self, first=True, last=True):
        """Loss (into self.loss_sum) and gradients (into self.g) for the staged batch; with gradient
        accumulation, call once per observation (first / last mark the step's first and last).
        With data parallelism the exchange overlaps the backward pass (`grad_buckets`)."""
        if not (last and self.overlapped_exchange()):
            self._local_forward_backward(first)
            if last:
                self._exchange()
            return
        self._buckets = self.grad_buckets()
        works = []
        for tag in self._local_forward_backward_gen(first):
            self._bucket_reduce(tag, works)
        self._finish_exchange(works)

    def optimizer_step(self):
        """Adam::update (crates/sejong-train/src/lib.rs:199-238) or the dense SGD step, in two launches."""
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        tc = self.tc
        total = self.layout.total
        sb = self.layout.shared_begin
        self._call("sj_grad_sumsq", _ptr(self.g, sb), total - sb, _ptr(self.partials), self.stream)
        self._call("sj_optim_prepare", _ptr(self.partials), self.n_partials, _ptr(self.opt_state), _ptr(self.hyper),
             tc.learning_rate, tc.min_learning_rate, tc.warmup_steps, tc.steps, tc.beta1, tc.beta2, tc.clip_norm,
             int(tc.clip_enabled), tc.loss_scale, self.stream)
        if tc.optimizer == "adamw":
            self._call("sj_adamw", _ptr(self.w), _ptr(self.g), _ptr(self.m), _ptr(self.v), _ptr(self.wb), total,
                 self.layout.n_decay, _ptr(self.hyper), tc.beta1, tc.beta2, tc.epsilon, tc.weight_decay, self.stream)
        else:
            self._call("sj_sgd", _ptr(self.w), _ptr(self.g), _ptr(self.wb), total, self.layout.n_decay, _ptr(self.hyper),
                 tc.weight_decay, self.stream)

    def step(self):
        self.forward_backward()
        self.optimizer_step()

    def stage_batch(self, ids, targets, non_blocking=True):
        """Copy a batch (host or device int32 tensors) into the step's input buffers."""
        self.ids.copy_(torch.as_tensor(ids, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)
        self.targets.copy_(torch.as_tensor(targets, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)

    def stage_requests(self, ids, sel, labels, non_blocking=True):
        """NativeValue mode: a batch of requests (sejong_b200.value.request_batch) and their labels."""
        if not self.values:
            raise ValueError("stage_requests needs a trainer built with TrainConfig.values > 0")
        self.ids.copy_(torch.as_tensor(ids, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)
        self.sel.copy_(torch.as_tensor(sel, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)
        self.labels.copy_(torch.as_tensor(labels, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)

    # ------------------------------------------------------------------ artifacts
    def save_checkpoint(self, directory, data_fingerprint=None, rng_state=None, model_id="sejong", precision="f16"):
        """save_training (crates/sejong-train/src/lib.rs:472-491) and the SGD route's `save`
        (crates/sejong-train/src/control_variate.rs:389-406): the FP32 master weights under the
        reference's parameter names, the optimizer step (the device optimizer state), the training
        config, the data fingerprint and the data generator's state, written atomically, with the
        optimizer state: AdamW moments as m.<name> / v.<name>, or the SGD state of
        SgdState::tensors (control_variate.rs:208-233: sgd.version, and the sampling, basis and
        parameter-VJP generators as four 16-bit words each)."""
        from . import checkpoint
        if self.ep is not None:
            raise checkpoint.ArtifactError("checkpoints of an expert-parallel trainer are not supported: each rank "
                                           "holds only its own experts")
        torch.cuda.synchronize(self.dev)
        params = self.layout.unpack(self.w.cpu().numpy())
        optimizer = None
        if self.tc.optimizer == "adamw":
            optimizer = {}
            for prefix, buf in (("m", self.m), ("v", self.v)):
                for name, value in self.layout.unpack(buf.cpu().numpy()).items():
                    optimizer[f"{prefix}.{name}"] = value
        else:
            optimizer = checkpoint.sgd_state_tensors(self.tc.seed, self.vjp_rng_state() if self.vjp is not None
                                                     else None)
        step = int(self.opt_state[0].item())
        return checkpoint.save(directory, self.c, params, step, optimizer, checkpoint.train_config_json(self.tc),
                               data_fingerprint, rng_state, model_id=model_id, precision=precision)

    def load_checkpoint(self, directory):
        """Resume from an artifact directory (Model::load, crates/sejong-model/src/lib.rs:134-170):
        weights, moments when present, and the optimizer step.  The artifact's model must have this
        trainer's parameter layout.  Returns the manifest."""
        from . import checkpoint
        config, params, manifest, optimizer = checkpoint.load(directory, self.c.init_std)
        if reference_layout(config) != reference_layout(self.c):
            raise checkpoint.ArtifactError("artifact model layout differs from this trainer's")
        torch.cuda.synchronize(self.dev)
        self.w.copy_(torch.from_numpy(self.layout.pack(params)).to(self.dev))
        if self.tc.optimizer != "adamw":
            # SgdState::load (control_variate.rs:122-195): the version, the generators, and nothing else
            if optimizer is None:
                raise checkpoint.ArtifactError("resume requires SGD optimizer state")
            rngs = checkpoint.read_sgd_state(optimizer, self.vjp is not None)
            if self.vjp is not None:
                self.vjp_rng.copy_(torch.from_numpy(np.array([rngs["sgd.parameter_rng"]], dtype=np.uint64)
                                                    .view(np.int64)).to(self.dev))
            self.m.zero_()
            self.v.zero_()
        elif optimizer is not None:
            for prefix, buf in (("m", self.m), ("v", self.v)):
                named = {k[len(prefix) + 1:]: v for k, v in optimizer.items() if k.startswith(prefix + ".")}
                if set(named) != set(params):
                    raise checkpoint.ArtifactError(f"optimizer state {prefix} does not cover every parameter")
                buf.copy_(torch.from_numpy(self.layout.pack(named)).to(self.dev))
        else:
            self.m.zero_()
            self.v.zero_()
        self.opt_state[0] = float(manifest["step"])
        call("sj_cast", _ptr(self.w), SJ_F32, _ptr(self.wb), SJ_BF16, self.layout.total,
             torch.cuda.current_stream(self.dev).cuda_stream)
        torch.cuda.synchronize(self.dev)
        return manifest

    def capture(self):
        """Capture the step as CUDA graphs (replayed by `replay`).

        One graph (forward + backward + update) on a single GPU.  With data parallelism the
        forward / backward is one graph per phase between gradient buckets and the update one more;
        the NCCL all-reduces of the buckets run between the replays, on NCCL's stream, overlapping the
        later phases (expert parallelism and the NativeValue head: one forward / backward graph, the
        exchange, the update), so no collective is captured."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        graphs = []
        with torch.cuda.stream(s):
            if self.world == 1:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    self.step()
                graphs.append(g)
            elif self.overlapped_exchange():
                # one graph per phase of the forward / backward, split where gradient buckets become
                # final; replay starts each bucket's all-reduce between the phases (no collective is
                # captured), then the update graph
                self._buckets = self.grad_buckets()
                gen = self._local_forward_backward_gen()
                done = False
                while not done:
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=s):
                        try:
                            tag = next(gen)
                        except StopIteration:
                            tag, done = None, True
                    graphs.append((g, tag))
                g2 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g2, stream=s):
                    self.optimizer_step()
                graphs.append((g2, "update"))
            else:
                g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                with torch.cuda.graph(g1, stream=s):
                    self._local_forward_backward()
                with torch.cuda.graph(g2, stream=s):
                    self.optimizer_step()
                graphs += [g1, g2]
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = graphs
        return graphs

    def replay(self):
        if len(self.graph) == 1:
            self.graph[0].replay()
        elif isinstance(self.graph[0], tuple):
            works = []
            for g, tag in self.graph[:-1]:
                g.replay()
                if tag is not None:
                    self._bucket_reduce(tag, works)
            self._finish_exchange(works)
            self.graph[-1][0].replay()
        else:
            self.graph[0].replay()
            self._exchange()
            self.graph[1].replay()

    def release_graphs(self):
        """Drop captured graphs (before destroying a process group)."""
        self.graph = None

    def close(self):
        """Release the expert-parallel heap (every rank, after its last step; then a barrier)."""
        self.graph = None
        if self.ep is not None:
            torch.cuda.synchronize(self.dev)
            if self.pg is not None:
                torch.distributed.barrier(self.pg)
            self.ep.close()

    # ------------------------------------------------------------------ inspection
    def loss(self):
        return float(self.loss_sum.item())

    def gradients(self):
        """Reference-named f32 gradients of the last forward_backward."""
        return self.layout.unpack(self.g.detach().cpu().numpy())

    def parameters(self):
        return self.layout.unpack(self.w.detach().cpu().numpy())

    def device_error(self):
        code = ctypes.c_int(0)
        self._call("sj_device_error", ctypes.byref(code), 1, self.stream)
        return code.value

    def routed_rows(self):
        """Rows an MoE layer sends to its experts (rows x top-k of the MoE stage; 0 without experts)."""
        for run in self.runs.values():
            if run.moe:
                return run.rows * run.stage.experts.top_k
        return 0

    def step_flops(self):
        """Algorithmic FLOPs of one step (FMA = 2; attention 4*B*H*64*pairs fwd, 8*... bwd; no recompute)."""
        c, tc = self.c, self.tc
        b, t = tc.batch, tc.sequence
        lin = 0
        att = 0

        def stage_cost(s, rows, seq):
            nonlocal lin, att
            d, kv = s.width, s.kv_heads * HEAD_DIM
            if s.experts is None:
                per = d * d + 2 * d * kv + d * d + 3 * d * s.ffn
                lin += 2 * rows * per * s.layers
            else:  # router for every row, the chosen experts' SwiGLU FFN for every routed row
                e = s.experts
                per = d * d + 2 * d * kv + d * d + d * e.count
                lin += 2 * rows * per * s.layers + 2 * rows * e.top_k * 3 * d * e.ffn_width * s.layers
            w = s.window or seq
            pairs = sum(min(q + 1, w) for q in range(seq))
            att += 4 * (rows // seq) * s.heads * HEAD_DIM * pairs * s.layers

        h = c.hierarchy
        if h is None:
            stage_cost(global_stage(c), b * t, t)
            lin += 2 * b * c.width * self.values if self.values else 2 * b * t * c.width * VOCAB
        else:
            p = t // h.patch_size
            stage_cost(local_stage(c, True), b * t, t)
            stage_cost(global_stage(c), b * p, p)
            stage_cost(local_stage(c, False), b * t, t)
            lin += 2 * b * p * h.encoder_width * c.width            # encoder_to_global
            lin += 2 * b * p * c.width * h.decoder_width            # global_to_decoder
            lin += 2 * b * t * h.encoder_width * h.decoder_width    # encoder_to_decoder
            lin += 2 * b * t * h.decoder_width * c.width            # output_projection
            lin += 2 * b * c.width * self.values if self.values else 2 * b * t * c.width * VOCAB  # head
            if self.values:
                lin += 2 * b * t * c.width * h.encoder_width        # input_projection
        total = 3 * lin + 3 * att  # fwd + (dX + dW) for linear; fwd (4) + bwd (8) for attention
        if self.vjp is not None:
            # executed work of the parameter VJP instead of the dense dW of each compressed group:
            # basis (donor columns 2nar, once per (rows, rank)), prepare (left 2nar, residual rows
            # 2nkr), coefficients 2(r+k)nB, factored gradient 2aBr
            for g in self.vjp.groups.values():
                n, a, r, k = g.rows, g.features, g.rank, g.k
                width = sum(m.width for m in g.members)
                active = sum(g.members[i].width for i in g.active)
                total -= 2 * n * a * active
                total += 2 * n * a * r * (2 if g.new_basis else 1) + 2 * n * k * r
                total += 2 * (r + k) * n * width + 2 * a * active * r
        return total


def gradient_buckets(layout, c):
    """The flat gradient's buckets for the overlapped data-parallel exchange, as (tag, begin, end): the
    range becomes final when the backward yields `tag` (tag None: at its end).  The rank > 1 tensors lie
    in the forward order of the model, so the backward finishes them from the end: the decoder blocks
    and heads first, then the upper and the lower half of the global blocks, then the rest together
    with the norm vectors."""
    nd = layout.n_decay
    ents = list(layout.entries.values())

    def first(prefix):
        return min(e.offset for e in ents if e.name.startswith(prefix) and e.decay)

    half = global_stage(c).layers // 2
    g0 = first("layers.0.")
    gh = first(f"layers.{half}.") if half > 0 else g0
    if c.hierarchy is not None:
        dec = first("decoder.")
        out = [("decoder", dec, nd), ("global_half", gh, dec), ("global", g0, gh)]
        out += [(None, 0, g0), (None, nd, layout.total)]
    else:
        out = [("global_half", gh, nd), (None, 0, gh), (None, nd, layout.total)]
    return [b for b in out if b[2] > b[1]]


def synthetic_corpus_tokens(seed, length, s=1.1):
    """Token stream of one synthetic Zipf document: EOS + bytes + EOS (Corpus layout, lib.rs:24-71)."""
    buf = np.empty(length, dtype=np.uint8)
    call("sj_zipf_bytes", seed, float(s), buf.ctypes.data, length)
    toks = np.empty(length + 2, dtype=np.int32)
    toks[0] = 256
    toks[1:-1] = buf
    toks[-1] = 256
    return toks


def corpus_batch(tokens, rng_state, batch, sequence):
    """Corpus::batch (crates/sejong-train/src/lib.rs:72-88) via the library's Rng; rng_state: ctypes.c_uint64."""
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    inputs = np.empty(batch * sequence, dtype=np.int32)
    targets = np.empty(batch * sequence, dtype=np.int32)
    call("sj_corpus_batch", tokens.ctypes.data, tokens.size, ctypes.byref(rng_state), batch, sequence,
         inputs.ctypes.data, targets.ctypes.data)
    return inputs, targets
