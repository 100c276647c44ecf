"""The dense byte-model training step in f32 arithmetic ("one training step in
fp32"; the reference's DType::F32 precision, under which Model::bind casts nothing,
crates/sejong-model/src/lib.rs:206-219).

The same schedule as `ByteTrainer` for the dense model (crates/sejong-model/src/architecture.rs:
201-246, 330-393; tape rules crates/sejong-gpu/src/graph.rs:817-913; Adam::update
crates/sejong-train/src/lib.rs:199-238): embedding -> blocks [RMSNorm, QKV GEMM + RoPE, GQA
attention, Wo GEMM + residual, RMSNorm, gate/up GEMM + SwiGLU, down GEMM + residual] -> final norm
-> head -> cross entropy, the backward in reverse, AdamW.  Every activation, GEMM operand and
gradient is f32; the GEMMs and attention run on the f32 kernels of csrc/f32.cu (CUDA-core FMA),
the master weights are read directly (no compute-precision copy).
"""
import ctypes

import torch

from . import _lib, distributed
from ._lib import EPI_ACCUM, EPI_RESIDUAL, EPI_ROPE, EPI_STORE, EPI_SWIGLU, SJ_F32, call
from .model import HEAD_DIM, VOCAB, VOCAB_PAD, FlatLayout, global_stage, initialize
from .train import TrainConfig  # noqa: F401  (the same configuration object)


def _ptr(t, offset_elems=0):
    return t.data_ptr() + offset_elems * t.element_size()


class F32Trainer:
    """One data-parallel replica of the dense byte-model step in f32 on the current CUDA device."""

    KERNELS = {"sj_rmsnorm_bwd": 2, "sj_rmsnorm_bwd_ex": 2, "sj_attn_f32_bwd": 3}

    def __init__(self, config, train, device=None, params=None, process_group=None):
        if config.hierarchy is not None or config.experts is not None:
            raise ValueError("the f32 step covers the dense byte model (BASELINE C1)")
        if train.parameter_vjp is not None or train.values:
            raise ValueError("the f32 step is the AdamW / SGD byte step")
        self.c, self.tc = config, train
        self.launches = 0
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        torch.cuda.set_device(self.dev)
        self.lib = _lib.load()
        call("sj_device_init", self.dev.index)
        self.pg = process_group
        self.world = torch.distributed.get_world_size(process_group) if process_group is not None else 1
        self.layout = FlatLayout(config)
        if params is None:
            params = initialize(config, self.lib)
        total = self.layout.total
        f32 = torch.float32
        self.w = torch.from_numpy(self.layout.pack(params)).to(self.dev)
        self.g = torch.zeros(total, dtype=f32, device=self.dev)
        self.m = torch.zeros(total, dtype=f32, device=self.dev)
        self.v = torch.zeros(total, dtype=f32, device=self.dev)
        self.n_partials = self.lib.sj_sumsq_partials(total)
        self.partials = torch.zeros(self.n_partials, dtype=torch.float64, device=self.dev)
        self.opt_state = torch.zeros(2, dtype=torch.float64, device=self.dev)
        self.hyper = torch.zeros(8, dtype=f32, device=self.dev)
        self.loss_sum = torch.zeros(1, dtype=torch.float64, device=self.dev)
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream

        b, t = train.batch, train.sequence
        self.rows = n = b * t
        self.s = s = global_stage(config)
        d, f, cq = s.width, s.ffn, s.qkv_width
        e = lambda *shape: torch.empty(*shape, dtype=f32, device=self.dev)  # noqa: E731
        self.ids = torch.zeros(n, dtype=torch.int32, device=self.dev)
        self.targets = torch.zeros(n, dtype=torch.int32, device=self.dev)
        self.x = [e(n, d) for _ in range(s.layers + 1)]
        self.layers = [dict(z1=e(n, d), inv1=e(n), qkv=e(n, cq), o=e(n, d), lse=e(n * s.heads), x1=e(n, d),
                            z2=e(n, d), inv2=e(n), gu=e(n, 2 * f), h=e(n, f)) for _ in range(s.layers)]
        self.dx, self.dz, self.do = e(n, d), e(n, d), e(n, d)
        self.dh, self.dgu, self.dqkv = e(n, f), e(n, 2 * f), e(n, cq)
        self.delta = e(self.lib.sj_attn_f32_workspace(b, t, s.heads))
        self.norm_partials = e(self.lib.sj_rmsnorm_workspace(n, d))
        self.hf, self.invF = e(n, d), e(n)
        self.logits, self.dlogits, self.dhead = e(n, VOCAB_PAD), e(n, VOCAB_PAD), e(n, d)
        self.rope = e(t * HEAD_DIM)
        call("sj_rope_table", _ptr(self.rope), t, HEAD_DIM, 0, float(config.rope_theta), self.stream)
        self.graph = None

    # ------------------------------------------------------------------ primitives
    @classmethod
    def kernels_of(cls, name, args):
        return cls.KERNELS.get(name, 1)

    def _call(self, name, *args):
        call(name, *args)
        self.launches += self.kernels_of(name, args)

    def w_ptr(self, name):
        return _ptr(self.w, self.layout[name].offset)

    def g_ptr(self, name):
        return _ptr(self.g, self.layout[name].offset)

    def _gemm(self, a, lda, a_trans, b, ldb, b_trans, c, ldc, m, n, k, epi=EPI_STORE, aux=0, ld_aux=0, rope_cols=0):
        self._call("sj_sgemm", a, lda, a_trans, b, ldb, b_trans, c, ldc, m, n, k, epi, aux, ld_aux,
                   _ptr(self.rope) if epi == EPI_ROPE else 0, rope_cols, self.tc.sequence, self.stream)

    def _norm(self, x, wname, y, inv, rows, d):
        self._call("sj_rmsnorm_fwd_f32", _ptr(x), self.w_ptr(wname), _ptr(y), _ptr(inv), rows, d,
                   float(self.c.norm_epsilon), self.stream)

    def _norm_bwd(self, x, wname, inv, dz, dres, rows, d, accumulate=True):
        self._call("sj_rmsnorm_bwd_ex", _ptr(x), SJ_F32, self.w_ptr(wname), _ptr(inv), _ptr(dz), _ptr(dres), 0,
                   self.g_ptr(wname), _ptr(self.norm_partials), rows, d, int(accumulate), self.stream)

    def _zero(self, t):
        self._call("sj_zero", _ptr(t), t.numel() * t.element_size(), self.stream)

    # ------------------------------------------------------------------ step
    def _block_fwd(self, i):
        s, a = self.s, self.layers[i]
        n, d, f, cq, t = self.rows, s.width, s.ffn, s.qkv_width, self.tc.sequence
        p = f"{s.prefix}.{i}"
        x, xn = self.x[i], self.x[i + 1]
        self._norm(x, f"{p}.attention_norm", a["z1"], a["inv1"], n, d)
        self._gemm(_ptr(a["z1"]), d, 0, self.w_ptr(f"{p}.qkv"), cq, 0, _ptr(a["qkv"]), cq, n, cq, d, EPI_ROPE,
                   rope_cols=(s.heads + s.kv_heads) * HEAD_DIM)
        qkv = a["qkv"]
        self._call("sj_attn_f32_fwd", _ptr(qkv), cq, _ptr(qkv, s.heads * HEAD_DIM), cq,
                   _ptr(qkv, (s.heads + s.kv_heads) * HEAD_DIM), cq, _ptr(a["o"]), d, _ptr(a["lse"]), self.tc.batch,
                   t, s.heads, s.kv_heads, HEAD_DIM, s.window, self.stream)
        self._gemm(_ptr(a["o"]), d, 0, self.w_ptr(f"{p}.attention_output"), d, 0, _ptr(a["x1"]), d, n, d, d,
                   EPI_RESIDUAL, aux=_ptr(x), ld_aux=d)
        self._norm(a["x1"], f"{p}.ffn_norm", a["z2"], a["inv2"], n, d)
        self._gemm(_ptr(a["z2"]), d, 0, self.w_ptr(f"{p}.gate_up"), 2 * f, 0, _ptr(a["gu"]), 2 * f, n, 2 * f, d,
                   EPI_SWIGLU, aux=_ptr(a["h"]), ld_aux=f)
        self._gemm(_ptr(a["h"]), f, 0, self.w_ptr(f"{p}.down"), d, 0, _ptr(xn), d, n, d, f, EPI_RESIDUAL,
                   aux=_ptr(a["x1"]), ld_aux=d)

    def _block_bwd(self, i):
        """self.dx holds dL/d(block output); on return dL/d(block input)."""
        s, a = self.s, self.layers[i]
        n, d, f, cq, t = self.rows, s.width, s.ffn, s.qkv_width, self.tc.sequence
        p = f"{s.prefix}.{i}"
        dx = self.dx
        self._gemm(_ptr(a["h"]), f, 1, _ptr(dx), d, 0, self.g_ptr(f"{p}.down"), d, f, d, n, EPI_ACCUM)
        self._gemm(_ptr(dx), d, 0, self.w_ptr(f"{p}.down"), d, 1, _ptr(self.dh), f, n, f, d)
        self._call("sj_swiglu_bwd_f32", _ptr(a["gu"]), _ptr(self.dh), _ptr(self.dgu), n, f, self.stream)
        self._gemm(_ptr(a["z2"]), d, 1, _ptr(self.dgu), 2 * f, 0, self.g_ptr(f"{p}.gate_up"), 2 * f, d, 2 * f, n,
                   EPI_ACCUM)
        self._gemm(_ptr(self.dgu), 2 * f, 0, self.w_ptr(f"{p}.gate_up"), 2 * f, 1, _ptr(self.dz), d, n, d, 2 * f)
        self._norm_bwd(a["x1"], f"{p}.ffn_norm", a["inv2"], self.dz, dx, n, d)
        self._gemm(_ptr(a["o"]), d, 1, _ptr(dx), d, 0, self.g_ptr(f"{p}.attention_output"), d, d, d, n, EPI_ACCUM)
        self._gemm(_ptr(dx), d, 0, self.w_ptr(f"{p}.attention_output"), d, 1, _ptr(self.do), d, n, d, d)
        qkv, dqkv = a["qkv"], self.dqkv
        kq, vq = s.heads * HEAD_DIM, (s.heads + s.kv_heads) * HEAD_DIM
        self._call("sj_attn_f32_bwd", _ptr(qkv), cq, _ptr(qkv, kq), cq, _ptr(qkv, vq), cq, _ptr(a["o"]), d,
                   _ptr(a["lse"]), _ptr(self.do), d, _ptr(dqkv), cq, _ptr(dqkv, kq), cq, _ptr(dqkv, vq), cq,
                   _ptr(self.delta), self.tc.batch, t, s.heads, s.kv_heads, HEAD_DIM, s.window, _ptr(self.rope),
                   self.stream)
        self._gemm(_ptr(a["z1"]), d, 1, _ptr(dqkv), cq, 0, self.g_ptr(f"{p}.qkv"), cq, d, cq, n, EPI_ACCUM)
        self._gemm(_ptr(dqkv), cq, 0, self.w_ptr(f"{p}.qkv"), cq, 1, _ptr(self.dz), d, n, d, cq)
        self._norm_bwd(self.x[i], f"{p}.attention_norm", a["inv1"], self.dz, dx, n, d)

    def _local_forward_backward(self):
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        c, n, d = self.c, self.rows, self.c.width
        self._zero(self.g)
        self._zero(self.loss_sum)
        self._call("sj_embedding_fwd_f32", self.w_ptr("embedding"), _ptr(self.ids), _ptr(self.x[0]), n, d, VOCAB,
                   self.stream)
        for i in range(self.s.layers):
            self._block_fwd(i)
        top = self.x[-1]
        self._norm(top, "final_norm", self.hf, self.invF, n, d)
        self._gemm(_ptr(self.hf), d, 0, self.w_ptr("output"), VOCAB_PAD, 0, _ptr(self.logits), VOCAB_PAD, n, VOCAB, d)
        self._call("sj_cross_entropy_f32", _ptr(self.logits), VOCAB_PAD, _ptr(self.targets), n, VOCAB,
                   distributed.ce_seed(n, self.world, self.tc.loss_scale), 0, _ptr(self.dlogits), VOCAB_PAD,
                   _ptr(self.loss_sum), distributed.ce_seed(n, self.world), self.stream)
        # backward
        self._gemm(_ptr(self.hf), d, 1, _ptr(self.dlogits), VOCAB_PAD, 0, self.g_ptr("output"), VOCAB_PAD, d, VOCAB,
                   n, EPI_ACCUM)
        self._gemm(_ptr(self.dlogits), VOCAB_PAD, 0, self.w_ptr("output"), VOCAB_PAD, 1, _ptr(self.dhead), d, n, d,
                   VOCAB)
        self._norm_bwd(top, "final_norm", self.invF, self.dhead, self.dx, n, d, accumulate=False)
        for i in reversed(range(self.s.layers)):
            self._block_bwd(i)
        self._call("sj_embedding_bwd", _ptr(self.dx), _ptr(self.ids), self.g_ptr("embedding"), n, d, VOCAB,
                   self.stream)

    def _exchange(self):
        if self.world > 1:
            distributed.exchange(self.g, self.loss_sum, self.pg)

    def forward_backward(self):
        self._local_forward_backward()
        self._exchange()

    def optimizer_step(self):
        """Adam::update (crates/sejong-train/src/lib.rs:199-238) or the dense SGD step."""
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        tc, total = self.tc, self.layout.total
        self._call("sj_grad_sumsq", _ptr(self.g), total, _ptr(self.partials), self.stream)
        self._call("sj_optim_prepare", _ptr(self.partials), self.n_partials, _ptr(self.opt_state), _ptr(self.hyper),
                   tc.learning_rate, tc.min_learning_rate, tc.warmup_steps, tc.steps, tc.beta1, tc.beta2,
                   tc.clip_norm, int(tc.clip_enabled), tc.loss_scale, self.stream)
        if tc.optimizer == "adamw":
            self._call("sj_adamw", _ptr(self.w), _ptr(self.g), _ptr(self.m), _ptr(self.v), 0, total,
                       self.layout.n_decay, _ptr(self.hyper), tc.beta1, tc.beta2, tc.epsilon, tc.weight_decay,
                       self.stream)
        else:
            self._call("sj_sgd", _ptr(self.w), _ptr(self.g), 0, total, self.layout.n_decay, _ptr(self.hyper),
                       tc.weight_decay, self.stream)

    def step(self):
        self.forward_backward()
        self.optimizer_step()

    def stage_batch(self, ids, targets, non_blocking=True):
        self.ids.copy_(torch.as_tensor(ids, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)
        self.targets.copy_(torch.as_tensor(targets, dtype=torch.int32).reshape(-1), non_blocking=non_blocking)

    def capture(self):
        """The step as CUDA graphs: one on a single GPU; with data parallelism forward/backward and
        the update, the NCCL exchange between them (as ByteTrainer.capture)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        graphs = []
        with torch.cuda.stream(s):
            if self.world == 1:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    self.step()
                graphs.append(g)
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
        self.graph[0].replay()
        if len(self.graph) > 1:
            self._exchange()
            self.graph[1].replay()

    def release_graphs(self):
        self.graph = None

    def close(self):
        self.graph = None

    def loss(self):
        return float(self.loss_sum.item())

    def gradients(self):
        return self.layout.unpack(self.g.detach().cpu().numpy())

    def parameters(self):
        return self.layout.unpack(self.w.detach().cpu().numpy())

    def device_error(self):
        code = ctypes.c_int(0)
        call("sj_device_error", ctypes.byref(code), 1, self.stream)
        return code.value

    def routed_rows(self):
        return 0

    def step_flops(self):
        """Algorithmic FLOPs of one step: 3 x 2 rows params for the linear layers, attention 4 B H 64
        pairs forward and 8 B H 64 pairs backward (exact causal pairs)."""
        c, b, t, s = self.c, self.tc.batch, self.tc.sequence, self.s
        d, kv = s.width, s.kv_heads * HEAD_DIM
        per = d * d + 2 * d * kv + d * d + 3 * d * s.ffn
        lin = 2 * b * t * (per * s.layers + d * VOCAB)
        pairs = t * (t + 1) // 2 if s.window <= 0 else sum(min(i + 1, s.window) for i in range(t))
        att = 4 * b * s.heads * HEAD_DIM * pairs * s.layers
        return 3 * lin + 3 * att
