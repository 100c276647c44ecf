"""Byte-Transformer training step restated on the CPU (FP64 by default).

Follows crates/sejong-model/src/architecture.rs:
  * parameter layout and names: `layout` (architecture.rs:63-137)
  * pre-norm GQA + SwiGLU block: `Block::apply` (architecture.rs:201-246)
  * hierarchy: encoder -> patch mean-pool -> global -> previous-patch broadcast
    (+ projected BOS) added to encoder_to_decoder(bytes) -> decoder ->
    output_projection -> final_norm (architecture.rs:330-393,
    crates/sejong-model/src/lib.rs:254-340)
  * output head on the FP32-cast hidden (lib.rs:336-340, architecture.rs:160-167)
  * MoE FFN: router GEMM, softmax top-k, per-expert FFN, gate-weighted combine
    (architecture.rs:229-241; hierarchy.py:175-251) — no capacity limit, no
    auxiliary loss, gate = full-softmax probability.
Training step (crates/sejong-train/src/lib.rs:387-453): mean next-byte CE,
FP64 global gradient norm / loss_scale, clip to clip_norm, AdamW per tensor with
decoupled decay on rank>1 tensors only (lib.rs:199-238); parameters without a
gradient (e.g. `input_projection` when nothing is injected) get a zero gradient
and are still updated.

Gradients are exact FP64 derivatives of the forward (torch autograd); the
reference's explicit backward kernels are pinned separately in `ops.py`.
"""
import math
from dataclasses import dataclass, field, replace
from typing import Optional

import numpy as np
import torch

from . import ops
from .rng import Rng

VOCAB = 257


@dataclass
class HierarchyConfig:
    patch_size: int
    encoder_width: int
    encoder_layers: int
    encoder_heads: int
    encoder_ffn_width: int
    decoder_width: int
    decoder_layers: int
    decoder_heads: int
    decoder_ffn_width: int
    local_window: int


@dataclass
class ExpertConfig:
    count: int
    top_k: int
    ffn_width: int


@dataclass
class ModelConfig:
    width: int
    layers: int
    heads: int
    ffn_width: int
    kv_heads: Optional[int] = None
    context: int = 8192
    rope_theta: float = 10000.0
    norm_epsilon: float = 1e-6
    hierarchy: Optional[HierarchyConfig] = None
    experts: Optional[ExpertConfig] = None
    seed: int = 42
    init_std: float = 0.02       # 0 selects the reference's fan-in init (lib.rs:82-116)
    router_std: float = 0.02
    # MoE additions that the reference lacks (0 keeps its semantics): expert capacity factor and the
    # weight of the load-balancing loss, restated from their definitions in sejong_b200/csrc/moe.cu
    moe_capacity_factor: float = 0.0
    moe_aux_weight: float = 0.0


@dataclass
class TrainConfig:
    sequence: int
    batch: int
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


@dataclass
class Stage:
    prefix: str
    width: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    window: Optional[int]
    experts: Optional[ExpertConfig] = None


def global_stage(c):
    return Stage("layers", c.width, c.layers, c.heads, c.kv_heads or c.heads, c.ffn_width, None, c.experts)


def local_stage(c, encoder):
    h = c.hierarchy
    if encoder:
        return Stage("encoder", h.encoder_width, h.encoder_layers, h.encoder_heads, h.encoder_heads,
                     h.encoder_ffn_width, h.local_window)
    return Stage("decoder", h.decoder_width, h.decoder_layers, h.decoder_heads, h.decoder_heads,
                 h.decoder_ffn_width, h.local_window)


def stage_layout(s, out):
    d = s.width
    kv = d // s.heads * s.kv_heads
    for i in range(s.layers):
        p = f"{s.prefix}.{i}"
        out.append((f"{p}.attention_norm", (d,), True))
        out.append((f"{p}.ffn_norm", (d,), True))
        for name, w in (("query", d), ("key", kv), ("value", kv), ("attention_output", d)):
            out.append((f"{p}.{name}", (d, w), False))
        if s.experts is not None:
            for e in range(s.experts.count):
                for name in ("gate", "up"):
                    out.append((f"{p}.experts.{e}.{name}", (d, s.experts.ffn_width), False))
                out.append((f"{p}.experts.{e}.down", (s.experts.ffn_width, d), False))
            out.append((f"{p}.router", (d, s.experts.count), False))
        else:
            for name in ("gate", "up"):
                out.append((f"{p}.{name}", (d, s.ffn), False))
            out.append((f"{p}.down", (s.ffn, d), False))


def layout(c):
    """architecture.rs:93-137: (name, shape, is_norm) in parameter order."""
    h = c.hierarchy
    out = [("embedding", (VOCAB, h.encoder_width if h else c.width), False)]
    if h is not None:
        stage_layout(local_stage(c, True), out)
        out.append(("encoder_norm", (h.encoder_width,), True))
        out.append(("input_projection", (c.width, h.encoder_width), False))
        out.append(("encoder_to_global", (h.encoder_width, c.width), False))
        out.append(("encoder_to_decoder", (h.encoder_width, h.decoder_width), False))
        out.append(("global_to_decoder", (c.width, h.decoder_width), False))
        out.append(("global_bos", (1, c.width), False))
        out.append(("global_norm", (c.width,), True))
        stage_layout(global_stage(c), out)
        stage_layout(local_stage(c, False), out)
        out.append(("decoder_norm", (h.decoder_width,), True))
        out.append(("output_projection", (h.decoder_width, c.width), False))
    else:
        stage_layout(global_stage(c), out)
    out.append(("final_norm", (c.width,), True))
    out.append(("output", (c.width, VOCAB), False))
    return out


def initialize(c):
    """FP32 master weights drawn from Rng(c.seed) in layout order.

    init_std > 0: every matrix N(0, init_std) (router N(0, router_std)), norms 1.
    init_std == 0: the reference's rule (crates/sejong-model/src/lib.rs:82-116):
    std 1/sqrt(fan_in) (embedding: 1/sqrt(width)), `.down`/`.attention_output`
    scaled by 1/sqrt(2 depth), `global_bos` zero.
    Each non-norm element consumes one `Rng::normal` (two uniforms) in order.
    """
    rng = Rng(c.seed)
    params = {}
    for name, shape, norm in layout(c):
        n = int(np.prod(shape))
        if norm:
            params[name] = np.ones(shape, dtype=np.float32)
            continue
        if c.init_std > 0:
            std = c.router_std if name.endswith(".router") else c.init_std
            params[name] = (rng.bulk_normal(n) * np.float32(std)).astype(np.float32).reshape(shape)
            continue
        std = 1.0 / np.sqrt(np.float32(shape[1] if name == "embedding" else shape[0]), dtype=np.float32)
        h = c.hierarchy
        depth = c.layers
        if h is not None:
            if name.startswith("encoder."):
                depth = h.encoder_layers
            elif name.startswith("decoder."):
                depth = h.decoder_layers
        if name.endswith(".down") or name.endswith(".attention_output"):
            std = std / np.sqrt(np.float32(2.0 * depth), dtype=np.float32)
        if name == "global_bos":  # written as 0 without consuming draws (lib.rs:104-110)
            params[name] = np.zeros(shape, dtype=np.float32)
            continue
        params[name] = (rng.bulk_normal(n) * np.float32(std)).astype(np.float32).reshape(shape)
    return params


# Every parameter matmul goes through `mm`, in the reference's node-creation order, so that a
# recorder (param_vjp.py) can replay the tape's backward visit order (graph.rs:567-913).
MATMUL_HOOK = None
# Test hook: {block prefix: LongTensor [rows, top_k]} of expert ids to use instead of the top-k of the
# oracle's own router logits (the gates stay the full-softmax probabilities of those experts).  A
# parity test sets it to the routing the GPU chose, so that the FP64 arithmetic is compared on the
# same routing decisions; near-tied router logits may otherwise pick different experts in FP64.
ROUTE_OVERRIDE = None
# Test hook for the load-balancing loss: {block prefix: LongTensor [rows, top_k]} of the top-k choices
# (before any capacity drop) whose shares f_e the loss uses.  f is piecewise constant in the logits, so a
# near tie that rounds the other way changes it by a whole choice; a parity test passes the GPU's own
# choices so that both sides weigh the same shares.
AUX_CHOICES = None


def mm(x, p, name):
    y = x @ p[name]
    if MATMUL_HOOK is not None:
        MATMUL_HOOK(name, x, y)
    return y


AUX_TERMS = []   # load-balancing losses of the current forward (summed into the loss)


def apply_capacity(ids, experts, capacity):
    """Expert capacity: each expert keeps at most `capacity` slots; every row's first choice before any
    second choice, rows in order within one choice; dropped slots become -1."""
    out = ids.clone()
    fill = torch.zeros(experts, dtype=torch.int64)
    for j in range(ids.shape[1]):
        col = ids[:, j]
        onehot = torch.nn.functional.one_hot(col, experts)           # [rows, E]
        rank = torch.cumsum(onehot, dim=0) - onehot + fill[None, :]  # slots of e before this row
        keep = (rank * onehot).sum(1) < capacity
        out[~keep, j] = -1
        fill += onehot.sum(0)
    return out


def aux_loss(logits, ids_topk, experts, weight):
    """Load-balancing loss weight * E * sum_e f_e P_e: f_e the share of the top-k choices (before any
    capacity drop) that picked e, P_e the mean router probability (differentiable) of e."""
    p = torch.softmax(logits, dim=1)
    f = torch.nn.functional.one_hot(ids_topk.reshape(-1), experts).to(p.dtype).mean(0)
    return weight * experts * (f * p.mean(0)).sum()


def _block(p, prefix, s, x, seq, theta, eps, c=None):
    z = ops.rmsnorm(x, p[f"{prefix}.attention_norm"], eps)
    q = mm(z, p, f"{prefix}.query")
    k = mm(z, p, f"{prefix}.key")
    v = mm(z, p, f"{prefix}.value")
    q = ops.rope(q, seq, 0, s.heads, theta)
    k = ops.rope(k, seq, 0, s.kv_heads, theta)
    a, _ = ops.grouped_attention(q, k, v, seq, s.heads, s.kv_heads, s.window)
    x = x + mm(a, p, f"{prefix}.attention_output")
    z = ops.rmsnorm(x, p[f"{prefix}.ffn_norm"], eps)
    if s.experts is not None:
        logits = mm(z, p, f"{prefix}.router")
        gates, ids = ops.route_topk(logits, s.experts.top_k)
        if ROUTE_OVERRIDE is not None and prefix in ROUTE_OVERRIDE:
            ids = ROUTE_OVERRIDE[prefix].to(ids.device)
            gates = torch.softmax(logits, dim=1).gather(1, ids.clamp(min=0))
        if c is not None and c.moe_aux_weight > 0:
            choices = (AUX_CHOICES[prefix] if AUX_CHOICES is not None and prefix in AUX_CHOICES
                       else ops.route_topk(logits.detach(), s.experts.top_k)[1])
            AUX_TERMS.append(aux_loss(logits, choices, s.experts.count, c.moe_aux_weight))
        if c is not None and c.moe_capacity_factor > 0 and (ROUTE_OVERRIDE is None or prefix not in ROUTE_OVERRIDE):
            rows, k = ids.shape
            ids = apply_capacity(ids, s.experts.count, max(1, math.ceil(c.moe_capacity_factor * rows * k /
                                                                         s.experts.count)))
        update = torch.zeros_like(z)
        for e in range(s.experts.count):
            rows, slot = torch.nonzero(ids == e, as_tuple=True)
            if rows.numel() == 0:
                continue
            xe = z[rows]
            he = ops.swiglu(mm(xe, p, f"{prefix}.experts.{e}.gate"), mm(xe, p, f"{prefix}.experts.{e}.up"))
            ye = mm(he, p, f"{prefix}.experts.{e}.down")
            update = update.index_add(0, rows, ye * gates[rows, slot][:, None])
    else:
        h = ops.swiglu(mm(z, p, f"{prefix}.gate"), mm(z, p, f"{prefix}.up"))
        update = mm(h, p, f"{prefix}.down")
    return x + update


def _blocks(p, s, x, seq, c):
    for i in range(s.layers):
        x = _block(p, f"{s.prefix}.{i}", s, x, seq, c.rope_theta, c.norm_epsilon, c)
    return x


def hidden(p, c, ids, seq):
    """crates/sejong-model/src/lib.rs:254-277 + architecture.rs:330-393."""
    return hidden_from(p, c, ops.embedding(p["embedding"], ids), seq)


def hidden_from(p, c, x, seq, project=False):
    """The body from its input rows x (architecture.rs:353-393).  `project`: x is an injected input
    of the model width (hidden_from, architecture.rs:360-365), mapped to the encoder width by
    input_projection before the encoder; the byte LM embeds at the encoder width directly."""
    eps = c.norm_epsilon
    h = c.hierarchy
    if h is None:
        x = _blocks(p, global_stage(c), x, seq, c)
        return ops.rmsnorm(x, p["final_norm"], eps)
    if project:
        x = mm(x, p, "input_projection")
    x = _blocks(p, local_stage(c, True), x, seq, c)
    x = ops.rmsnorm(x, p["encoder_norm"], eps)
    pooled = ops.patch_pool(x, seq, h.patch_size)
    z = mm(pooled, p, "encoder_to_global")
    patches = -(-seq // h.patch_size)
    z = _blocks(p, global_stage(c), z, patches, c)
    z = ops.rmsnorm(z, p["global_norm"], eps)
    z = mm(z, p, "global_to_decoder")
    bos = mm(p["global_bos"], p, "global_to_decoder")
    z = ops.patch_broadcast(z, bos, seq, h.patch_size)
    x = mm(x, p, "encoder_to_decoder") + z
    x = _blocks(p, local_stage(c, False), x, seq, c)
    x = ops.rmsnorm(x, p["decoder_norm"], eps)
    x = mm(x, p, "output_projection")
    return ops.rmsnorm(x, p["final_norm"], eps)


def compute_cast(params, cast):
    """The per-step cast of every leaf to the compute precision (crates/sejong-model/src/lib.rs:206-219).

    `cast="bf16"` rounds every matrix (rank > 1) to bfloat16 -- the weights the bf16 compute path
    binds -- and keeps the norm vectors (f32 in the compute path).  The reference's Cast backward
    passes the gradient through unchanged (crates/sejong-gpu/src/graph.rs:807-812), so gradients
    taken at the cast weights are the gradients of the f32 master weights.
    """
    if cast is None:
        return params
    if cast != "bf16":
        raise ValueError(cast)
    out = {}
    for k, v in params.items():
        if np.ndim(v) > 1:
            out[k] = torch.tensor(np.asarray(v, dtype=np.float32)).to(torch.bfloat16).float().numpy()
        else:
            out[k] = v
    return out


def loss_and_grads(params, c, ids, targets, seq, dtype=torch.float64, scale=1.0, cast=None):
    """Mean next-byte CE and its gradients (seed scale/rows per row, graph.rs:539-549), in `dtype`
    arithmetic at the weights `compute_cast(params, cast)`."""
    params = compute_cast(params, cast)
    p = {k: torch.tensor(v, dtype=dtype, requires_grad=True) for k, v in params.items()}
    ids = torch.as_tensor(np.asarray(ids, dtype=np.int64))
    targets = torch.as_tensor(np.asarray(targets, dtype=np.int64))
    AUX_TERMS.clear()
    h = hidden(p, c, ids, seq)
    logits = mm(h, p, "output")
    per_row = ops.cross_entropy(logits, targets)
    loss = per_row.mean()
    for term in AUX_TERMS:
        loss = loss + term
    AUX_TERMS.clear()
    (loss * scale).backward()
    grads = {k: (t.grad.detach().numpy().copy() if t.grad is not None
                 else np.zeros(t.shape, dtype=np.float64 if dtype == torch.float64 else np.float32))
             for k, t in p.items()}
    return float(loss.detach()), grads


def forward_logits(params, c, ids, seq, dtype=torch.float64):
    p = {k: torch.tensor(v, dtype=dtype) for k, v in params.items()}
    ids = torch.as_tensor(np.asarray(ids, dtype=np.int64))
    with torch.no_grad():
        return (hidden(p, c, ids, seq) @ p["output"]).numpy()


@dataclass
class AdamState:
    step: int = 0
    m: dict = field(default_factory=dict)
    v: dict = field(default_factory=dict)


def adam_update(params, grads, state, tc, layout_names=None):
    """Adam::update (crates/sejong-train/src/lib.rs:199-238) in FP64.

    Returns (new params, gradient norm).  lr is taken at the pre-increment step
    (lib.rs:417), bias correction at the post-increment step.
    """
    norm = float(np.sqrt(sum(float(np.sum(np.asarray(g, dtype=np.float64) ** 2)) for g in grads.values())))
    norm /= tc.loss_scale
    clipping = tc.clip_norm / norm if (tc.clip_enabled and norm > tc.clip_norm) else 1.0
    scale = clipping / tc.loss_scale
    lr = ops.lr_schedule(state.step, tc.learning_rate, tc.min_learning_rate, tc.warmup_steps, tc.steps)
    state.step += 1
    out = {}
    for name, w in params.items():
        g = torch.tensor(np.asarray(grads[name], dtype=np.float64))
        m = torch.tensor(state.m.get(name, np.zeros(w.shape)), dtype=torch.float64)
        v = torch.tensor(state.v.get(name, np.zeros(w.shape)), dtype=torch.float64)
        decay = tc.weight_decay if np.ndim(w) > 1 else 0.0
        nw, nm, nv = ops.adamw(torch.tensor(np.asarray(w, dtype=np.float64)), g, m, v, state.step, lr,
                               tc.beta1, tc.beta2, tc.epsilon, decay, scale)
        out[name] = nw.numpy()
        state.m[name] = nm.numpy()
        state.v[name] = nv.numpy()
    return out, norm


# ---- BASELINE.json configurations --------------------------------------------------------

def config_c1():
    """Dense byte Transformer (d256 L4 HQ4/HK2 FFN1024)."""
    return ModelConfig(width=256, layers=4, heads=4, kv_heads=2, ffn_width=1024)


def config_c3():
    """Hierarchical byte model: local d256 x(2+2) H4 W128 FFN768, global d768 L8 HQ12/HK4 FFN2048, P8."""
    return ModelConfig(width=768, layers=8, heads=12, kv_heads=4, ffn_width=2048,
                       hierarchy=HierarchyConfig(8, 256, 2, 4, 768, 256, 2, 4, 768, 128))


def config_c5():
    """Byte MoE: global d1024 L12 HQ16/HK4, 8 experts FFN2816 top-2; local d256 x(2+2)."""
    return ModelConfig(width=1024, layers=12, heads=16, kv_heads=4, ffn_width=2816,
                       experts=ExpertConfig(8, 2, 2816), router_std=0.006,
                       hierarchy=HierarchyConfig(8, 256, 2, 4, 768, 256, 2, 4, 768, 128))


def small_hierarchy(width=128, layers=2, heads=4, kv_heads=2, ffn=256, local=64, local_heads=2,
                    local_ffn=192, patch=8, window=16, experts=None):
    """A reduced hierarchical model for CPU-speed parity tests (same code path as C3)."""
    return ModelConfig(width=width, layers=layers, heads=heads, kv_heads=kv_heads, ffn_width=ffn,
                       experts=experts,
                       hierarchy=HierarchyConfig(patch, local, 1, local_heads, local_ffn, local, 1,
                                                 local_heads, local_ffn, window))


def with_(c, **kw):
    return replace(c, **kw)
