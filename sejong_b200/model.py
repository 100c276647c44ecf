"""Model configuration, parameter layout and the flat GEMM-ready parameter store.

Configuration fields mirror sejong_core::ModelConfig / HierarchyConfig / ExpertConfig
(crates/sejong-core/src/lib.rs:60-118).  `reference_layout` lists the reference's
parameters in its order and with its names and shapes (crates/sejong-model/src/
architecture.rs:63-137); initialisation draws them in that order from the
reference Rng (crates/sejong-model/src/lib.rs:82-116).

On the device the parameters live in ONE flat f32 buffer (master weights, and
the same layout for gradients and Adam moments) plus one flat bf16 copy that the
GEMMs read.  Within it each transformer block's Q/K/V matrices are concatenated
column-wise into `qkv` [d, (hq+2hk)*64] and gate/up are interleaved in blocks of
16 columns into `gate_up` [d, 2F] (the SwiGLU epilogue of sj_gemm then sees the
gate and up value of one feature in the same thread).  The output head is padded
from 257 to 264 columns so its row stride meets TMA's 16-byte rule.  Tensors with
rank > 1 (decoupled weight decay, crates/sejong-train/src/lib.rs:228-236) come
first, norm weights last, every tensor 64-element aligned.  `pack`/`unpack` map
between reference-named arrays and the flat layout.
"""
from dataclasses import dataclass, replace
from typing import Optional

import numpy as np

VOCAB = 257
EOS = 256
VOCAB_PAD = 264
HEAD_DIM = 64
ALIGN = 64
INTERLEAVE = 16


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
    init_std: float = 0.02      # 0 selects the reference's fan-in rule (crates/sejong-model/src/lib.rs:82-116)
    router_std: float = 0.02


@dataclass
class Stage:
    prefix: str
    width: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    window: int          # 0 = full causal
    experts: Optional[ExpertConfig] = None

    @property
    def qkv_width(self):
        return (self.heads + 2 * self.kv_heads) * HEAD_DIM


def global_stage(c):
    return Stage("layers", c.width, c.layers, c.heads, c.kv_heads or c.heads, c.ffn_width, 0, c.experts)


def local_stage(c, encoder):
    h = c.hierarchy
    if encoder:
        return Stage("encoder", h.encoder_width, h.encoder_layers, h.encoder_heads, h.encoder_heads,
                     h.encoder_ffn_width, h.local_window)
    return Stage("decoder", h.decoder_width, h.decoder_layers, h.decoder_heads, h.decoder_heads,
                 h.decoder_ffn_width, h.local_window)


def stages(c):
    if c.hierarchy is None:
        return [global_stage(c)]
    return [local_stage(c, True), global_stage(c), local_stage(c, False)]


def _stage_layout(s, out):
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
                out.append((f"{p}.experts.{e}.gate", (d, s.experts.ffn_width), False))
                out.append((f"{p}.experts.{e}.up", (d, s.experts.ffn_width), False))
                out.append((f"{p}.experts.{e}.down", (s.experts.ffn_width, d), False))
            out.append((f"{p}.router", (d, s.experts.count), False))
        else:
            out.append((f"{p}.gate", (d, s.ffn), False))
            out.append((f"{p}.up", (d, s.ffn), False))
            out.append((f"{p}.down", (s.ffn, d), False))


def reference_layout(c):
    """(name, shape, is_norm) in the reference's parameter order (architecture.rs:93-137)."""
    h = c.hierarchy
    out = [("embedding", (VOCAB, h.encoder_width if h else c.width), False)]
    if h is not None:
        _stage_layout(local_stage(c, True), out)
        out.append(("encoder_norm", (h.encoder_width,), True))
        out.append(("input_projection", (c.width, h.encoder_width), False))
        out.append(("encoder_to_global", (h.encoder_width, c.width), False))
        out.append(("encoder_to_decoder", (h.encoder_width, h.decoder_width), False))
        out.append(("global_to_decoder", (c.width, h.decoder_width), False))
        out.append(("global_bos", (1, c.width), False))
        out.append(("global_norm", (c.width,), True))
        _stage_layout(global_stage(c), out)
        _stage_layout(local_stage(c, False), out)
        out.append(("decoder_norm", (h.decoder_width,), True))
        out.append(("output_projection", (h.decoder_width, c.width), False))
    else:
        _stage_layout(global_stage(c), out)
    out.append(("final_norm", (c.width,), True))
    out.append(("output", (c.width, VOCAB), False))
    return out


def parameter_count(c):
    return sum(int(np.prod(s)) for _, s, _ in reference_layout(c))


# ---------------------------------------------------------------- flat fused layout
@dataclass
class Entry:
    name: str            # fused name
    shape: tuple         # fused shape (row-major)
    offset: int          # element offset in the flat buffers
    decay: bool
    parts: tuple         # reference names packed into this entry

    @property
    def size(self):
        return int(np.prod(self.shape))


def _interleave_cols(gate, up):
    """[d, F] x2 -> [d, 2F]: column blocks of 16 gate features then the same 16 up features."""
    d, f = gate.shape
    g = gate.reshape(d, f // INTERLEAVE, INTERLEAVE)
    u = up.reshape(d, f // INTERLEAVE, INTERLEAVE)
    return np.concatenate([g, u], axis=2).reshape(d, 2 * f)


def _deinterleave_cols(gu):
    d, f2 = gu.shape
    x = gu.reshape(d, f2 // (2 * INTERLEAVE), 2, INTERLEAVE)
    return x[:, :, 0, :].reshape(d, f2 // 2), x[:, :, 1, :].reshape(d, f2 // 2)


def router_pad(experts):
    """Columns of a router weight in the flat buffers: the expert count rounded up to 8."""
    return (experts + 7) // 8 * 8


NATIVE_VOCAB = 259          # 256 bytes, PAD 256, BOS 257, SEP 258 (value.rs:15-17)
NATIVE_PAD, NATIVE_BOS, NATIVE_SEP = 256, 257, 258


def value_layout(c, values):
    """(name, shape, is_norm) of NativeValue's own parameters (value.rs:84-106, 53-67)."""
    return [("native_embedding", (NATIVE_VOCAB, c.width), False),
            ("native_value", (c.width, values), False),
            ("native_bias", (1, values), False)]


class FlatLayout:
    """Placement of every (fused) parameter in the flat master / gradient / moment buffers.

    With `expert_shard=(rank, world)` (expert parallelism) the layout holds only this rank's experts
    of every MoE layer, experts [rank * E/world, (rank + 1) * E/world), and places them first:
    [0, shared_begin) is rank-local, [shared_begin, total) is replicated on every rank (the range
    the data-parallel all-reduce covers).  Without it shared_begin is 0."""

    def __init__(self, c, expert_shard=None, values=0):
        self.config = c
        self.expert_shard = expert_shard
        self.values = values
        ref = reference_layout(c)
        if values:
            # NativeValue (crates/sejong-model/src/native/value.rs:84-106): the body without its byte
            # embedding and output head, plus the 259-row native embedding and the f32 value head
            ref = [r for r in ref if r[0] not in ("embedding", "output")] + value_layout(c, values)
        shapes = {n: s for n, s, _ in ref}
        entries = []
        fused_done = set()
        for name, shape, norm in ref:
            if name in fused_done:
                continue
            if name.endswith(".query"):
                p = name[: -len(".query")]
                d = shape[0]
                kv = shapes[f"{p}.key"][1]
                entries.append((f"{p}.qkv", (d, shape[1] + 2 * kv), True,
                                (f"{p}.query", f"{p}.key", f"{p}.value")))
                fused_done.update({f"{p}.key", f"{p}.value"})
            elif name.endswith(".gate"):
                p = name[: -len(".gate")]
                d, f = shape
                entries.append((f"{p}.gate_up", (d, 2 * f), True, (f"{p}.gate", f"{p}.up")))
                fused_done.add(f"{p}.up")
            elif name == "output":
                entries.append(("output", (shape[0], VOCAB_PAD), True, ("output",)))
            elif name.endswith(".router"):  # columns padded to 8 (16-byte rows for TMA), padding zero
                entries.append((name, (shape[0], router_pad(shape[1])), True, (name,)))
            else:
                entries.append((name, shape, (not norm) and len(shape) > 1, (name,)))
        # the experts of an MoE layer: all fused gate/up matrices, then all down matrices, each run
        # contiguous, so that a grouped GEMM reads expert g's matrix as the g-th block of one stack
        grouped = []
        i = 0
        while i < len(entries):
            if ".experts." not in entries[i][0]:
                grouped.append(entries[i])
                i += 1
                continue
            layer = entries[i][0].split(".experts.")[0]
            j = i
            while j < len(entries) and entries[j][0].startswith(layer + ".experts."):
                j += 1
            run = entries[i:j]
            grouped += [e for e in run if e[0].endswith(".gate_up")] + [e for e in run if e[0].endswith(".down")]
            i = j
        entries = grouped
        experts_first = []
        if expert_shard is not None:
            rank, world = expert_shard
            count = c.experts.count if c.experts is not None else 0
            if count == 0 or count % world or not 0 <= rank < world:
                raise ValueError(f"expert shard {expert_shard} of {count} experts")
            local = range(rank * count // world, (rank + 1) * count // world)
            mine = {f".experts.{x}." for x in local}
            experts_first = [e for e in entries if ".experts." in e[0] and any(m in e[0] for m in mine)]
            entries = [e for e in entries if ".experts." not in e[0]]
        ordered = experts_first + [e for e in entries if e[2]] + [e for e in entries if not e[2]]
        self.entries = {}
        off = 0
        self.n_decay = 0
        self.shared_begin = 0
        for i, (name, shape, decay, parts) in enumerate(ordered):
            self.entries[name] = Entry(name, tuple(shape), off, decay, parts)
            off += int(np.prod(shape))
            off = (off + ALIGN - 1) // ALIGN * ALIGN
            if decay:
                self.n_decay = off
            if i + 1 == len(experts_first):
                self.shared_begin = off
        self.total = off

    def __getitem__(self, name):
        return self.entries[name]

    def pack(self, params):
        """Reference-named f32 arrays -> flat f32 array."""
        flat = np.zeros(self.total, dtype=np.float32)
        for e in self.entries.values():
            if e.name.endswith(".qkv"):
                v = np.concatenate([params[p] for p in e.parts], axis=1)
            elif e.name.endswith(".gate_up"):
                v = _interleave_cols(params[e.parts[0]], params[e.parts[1]])
            elif e.name == "output":
                v = np.zeros(e.shape, dtype=np.float32)
                v[:, :VOCAB] = params["output"]
            elif e.name.endswith(".router"):
                v = np.zeros(e.shape, dtype=np.float32)
                v[:, :params[e.name].shape[1]] = params[e.name]
            else:
                v = params[e.name]
            flat[e.offset:e.offset + e.size] = np.asarray(v, dtype=np.float32).reshape(-1)
        return flat

    def unpack(self, flat):
        """Flat array -> dict of reference-named arrays (same dtype as `flat`)."""
        flat = np.asarray(flat)
        out = {}
        ref_shapes = {n: s for n, s, _ in reference_layout(self.config)}
        for e in self.entries.values():
            v = flat[e.offset:e.offset + e.size].reshape(e.shape)
            if e.name.endswith(".qkv"):
                q, k, _ = e.parts
                wq, wk = ref_shapes[q][1], ref_shapes[k][1]
                out[e.parts[0]] = v[:, :wq].copy()
                out[e.parts[1]] = v[:, wq:wq + wk].copy()
                out[e.parts[2]] = v[:, wq + wk:].copy()
            elif e.name.endswith(".gate_up"):
                g, u = _deinterleave_cols(v)
                out[e.parts[0]] = g.copy()
                out[e.parts[1]] = u.copy()
            elif e.name == "output":
                out["output"] = v[:, :VOCAB].copy()
            elif e.name.endswith(".router"):
                out[e.name] = v[:, :ref_shapes[e.name][1]].copy()
            else:
                out[e.name] = v.copy()
        return out


def initialize(c, lib=None):
    """Reference-named f32 master weights drawn from Rng(c.seed) in reference layout order.

    Every non-norm element consumes one Rng::normal; init_std > 0 gives N(0, init_std)
    (router N(0, router_std)), init_std == 0 the reference's fan-in rule with global_bos = 0
    (crates/sejong-model/src/lib.rs:82-116).  The draws run in the library's C Rng.
    """
    import ctypes

    from . import _lib
    lib = lib or _lib.load()
    state = ctypes.c_uint64(c.seed)
    params = {}
    for name, shape, norm in reference_layout(c):
        n = int(np.prod(shape))
        if norm:
            params[name] = np.ones(shape, dtype=np.float32)
            continue
        if c.init_std > 0:
            std = c.router_std if name.endswith(".router") else c.init_std
        else:
            if name == "global_bos":
                params[name] = np.zeros(shape, dtype=np.float32)
                continue
            std = np.float32(1.0) / np.sqrt(np.float32(shape[1] if name == "embedding" else shape[0]))
            depth = c.layers
            if c.hierarchy is not None:
                if name.startswith("encoder."):
                    depth = c.hierarchy.encoder_layers
                elif name.startswith("decoder."):
                    depth = c.hierarchy.decoder_layers
            if name.endswith(".down") or name.endswith(".attention_output"):
                std = std / np.sqrt(np.float32(2.0 * depth))
        buf = np.empty(n, dtype=np.float32)
        _lib.call("sj_rng_normal_fill", ctypes.byref(state), buf.ctypes.data, n, float(std))
        params[name] = buf.reshape(shape)
    return params


# ---------------------------------------------------------------- BASELINE.json configurations
def config_c1():
    """Dense byte Transformer: d256, 4 layers, HQ4/HK2, SwiGLU 1024, eps 1e-6, RoPE 1e4."""
    return ModelConfig(width=256, layers=4, heads=4, kv_heads=2, ffn_width=1024)


def config_c3():
    """Hierarchical byte model: local d256 (2 enc + 2 dec layers, 4 heads, window 128, FFN 768),
    global d768 x 8 layers, HQ12/HK4, SwiGLU 2048, patch 8."""
    return ModelConfig(width=768, layers=8, heads=12, kv_heads=4, ffn_width=2048,
                       hierarchy=HierarchyConfig(8, 256, 2, 4, 768, 256, 2, 4, 768, 128))


def config_c5():
    """Byte MoE: global d1024 x 12, HQ16/HK4, 8 SwiGLU experts of 2816, top-2; local as C3."""
    return ModelConfig(width=1024, layers=12, heads=16, kv_heads=4, ffn_width=2816,
                       experts=ExpertConfig(8, 2, 2816), router_std=0.006,
                       hierarchy=HierarchyConfig(8, 256, 2, 4, 768, 256, 2, 4, 768, 128))


def small_hierarchy(width=256, layers=2, heads=4, kv_heads=2, ffn=512, local=128, local_heads=2,
                    local_ffn=384, patch=8, window=32):
    """Reduced hierarchical model (same code path as C3) for quick parity checks."""
    return ModelConfig(width=width, layers=layers, heads=heads, kv_heads=kv_heads, ffn_width=ffn,
                       hierarchy=HierarchyConfig(patch, local, 1, local_heads, local_ffn, local, 1,
                                                 local_heads, local_ffn, window))


def with_(c, **kw):
    return replace(c, **kw)
