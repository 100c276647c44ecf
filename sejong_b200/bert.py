"""MiniLM-shaped BERT encoder forward on the B200 kernels.

Restates `BertEncoder::hidden` (crates/sejong-model/src/native/bert.rs:360-411), the frozen text
encoder of the reference's native models: embeddings (word + position + token type 0) and
LayerNorm, then per layer (post-LN)
    q, k, v = x Wq^T + bq, x Wk^T + bk, x Wv^T + bv      (one GEMM over the fused [Wq; Wk; Wv])
    a = attention(q, k, v) (non-causal, 12 heads of 32)
    x = LayerNorm(x + a Wo^T + bo)
    x = LayerNorm(x + gelu(x W1^T + b1) W2^T + b2)
with LayerNorm eps 1e-12 and erf GELU.  The reference encodes one sequence at a time, unpadded; here
a batch of sequences is packed row after row (cu_seqlens), which gives the same arithmetic per
sequence and lets every launch cover the whole batch.  Weights are the reference's parameter names
(the HuggingFace BERT layout `bert.rs` reads).  Activations and GEMM operands are bf16 with f32
accumulation; the residual stream, LayerNorm statistics and the output are f32.
"""
import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL, SJ_BF16, SJ_F32, call

CLS, SEP = 101, 102


@dataclass
class MiniLMConfig:
    """BertConfig fields bert.rs uses; defaults are BASELINE C2 (MiniLM-L6 shape)."""
    vocab: int = 30522
    hidden: int = 384
    layers: int = 6
    heads: int = 12
    ffn: int = 1536
    max_position: int = 512
    type_vocab: int = 2
    layer_norm_eps: float = 1e-12
    seed: int = 2024
    init_std: float = 0.02


def bert_layout(c):
    """(name, shape, kind) in parameter order; kind: "matrix", "bias", "ln_weight", "ln_bias"."""
    d, f = c.hidden, c.ffn
    out = [("embeddings.word_embeddings.weight", (c.vocab, d), "matrix"),
           ("embeddings.position_embeddings.weight", (c.max_position, d), "matrix"),
           ("embeddings.token_type_embeddings.weight", (c.type_vocab, d), "matrix"),
           ("embeddings.LayerNorm.weight", (d,), "ln_weight"),
           ("embeddings.LayerNorm.bias", (d,), "ln_bias")]
    for i in range(c.layers):
        p = f"encoder.layer.{i}"
        for name in ("query", "key", "value"):
            out.append((f"{p}.attention.self.{name}.weight", (d, d), "matrix"))
            out.append((f"{p}.attention.self.{name}.bias", (d,), "bias"))
        out += [(f"{p}.attention.output.dense.weight", (d, d), "matrix"),
                (f"{p}.attention.output.dense.bias", (d,), "bias"),
                (f"{p}.attention.output.LayerNorm.weight", (d,), "ln_weight"),
                (f"{p}.attention.output.LayerNorm.bias", (d,), "ln_bias"),
                (f"{p}.intermediate.dense.weight", (f, d), "matrix"),
                (f"{p}.intermediate.dense.bias", (f,), "bias"),
                (f"{p}.output.dense.weight", (d, f), "matrix"),
                (f"{p}.output.dense.bias", (d,), "bias"),
                (f"{p}.output.LayerNorm.weight", (d,), "ln_weight"),
                (f"{p}.output.LayerNorm.bias", (d,), "ln_bias")]
    return out


def initialize(c, lib=None):
    """Random weights as BASELINE C2 specifies: every matrix N(0, init_std) drawn with the reference
    Rng (Rng::normal, one per element, in layout order from Rng(seed)), biases 0, LayerNorm weight 1
    and bias 0."""
    lib = lib or _lib.load()
    state = ctypes.c_uint64(c.seed)
    params = {}
    for name, shape, kind in bert_layout(c):
        if kind == "matrix":
            buf = np.empty(int(np.prod(shape)), dtype=np.float32)
            call("sj_rng_normal_fill", ctypes.byref(state), buf.ctypes.data, buf.size, float(c.init_std))
            params[name] = buf.reshape(shape)
        else:
            params[name] = (np.ones if kind == "ln_weight" else np.zeros)(shape, dtype=np.float32)
    return params


def synthetic_batch(seed, batch, max_len=128, min_len=16, vocab=30522):
    """BASELINE C2 inputs: per row a length uniform in [min_len, max_len], [CLS] first, [SEP] last,
    the rest uniform in [1000, vocab); drawn with the reference Rng (Rng::index) from Rng(seed).
    Returns (list of int32 arrays, one per sequence)."""
    lib = _lib.load()
    state = ctypes.c_uint64(seed)
    seqs = []
    for _ in range(batch):
        n = min_len + int(lib.sj_rng_index(ctypes.byref(state), max_len - min_len + 1))
        body = [1000 + int(lib.sj_rng_index(ctypes.byref(state), vocab - 1000)) for _ in range(n - 2)]
        seqs.append(np.array([CLS] + body + [SEP], dtype=np.int32))
    return seqs


def pack(seqs):
    """Packed ids [rows] and cu_seqlens [batch + 1] (int32) of a list of sequences."""
    lens = np.array([len(s) for s in seqs], dtype=np.int64)
    cu = np.zeros(len(seqs) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    return np.concatenate(seqs).astype(np.int32), cu


def _ptr(t, offset=0):
    return t.data_ptr() + offset * t.element_size()


class MiniLM:
    """The encoder on one GPU.  `forward(ids, cu_seqlens)` returns the f32 hidden states
    [rows, hidden] of every packed row (BertEncoder::hidden for each sequence)."""

    KERNELS_PER_LAYER = 7   # QKV GEMM, attention, Wo GEMM, LayerNorm, W1 GEMM, W2 GEMM, LayerNorm

    def __init__(self, config, params=None, device=None):
        self.c = c = config
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        torch.cuda.set_device(self.dev)
        self.lib = _lib.load()
        call("sj_device_init", self.dev.index)
        if params is None:
            params = initialize(c, self.lib)
        f32, bf = torch.float32, torch.bfloat16

        def dev(a, dt=f32):
            return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(self.dev, dt)
        self.word = dev(params["embeddings.word_embeddings.weight"])
        self.position = dev(params["embeddings.position_embeddings.weight"])
        self.type0 = dev(params["embeddings.token_type_embeddings.weight"][0])
        self.ln_e = (dev(params["embeddings.LayerNorm.weight"]), dev(params["embeddings.LayerNorm.bias"]))
        self.layers = []
        for i in range(c.layers):
            p = f"encoder.layer.{i}"
            qkv_w = np.concatenate([params[f"{p}.attention.self.{n}.weight"] for n in ("query", "key", "value")])
            qkv_b = np.concatenate([params[f"{p}.attention.self.{n}.bias"] for n in ("query", "key", "value")])
            self.layers.append({
                "wqkv": dev(qkv_w, bf), "bqkv": dev(qkv_b),
                "wo": dev(params[f"{p}.attention.output.dense.weight"], bf),
                "bo": dev(params[f"{p}.attention.output.dense.bias"]),
                "ln1": (dev(params[f"{p}.attention.output.LayerNorm.weight"]),
                        dev(params[f"{p}.attention.output.LayerNorm.bias"])),
                "w1": dev(params[f"{p}.intermediate.dense.weight"], bf),
                "b1": dev(params[f"{p}.intermediate.dense.bias"]),
                "w2": dev(params[f"{p}.output.dense.weight"], bf),
                "b2": dev(params[f"{p}.output.dense.bias"]),
                "ln2": (dev(params[f"{p}.output.LayerNorm.weight"]), dev(params[f"{p}.output.LayerNorm.bias"])),
            })
        self.capacity = 0
        self.launches = 0
        self._call = call  # every kernel launch goes through here (a profiler may wrap it)

    def _buffers(self, rows):
        if rows <= self.capacity:
            return
        d, f = self.c.hidden, self.c.ffn
        e = lambda *s, dt=torch.bfloat16: torch.empty(*s, dtype=dt, device=self.dev)  # noqa: E731
        self.x = e(rows, d, dt=torch.float32)
        self.xb = e(rows, d)
        self.sum = e(rows, d, dt=torch.float32)
        self.qkv = e(rows, 3 * d)
        self.ctx = e(rows, d)
        self.h = e(rows, f)
        self.capacity = rows

    def _gemm(self, a, w, out, out_dtype, m, n, k, epi, bias, aux=None, stream=None):
        """out[m, n] = epi(a[m, k] w[n, k]^T + bias) (w is the reference's [out, in] weight)."""
        self._call("sj_gemm_bias", _ptr(a), k, 0, _ptr(w), k, 1, _ptr(out), n, out_dtype, m, n, k, epi, 1.0, _ptr(bias),
             _ptr(aux) if aux is not None else 0, n if aux is not None else 0, stream)
        self.launches += 1

    def reserve(self, rows):
        """Allocate activation buffers for up to `rows` packed rows (before capturing a graph)."""
        self._buffers(rows)

    def forward(self, ids, cu_seqlens, max_len=None, stream=None):
        """ids int32 [rows] and cu_seqlens int32 [batch + 1], device tensors; returns x f32 [rows, d]
        (a view of an internal buffer, valid until the next call)."""
        c = self.c
        d, f = c.hidden, c.ffn
        rows = int(ids.shape[0])
        batch = int(cu_seqlens.shape[0]) - 1
        max_len = max_len or 128
        self._buffers(rows)
        s = stream if stream is not None else torch.cuda.current_stream(self.dev).cuda_stream
        eps = float(c.layer_norm_eps)
        self._call("sj_bert_embed", _ptr(ids), _ptr(cu_seqlens), batch, _ptr(self.word), c.vocab, _ptr(self.position),
             c.max_position, _ptr(self.type0), _ptr(self.ln_e[0]), _ptr(self.ln_e[1]), eps, _ptr(self.x),
             _ptr(self.xb), rows, d, s)
        self.launches += 1
        for L in self.layers:
            self._gemm(self.xb, L["wqkv"], self.qkv, SJ_BF16, rows, 3 * d, d, EPI_BIAS, L["bqkv"], stream=s)
            self._call("sj_bert_attention", _ptr(self.qkv), 3 * d, _ptr(cu_seqlens), batch, max_len, c.heads,
                 d // c.heads, _ptr(self.ctx), d, s)
            self._gemm(self.ctx, L["wo"], self.sum, SJ_F32, rows, d, d, EPI_BIAS_RESIDUAL, L["bo"], aux=self.x,
                       stream=s)
            self._call("sj_layernorm", _ptr(self.sum), _ptr(L["ln1"][0]), _ptr(L["ln1"][1]), eps, _ptr(self.x),
                 _ptr(self.xb), rows, d, s)
            self._gemm(self.xb, L["w1"], self.h, SJ_BF16, rows, f, d, EPI_BIAS_GELU, L["b1"], stream=s)
            self._gemm(self.h, L["w2"], self.sum, SJ_F32, rows, d, f, EPI_BIAS_RESIDUAL, L["b2"], aux=self.x,
                       stream=s)
            self._call("sj_layernorm", _ptr(self.sum), _ptr(L["ln2"][0]), _ptr(L["ln2"][1]), eps, _ptr(self.x),
                 _ptr(self.xb), rows, d, s)
            self.launches += 3
        return self.x[:rows]

    def flops(self, cu_seqlens):
        """Algorithmic FLOPs of one forward over valid tokens only: 2 rows params for every linear
        layer, 4 len^2 hidden for attention scores and values per sequence."""
        c = self.c
        lens = np.diff(np.asarray(cu_seqlens, dtype=np.int64))
        rows = int(lens.sum())
        per_layer = 2 * rows * (4 * c.hidden * c.hidden + 2 * c.hidden * c.ffn)
        attn = 4 * int((lens * lens).sum()) * c.hidden
        return c.layers * (per_layer + attn)
