"""KV-cached inference and generation for the byte model.

Restates `Model::forward_cached` / `hidden_cached` (crates/sejong-model/src/lib.rs:362-390,
architecture.rs:395-533, 651-799 dense branch) and the runtime's `generate` / `sample`
(crates/sejong-runtime/src/lib.rs:27-126) on the library's kernels:

  * a cache of K and V rows (bf16) per layer, `context` positions long;
  * a chunk of new tokens at position `length`: embedding, then per block RMSNorm, the QKV GEMM with
    the RoPE epilogue reading the RoPE table from row `length` on, the chunk's K/V rows appended to
    the cache (sj_copy_rows), attention -- the tcgen05 kernel for a prefill (length 0), the cached
    kernel (sj_attn_cached) over every position up to the row otherwise -- and the rest of the block
    as in training; the final norm; the head on the chunk's last row (f32 logits);
  * `generate`: the prompt after EOS, prefilled, then one byte at a time: sample (temperature,
    top-k, top-p with Rng(seed)), stop at EOS or max_bytes; when the cache is full it restarts from
    the last `context` tokens, as the reference does.

`sample` runs on the host with the reference's ordering and f32 arithmetic (numpy float32; the
exponential may differ from the Rust libm by an ulp).
"""
import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import EPI_RESIDUAL, EPI_ROPE, EPI_STORE, EPI_SWIGLU, SJ_BF16, SJ_F32, call
from .model import EOS, HEAD_DIM, VOCAB, VOCAB_PAD, FlatLayout, global_stage, initialize


def _ptr(t, offset_elems=0):
    return t.data_ptr() + offset_elems * t.element_size()


@dataclass
class Sampling:
    """sejong_runtime::Sampling (crates/sejong-runtime/src/lib.rs:9-26)."""
    max_bytes: int = 512
    temperature: float = 0.8
    top_k: int = 0
    top_p: float = 0.95
    seed: int = 42


def _uniform(state):
    """Rng::uniform: ((next_u64 >> 40) + 0.5) / 2^24 in f64, rounded to f32."""
    x = _lib.load().sj_rng_next_u64(ctypes.byref(state))
    return np.float32(((x >> 40) + 0.5) / 16777216.0)


def sample(logits, options, state):
    """sample_prepared (lib.rs:44-78): rank by logit (stable, descending), argmax at temperature 0,
    else top-k, exp((v - max) / T), the top-p prefix, and a draw of Rng::uniform * total."""
    if options.temperature != options.temperature or options.temperature < 0 or not 0 < options.top_p <= 1:
        raise ValueError("sampling requires temperature >= 0 and top_p in (0, 1]")
    x = np.asarray(logits, dtype=np.float32)
    if not np.all(np.isfinite(x)):
        raise ValueError("sampling requires finite logits")
    order = np.argsort(-x, kind="stable")
    if options.temperature == 0:
        return int(order[0])
    if options.top_k > 0:
        order = order[:options.top_k]
    ranked = x[order]
    t = np.float32(options.temperature)
    vals = np.exp((ranked - ranked[0]) / t).astype(np.float32)
    total = np.float32(0)
    for v in vals:
        total = np.float32(total + v)
    cumulative = np.float32(0)
    keep = len(vals)
    for i, v in enumerate(vals):
        cumulative = np.float32(cumulative + v / total)
        if cumulative >= np.float32(options.top_p):
            keep = i + 1
            break
    vals = vals[:keep]
    total = np.float32(0)
    for v in vals:
        total = np.float32(total + v)
    threshold = np.float32(_uniform(state) * total)
    acc = np.float32(0)
    for i, v in enumerate(vals):
        acc = np.float32(acc + v)
        if acc >= threshold:
            return int(order[i])
    return int(order[keep - 1])


class Generator:
    """KV-cached forward of the dense byte model on one GPU.  `forward_cached(tokens)` appends the
    tokens to the cache and returns the f32 logits [257] of the last one; `reset()` empties the
    cache; `generate(prompt, Sampling)` returns (bytes, ended)."""

    def __init__(self, config, params=None, device=None, context=None):
        if config.hierarchy is not None or config.experts is not None:
            raise ValueError("cached inference covers the dense byte model")
        self.c = c = config
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        torch.cuda.set_device(self.dev)
        self.lib = _lib.load()
        call("sj_device_init", self.dev.index)
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        self.context = int(context or c.context)
        self.layout = FlatLayout(c)
        if params is None:
            params = initialize(c, self.lib)
        # the f32 master (norm weights are read in f32, as the training step does) and its bf16 copy
        self.w = torch.from_numpy(self.layout.pack(params)).to(self.dev)
        self.wb = torch.empty(self.layout.total, dtype=torch.bfloat16, device=self.dev)
        call("sj_cast", _ptr(self.w), SJ_F32, _ptr(self.wb), SJ_BF16, self.layout.total, self.stream)
        self.s = s = global_stage(c)
        L, d, f, cq = self.context, s.width, s.ffn, s.qkv_width
        self.kvw = s.kv_heads * HEAD_DIM
        bf, f32 = torch.bfloat16, torch.float32
        e = lambda *shape, dt=bf: torch.empty(*shape, dtype=dt, device=self.dev)  # noqa: E731
        self.k_cache = [e(L, self.kvw) for _ in range(s.layers)]
        self.v_cache = [e(L, self.kvw) for _ in range(s.layers)]
        self.rope = e(L * HEAD_DIM, dt=f32)
        call("sj_rope_table", _ptr(self.rope), L, HEAD_DIM, 0, float(c.rope_theta), self.stream)
        self.ids = torch.zeros(L, dtype=torch.int32, device=self.dev)
        self.x, self.x1 = e(L, d, dt=f32), e(L, d, dt=f32)
        self.z, self.qkv, self.o = e(L, d), e(L, cq), e(L, d)
        self.gu, self.h = e(L, 2 * f), e(L, f)
        self.inv, self.lse = e(L, dt=f32), e(L * s.heads, dt=f32)
        self.logits = e(1, VOCAB_PAD, dt=f32)
        self.length = 0

    def wb_ptr(self, name):
        return _ptr(self.wb, self.layout[name].offset)

    def _gemm(self, a, lda, b, ldb, c, ldc, c_dtype, m, n, k, epi=EPI_STORE, aux=0, ld_aux=0, rope_cols=0, rope_t=0):
        call("sj_gemm", a, lda, 0, b, ldb, 0, c, ldc, c_dtype, m, n, k, epi, 1.0, aux, ld_aux, rope_cols, rope_t,
             float(self.c.rope_theta) if epi == EPI_ROPE else 0.0, 0, self.stream)

    def _norm(self, x, name, rows):
        call("sj_rmsnorm_fwd", _ptr(x), SJ_F32, _ptr(self.w, self.layout[name].offset), _ptr(self.z), _ptr(self.inv),
             rows, self.s.width, float(self.c.norm_epsilon), self.stream)

    def reset(self):
        self.length = 0

    def hidden_cached(self, tokens):
        """Append `tokens` at position `length`; returns the final-norm rows of the chunk (bf16 view)."""
        tokens = np.asarray(tokens, dtype=np.int32).reshape(-1)
        n, off = len(tokens), self.length
        if n == 0 or np.any(tokens < 0) or np.any(tokens > EOS):
            raise ValueError("input tokens must be bytes or EOS")
        if off + n > self.context:
            raise ValueError("KV cache context limit reached")
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        s, c = self.s, self.c
        d, f, cq, kvw = s.width, s.ffn, s.qkv_width, self.kvw
        kq, vq = s.heads * HEAD_DIM, (s.heads + s.kv_heads) * HEAD_DIM
        self.ids[:n].copy_(torch.from_numpy(tokens), non_blocking=False)
        call("sj_embedding_fwd", self.wb_ptr("embedding"), _ptr(self.ids), _ptr(self.x), SJ_F32, n, d, VOCAB,
             self.stream)
        for i in range(s.layers):
            p = f"{s.prefix}.{i}"
            self._norm(self.x, f"{p}.attention_norm", n)
            self._gemm(_ptr(self.z), d, self.wb_ptr(f"{p}.qkv"), cq, _ptr(self.qkv), cq, SJ_BF16, n, cq, d, EPI_ROPE,
                       aux=_ptr(self.rope, off * HEAD_DIM), rope_cols=vq, rope_t=self.context - off)
            for cache, col in ((self.k_cache[i], kq), (self.v_cache[i], vq)):
                call("sj_copy_rows", _ptr(self.qkv, col), cq * 2, _ptr(cache, off * kvw), kvw * 2, n, kvw * 2,
                     self.stream)
            if off == 0:
                call("sj_attn_gqa_fwd", _ptr(self.qkv), cq, _ptr(self.qkv, kq), cq, _ptr(self.qkv, vq), cq,
                     _ptr(self.o), d, _ptr(self.lse), 1, n, s.heads, s.kv_heads, HEAD_DIM, s.window, self.stream)
            else:
                call("sj_attn_cached", _ptr(self.qkv), cq, _ptr(self.k_cache[i]), kvw, _ptr(self.v_cache[i]), kvw,
                     _ptr(self.o), d, n, off, s.heads, s.kv_heads, HEAD_DIM, s.window, self.stream)
            self._gemm(_ptr(self.o), d, self.wb_ptr(f"{p}.attention_output"), d, _ptr(self.x1), d, SJ_F32, n, d, d,
                       EPI_RESIDUAL, aux=_ptr(self.x), ld_aux=d)
            self._norm(self.x1, f"{p}.ffn_norm", n)
            self._gemm(_ptr(self.z), d, self.wb_ptr(f"{p}.gate_up"), 2 * f, _ptr(self.gu), 2 * f, SJ_BF16, n, 2 * f,
                       d, EPI_SWIGLU, aux=_ptr(self.h), ld_aux=f)
            self._gemm(_ptr(self.h), f, self.wb_ptr(f"{p}.down"), d, _ptr(self.x), d, SJ_F32, n, d, f, EPI_RESIDUAL,
                       aux=_ptr(self.x1), ld_aux=d)
        self._norm(self.x, "final_norm", n)
        self.length = off + n
        return self.z[:n]

    def forward_cached(self, tokens):
        """lib.rs:362-372: the chunk, then the head on its last row: f32 logits [257] (device)."""
        h = self.hidden_cached(tokens)
        n, d = h.shape[0], self.s.width
        self._gemm(_ptr(self.z, (n - 1) * d), d, self.wb_ptr("output"), VOCAB_PAD, _ptr(self.logits), VOCAB_PAD, SJ_F32,
                   1, VOCAB, d)
        return self.logits[0, :VOCAB]

    def generate(self, prompt, options=None):
        """sejong_runtime::generate (lib.rs:84-126): returns (bytes, ended)."""
        options = options or Sampling()
        self.reset()
        tokens = [EOS] + list(bytes(prompt))
        if len(tokens) > self.context:
            tokens = tokens[-self.context:]
        logits = self.forward_cached(tokens)
        state = ctypes.c_uint64(int(options.seed) & (2**64 - 1))
        out = []
        for index in range(options.max_bytes):
            token = sample(logits.cpu().numpy(), options, state)
            if token == EOS:
                return bytes(out), True
            out.append(token)
            tokens.append(token)
            if index + 1 < options.max_bytes:
                if self.length == self.context:
                    self.reset()
                    tokens = tokens[-self.context:]
                    logits = self.forward_cached(tokens)
                else:
                    logits = self.forward_cached([token])
        return bytes(out), False
