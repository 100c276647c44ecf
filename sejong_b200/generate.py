"""KV-cached inference and generation for the byte model.

Restates `Model::forward_cached` / `hidden_cached` (crates/sejong-model/src/lib.rs:362-390,
architecture.rs:395-799, dense and hierarchical) and the runtime's `generate` / `sample`
(crates/sejong-runtime/src/lib.rs:27-126) on the library's kernels:

  * a cache of K and V rows (bf16) per layer, `context` positions long;
  * a chunk of new tokens at position `length`: embedding, then per block RMSNorm, the QKV GEMM with
    the RoPE epilogue reading the RoPE table from row `length` on, the chunk's K/V rows appended to
    the cache (sj_copy_rows), attention -- the tcgen05 kernel for a prefill (length 0), the cached
    kernel (sj_attn_cached) over every position up to the row otherwise -- and the rest of the block
    as in training; the final norm; the head on the chunk's last row (f32 logits);
  * the hierarchical model: a prefill runs encoder, global stage over the (partial) patches and
    decoder as in training and keeps the patch state -- the global context of the last completed
    patch (or the BOS projection), the running f32 sum of the encoded bytes of the open patch;
    afterwards bytes go through encoder and decoder (with the current global context added to
    every row) and, when a patch completes, its mean goes through the global stage at the patch's
    position and yields the next global context (architecture.rs:534-779);
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
from .model import EOS, HEAD_DIM, VOCAB, VOCAB_PAD, FlatLayout, global_stage, initialize, local_stage


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


class _Stage:
    """K/V caches, RoPE table and working buffers of one stage (encoder, global or decoder) for chunks
    of up to `rows` rows."""

    def __init__(self, stage, capacity, rows, dev, theta, stream):
        self.s = stage
        d, f, cq = stage.width, stage.ffn, stage.qkv_width
        self.kvw = stage.kv_heads * HEAD_DIM
        bf, f32 = torch.bfloat16, torch.float32
        e = lambda *shape, dt=bf: torch.empty(*shape, dtype=dt, device=dev)  # noqa: E731
        self.capacity = capacity
        self.k = [e(capacity, self.kvw) for _ in range(stage.layers)]
        self.v = [e(capacity, self.kvw) for _ in range(stage.layers)]
        self.rope = e(capacity * HEAD_DIM, dt=f32)
        call("sj_rope_table", _ptr(self.rope), capacity, HEAD_DIM, 0, float(theta), stream)
        self.x, self.x1 = e(rows, d, dt=f32), e(rows, d, dt=f32)
        self.z, self.qkv, self.o = e(rows, d), e(rows, cq), e(rows, d)
        self.gu, self.h = e(rows, 2 * f), e(rows, f)
        self.inv, self.lse = e(rows, dt=f32), e(rows * stage.heads, dt=f32)


class Generator:
    """KV-cached forward of the byte model (dense or hierarchical) on one GPU.  `forward_cached(tokens)`
    appends the tokens and returns the f32 logits [257] of the last one; `hidden_cached(tokens)`
    returns the final-norm rows of the chunk; `reset()` empties the cache; `generate(prompt,
    Sampling)` returns (bytes, ended)."""

    def __init__(self, config, params=None, device=None, context=None):
        if config.experts is not None:
            raise ValueError("cached inference covers the dense and hierarchical byte models without experts")
        self.c = c = config
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        torch.cuda.set_device(self.dev)
        self.lib = _lib.load()
        call("sj_device_init", self.dev.index)
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        self.context = L = int(context or c.context)
        self.layout = FlatLayout(c)
        if params is None:
            params = initialize(c, self.lib)
        # the f32 master (norm weights are read in f32, as the training step does) and its bf16 copy
        self.w = torch.from_numpy(self.layout.pack(params)).to(self.dev)
        self.wb = torch.empty(self.layout.total, dtype=torch.bfloat16, device=self.dev)
        call("sj_cast", _ptr(self.w), SJ_F32, _ptr(self.wb), SJ_BF16, self.layout.total, self.stream)
        bf, f32 = torch.bfloat16, torch.float32
        e = lambda *shape, dt=bf: torch.empty(*shape, dtype=dt, device=self.dev)  # noqa: E731
        self.ids = torch.zeros(L, dtype=torch.int32, device=self.dev)
        self.h = h = c.hierarchy
        if h is None:
            self.glob = _Stage(global_stage(c), L, L, self.dev, c.rope_theta, self.stream)
        else:
            P = h.patch_size
            self.patches_cap = -(-L // P)
            self.enc = _Stage(local_stage(c, True), L, L, self.dev, c.rope_theta, self.stream)
            self.glob = _Stage(global_stage(c), self.patches_cap, self.patches_cap, self.dev, c.rope_theta, self.stream)
            self.dec = _Stage(local_stage(c, False), L, L, self.dev, c.rope_theta, self.stream)
            de, dg, dd = h.encoder_width, c.width, h.decoder_width
            self.zE = e(L, de)                       # encoded bytes (encoder norm output)
            self.pooled = e(self.patches_cap, de)
            self.zd = e(self.patches_cap, dd)        # global contexts (global_to_decoder of each patch)
            self.bos = e(1, dd)
            self.gctx = e(1, dd)                     # the global context of the current patch
            self.patch_sum = e(de, dt=f32)
            self.y = e(L, dg, dt=f32)
            self.final = e(L, dg)
            self.patch_count = 0
            self.have_ctx = False
        self.logits = e(1, VOCAB_PAD, dt=f32)
        self.length = 0

    def wb_ptr(self, name):
        return _ptr(self.wb, self.layout[name].offset)

    def _gemm(self, a, lda, b, ldb, c, ldc, c_dtype, m, n, k, epi=EPI_STORE, aux=0, ld_aux=0, rope_cols=0, rope_t=0):
        call("sj_gemm", a, lda, 0, b, ldb, 0, c, ldc, c_dtype, m, n, k, epi, 1.0, aux, ld_aux, rope_cols, rope_t,
             float(self.c.rope_theta) if epi == EPI_ROPE else 0.0, 0, self.stream)

    def _norm(self, x, name, y, inv, rows, d):
        """y (a tensor or a device address) = RMSNorm(x) with the f32 norm weight `name`."""
        y = y if isinstance(y, int) else _ptr(y)
        call("sj_rmsnorm_fwd", _ptr(x), SJ_F32, _ptr(self.w, self.layout[name].offset), y, _ptr(inv), rows, d,
             float(self.c.norm_epsilon), self.stream)

    def reset(self):
        """HierarchyCache::reset and an empty cache (architecture.rs:406-412)."""
        self.length = 0
        if self.h is not None:
            self.patch_count = 0
            self.have_ctx = False

    def _blocks(self, st, n, offset):
        """cached_blocks (architecture.rs:474-533) on st.x [n, d] (f32, in place) at position `offset`."""
        s = st.s
        d, f, cq, kvw = s.width, s.ffn, s.qkv_width, st.kvw
        kq, vq = s.heads * HEAD_DIM, (s.heads + s.kv_heads) * HEAD_DIM
        if offset + n > st.capacity:
            raise ValueError("KV cache context limit reached")
        for i in range(s.layers):
            p = f"{s.prefix}.{i}"
            self._norm(st.x, f"{p}.attention_norm", st.z, st.inv, n, d)
            self._gemm(_ptr(st.z), d, self.wb_ptr(f"{p}.qkv"), cq, _ptr(st.qkv), cq, SJ_BF16, n, cq, d, EPI_ROPE,
                       aux=_ptr(st.rope, offset * HEAD_DIM), rope_cols=vq, rope_t=st.capacity - offset)
            for cache, col in ((st.k[i], kq), (st.v[i], vq)):
                call("sj_copy_rows", _ptr(st.qkv, col), cq * 2, _ptr(cache, offset * kvw), kvw * 2, n, kvw * 2,
                     self.stream)
            if offset == 0:
                call("sj_attn_gqa_fwd", _ptr(st.qkv), cq, _ptr(st.qkv, kq), cq, _ptr(st.qkv, vq), cq, _ptr(st.o), d,
                     _ptr(st.lse), 1, n, s.heads, s.kv_heads, HEAD_DIM, s.window, self.stream)
            else:
                call("sj_attn_cached", _ptr(st.qkv), cq, _ptr(st.k[i]), kvw, _ptr(st.v[i]), kvw, _ptr(st.o), d, n,
                     offset, s.heads, s.kv_heads, HEAD_DIM, s.window, self.stream)
            self._gemm(_ptr(st.o), d, self.wb_ptr(f"{p}.attention_output"), d, _ptr(st.x1), d, SJ_F32, n, d, d,
                       EPI_RESIDUAL, aux=_ptr(st.x), ld_aux=d)
            self._norm(st.x1, f"{p}.ffn_norm", st.z, st.inv, n, d)
            self._gemm(_ptr(st.z), d, self.wb_ptr(f"{p}.gate_up"), 2 * f, _ptr(st.gu), 2 * f, SJ_BF16, n, 2 * f, d,
                       EPI_SWIGLU, aux=_ptr(st.h), ld_aux=f)
            self._gemm(_ptr(st.h), f, self.wb_ptr(f"{p}.down"), d, _ptr(st.x), d, SJ_F32, n, d, f, EPI_RESIDUAL,
                       aux=_ptr(st.x1), ld_aux=d)

    def _embed(self, tokens, x, d, start=0):
        n = len(tokens)
        self.ids[start:start + n].copy_(torch.from_numpy(np.asarray(tokens, dtype=np.int32)), non_blocking=False)
        call("sj_embedding_fwd", self.wb_ptr("embedding"), _ptr(self.ids, start), _ptr(x), SJ_F32, n, d, VOCAB,
             self.stream)

    def _decoder_tail(self, n, row0):
        """decoder blocks -> decoder norm -> output projection -> final norm into self.final[row0:row0+n]."""
        h, c = self.h, self.c
        dd, dg = h.decoder_width, c.width
        dec = self.dec
        self._norm(dec.x, "decoder_norm", dec.z, dec.inv, n, dd)
        self._gemm(_ptr(dec.z), dd, self.wb_ptr("output_projection"), dg, _ptr(self.y), dg, SJ_F32, n, dg, dd)
        self._norm(self.y, "final_norm", _ptr(self.final, row0 * dg), dec.inv, n, dg)

    def hidden_cached(self, tokens):
        """Model::hidden_cached (architecture.rs:651-799): append `tokens` at position `length`; returns
        the final-norm rows of the chunk (bf16)."""
        tokens = [int(t) for t in np.asarray(tokens).reshape(-1)]
        if not tokens or min(tokens) < 0 or max(tokens) > EOS:
            raise ValueError("input tokens must be bytes or EOS")
        if self.length + len(tokens) > self.context:
            raise ValueError("KV cache context limit reached")
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream
        c, h = self.c, self.h
        if h is None:
            n = len(tokens)
            g = self.glob
            self._embed(tokens, g.x, c.width)
            self._blocks(g, n, self.length)
            self._norm(g.x, "final_norm", g.z, g.inv, n, c.width)
            self.length += n
            return g.z[:n]
        if self.length == 0 and len(tokens) >= h.patch_size:
            return self._prefill(tokens)
        return self._decode(tokens)

    def _bos(self):
        c, h = self.c, self.h
        self._gemm(self.wb_ptr("global_bos"), c.width, self.wb_ptr("global_to_decoder"), h.decoder_width,
                   _ptr(self.bos), h.decoder_width, SJ_BF16, 1, h.decoder_width, c.width)

    def _prefill(self, tokens):
        """hierarchical_prefill (architecture.rs:534-650)."""
        c, h = self.c, self.h
        n, P = len(tokens), h.patch_size
        de, dg, dd = h.encoder_width, c.width, h.decoder_width
        enc, glob, dec = self.enc, self.glob, self.dec
        np_ = -(-n // P)
        self._embed(tokens, enc.x, de)
        self._blocks(enc, n, 0)
        self._norm(enc.x, "encoder_norm", self.zE, enc.inv, n, de)
        call("sj_patch_pool_fwd", _ptr(self.zE), _ptr(self.pooled), 1, n, de, P, self.stream)
        self._gemm(_ptr(self.pooled), de, self.wb_ptr("encoder_to_global"), dg, _ptr(glob.x), dg, SJ_F32, np_, dg, de)
        self._blocks(glob, np_, 0)
        self._norm(glob.x, "global_norm", glob.z, glob.inv, np_, dg)
        self._gemm(_ptr(glob.z), dg, self.wb_ptr("global_to_decoder"), dd, _ptr(self.zd), dd, SJ_BF16, np_, dd, dg)
        self._bos()
        self._gemm(_ptr(self.zE), de, self.wb_ptr("encoder_to_decoder"), dd, _ptr(dec.x), dd, SJ_F32, n, dd, de)
        call("sj_patch_broadcast_fwd", _ptr(self.zd), _ptr(self.bos), _ptr(dec.x), SJ_F32, 1, 1, n, dd, P, self.stream)
        self._blocks(dec, n, 0)
        self._decoder_tail(n, 0)
        completed = n // P
        src = self.bos if completed == 0 else self.zd[completed - 1:completed]
        call("sj_copy_rows", _ptr(src), dd * 2, _ptr(self.gctx), dd * 2, 1, dd * 2, self.stream)
        self.have_ctx = True
        self.patch_count = n % P
        if self.patch_count:
            call("sj_rows_sum_f32", _ptr(self.zE, (n - self.patch_count) * de), de, self.patch_count, de,
                 _ptr(self.patch_sum), 1, self.stream)
        self.length = n
        return self.final[:n]

    def _decode(self, tokens):
        """The patch-by-patch branch of hidden_cached (architecture.rs:672-779)."""
        c, h = self.c, self.h
        P = h.patch_size
        de, dg, dd = h.encoder_width, c.width, h.decoder_width
        enc, glob, dec = self.enc, self.glob, self.dec
        total, i = len(tokens), 0
        while i < total:
            count = min(P - self.patch_count, total - i)
            position = self.length + i
            self._embed(tokens[i:i + count], enc.x, de, start=i)
            self._blocks(enc, count, position)
            self._norm(enc.x, "encoder_norm", self.zE, enc.inv, count, de)
            if not self.have_ctx:
                self._bos()
                call("sj_copy_rows", _ptr(self.bos), dd * 2, _ptr(self.gctx), dd * 2, 1, dd * 2, self.stream)
                self.have_ctx = True
            self._gemm(_ptr(self.zE), de, self.wb_ptr("encoder_to_decoder"), dd, _ptr(dec.x), dd, SJ_F32, count, dd,
                       de)
            # bias_add of the global context: every row of the piece lies in the current patch, so the
            # broadcast's BOS row (patch index -1) is the context for all of them
            call("sj_patch_broadcast_fwd", _ptr(self.zd), _ptr(self.gctx), _ptr(dec.x), SJ_F32, 1, 1, count, dd, P,
                 self.stream)
            self._blocks(dec, count, position)
            self._decoder_tail(count, i)
            call("sj_rows_sum_f32", _ptr(self.zE), de, count, de, _ptr(self.patch_sum), int(self.patch_count == 0),
                 self.stream)
            self.patch_count += count
            if self.patch_count == P:
                call("sj_scale_to_bf16", _ptr(self.patch_sum), de, 1.0 / P, _ptr(self.pooled), self.stream)
                self._gemm(_ptr(self.pooled), de, self.wb_ptr("encoder_to_global"), dg, _ptr(glob.x), dg, SJ_F32, 1,
                           dg, de)
                self._blocks(glob, 1, position // P)
                self._norm(glob.x, "global_norm", glob.z, glob.inv, 1, dg)
                self._gemm(_ptr(glob.z), dg, self.wb_ptr("global_to_decoder"), dd, _ptr(self.gctx), dd, SJ_BF16, 1, dd,
                           dg)
                self.patch_count = 0
            i += count
        self.length += total
        return self.final[:total]

    def forward_cached(self, tokens):
        """lib.rs:362-372: the chunk, then the head on its last row: f32 logits [257] (device)."""
        hs = self.hidden_cached(tokens)
        n, d = hs.shape[0], self.c.width
        self._gemm(_ptr(hs, (n - 1) * d), d, self.wb_ptr("output"), VOCAB_PAD, _ptr(self.logits), VOCAB_PAD, SJ_F32,
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

