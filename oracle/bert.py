"""FP64 restatement of BertEncoder::hidden (crates/sejong-model/src/native/bert.rs:360-411).

Test infrastructure only (the checker of sejong_b200/bert.py): nothing in the product imports it.

One sequence at a time, unpadded, as the reference runs it:
    x = LayerNorm(word[ids] + position[0:len] + token_type[0])          (bert.rs:364-385)
    per layer i:
        q, k, v = linear(x, query / key / value)                        (bert.rs:388-391)
        a = attention(q, k, v, len, heads, causal = False)              (bert.rs:392-401)
        x = LayerNorm(x + linear(a, attention.output.dense))            (bert.rs:402-404)
        x = LayerNorm(x + linear(gelu(linear(x, intermediate.dense)), output.dense))  (bert.rs:405-409)
with linear(x, p) = x W^T + b (bert.rs:335-347), the erf GELU, LayerNorm and non-causal attention
of oracle.ops (each pinned against the reference's own kernels in tests/test_oracle_pins.py).

`matrix_dtype` lets a test evaluate the layers at the weights the compute path binds (bf16
matrices), so that the comparison measures the arithmetic of the bf16 path, as the byte-model
tests do.
"""
import numpy as np
import torch

from . import ops


COMPUTE = torch.float64  # the arithmetic type (bench.py's CPU baseline sets float32)


def _w(params, name, dtype=None):
    t = torch.as_tensor(np.asarray(params[name]))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(COMPUTE)


def hidden(params, ids, layers, heads, eps=1e-12, matrix_dtype=None):
    """Hidden states [len, d] (COMPUTE type) of one unpadded sequence `ids` (int array)."""
    ids = torch.as_tensor(np.asarray(ids, dtype=np.int64))
    n = ids.shape[0]
    word = _w(params, "embeddings.word_embeddings.weight")
    pos = _w(params, "embeddings.position_embeddings.weight")
    typ = _w(params, "embeddings.token_type_embeddings.weight")
    x = (word[ids] + pos[:n]) + typ[0][None, :]
    x = ops.layernorm(x, _w(params, "embeddings.LayerNorm.weight"), _w(params, "embeddings.LayerNorm.bias"), eps)

    def linear(x, prefix, act_dtype=None):
        w = _w(params, f"{prefix}.weight", matrix_dtype)
        b = _w(params, f"{prefix}.bias")
        if act_dtype is not None:
            x = x.to(act_dtype).to(COMPUTE)
        return x @ w.T + b

    act = matrix_dtype  # GEMM operands are rounded to the same type as the matrices
    for i in range(layers):
        p = f"encoder.layer.{i}"
        q = linear(x, f"{p}.attention.self.query", act)
        k = linear(x, f"{p}.attention.self.key", act)
        v = linear(x, f"{p}.attention.self.value", act)
        if act is not None:
            q, k, v = (t.to(act).to(COMPUTE) for t in (q, k, v))
        a, _ = ops.attention(q, k, v, n, heads, causal=False)
        x = ops.layernorm(x + linear(a, f"{p}.attention.output.dense", act),
                          _w(params, f"{p}.attention.output.LayerNorm.weight"),
                          _w(params, f"{p}.attention.output.LayerNorm.bias"), eps)
        h = ops.gelu(linear(x, f"{p}.intermediate.dense", act))
        x = ops.layernorm(x + linear(h, f"{p}.output.dense", act), _w(params, f"{p}.output.LayerNorm.weight"),
                          _w(params, f"{p}.output.LayerNorm.bias"), eps)
    return x


def hidden_batch(params, seqs, layers, heads, eps=1e-12, matrix_dtype=None):
    """Rows of every sequence, concatenated in order (the packed layout)."""
    return torch.cat([hidden(params, s, layers, heads, eps, matrix_dtype) for s in seqs])
