"""FP64 restatement of the NativeValue step (test infrastructure: the checker of the product's value
mode, sejong_b200/value.py and ByteTrainer with TrainConfig.values > 0; nothing in the product
imports it).

* request layout: NativeValue::forward_batch (crates/sejong-model/src/native/value.rs:117-137): per
  request BOS 257, the prompt bytes, SEP 258, PAD 256 up to the batch's longest prompt + 2; the SEP
  row of each request is selected (value.rs:136);
* forward: the native embedding cast to the compute precision (value.rs:139-141), the body from
  that input (hidden_from, architecture.rs:353-393), the selected rows cast to f32 and an f32 affine
  head (value.rs:144-150);
* loss: the cross entropy of each request against its label, averaged over the batch (the seed
  1 / batch of Graph::backward, crates/sejong-gpu/src/graph.rs:539-549; memory.rs:958-966);
* initialisation: value.rs:39-76 (Rng(seed ^ 0x76616c7565), normal() / sqrt(width), bias 0).
"""
import numpy as np
import torch

from . import model as om
from . import ops
from .rng import Rng

NATIVE_VOCAB, PAD, BOS, SEP = 259, 256, 257, 258


def layout_requests(prompts):
    """value.rs:117-137: (ids int64 [batch * sequence], selected rows, sequence)."""
    raw = [p.encode() if isinstance(p, str) else bytes(p) for p in prompts]
    sequence = max(len(p) for p in raw) + 2
    ids = [PAD] * (len(raw) * sequence)
    selected = []
    for row, p in enumerate(raw):
        start = row * sequence
        ids[start] = BOS
        for i, byte in enumerate(p):
            ids[start + 1 + i] = byte
        ids[start + 1 + len(p)] = SEP
        selected.append(start + 1 + len(p))
    return np.array(ids, dtype=np.int64), np.array(selected, dtype=np.int64), sequence


def initialize(c, values):
    rng = Rng(int(c.seed) ^ 0x76616C7565)
    d = c.width
    scale = np.float32(np.sqrt(np.float32(d)))
    emb = (rng.bulk_normal(NATIVE_VOCAB * d).astype(np.float32) / scale).astype(np.float32)
    head = (rng.bulk_normal(d * values).astype(np.float32) / scale).astype(np.float32)
    return {"native_embedding": emb.reshape(NATIVE_VOCAB, d), "native_value": head.reshape(d, values),
            "native_bias": np.zeros((1, values), dtype=np.float32)}


def loss_and_grads(params, c, prompts, labels, dtype=torch.float64, cast=None, scale=1.0, logits_out=None):
    """Mean value cross entropy and the gradients of every parameter (body, native embedding, head).

    `cast="bf16"` evaluates the body and the native embedding at their bf16-rounded values (the
    reference binds them in the compute precision, crates/sejong-model/src/lib.rs:206-219, and
    casts the native embedding, value.rs:140); the head and bias stay f32."""
    head_names = ("native_value", "native_bias")
    body = om.compute_cast({k: v for k, v in params.items() if k not in head_names}, cast)
    body.update({k: params[k] for k in head_names})
    p = {k: torch.tensor(np.asarray(v), dtype=dtype, requires_grad=True) for k, v in body.items()}
    ids, selected, sequence = layout_requests(prompts)
    x = ops.embedding(p["native_embedding"], torch.as_tensor(ids))
    h = om.hidden_from(p, c, x, sequence, project=c.hierarchy is not None)
    sel = h[torch.as_tensor(selected)]
    if cast is not None:  # the final-norm output is a compute-precision tensor before the f32 cast
        sel = sel.to(torch.bfloat16).to(dtype)
    logits = sel @ p["native_value"] + p["native_bias"]
    if logits_out is not None:
        logits_out.append(logits.detach().numpy().copy())
    per = ops.cross_entropy(logits, torch.as_tensor(np.asarray(labels, dtype=np.int64)))
    loss = per.mean()
    (loss * scale).backward()
    grads = {k: (t.grad.detach().numpy().copy() if t.grad is not None else np.zeros(t.shape))
             for k, t in p.items()}
    return float(loss.detach()), grads
