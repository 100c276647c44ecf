"""FP64 restatement of the reference kernels on the training-step path.

Every function names the reference kernel (python/sejong_kernels/ops/...) it
restates.  All functions are written with differentiable torch operations so
that `model.py` can take exact FP64 gradients with autograd; the explicit
backward formulas the reference kernels use are restated too (`*_backward`) so
they can be pinned one by one against the interpreter-run reference kernels.

Layouts follow the reference: activations are row-major [rows, features];
attention heads are packed [rows, heads*head_dim] with row = batch*T + t.
"""
import math

import torch


def embedding(w, ids):
    """kernels.py:41-45 — row gather."""
    return w[ids.long()]


def embedding_backward(dy, ids, vocab):
    """kernels.py:47-52 — scatter-add of rows into a zero [vocab, D] gradient."""
    dw = torch.zeros(vocab, dy.shape[1], dtype=dy.dtype)
    dw.index_add_(0, ids.long(), dy)
    return dw


def rmsnorm(x, w, eps):
    """kernels.py:54-61 — y = x * w / sqrt(mean(x^2) + eps) per row."""
    inv = 1.0 / torch.sqrt((x * x).mean(dim=1, keepdim=True) + eps)
    return x * inv * w


def rmsnorm_backward(x, w, dy, eps):
    """kernels.py:63-87 — dx per row; dw = sum_rows dy * x * inv."""
    d = x.shape[1]
    inv = torch.rsqrt((x * x).sum(1) / d + eps)[:, None]
    g = dy * w[None, :]
    dx = inv * (g - x * ((g * x).sum(1) / d)[:, None] * inv * inv)
    dw = (dy * x * inv).sum(0)
    return dx, dw


def swiglu(g, u):
    """kernels.py:89-93 — h = g * sigmoid(g) * u."""
    return g * torch.sigmoid(g) * u


def swiglu_backward(g, u, dy):
    """kernels.py:95-101."""
    s = torch.sigmoid(g)
    return dy * u * s * (1 + g * (1 - s)), dy * g * s


def rope(x, t, offset, heads, theta, inverse=False):
    """kernels.py:103-113 — interleaved pairs (2i, 2i+1) of each head.

    angle = (row mod T + offset) * exp((-2 i / D) * ln(theta)); the inverse
    (used for the backward, crates/sejong-gpu/src/graph.rs:879-882) negates sin.
    """
    n, width = x.shape
    d = width // heads
    pos = (torch.arange(n, dtype=torch.float64) % t + offset)[:, None, None]
    pair = torch.arange(d // 2, dtype=torch.float64)[None, None, :]
    angle = pos * torch.exp((-2.0 * pair / d) * math.log(theta))
    cos, sin = torch.cos(angle).to(x.dtype), torch.sin(angle).to(x.dtype)
    if inverse:
        sin = -sin
    xv = x.reshape(n, heads, d // 2, 2)
    a, b = xv[..., 0], xv[..., 1]
    y = torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1)
    return y.reshape(n, width)


def grouped_attention(q, k, v, t, hq, hk, window=None, offset=0):
    """hierarchy.py:7-39 — causal GQA with optional sliding window.

    Query (b, t, h) attends keys s of kv head h // (hq/hk) with
    max(0, t + offset + 1 - W) <= s <= t + offset (no lower bound without a
    window); scale D^-1/2; returns O [rows, hq*D] and LSE (natural log) laid out
    [rows*hq] with index row*hq + h.
    """
    rows = q.shape[0]
    d = q.shape[1] // hq
    b = rows // t
    tk = k.shape[0] // b
    qh = q.reshape(b, t, hq, d).permute(0, 2, 1, 3)
    kh = k.reshape(b, tk, hk, d).permute(0, 2, 1, 3)
    vh = v.reshape(b, tk, hk, d).permute(0, 2, 1, 3)
    group = hq // hk
    kh = kh.repeat_interleave(group, dim=1)
    vh = vh.repeat_interleave(group, dim=1)
    s = torch.matmul(qh, kh.transpose(-1, -2)) * (d ** -0.5)
    qpos = torch.arange(t)[:, None] + offset
    kpos = torch.arange(tk)[None, :]
    allowed = kpos <= qpos
    if window:
        allowed = allowed & (kpos >= qpos + 1 - window)
    s = s.masked_fill(~allowed, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    o = torch.matmul(p, vh)
    o = o.permute(0, 2, 1, 3).reshape(rows, hq * d)
    lse = lse.permute(0, 2, 1).reshape(rows * hq)
    return o, lse


def attention(q, k, v, t, heads, causal=True):
    """kernels.py:115-136 — multi-head attention; non-causal for the BERT path."""
    if causal:
        return grouped_attention(q, k, v, t, heads, heads, None)
    rows = q.shape[0]
    d = q.shape[1] // heads
    b = rows // t
    qh = q.reshape(b, t, heads, d).permute(0, 2, 1, 3)
    kh = k.reshape(b, t, heads, d).permute(0, 2, 1, 3)
    vh = v.reshape(b, t, heads, d).permute(0, 2, 1, 3)
    s = torch.matmul(qh, kh.transpose(-1, -2)) * (d ** -0.5)
    lse = torch.logsumexp(s, dim=-1)
    o = torch.matmul(torch.exp(s - lse[..., None]), vh)
    return o.permute(0, 2, 1, 3).reshape(rows, heads * d), lse.permute(0, 2, 1).reshape(rows * heads)


def patch_pool(x, t, patch):
    """hierarchy.py:107-119 — mean of each patch's rows (partial last patch by count)."""
    rows, d = x.shape
    b = rows // t
    patches = -(-t // patch)
    out = []
    xb = x.reshape(b, t, d)
    for p in range(patches):
        s = p * patch
        out.append(xb[:, s:min(s + patch, t)].mean(dim=1))
    return torch.stack(out, dim=1).reshape(b * patches, d)


def patch_broadcast(x, bos, t, patch):
    """hierarchy.py:134-143 — byte t receives patch (t//P - 1); the first patch gets BOS."""
    d = x.shape[1]
    patches = -(-t // patch)
    b = x.shape[0] // patches
    xb = x.reshape(b, patches, d)
    src = torch.arange(t) // patch - 1
    body = xb[:, src.clamp(min=0)]
    first = (src < 0)[None, :, None]
    y = torch.where(first, bos.reshape(1, 1, d).expand(b, t, d), body)
    return y.reshape(b * t, d)


def cross_entropy(logits, targets):
    """kernels.py:176-183 — per-row logsumexp - logit[target]."""
    return torch.logsumexp(logits, dim=1) - logits.gather(1, targets.long()[:, None])[:, 0]


def cross_entropy_backward(logits, targets, dy):
    """kernels.py:185-191 — (softmax - onehot) * dy."""
    p = torch.softmax(logits, dim=1)
    p[torch.arange(logits.shape[0]), targets.long()] -= 1.0
    return p * dy[:, None]


def gelu(x):
    """kernels.py:227-232 — erf GELU."""
    return 0.5 * x * (1 + torch.erf(x * 0.7071067811865476))


def layernorm(x, w, b, eps):
    """common.py:6-14 — post-LN."""
    mean = x.mean(dim=1, keepdim=True)
    c = x - mean
    inv = 1.0 / torch.sqrt((c * c).mean(dim=1, keepdim=True) + eps)
    return c * inv * w + b


def route_topk(logits, k):
    """hierarchy.py:175-191 — softmax over experts, top-k ids (lowest index on
    ties), gate = full-softmax probability of the selected expert."""
    p = torch.softmax(logits, dim=1)
    ids = torch.empty(logits.shape[0], k, dtype=torch.int64)
    scores = logits.detach().clone()
    for slot in range(k):
        best = scores.max(dim=1, keepdim=True).values
        idx = torch.where(scores == best, torch.arange(scores.shape[1])[None, :],
                          torch.full_like(scores, scores.shape[1], dtype=torch.int64)).min(dim=1).values
        ids[:, slot] = idx
        scores[torch.arange(scores.shape[0]), idx] = float("-inf")
    return p.gather(1, ids), ids


def adamw(w, g, m, v, step, lr, beta1, beta2, eps, decay, scale):
    """kernels.py:193-202 with the host constants of crates/sejong-gpu/src/lib.rs:925-957.

    INV_B1 = 1/(1 - beta1^step), INV_B2 = 1/(1 - beta2^step) (computed in f32 by
    the host), g scaled by SCALE = clip / loss_scale; step = 0 where the
    denominator is 0.  Returns new (w, m, v).
    """
    inv_b1 = 1.0 / (1.0 - float(torch.tensor(beta1, dtype=torch.float32) ** step))
    inv_b2 = 1.0 / (1.0 - float(torch.tensor(beta2, dtype=torch.float32) ** step))
    g = g * scale
    m = beta1 * m + (1 - beta1) * g
    v = beta2 * v + (1 - beta2) * g * g
    den = torch.sqrt(v * inv_b2) + eps
    upd = torch.where(den > 0, (m * inv_b1) / torch.where(den > 0, den, torch.ones_like(den)),
                      torch.zeros_like(den))
    return w * (1 - lr * decay) - lr * upd, m, v


def lr_schedule(step, learning_rate, min_learning_rate, warmup_steps, steps):
    """crates/sejong-core/src/lib.rs:422-433 — linear warm-up then cosine."""
    if step < warmup_steps:
        return learning_rate * (step + 1) / warmup_steps
    span = max(steps - warmup_steps, 1)
    phase = min(max(step - warmup_steps, 0) / span, 1.0)
    return min_learning_rate + 0.5 * (learning_rate - min_learning_rate) * (1.0 + math.cos(math.pi * phase))
