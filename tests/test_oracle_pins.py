"""Pin the CPU oracle against the reference's own kernels (golden vectors).

`tests/golden/reference_kernels.npz` holds inputs and outputs of the unmodified
reference Triton kernels run in Triton's CPU interpreter (generator:
tests/golden/make_golden.py).  Each oracle function must reproduce them at the
reference's own FP32 contract tolerances (crates/sejong-gpu/examples/
hierarchy_check.rs:113-116 uses 2e-5 max-abs for attention), and bit-exactly
for integer outputs (routing ids, packing, parameter indices).
"""
import os

import numpy as np
import pytest
import torch

from oracle import ops
from oracle.rng import Rng

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))


def g(prefix, key):
    return GOLD[f"{prefix}/{key}"]


def t64(a):
    return torch.tensor(np.asarray(a), dtype=torch.float64)


def close(a, b, tol):
    if torch.is_tensor(a):
        a = a.detach().numpy()
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    err = np.max(np.abs(a - b)) if a.size else 0.0
    scale = max(1.0, float(np.max(np.abs(b)))) if b.size else 1.0
    assert err <= tol * scale, f"max abs err {err} > {tol} * {scale}"


def test_rmsnorm_f32_f64():
    for tag, tol in (("f32", 2e-6), ("f64", 1e-13)):
        p = f"rmsnorm_{tag}"
        close(ops.rmsnorm(t64(g(p, "x")), t64(g(p, "w")), float(g(p, "eps"))), g(p, "y"), tol)


def test_rmsnorm_backward():
    p = "rmsnorm_backward"
    dx, dw = ops.rmsnorm_backward(t64(g(p, "x")), t64(g(p, "w")), t64(g(p, "dy")), float(g(p, "eps")))
    close(dx, g(p, "dx"), 1e-5)
    close(dw, g(p, "dw"), 1e-5)
    # the explicit formula is the exact derivative of the forward
    x = t64(g(p, "x")).requires_grad_()
    w = t64(g(p, "w")).requires_grad_()
    (ops.rmsnorm(x, w, 1e-6) * t64(g(p, "dy"))).sum().backward()
    close(x.grad, dx, 1e-12)
    close(w.grad, dw, 1e-12)


def test_swiglu_and_backward():
    p = "swiglu"
    gg, u, dy = t64(g(p, "g")), t64(g(p, "u")), t64(g(p, "dy"))
    close(ops.swiglu(gg, u), g(p, "h"), 2e-6)
    dg, du = ops.swiglu_backward(gg, u, dy)
    close(dg, g(p, "dg"), 2e-6)
    close(du, g(p, "du"), 2e-6)


def test_gelu():
    p = "gelu"
    close(ops.gelu(t64(g(p, "x"))), g(p, "y"), 2e-6)


def test_rope_forward_and_inverse():
    for kind, inverse in (("forward", False), ("inverse", True)):
        p = f"rope_{kind}"
        y = ops.rope(t64(g(p, "x")), int(g(p, "t")), 0, int(g(p, "heads")), float(g(p, "theta")), inverse)
        close(y, g(p, "y"), 2e-5)


def test_embedding_forward_backward():
    p = "embedding"
    ids = torch.tensor(g(p, "ids"))
    close(ops.embedding(t64(g(p, "w")), ids), g(p, "y"), 0)
    close(ops.embedding_backward(t64(g(p, "dy")), ids, 257), g(p, "dw"), 2e-6)


def test_cross_entropy():
    p = "cross_entropy"
    x, tg = t64(g(p, "x")), torch.tensor(g(p, "targets"))
    close(ops.cross_entropy(x, tg), g(p, "loss"), 2e-6)
    close(ops.cross_entropy_backward(x, tg, t64(g(p, "dy"))), g(p, "dx"), 2e-6)


def test_layernorm():
    p = "layernorm"
    close(ops.layernorm(t64(g(p, "x")), t64(g(p, "w")), t64(g(p, "b")), float(g(p, "eps"))), g(p, "y"), 2e-6)


def test_adamw_transition():
    p = "adamw"
    step, lr, b1, b2, eps, decay, scale = g(p, "hyper")
    w, m, v = ops.adamw(t64(g(p, "w0")), t64(g(p, "g")), t64(g(p, "m0")), t64(g(p, "v0")), int(step), lr, b1, b2,
                        eps, decay, scale)
    # crates/sejong-train/examples/system_check.rs:135-163 holds the transition to 2e-7
    close(w, g(p, "w"), 2e-7)
    close(m, g(p, "m"), 2e-7)
    close(v, g(p, "v"), 2e-7)


@pytest.mark.parametrize("window", [0, 3])
@pytest.mark.parametrize("tag", ["f32", "f64"])
def test_grouped_attention_forward(window, tag):
    p = f"attention_w{window}_{tag}"
    o, lse = ops.grouped_attention(t64(g(p, "q")), t64(g(p, "k")), t64(g(p, "v")), int(g(p, "t")), int(g(p, "hq")),
                                   int(g(p, "hk")), window or None)
    tol = 2e-5 if tag == "f32" else 1e-12
    close(o, g(p, "o"), tol)
    close(lse, g(p, "lse"), tol)


@pytest.mark.parametrize("window", [0, 3])
def test_grouped_attention_backward(window):
    p = f"attention_backward_w{window}"
    q, k, v = (t64(g(p, n)).requires_grad_() for n in ("q", "k", "v"))
    o, _ = ops.grouped_attention(q, k, v, int(g(p, "t")), int(g(p, "hq")), int(g(p, "hk")), window or None)
    (o * t64(g(p, "do"))).sum().backward()
    close(q.grad, g(p, "dq"), 2e-5)
    close(k.grad, g(p, "dk"), 2e-5)
    close(v.grad, g(p, "dv"), 2e-5)
    delta = (t64(g(p, "do")) * t64(g(p, "o"))).reshape(-1, q.shape[1] // int(g(p, "hq"))).sum(1)
    close(delta, g(p, "delta"), 2e-5)


def test_noncausal_attention():
    p = "attention_noncausal"
    o, lse = ops.attention(t64(g(p, "q")), t64(g(p, "k")), t64(g(p, "v")), int(g(p, "t")), int(g(p, "heads")), False)
    close(o, g(p, "o"), 2e-5)
    close(lse, g(p, "lse"), 2e-5)


def test_patch_pool_and_backward():
    p = "patch_pool"
    t, patch = int(g(p, "t")), int(g(p, "patch"))
    x = t64(g(p, "x")).requires_grad_()
    y = ops.patch_pool(x, t, patch)
    close(y, g(p, "y"), 2e-6)
    (y * t64(g(p, "dy"))).sum().backward()
    close(x.grad, g(p, "dx"), 2e-6)


def test_patch_broadcast_and_backward():
    p = "patch_broadcast"
    t, patch = int(g(p, "t")), int(g(p, "patch"))
    x = t64(g(p, "x")).requires_grad_()
    bos = t64(g(p, "bos")).requires_grad_()
    y = ops.patch_broadcast(x, bos, t, patch)
    close(y, g(p, "y"), 0)
    (y * t64(g(p, "dy"))).sum().backward()
    close(x.grad, g(p, "dx"), 2e-6)
    close(bos.grad.reshape(-1), g(p, "dbos"), 2e-6)


def test_route_topk_ids_bit_exact_and_backward():
    p = "route"
    logits = t64(g(p, "logits")).requires_grad_()
    gates, ids = ops.route_topk(logits, int(g(p, "k")))
    assert np.array_equal(ids.numpy(), g(p, "ids").astype(np.int64))
    close(gates.detach(), g(p, "gates"), 2e-6)
    (gates * t64(g(p, "dy"))).sum().backward()
    close(logits.grad, g(p, "dx"), 2e-6)


def test_route_pack_order_bit_exact():
    """hierarchy.py:212-225: per expert, routed (row, slot) pairs in slot order."""
    p = "route"
    ids = g(p, "ids").reshape(-1)
    r = ids.size
    counts = g(p, "counts")
    tokens, slots = g(p, "tokens"), g(p, "slots")
    k = int(g(p, "k"))
    for e in range(counts.size):
        sel = np.nonzero(ids == e)[0]
        assert counts[e] == sel.size
        assert np.array_equal(slots[e * r:e * r + sel.size], sel)
        assert np.array_equal(tokens[e * r:e * r + sel.size], sel // k)


def test_projections_and_matmul():
    p = "projection_qkv"
    x = t64(g(p, "x"))
    close(x @ t64(g(p, "wq")), g(p, "q"), 1e-5)
    close(x @ t64(g(p, "wk")), g(p, "k"), 1e-5)
    close(x @ t64(g(p, "wv")), g(p, "v"), 1e-5)
    p = "projection_gate_up"
    x = t64(g(p, "x"))
    gg, u = x @ t64(g(p, "wg")), x @ t64(g(p, "wu"))
    close(gg, g(p, "g"), 1e-5)
    close(ops.swiglu(gg, u), g(p, "h"), 1e-4)
    for ta in (0, 1):
        for tb in (0, 1):
            p = f"matmul_{ta}{tb}"
            a, b = t64(g(p, "a")), t64(g(p, "b"))
            close((a.T if ta else a) @ (b.T if tb else b), g(p, "c"), 1e-5)


def test_rng_pinned_by_parameter_indices():
    """The reference's in-kernel SplitMix64 + rejection draw (parameter.py:6-22) equals Rng::index."""
    p = "parameter_indices"
    a, bcols, nb, s, r, group = (int(v) for v in g(p, "shape"))
    rng = Rng(int(g(p, "seed")))
    cols = list(range(bcols))
    picked = []
    for i in range(r):
        j = i + rng.index(bcols - i)
        cols[i], cols[j] = cols[j], cols[i]
        picked.append(cols[i])
    assert picked == list(g(p, "columns"))
    blocks = list(range(nb))
    rows = []
    for i in range(s):
        j = i + rng.index(nb - i)
        blocks[i], blocks[j] = blocks[j], blocks[i]
        for o in range(group):
            idx = blocks[i] * group + o
            rows.append(idx if idx < a else -1)
    assert rows == list(g(p, "rows"))


@pytest.mark.parametrize("case", ["parameter_indices"] + [f"parameter_indices_{i}" for i in range(4)])
def test_param_vjp_indices_pinned(case):
    """oracle.param_vjp.parameter_indices reproduces the reference kernel (parameter.py:25-62) bit for
    bit, including the zero-size draws of a reused basis or selection."""
    from oracle import param_vjp as pv
    a, bcols, nb, s, r, group = (int(v) for v in g(case, "shape"))
    columns, rows, row_map = pv.parameter_indices(int(g(case, "seed")), a, bcols, nb, s, r, group)
    assert list(columns) == list(g(case, "columns"))
    assert list(rows) == list(g(case, "rows"))
    assert list(row_map) == list(g(case, "map"))


@pytest.mark.parametrize("tag", ["register", "streaming"])
def test_param_vjp_basis_pinned(tag):
    """oracle.param_vjp.basis_cgs2 (FP64) matches the reference's f32 CGS2 (parameter.py:65-129),
    including the column the small-norm cutoff zeroes."""
    from oracle import param_vjp as pv
    p = f"parameter_basis_{tag}"
    y, cols = g(p, "y"), g(p, "columns")
    n, r = y.shape[0], len(cols)
    eps = pv.basis_eps(n, r)
    assert np.float32(eps) == g(p, "eps")
    q = pv.basis_cgs2(y[:, cols], eps)
    ref = g(p, "q")
    zero = np.all(ref == 0, axis=0)
    assert list(np.all(q == 0, axis=0)) == list(zero)
    close(q, ref, 2e-5)


def test_param_vjp_prepare_pinned():
    """oracle.param_vjp.prepare_factors matches parameter_prepare (parameter.py:131-166)."""
    from oracle import param_vjp as pv
    p = "parameter_prepare"
    n, m, r, k = (int(v) for v in g(p, "shape"))
    row_map = g(p, "map")
    rows = np.full(k, -1)
    for row, pos in enumerate(row_map):
        if pos >= 0:
            rows[pos] = row
    left, e = pv.prepare_factors(g(p, "x"), g(p, "q"), rows, float(g(p, "inverse")))
    close(left, g(p, "left"), 1e-5)
    close(e, g(p, "e"), 1e-5)
