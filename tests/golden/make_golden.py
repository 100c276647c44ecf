"""Generate golden vectors by running the reference's own Triton kernels on the CPU.

Run in a container that holds the reference source (read-only); point
SEJONG_REFERENCE at its checkout (the directory that contains python/sejong_kernels):

    SEJONG_REFERENCE=<reference checkout> python tests/golden/make_golden.py

The reference kernels (python/sejong_kernels/ops/{kernels,hierarchy,projection,
common,parameter}.py) are imported unmodified and executed by Triton's CPU
interpreter (TRITON_INTERPRET=1).  Under the interpreter `libdevice` calls
return nothing, so the modules' `math` name is pointed at small jitted
wrappers of tl.sqrt/tl.exp/tl.log/tl.math.erf before launch; no reference file
is edited.  Inputs are seeded; inputs and outputs are stored in
`reference_kernels.npz` next to this script.  The GPU box never runs this
script: the tests read only the committed .npz.
"""
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"
REFERENCE = os.environ.get("SEJONG_REFERENCE")
if not REFERENCE or not os.path.isdir(os.path.join(REFERENCE, "python", "sejong_kernels")):
    sys.exit("set SEJONG_REFERENCE to the reference checkout (the directory holding python/sejong_kernels)")
sys.path.insert(0, os.path.join(REFERENCE, "python"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


@triton.jit
def _sqrt(x):
    return tl.sqrt(x)


@triton.jit
def _exp(x):
    return tl.exp(x)


@triton.jit
def _log(x):
    return tl.log(x)


@triton.jit
def _erf(x):
    return tl.math.erf(x)


SHIM = types.SimpleNamespace(sqrt=_sqrt, exp=_exp, log=_log, erf=_erf)

from sejong_kernels.ops import common as C  # noqa: E402
from sejong_kernels.ops import hierarchy as H  # noqa: E402
from sejong_kernels.ops import kernels as K  # noqa: E402
from sejong_kernels.ops import parameter as PV  # noqa: E402
from sejong_kernels.ops import projection as PJ  # noqa: E402

for module in (K, H, C):
    module.math = SHIM

OUT = {}
G = torch.Generator().manual_seed(20261201)


def randn(*shape, dtype=torch.float32):
    return torch.randn(*shape, generator=G, dtype=torch.float64).to(dtype)


def save(prefix, **arrays):
    for k, v in arrays.items():
        OUT[f"{prefix}/{k}"] = v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v)


def npow2(n):
    return 1 << (int(n) - 1).bit_length()


def rmsnorm_cases():
    for dtype, tag in ((torch.float32, "f32"), (torch.float64, "f64")):
        r, d = 6, 48
        x = randn(r, d, dtype=dtype)
        w = 1 + 0.1 * randn(d, dtype=dtype)
        y = torch.empty_like(x)
        K.rmsnorm[(r,)](x, w, y, D=d, EPS=1e-6, BLOCK=npow2(d))
        save(f"rmsnorm_{tag}", x=x, w=w, y=y, eps=1e-6)
    r, d, br = 10, 48, 4
    x, w, dy = randn(r, d), 1 + 0.1 * randn(d), randn(r, d)
    dx = torch.empty_like(x)
    groups = -(-r // br)
    partial = torch.empty(groups, d)
    dw = torch.empty(d)
    K.rmsnorm_backward_partial[(groups,)](x, w, dy, dx, partial, r, D=d, EPS=1e-6, BR=br, BD=npow2(d))
    K.rmsnorm_backward_reduce[(-(-d // 32),)](partial, dw, groups, D=d, BG=4, BD=32)
    save("rmsnorm_backward", x=x, w=w, dy=dy, dx=dx, dw=dw, eps=1e-6)


def elementwise_cases():
    n = 300
    g, u, dy = randn(n), randn(n), randn(n)
    h, dg, du = torch.empty(n), torch.empty(n), torch.empty(n)
    K.swiglu[(-(-n // 256),)](g, u, h, n, BLOCK=256)
    K.swiglu_backward[(-(-n // 256),)](g, u, dy, dg, du, n, BLOCK=256)
    save("swiglu", g=g, u=u, dy=dy, h=h, dg=dg, du=du)
    x = randn(n)
    y = torch.empty(n)
    dx = torch.empty(n)
    K.gelu[(-(-n // 256),)](x, y, n, BLOCK=256)
    K.gelu_backward[(-(-n // 256),)](x, dy, dx, n, BLOCK=256)
    save("gelu", x=x, dy=dy, y=y, dx=dx)
    # RoPE: [N, H*D] with N = B*T rows
    b, t, heads, d, offset = 2, 5, 3, 8, 0
    rows = b * t
    x = randn(rows, heads * d)
    for inverse in (False, True):
        y = torch.empty_like(x)
        total = x.numel()
        K.rope[(-(-(total // 2) // 256),)](x, y, total, t, offset, D=d, H=heads, THETA=10000.0,
                                           INVERSE=inverse, BLOCK=256)
        save(f"rope_{'inverse' if inverse else 'forward'}", x=x, y=y, t=t, heads=heads, theta=10000.0)
    # embedding fwd / bwd
    vocab, d, n_ids = 257, 16, 20
    w = randn(vocab, d)
    ids = torch.randint(0, vocab, (n_ids,), generator=G, dtype=torch.int32)
    y = torch.empty(n_ids, d)
    K.embedding[(-(-n_ids * d // 256),)](w, ids, y, n_ids, d, BLOCK=256)
    dy = randn(n_ids, d)
    dw = torch.zeros(vocab, d)
    K.embedding_backward[(-(-n_ids * d // 256),)](dy, ids, dw, n_ids, d, BLOCK=256)
    save("embedding", w=w, ids=ids, y=y, dy=dy, dw=dw)
    # cross entropy fwd / bwd over 257-way rows
    r, v = 7, 257
    x = randn(r, v) * 3
    tg = torch.randint(0, v, (r,), generator=G, dtype=torch.int32)
    loss = torch.empty(r)
    K.cross_entropy[(r,)](x, tg, loss, V=v, BLOCK=512)
    dyr = randn(r)
    dx = torch.empty(r, v)
    K.cross_entropy_backward[(r,)](x, tg, dyr, dx, V=v, BLOCK=512)
    save("cross_entropy", x=x, targets=tg, loss=loss, dy=dyr, dx=dx)
    # layernorm
    x, w, bb = randn(5, 24), 1 + 0.1 * randn(24), randn(24)
    y = torch.empty_like(x)
    C.layernorm[(5,)](x, w, bb, y, D=24, EPS=1e-12, BLOCK=32)
    save("layernorm", x=x, w=w, b=bb, y=y, eps=1e-12)


def adamw_cases():
    n = 300
    w, g = randn(n), randn(n)
    m, v = 0.1 * randn(n), randn(n).abs() * 0.01
    w0, m0, v0 = w.clone(), m.clone(), v.clone()
    step, lr, b1, b2, eps, decay, scale = 3, 3e-4, 0.9, 0.95, 1e-8, 0.1, 0.5
    inv_b1 = float(np.float32(1.0) / (np.float32(1.0) - np.float32(b1) ** np.float32(step)))
    inv_b2 = float(np.float32(1.0) / (np.float32(1.0) - np.float32(b2) ** np.float32(step)))
    K.adamw[(-(-n // 256),)](w, g, m, v, n, lr, b1, b2, eps, decay, inv_b1, inv_b2, scale, BLOCK=256)
    save("adamw", w0=w0, g=g, m0=m0, v0=v0, w=w, m=m, v=v,
         hyper=np.array([step, lr, b1, b2, eps, decay, scale], dtype=np.float64))


def attention_cases():
    b, t, hq, hk, d = 2, 7, 4, 2, 8
    rows = b * t
    for window in (0, 3):
        for dtype, tag in ((torch.float32, "f32"), (torch.float64, "f64")):
            q, k, v = randn(rows, hq * d, dtype=dtype), randn(rows, hk * d, dtype=dtype), randn(rows, hk * d, dtype=dtype)
            o = torch.empty_like(q)
            lse = torch.empty(rows * hq, dtype=dtype)
            H.hierarchy_attention[(rows * hq,)](q, k, v, o, lse, t, t, 0, HQ=hq, HK=hk, D=d, BD=d, BK=8,
                                                WINDOW=window, FP64=dtype == torch.float64)
            save(f"attention_w{window}_{tag}", q=q, k=k, v=v, o=o, lse=lse, t=t, hq=hq, hk=hk)
            if dtype != torch.float32:
                continue
            do = randn(rows, hq * d)
            dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
            delta = torch.empty(rows * hq)
            H.hierarchy_attention_dq[(rows * hq,)](q, k, v, o, lse, do, dq, delta, t, HQ=hq, HK=hk, D=d, BD=d,
                                                   BK=8, WINDOW=window)
            H.hierarchy_attention_dkv[(rows * hk,)](q, k, v, lse, do, delta, dk, dv, t, HQ=hq, HK=hk, D=d, BD=d,
                                                    BK=8, WINDOW=window)
            save(f"attention_backward_w{window}", q=q, k=k, v=v, o=o, lse=lse, do=do, dq=dq, dk=dk, dv=dv,
                 delta=delta, t=t, hq=hq, hk=hk)
    # non-causal multi-head attention (BERT path)
    heads = 2
    q, k, v = randn(rows, heads * d), randn(rows, heads * d), randn(rows, heads * d)
    o = torch.empty_like(q)
    lse = torch.empty(rows * heads)
    K.attention[(rows * heads,)](q, k, v, o, lse, t, t, 0, H=heads, D=d, BD=d, BK=8, CAUSAL=False, FP64=False)
    save("attention_noncausal", q=q, k=k, v=v, o=o, lse=lse, t=t, heads=heads)


def hierarchy_cases():
    b, t, d, patch = 2, 13, 6, 4
    patches = -(-t // patch)
    x = randn(b * t, d)
    y = torch.empty(b * patches, d)
    H.hierarchy_patch_pool[(b * patches, 1)](x, y, t, d, PATCH=patch, BLOCK=8)
    dy = randn(b * patches, d)
    dx = torch.empty(b * t, d)
    H.hierarchy_patch_pool_backward[(-(-b * t * d // 64),)](dy, dx, b * t * d, t, d, PATCH=patch, BLOCK=64)
    save("patch_pool", x=x, y=y, dy=dy, dx=dx, t=t, patch=patch)
    z = randn(b * patches, d)
    bos = randn(1, d)
    yb = torch.empty(b * t, d)
    n = b * t * d
    H.hierarchy_patch_broadcast[(-(-n // 64),)](z, bos, yb, n, t, d, PATCH=patch, BLOCK=64)
    dyb = randn(b * t, d)
    dz = torch.empty(b * patches, d)
    dbos = torch.empty(d)
    body_tiles = -(-(b * patches * d) // 64)
    H.hierarchy_patch_broadcast_backward[(body_tiles + -(-d // 64),)](dyb, dz, dbos, n, t, d, PATCH=patch,
                                                                        BLOCK=64)
    save("patch_broadcast", x=z, bos=bos, y=yb, dy=dyb, dx=dz, dbos=dbos, t=t, patch=patch)
    # router top-k (+ ties) and its backward
    r, e, kk = 9, 5, 2
    logits = randn(r, e)
    logits[3, 1] = logits[3, 4] = logits[3].max() + 1.0  # tie -> lowest index first
    ids = torch.empty(r, kk, dtype=torch.int32)
    gates = torch.empty(r, kk)
    H.hierarchy_route_topk[(r,)](logits, ids, gates, E=e, K=kk, BLOCK=8)
    dg = randn(r, kk)
    dl = torch.empty(r, e)
    H.hierarchy_route_backward[(r,)](logits, ids, gates, dg, dl, E=e, K=kk, BLOCK=8)
    tokens = torch.full((e * r * kk,), -7, dtype=torch.int32)
    slots = torch.full((e * r * kk,), -7, dtype=torch.int32)
    counts = torch.empty(e, dtype=torch.int32)
    H.hierarchy_route_pack[(e,)](ids, tokens, slots, counts, r * kk, K=kk, BLOCK=8)
    save("route", logits=logits, ids=ids, gates=gates, dy=dg, dx=dl, tokens=tokens, slots=slots, counts=counts,
         k=kk)


def projection_cases():
    m, kdim, n, kv = 20, 24, 40, 16
    x, wq, wk, wv = randn(m, kdim), randn(kdim, n), randn(kdim, kv), randn(kdim, kv)
    q, ko, vo = torch.empty(m, n), torch.empty(m, kv), torch.empty(m, kv)
    PJ.projection_qkv[(-(-m // 16), -(-n // 32))](x, wq, wk, wv, q, ko, vo, m, n, kdim, kv, BM=16, BN=32, BK=32)
    save("projection_qkv", x=x, wq=wq, wk=wk, wv=wv, q=q, k=ko, v=vo)
    wg, wu = randn(kdim, n), randn(kdim, n)
    g, u, h = torch.empty(m, n), torch.empty(m, n), torch.empty(m, n)
    PJ.projection_gate_up[(-(-m // 16), -(-n // 32))](x, wg, wu, g, u, h, m, n, kdim, BM=16, BN=32, BK=32)
    save("projection_gate_up", x=x, wg=wg, wu=wu, g=g, u=u, h=h)
    for ta in (False, True):
        for tb in (False, True):
            mm, nn, kk = 19, 35, 21
            a = randn(kk, mm) if ta else randn(mm, kk)
            bmat = randn(nn, kk) if tb else randn(kk, nn)
            cmat = torch.empty(mm, nn)
            K.matmul[(-(-mm // 16), -(-nn // 32))](a, bmat, cmat, mm, nn, kk, TA=ta, TB=tb, BM=16, BN=32, BK=32)
            save(f"matmul_{int(ta)}{int(tb)}", a=a, b=bmat, c=cmat)


def parameter_index_cases():
    # partial Fisher-Yates draws driven by the in-kernel SplitMix64 (_random/_draw)
    a, bcols, nb, s, r, group = 71, 23, 5, 2, 6, 16
    seed = 0x0123456789ABCDEF
    scratch = torch.empty(bcols + nb, dtype=torch.int32)
    columns = torch.empty(r, dtype=torch.int32)
    rows = torch.empty(s * group, dtype=torch.int32)
    row_map = torch.empty(a, dtype=torch.int32)
    lo = np.int64(seed & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    hi = np.int64(seed >> 32).astype(np.uint32).view(np.int32)
    PV.parameter_indices[(1,)](scratch, columns, rows, row_map, a, bcols, nb, s, r, int(lo), int(hi),
                               GROUP=group, BLOCK=512)
    save("parameter_indices", columns=columns, rows=rows, map=row_map,
         shape=np.array([a, bcols, nb, s, r, group], dtype=np.int64), seed=np.uint64(seed))
    # the hierarchical model's two preparations (local d256 / FFN 768, global d768 / FFN 2048), a
    # basis-only and a selection-only draw (the zero sizes of a reused basis or selection)
    cases = [(256, 768, 8, 2, 16, 32), (768, 2048, 24, 6, 16, 32), (0, 300, 0, 0, 16, 32), (200, 0, 7, 2, 0, 32)]
    for idx, (a, bcols, nb, s, r, group) in enumerate(cases):
        seed = (0x9E3779B97F4A7C15 * (idx + 3)) & 0xFFFFFFFFFFFFFFFF
        scratch = torch.empty(max(bcols + nb, 1), dtype=torch.int32)
        columns = torch.full((max(r, 1),), -7, dtype=torch.int32)
        rows = torch.full((max(s * group, 1),), -7, dtype=torch.int32)
        row_map = torch.full((max(a, 1),), -7, dtype=torch.int32)
        lo = np.int64(seed & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
        hi = np.int64(seed >> 32).astype(np.uint32).view(np.int32)
        PV.parameter_indices[(1,)](scratch, columns, rows, row_map, a, bcols, nb, s, r, int(lo), int(hi),
                                   GROUP=group, BLOCK=512)
        save(f"parameter_indices_{idx}", columns=columns[:r], rows=rows[:s * group], map=row_map[:a],
             shape=np.array([a, bcols, nb, s, r, group], dtype=np.int64), seed=np.uint64(seed))


def parameter_basis_cases():
    # CGS2 of selected donor columns: the register form (small N) and the streaming form; the
    # streaming case selects a column twice so the small-norm cutoff zeroes one basis column
    for tag, n, bcols, cols in (("register", 40, 20, [3, 17, 0, 9, 11, 5]),
                                ("streaming", 300, 37, [4, 30, 12, 4, 7, 21, 0, 36, 15, 2, 8, 25, 33, 19, 1, 28])):
        y = randn(n, bcols)
        columns = torch.tensor(cols, dtype=torch.int32)
        r = len(cols)
        q = torch.full((n, r), float("nan"))
        operations = n * (4.0 * r + 1.0)
        roundoff = operations * (np.finfo(np.float32).eps / 2.0)
        eps = float(np.float32(roundoff / (1.0 - roundoff)))
        if tag == "register":
            PV.parameter_basis_register[(1,)](y, columns, q, n, bcols, eps, R=r, NR=npow2(n), NC=npow2(r))
        else:
            PV.parameter_basis[(1,)](y, columns, q, n, bcols, eps, R=r, BR=16, BC=32)
        save(f"parameter_basis_{tag}", y=y, columns=columns, q=q, eps=np.float32(eps))


def parameter_prepare_cases():
    # left = X^T Q and E = [Q^T ; (X - Q left^T)[:, rows] * INVERSE] with the rows of a draw
    n, m, r, group, nb, s = 96, 70, 5, 16, 5, 2
    x = randn(n, m)
    q = torch.linalg.qr(randn(n, r, dtype=torch.float64))[0].float().contiguous()  # QR returns column-major
    rows = [16 * 3 + o for o in range(16)] + [16 * 4 + o for o in range(16)]
    row_map = torch.full((m,), -1, dtype=torch.int32)
    for pos, row in enumerate(rows):
        if row < m:
            row_map[row] = pos
    k = s * group
    inverse = float(np.float32(nb) / np.float32(s))
    a_out = torch.full((m, r), float("nan"))
    e = torch.zeros(r + k, n)
    PV.parameter_prepare[(-(-m // 16),)](x, q, a_out, row_map, e, m, n, k, r, inverse, BM=16, BN=32, BK=32)
    save("parameter_prepare", x=x, q=q, map=row_map, left=a_out, e=e,
         shape=np.array([n, m, r, k], dtype=np.int64), inverse=np.float32(inverse))


def main():
    rmsnorm_cases()
    elementwise_cases()
    adamw_cases()
    attention_cases()
    hierarchy_cases()
    projection_cases()
    parameter_index_cases()
    parameter_basis_cases()
    parameter_prepare_cases()
    path =os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kernels.npz")
    np.savez_compressed(path, **OUT)
    print(f"wrote {len(OUT)} arrays to {path}")


if __name__ == "__main__":
    main()
