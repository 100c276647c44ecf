"""GPU parity of each kernel, called through the C ABI, against the CPU oracle / an fp32 torch
reference of the same op on the same seeded inputs.

Tolerances: GEMMs with f32 output must match an f32 product of the same bf16 operands to
1e-4 relative L2 (only summation order differs); bf16 outputs to 1e-2 (one bf16 rounding);
other bf16 kernels to 2e-2 relative L2 (the bf16 bar of the path); integer work bit-exact.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def lib():
    from sejong_b200 import _lib
    lib = _lib.load()
    _lib.call("sj_device_init", 0)
    return lib


def call(name, *args):
    from sejong_b200 import _lib
    return _lib.call(name, *args)


def ptr(t, off=0):
    return t.data_ptr() + off * t.element_size()


def stream():
    return torch.cuda.current_stream().cuda_stream


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / max(b.norm(), 1e-30))


def bf(x):
    return x.to(torch.bfloat16)


def check_device_error():
    code = ctypes.c_int(0)
    call("sj_device_error", ctypes.byref(code), 1, stream())
    assert code.value == 0, f"device error word {code.value}"


GEN = torch.Generator().manual_seed(1234)


def randn(*shape, scale=1.0):
    return (torch.randn(*shape, generator=GEN) * scale).to(DEV)


# ------------------------------------------------------------------------------------- GEMM
def gemm(a, a_trans, b, b_trans, m, n, k, c_dtype=torch.float32, epi=0, aux=None, ld_aux=0, rope_cols=0, rope_t=0,
         theta=0.0, split_k=0, c=None, alpha=1.0):
    from sejong_b200._lib import SJ_BF16, SJ_F32
    if c is None:
        c = torch.zeros(m, n, dtype=c_dtype, device=DEV)
    call("sj_gemm", ptr(a), a.shape[1], int(a_trans), ptr(b), b.shape[1], int(b_trans), ptr(c), c.shape[1],
         SJ_F32 if c.dtype == torch.float32 else SJ_BF16, m, n, k, epi, alpha, ptr(aux) if aux is not None else 0,
         ld_aux, rope_cols, rope_t, theta, split_k, stream())
    torch.cuda.synchronize()
    check_device_error()
    return c


def ref_mm(a, a_trans, b, b_trans):
    a32 = a.float().T if a_trans else a.float()
    b32 = b.float().T if b_trans else b.float()
    return a32 @ b32


@pytest.mark.parametrize("a_trans,b_trans", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (256, 256, 256), (200, 136, 104), (1024, 768, 256),
                                   (4096, 1280, 768), (384, 2048, 768)])
def test_gemm_layouts_f32_out(a_trans, b_trans, m, n, k):
    a = bf(randn(k, m) if a_trans else randn(m, k))
    b = bf(randn(n, k) if b_trans else randn(k, n))
    c = gemm(a, a_trans, b, b_trans, m, n, k)
    assert rel(c, ref_mm(a, a_trans, b, b_trans)) < 1e-4


@pytest.mark.parametrize("m,n,k", [(512, 384, 192), (4096, 257, 768)])
def test_gemm_bf16_out(m, n, k):
    a = bf(randn(m, k))
    b = torch.zeros(k, 264 if n == 257 else n, dtype=torch.bfloat16, device=DEV)
    b[:, :n] = bf(randn(k, n))
    c = torch.zeros(m, b.shape[1], dtype=torch.bfloat16, device=DEV)  # C rows padded to 16-byte multiples
    call("sj_gemm", ptr(a), k, 0, ptr(b), b.shape[1], 0, ptr(c), c.shape[1], 4, m, n, k, 0, 1.0, 0, 0, 0, 0, 0.0, 0,
         stream())
    torch.cuda.synchronize()
    assert rel(c[:, :n], a.float() @ b[:, :n].float()) < 1e-2
    assert float(c[:, n:].float().abs().max() if c.shape[1] > n else 0.0) == 0.0  # padding untouched


@pytest.mark.parametrize("split_k", [0, 1, 7])
def test_gemm_accumulate_split_k(split_k):
    m, n, k = 256, 768, 8192
    a = bf(randn(k, m, scale=0.1))   # weight-gradient form: A^T * B
    b = bf(randn(k, n, scale=0.1))
    c0 = randn(m, n)
    c = c0.clone()
    gemm(a, 1, b, 0, m, n, k, epi=1, c=c, split_k=split_k)
    assert rel(c, c0 + ref_mm(a, 1, b, 0)) < 1e-4


def test_gemm_residual_epilogue():
    m, n, k = 640, 256, 768
    a, b = bf(randn(m, k)), bf(randn(k, n))
    res = bf(randn(m, n))
    c = gemm(a, 0, b, 0, m, n, k, c_dtype=torch.bfloat16, epi=2, aux=res, ld_aux=n)
    assert rel(c, res.float() + a.float() @ b.float()) < 1e-2
    res32 = randn(m, n)
    c32 = gemm(a, 0, b, 0, m, n, k, c_dtype=torch.float32, epi=2, aux=res32, ld_aux=n)
    assert rel(c32, res32 + a.float() @ b.float()) < 1e-5


@pytest.mark.parametrize("epi", [0, 2])
@pytest.mark.parametrize("in_place", [False, True])
def test_gemm_f32_strided_store_residual(epi, in_place):
    """f32 STORE / RESIDUAL products with a strided C holding stale values, the residual in place or
    in its own buffer: columns past N stay untouched."""
    if epi == 0 and in_place:
        pytest.skip("in place applies to the residual only")
    m, n, k, ldc = 4096, 768, 2048, 776
    a, b = bf(randn(m, k, scale=0.1)), bf(randn(k, n, scale=0.1))
    c = randn(m, ldc) * 100.0   # stale contents must not leak into a STORE
    res = c if in_place else randn(m, ldc)
    res0 = res[:, :n].clone()
    pad0 = c[:, n:].clone()
    from sejong_b200._lib import SJ_F32
    call("sj_gemm", ptr(a), k, 0, ptr(b), n, 0, ptr(c), ldc, SJ_F32, m, n, k, epi, 1.0,
         ptr(res) if epi == 2 else 0, ldc if epi == 2 else 0, 0, 0, 0.0, 0, stream())
    torch.cuda.synchronize()
    check_device_error()
    ref = a.float() @ b.float() + (res0 if epi == 2 else 0)
    assert rel(c[:, :n], ref) < 1e-5
    assert torch.equal(c[:, n:], pad0)   # columns past N untouched


def test_gemm_swiglu_epilogue():
    from sejong_b200.model import _interleave_cols
    m, k, f = 512, 256, 768
    x = bf(randn(m, k))
    wg, wu = bf(randn(k, f, scale=0.1)), bf(randn(k, f, scale=0.1))
    wgu = torch.from_numpy(_interleave_cols(wg.float().cpu().numpy(), wu.float().cpu().numpy())).to(DEV)
    wgu = bf(wgu)
    h = torch.zeros(m, f, dtype=torch.bfloat16, device=DEV)
    gu = gemm(x, 0, wgu, 0, m, 2 * f, k, c_dtype=torch.bfloat16, epi=3, aux=h, ld_aux=f)
    g32, u32 = x.float() @ wg.float(), x.float() @ wu.float()
    assert rel(h, ops.swiglu(bf(g32).double().cpu(), bf(u32).double().cpu())) < 2e-2
    gu_ref = torch.from_numpy(_interleave_cols(g32.cpu().numpy(), u32.cpu().numpy()))
    assert rel(gu, gu_ref) < 1e-2


def gemm_plan(m, n, k, a_trans, b_trans, c_dtype, epi):
    import ctypes
    from sejong_b200 import _lib
    plan = (ctypes.c_int * 3)()
    assert _lib.load().sj_gemm_plan(m, n, k, a_trans, b_trans, c_dtype, epi, 0, plan) == 0
    return list(plan)


@pytest.mark.parametrize("m,n,k,b_trans", [(4224, 2048, 768, 0), (2048, 2304, 768, 1)])
def test_gemm_cta_pairs(m, n, k, b_trans):
    """Products the planner gives to CTA pairs (256-row tiles, tcgen05 cta_group::2), f32 and bf16
    C: 4224 rows end in a pair tile whose odd CTA holds only rows past M."""
    from sejong_b200._lib import SJ_BF16, SJ_F32
    for cdt in (SJ_F32, SJ_BF16):
        assert gemm_plan(m, n, k, 0, b_trans, cdt, 0) == [256, 1, 1]
    a = bf(randn(m, k))
    b = bf(randn(n, k) if b_trans else randn(k, n))
    ref = ref_mm(a, 0, b, b_trans)
    assert rel(gemm(a, 0, b, b_trans, m, n, k), ref) < 1e-4
    assert rel(gemm(a, 0, b, b_trans, m, n, k, c_dtype=torch.bfloat16), ref) < 1e-2
    check_device_error()


def test_gemm_swiglu_cta_pairs():
    """The global stage's gate/up product (4096 x 4096 x 768, SwiGLU epilogue) on CTA pairs."""
    from sejong_b200.model import _interleave_cols
    from sejong_b200._lib import SJ_BF16
    m, k, f = 4096, 768, 2048
    assert gemm_plan(m, 2 * f, k, 0, 0, SJ_BF16, 3) == [256, 1, 1]
    x = bf(randn(m, k))
    wg, wu = bf(randn(k, f, scale=0.1)), bf(randn(k, f, scale=0.1))
    wgu = bf(torch.from_numpy(_interleave_cols(wg.float().cpu().numpy(), wu.float().cpu().numpy())).to(DEV))
    h = torch.zeros(m, f, dtype=torch.bfloat16, device=DEV)
    gu = gemm(x, 0, wgu, 0, m, 2 * f, k, c_dtype=torch.bfloat16, epi=3, aux=h, ld_aux=f)
    g32, u32 = x.float() @ wg.float(), x.float() @ wu.float()
    assert rel(h, ops.swiglu(bf(g32).double().cpu(), bf(u32).double().cpu())) < 2e-2
    gu_ref = torch.from_numpy(_interleave_cols(g32.cpu().numpy(), u32.cpu().numpy()))
    assert rel(gu, gu_ref) < 1e-2
    check_device_error()


def test_gemm_rope_epilogue():
    m, k, hq, hk, t = 256, 256, 4, 2, 128
    cq = (hq + 2 * hk) * 64
    x, w = bf(randn(m, k)), bf(randn(k, cq, scale=0.1))
    c = gemm(x, 0, w, 0, m, cq, k, c_dtype=torch.bfloat16, epi=4, rope_cols=(hq + hk) * 64, rope_t=t, theta=10000.0)
    table = torch.empty(t * 64, device=DEV)
    call("sj_rope_table", ptr(table), t, 64, 0, 10000.0, stream())
    c_tab = gemm(x, 0, w, 0, m, cq, k, c_dtype=torch.bfloat16, epi=4, aux=table, rope_cols=(hq + hk) * 64, rope_t=t)
    y = (x.float() @ w.float()).double().cpu()
    q = ops.rope(y[:, :hq * 64], t, 0, hq, 10000.0)
    kk = ops.rope(y[:, hq * 64:(hq + hk) * 64], t, 0, hk, 10000.0)
    ref = torch.cat([q, kk, y[:, (hq + hk) * 64:]], dim=1)
    assert rel(c, ref) < 1e-2
    assert rel(c_tab, ref) < 1e-2


def test_gemm_rejects_bad_arguments():
    from sejong_b200._lib import SejongError
    a = bf(randn(64, 64))
    with pytest.raises(SejongError):
        call("sj_gemm", ptr(a), 63, 0, ptr(a), 64, 0, ptr(a), 64, 4, 64, 64, 64, 0, 1.0, 0, 0, 0, 0, 0.0, 0, stream())
    with pytest.raises(SejongError):  # split-K needs ACCUM
        call("sj_gemm", ptr(a), 64, 0, ptr(a), 64, 0, ptr(a), 64, 4, 64, 64, 64, 0, 1.0, 0, 0, 0, 0, 0.0, 4, stream())


# ------------------------------------------------------------------------------------- norms
@pytest.mark.parametrize("x_f32", [False, True])
@pytest.mark.parametrize("rows,d", [(1000, 256), (333, 768), (64, 1024)])
def test_rmsnorm_forward_backward(rows, d, x_f32):
    x = randn(rows, d) if x_f32 else bf(randn(rows, d))
    xdt = 0 if x_f32 else 4
    w = (1 + 0.1 * randn(d)).float()
    y = torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
    inv = torch.empty(rows, dtype=torch.float32, device=DEV)
    call("sj_rmsnorm_fwd", ptr(x), xdt, ptr(w), ptr(y), ptr(inv), rows, d, 1e-6, stream())
    ref = ops.rmsnorm(x.double().cpu(), w.double().cpu(), 1e-6)
    assert rel(y, ref) < 1e-2
    dz = randn(rows, d)
    dres0 = randn(rows, d)
    dres = dres0.clone()
    dres_b = torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
    dw = torch.zeros(d, device=DEV)
    from sejong_b200 import _lib
    partials = torch.empty(_lib.load().sj_rmsnorm_workspace(rows, d), device=DEV)
    call("sj_rmsnorm_bwd", ptr(x), xdt, ptr(w), ptr(inv), ptr(dz), ptr(dres), ptr(dres_b), ptr(dw), ptr(partials),
         rows, d, stream())
    torch.cuda.synchronize()
    rdx, rdw = ops.rmsnorm_backward(x.double().cpu(), w.double().cpu(), dz.double().cpu(), 1e-6)
    assert rel(dres - dres0, rdx) < 1e-4
    assert rel(dres_b, dres) < 1e-2
    assert rel(dw, rdw) < 1e-4


# ------------------------------------------------------------------------------------- attention
@pytest.mark.parametrize("b,t,hq,hk,window", [(8, 1024, 4, 4, 128), (20, 512, 6, 2, 0)])
def test_attention_more_items_than_sms(b, t, hq, hk, window):
    """The persistent forward and backward walk several work items per CTA (here 256 or more items
    on 148 SMs): outputs and gradients against an fp32 torch reference on the GPU, and no expired
    wait in the device error word."""
    d = 64
    n = b * t
    cq = (hq + 2 * hk) * d
    qkv = bf(randn(n, cq))
    ko, vo = hq * d, (hq + hk) * d
    o = torch.empty(n, hq * d, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(n * hq, dtype=torch.float32, device=DEV)
    call("sj_attn_gqa_fwd", ptr(qkv), cq, ptr(qkv, ko), cq, ptr(qkv, vo), cq, ptr(o), hq * d, ptr(lse), b, t, hq, hk,
         d, window, stream())
    do = bf(randn(n, hq * d))
    dqkv = torch.zeros(n, cq, dtype=torch.bfloat16, device=DEV)
    from sejong_b200 import _lib
    ws = torch.empty(_lib.load().sj_attn_workspace(b, t, hq, hk), dtype=torch.float32, device=DEV)
    call("sj_attn_gqa_bwd", ptr(qkv), cq, ptr(qkv, ko), cq, ptr(qkv, vo), cq, ptr(o), hq * d, ptr(lse), ptr(do),
         hq * d, ptr(dqkv), cq, ptr(dqkv, ko), cq, ptr(dqkv, vo), cq, ptr(ws), b, t, hq, hk, d, window, 0.0, 0, stream())
    torch.cuda.synchronize()
    check_device_error()
    # fp32 reference on the GPU
    q = qkv[:, :ko].float().reshape(b, t, hq, d).permute(0, 2, 1, 3).requires_grad_()
    k = qkv[:, ko:vo].float().reshape(b, t, hk, d).permute(0, 2, 1, 3).requires_grad_()
    v = qkv[:, vo:].float().reshape(b, t, hk, d).permute(0, 2, 1, 3).requires_grad_()
    kk, vv = k.repeat_interleave(hq // hk, dim=1), v.repeat_interleave(hq // hk, dim=1)
    s = q @ kk.transpose(-1, -2) * d ** -0.5
    pos = torch.arange(t, device=DEV)
    allowed = pos[None, :] <= pos[:, None]
    if window:
        allowed &= pos[None, :] > pos[:, None] - window
    s = s.masked_fill(~allowed, float("-inf"))
    ro = torch.softmax(s, dim=-1) @ vv
    rlse = torch.logsumexp(s, dim=-1)
    (ro * do.float().reshape(b, t, hq, d).permute(0, 2, 1, 3)).sum().backward()
    assert rel(o, ro.permute(0, 2, 1, 3).reshape(n, hq * d).detach()) < 2e-2
    assert float((lse - rlse.permute(0, 2, 1).reshape(-1)).abs().max()) < 2e-2
    assert rel(dqkv[:, :ko], q.grad.permute(0, 2, 1, 3).reshape(n, ko)) < 2e-2
    assert rel(dqkv[:, ko:vo], k.grad.permute(0, 2, 1, 3).reshape(n, hk * d)) < 2e-2
    assert rel(dqkv[:, vo:], v.grad.permute(0, 2, 1, 3).reshape(n, hk * d)) < 2e-2


@pytest.mark.parametrize("b,t,hq,hk,window", [(2, 128, 4, 2, 0), (1, 200, 4, 4, 0), (2, 256, 4, 4, 64),
                                              (1, 300, 6, 2, 100), (2, 512, 12, 4, 0), (1, 4096, 4, 4, 128),
                                              (3, 1000, 2, 2, 128), (2, 300, 2, 2, 100), (5, 700, 4, 4, 2)])
def test_attention_forward_backward(b, t, hq, hk, window):
    """Forward and backward against the FP64 restatement.  The windowed cases with one query head per
    kv head take the banded backward: (3, 1000, 2, 2, 128) has 48 key tiles, one per CTA, so every
    range starts with a halo step and ends with a query tile left to the next range; (2, 300, ...)
    ends on a partial tile; with window 2 most of each off-diagonal step is masked."""
    d = 64
    n = b * t
    cq = (hq + 2 * hk) * d
    qkv = bf(randn(n, cq))
    o = torch.empty(n, hq * d, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(n * hq, dtype=torch.float32, device=DEV)
    ko, vo = hq * d, (hq + hk) * d
    call("sj_attn_gqa_fwd", ptr(qkv), cq, ptr(qkv, ko), cq, ptr(qkv, vo), cq, ptr(o), hq * d, ptr(lse), b, t, hq, hk,
         d, window, stream())
    torch.cuda.synchronize()
    q = qkv[:, :ko].double().cpu().requires_grad_()
    k = qkv[:, ko:vo].double().cpu().requires_grad_()
    v = qkv[:, vo:].double().cpu().requires_grad_()
    ro, rlse = ops.grouped_attention(q, k, v, t, hq, hk, window or None)
    assert rel(o, ro.detach()) < 2e-2
    assert float((lse.double().cpu() - rlse.detach()).abs().max()) < 2e-2
    do = bf(randn(n, hq * d))
    (ro * do.double().cpu()).sum().backward()
    dqkv = torch.zeros(n, cq, dtype=torch.bfloat16, device=DEV)
    from sejong_b200 import _lib
    delta = torch.empty(_lib.load().sj_attn_workspace(b, t, hq, hk), dtype=torch.float32, device=DEV)
    call("sj_attn_gqa_bwd", ptr(qkv), cq, ptr(qkv, ko), cq, ptr(qkv, vo), cq, ptr(o), hq * d, ptr(lse), ptr(do),
         hq * d, ptr(dqkv), cq, ptr(dqkv, ko), cq, ptr(dqkv, vo), cq, ptr(delta), b, t, hq, hk, d, window, 0.0,
         0, stream())
    torch.cuda.synchronize()
    check_device_error()
    assert rel(dqkv[:, :ko], q.grad) < 2e-2
    assert rel(dqkv[:, ko:vo], k.grad) < 2e-2
    assert rel(dqkv[:, vo:], v.grad) < 2e-2


@pytest.mark.parametrize("b,t,hq,hk,window", [(1, 128, 2, 1, 0), (2, 384, 2, 2, 128)])
def test_attention_backward_inverse_rope(b, t, hq, hk, window):
    """dq and dk leave the kernel rotated back (table or inline angles); the second case runs the banded
    backward."""
    d = 64
    n, cq = b * t, (hq + 2 * hk) * 64
    qkv = bf(randn(n, cq))
    o = torch.empty(n, hq * d, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(n * hq, device=DEV)
    ko, vo = hq * d, (hq + hk) * d
    call("sj_attn_gqa_fwd", ptr(qkv), cq, ptr(qkv, ko), cq, ptr(qkv, vo), cq, ptr(o), hq * d, ptr(lse), b, t, hq, hk,
         d, window, stream())
    do = bf(randn(n, hq * d))
    table = torch.empty(t * 64, device=DEV)
    call("sj_rope_table", ptr(table), t, 64, 0, 10000.0, stream())
    outs = []
    for theta, tab in ((0.0, 0), (10000.0, 0), (0.0, ptr(table))):
        dqkv = torch.zeros(n, cq, dtype=torch.bfloat16, device=DEV)
        from sejong_b200 import _lib
        delta = torch.empty(_lib.load().sj_attn_workspace(b, t, hq, hk), device=DEV)
        call("sj_attn_gqa_bwd", ptr(qkv), cq, ptr(qkv, ko), cq, ptr(qkv, vo), cq, ptr(o), hq * d, ptr(lse), ptr(do),
             hq * d, ptr(dqkv), cq, ptr(dqkv, ko), cq, ptr(dqkv, vo), cq, ptr(delta), b, t, hq, hk, d, window, theta,
             tab, stream())
        outs.append(dqkv.double().cpu())
    plain = outs[0]
    for rotated in outs[1:]:
        assert rel(rotated[:, :ko], ops.rope(plain[:, :ko], t, 0, hq, 10000.0, inverse=True)) < 2e-2
        assert rel(rotated[:, ko:vo], ops.rope(plain[:, ko:vo], t, 0, hk, 10000.0, inverse=True)) < 2e-2
        assert rel(rotated[:, vo:], plain[:, vo:]) == 0.0


def test_rope_table_matches_reference_formula():
    t = 300
    table = torch.empty(t * 64, device=DEV)
    call("sj_rope_table", ptr(table), t, 64, 0, 10000.0, stream())
    torch.cuda.synchronize()
    tab = table.reshape(t, 32, 2).double().cpu()
    pos = torch.arange(t, dtype=torch.float64)[:, None]
    pair = torch.arange(32, dtype=torch.float64)[None, :]
    angle = pos * torch.exp((-2.0 * pair / 64) * np.log(10000.0))
    assert float((tab[..., 0] - torch.cos(angle)).abs().max()) < 5e-4
    assert float((tab[..., 1] - torch.sin(angle)).abs().max()) < 5e-4


# ------------------------------------------------------------------------------------- elementwise
def test_rope_standalone():
    rows, heads, t = 300, 3, 100
    x = bf(randn(rows, heads * 64))
    for inverse in (0, 1):
        y = torch.empty_like(x)
        call("sj_rope", ptr(x), ptr(y), rows, heads, 64, t, 0, 10000.0, inverse, stream())
        torch.cuda.synchronize()
        assert rel(y, ops.rope(x.double().cpu(), t, 0, heads, 10000.0, bool(inverse))) < 1e-2


def test_embedding_forward_backward():
    n, d = 5000, 256
    w = bf(randn(257, d))
    ids = torch.randint(0, 257, (n,), generator=GEN, dtype=torch.int32).to(DEV)
    ids[:1000] = 0  # a frequent byte
    y = torch.empty(n, d, dtype=torch.bfloat16, device=DEV)
    call("sj_embedding_fwd", ptr(w), ptr(ids), ptr(y), 4, n, d, 257, stream())
    y32 = torch.empty(n, d, dtype=torch.float32, device=DEV)
    call("sj_embedding_fwd", ptr(w), ptr(ids), ptr(y32), 0, n, d, 257, stream())
    torch.cuda.synchronize()
    assert torch.equal(y, w[ids.long()])
    assert torch.equal(y32, w[ids.long()].float())
    dy = randn(n, d)
    dw = torch.zeros(257, d, device=DEV)
    call("sj_embedding_bwd", ptr(dy), ptr(ids), ptr(dw), n, d, 257, stream())
    torch.cuda.synchronize()
    assert rel(dw, ops.embedding_backward(dy.double().cpu(), ids.cpu(), 257)) < 1e-5


def test_swiglu_backward():
    from sejong_b200.model import _deinterleave_cols
    rows, f = 300, 768
    gu = bf(randn(rows, 2 * f))
    dh = bf(randn(rows, f))
    dgu = torch.empty_like(gu)
    call("sj_swiglu_bwd", ptr(gu), ptr(dh), ptr(dgu), rows, f, stream())
    torch.cuda.synchronize()
    g, u = _deinterleave_cols(gu.float().cpu().numpy())
    dg_ref, du_ref = ops.swiglu_backward(torch.from_numpy(g).double(), torch.from_numpy(u).double(), dh.double().cpu())
    dg, du = _deinterleave_cols(dgu.float().cpu().numpy())
    assert rel(torch.from_numpy(dg), dg_ref) < 1e-2
    assert rel(torch.from_numpy(du), du_ref) < 1e-2


@pytest.mark.parametrize("t,patch", [(64, 8), (100, 8)])
def test_patch_pool_and_broadcast(t, patch):
    b, d = 3, 256
    patches = -(-t // patch)
    x = bf(randn(b * t, d))
    y = torch.empty(b * patches, d, dtype=torch.bfloat16, device=DEV)
    call("sj_patch_pool_fwd", ptr(x), ptr(y), b, t, d, patch, stream())
    torch.cuda.synchronize()
    assert rel(y, ops.patch_pool(x.double().cpu(), t, patch)) < 1e-2
    dy = randn(b * patches, d)
    dx0 = randn(b * t, d)
    dx = dx0.clone()
    call("sj_patch_pool_bwd", ptr(dy), ptr(dx), b, t, d, patch, stream())
    xx = x.double().cpu().requires_grad_()
    (ops.patch_pool(xx, t, patch) * dy.double().cpu()).sum().backward()
    torch.cuda.synchronize()
    assert rel(dx - dx0, xx.grad) < 1e-5
    z = bf(randn(b * patches, d))
    bos = bf(randn(1, d))
    base = bf(randn(b * t, d))
    yb = base.clone()
    call("sj_patch_broadcast_fwd", ptr(z), ptr(bos), ptr(yb), 4, 1, b, t, d, patch, stream())
    y32 = base.float().clone()
    call("sj_patch_broadcast_fwd", ptr(z), ptr(bos), ptr(y32), 0, 1, b, t, d, patch, stream())
    torch.cuda.synchronize()
    ref = base.double().cpu() + ops.patch_broadcast(z.double().cpu(), bos.double().cpu(), t, patch)
    assert rel(y32, ref) < 1e-6
    assert rel(yb, ref) < 1e-2
    dyb = randn(b * t, d)
    dz = torch.empty(b * patches, d, dtype=torch.bfloat16, device=DEV)
    dbos = torch.empty(d, dtype=torch.bfloat16, device=DEV)
    call("sj_patch_broadcast_bwd", ptr(dyb), ptr(dz), ptr(dbos), b, t, d, patch, stream())
    zz = z.double().cpu().requires_grad_()
    bb = bos.double().cpu().requires_grad_()
    (ops.patch_broadcast(zz, bb, t, patch) * dyb.double().cpu()).sum().backward()
    torch.cuda.synchronize()
    assert rel(dz, zz.grad) < 1e-2
    assert rel(dbos, bb.grad.reshape(-1)) < 1e-2


def test_cross_entropy_fused():
    rows, ld = 1000, 264
    logits = randn(rows, ld, scale=3.0)
    targets = torch.randint(0, 257, (rows,), generator=GEN, dtype=torch.int32).to(DEV)
    loss_rows = torch.empty(rows, device=DEV)
    dl = torch.empty(rows, ld, dtype=torch.bfloat16, device=DEV)
    total = torch.zeros(1, dtype=torch.float64, device=DEV)
    seed = 1.0 / rows
    call("sj_cross_entropy", ptr(logits), ld, ptr(targets), rows, 257, seed, ptr(loss_rows), ptr(dl), ld, ptr(total),
         1.0 / rows, stream())
    torch.cuda.synchronize()
    x = logits[:, :257].double().cpu()
    ref = ops.cross_entropy(x, targets.cpu())
    assert rel(loss_rows, ref) < 1e-5
    assert abs(float(total) - float(ref.mean())) < 1e-6
    g = ops.cross_entropy_backward(x, targets.cpu(), torch.full((rows,), seed, dtype=torch.float64))
    assert rel(dl[:, :257], g) < 1e-2
    assert float(dl[:, 257:].float().abs().max()) == 0.0


def test_adamw_and_grad_norm():
    n, n_decay = 100003, 60000
    w, g = randn(n), randn(n, scale=0.01)
    m, v = randn(n, scale=0.001), randn(n, scale=0.001).abs() * 1e-3
    w0, m0, v0 = w.clone(), m.clone(), v.clone()
    wb = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    from sejong_b200 import _lib
    parts = _lib.load().sj_sumsq_partials(n)
    partials = torch.zeros(parts, dtype=torch.float64, device=DEV)
    state = torch.tensor([4.0, 0.0], dtype=torch.float64, device=DEV)  # 4 steps already taken
    hyper = torch.zeros(8, device=DEV)
    call("sj_grad_sumsq", ptr(g), n, ptr(partials), stream())
    call("sj_optim_prepare", ptr(partials), parts, ptr(state), ptr(hyper), 3e-4, 3e-5, 0, 10, 0.9, 0.95, 1.0, 1, 1.0,
         stream())
    call("sj_adamw", ptr(w), ptr(g), ptr(m), ptr(v), ptr(wb), n, n_decay, ptr(hyper), 0.9, 0.95, 1e-8, 0.1, stream())
    torch.cuda.synchronize()
    norm = float(g.double().norm())
    assert abs(float(hyper[4]) - norm) < 1e-4 * norm
    assert float(state[0]) == 5.0
    lr = ops.lr_schedule(4, 3e-4, 3e-5, 0, 10)
    assert abs(float(hyper[0]) - lr) < 1e-9 + 1e-6 * lr
    scale = 1.0 / norm if norm > 1.0 else 1.0
    decay = torch.zeros(n, dtype=torch.float64)
    decay[:n_decay] = 0.1
    rw, rm, rv = ops.adamw(w0.double().cpu(), g.double().cpu(), m0.double().cpu(), v0.double().cpu(), 5, lr, 0.9, 0.95,
                           1e-8, decay, scale)
    assert rel(m, rm) < 1e-5 and rel(v, rv) < 1e-5
    assert float((w.double().cpu() - rw).abs().max()) < 1e-6
    assert rel(wb, w) < 1e-2
