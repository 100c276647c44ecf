"""MoE kernels on the GPU: routing ids bit-exact against the reference's own kernels (golden vectors,
ties included), the device-side pack against the reference's per-expert slot order, the router
backward, both grouped GEMM modes against fp32 (uneven and empty experts), and the dispatch /
combine data movement with their backwards."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))


def g(name):
    return GOLDEN[f"route/{name}"]


def st():
    return torch.cuda.current_stream().cuda_stream


def lib():
    from sejong_b200 import _lib
    return _lib.load()


def call(*a):
    from sejong_b200._lib import call as c
    return c(*a)


def route(logits, k):
    rows, e = logits.shape
    ld = logits.cuda().float().contiguous()
    ids = torch.empty(rows, k, dtype=torch.int32, device="cuda")
    gates = torch.empty(rows, k, device="cuda")
    call("sj_route_topk", ld.data_ptr(), e, rows, e, k, ids.data_ptr(), gates.data_ptr(), st())
    return ld, ids, gates


def pack(ids, experts):
    rows, k = ids.shape
    cap = lib().sj_moe_capacity(rows, k, experts)
    group_rows = torch.empty(experts + 1, dtype=torch.int32, device="cuda")
    pos = torch.empty(rows * k, dtype=torch.int32, device="cuda")
    row_slot = torch.empty(cap, dtype=torch.int32, device="cuda")
    call("sj_route_pack", ids.data_ptr(), rows, experts, k, group_rows.data_ptr(), pos.data_ptr(), row_slot.data_ptr(),
         cap, st())
    return cap, group_rows, pos, row_slot


def test_route_topk_matches_the_reference_kernel():
    k = int(g("k"))
    _, ids, gates = route(torch.from_numpy(g("logits")), k)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), g("ids"))
    np.testing.assert_allclose(gates.cpu().numpy(), g("gates"), rtol=1e-6, atol=1e-7)


def test_route_pack_matches_the_reference_order():
    k = int(g("k"))
    ids = torch.from_numpy(g("ids")).cuda()
    e = g("counts").size
    cap, group_rows, pos, row_slot = pack(ids, e)
    torch.cuda.synchronize()
    gr, ps, rs = group_rows.cpu().numpy(), pos.cpu().numpy(), row_slot.cpu().numpy()
    r = ids.numel()
    counts, slots = g("counts"), g("slots")
    assert gr[0] == 0 and np.all(np.diff(gr) % 128 == 0)
    for x in range(e):
        n = int(counts[x])
        seg = rs[gr[x]:gr[x + 1]]
        assert np.array_equal(seg[:n], slots[x * r:x * r + n])          # the reference's slot order
        assert np.all(seg[n:] == -1)                                     # padding routes nowhere
        assert np.array_equal(ps[seg[:n]], np.arange(gr[x], gr[x] + n))  # pos inverts row_slot
    assert np.all(rs[gr[e]:] == -1)


def test_route_backward_matches_the_reference_kernel():
    k = int(g("k"))
    logits = torch.from_numpy(g("logits"))
    rows, e = logits.shape
    ld, ids, gates = route(logits, k)
    dy = torch.from_numpy(g("dy")).cuda().float().contiguous()
    dl = torch.empty(rows, 8, dtype=torch.bfloat16, device="cuda")
    call("sj_route_topk_bwd", ld.data_ptr(), e, ids.data_ptr(), gates.data_ptr(), dy.data_ptr(), dl.data_ptr(), 8, rows,
         e, k, st())
    torch.cuda.synchronize()
    got = dl.float().cpu().numpy()
    np.testing.assert_allclose(got[:, :e], g("dx"), rtol=1e-2, atol=1e-3)
    assert np.all(got[:, e:] == 0)


def _segments(counts):
    gr = [0]
    for c in counts:
        gr.append(gr[-1] + (c + 127) // 128 * 128)
    return gr


@pytest.mark.parametrize("counts", [[300, 0, 129, 37], [128, 128, 1, 5, 700]])
def test_grouped_gemm_rows_and_reduction(counts):
    from sejong_b200._lib import EPI_ACCUM, EPI_STORE, SJ_BF16, SJ_F32
    torch.manual_seed(sum(counts))
    G, d, n = len(counts), 256, 320
    gr = _segments(counts)
    cap = gr[-1]
    a = torch.zeros(cap, d)
    for x in range(G):
        a[gr[x]:gr[x] + counts[x]] = torch.randn(counts[x], d)
    a = a.bfloat16()
    w = (0.05 * torch.randn(G * d, n)).bfloat16()       # B [k, n] per group, stacked along k
    ad, wd = a.cuda(), w.cuda()
    grd = torch.tensor(gr, dtype=torch.int32, device="cuda")
    c = torch.full((cap, n), float("nan"), device="cuda")
    call("sj_gemm_grouped", ad.data_ptr(), d, 0, wd.data_ptr(), n, 0, c.data_ptr(), n, SJ_F32, cap, n, d, EPI_STORE, 0, 0,
         G, grd.data_ptr(), 1, d, 0, st())
    # grouped reduction: C_g += A_g^T Y_g
    y = torch.zeros(cap, n)
    for x in range(G):
        y[gr[x]:gr[x] + counts[x]] = torch.randn(counts[x], n)
    y = y.bfloat16()
    yd = y.cuda()
    dw = torch.ones(G * d, n, device="cuda")
    call("sj_gemm_grouped", ad.data_ptr(), d, 1, yd.data_ptr(), n, 0, dw.data_ptr(), n, SJ_F32, d, n, cap, EPI_ACCUM, 0,
         0, G, grd.data_ptr(), 2, 0, d, st())
    torch.cuda.synchronize()
    got, gdw = c.cpu(), dw.cpu()
    for x in range(G):
        rows = slice(gr[x], gr[x] + counts[x])
        ref = a[rows].float() @ w[x * d:(x + 1) * d].float()
        if counts[x]:
            assert float((got[rows] - ref).norm() / ref.norm()) < 1e-4, x
        refw = 1 + a[rows].float().T @ y[rows].float()
        assert float((gdw[x * d:(x + 1) * d] - refw).abs().max()) < 1e-3 * max(1.0, float(refw.abs().max())), x


def test_dispatch_combine_and_backwards():
    torch.manual_seed(3)
    rows, E, k, d = 200, 6, 2, 128
    logits = torch.randn(rows, E)
    ld, ids, gates = route(logits, k)
    cap, group_rows, pos, row_slot = pack(ids, E)
    z = torch.randn(rows, d).bfloat16().cuda()
    a = torch.full((cap, d), 7.0, dtype=torch.bfloat16, device="cuda")
    call("sj_moe_dispatch", z.data_ptr(), d, row_slot.data_ptr(), cap, k, d, a.data_ptr(), st())
    out = torch.randn(cap, d).bfloat16().cuda()
    x = torch.randn(rows, d, device="cuda")
    y = torch.empty(rows, d, device="cuda")
    call("sj_moe_combine", out.data_ptr(), pos.data_ptr(), gates.data_ptr(), x.data_ptr(), y.data_ptr(), rows, k, d, st())
    dy = torch.randn(rows, d, device="cuda")
    d_out = torch.empty(cap, d, dtype=torch.bfloat16, device="cuda")
    d_gates = torch.empty(rows * k, device="cuda")
    call("sj_moe_combine_bwd", out.data_ptr(), row_slot.data_ptr(), gates.data_ptr(), dy.data_ptr(), d_out.data_ptr(),
         d_gates.data_ptr(), cap, k, d, st())
    da = torch.randn(cap, d, device="cuda")
    dz = torch.empty(rows, d, device="cuda")
    call("sj_moe_dispatch_bwd", da.data_ptr(), pos.data_ptr(), dz.data_ptr(), d, rows, k, d, st())
    torch.cuda.synchronize()
    rs, ps = row_slot.cpu(), pos.cpu().long()
    valid = rs >= 0
    tok = (rs[valid] // k).long()
    assert torch.equal(a.cpu()[valid], z.cpu()[tok]) and torch.all(a.cpu()[~valid] == 0)
    gsel = gates.cpu().reshape(-1)
    ref = x.cpu() + (gsel.reshape(rows, k, 1) * out.cpu().float()[ps].reshape(rows, k, d)).sum(1)
    assert float((y.cpu() - ref).abs().max()) < 1e-4
    ref_dout = torch.zeros(cap, d)
    ref_dout[valid] = gsel[rs[valid].long()][:, None] * dy.cpu()[tok]
    assert float((d_out.cpu().float() - ref_dout).abs().max()) < 2e-2 * float(ref_dout.abs().max())
    ref_dg = (out.cpu().float()[ps].reshape(rows * k, d) * dy.cpu().repeat_interleave(k, 0)).sum(1)
    assert float((d_gates.cpu() - ref_dg).abs().max()) < 1e-3 * float(ref_dg.abs().max())
    ref_dz = da.cpu()[ps].reshape(rows, k, d).sum(1)
    assert float((dz.cpu() - ref_dz).abs().max()) < 1e-5


def test_grouped_gemm_at_c5_shapes():
    """The C5 expert projections at their full size (8 experts, top-2 of 4,096 patch rows, d 1024,
    FFN 2816): gate/up with the SwiGLU epilogue and down, on the device-side layout of a real
    routing; checked against fp32 products on a sample of rows of every expert."""
    from sejong_b200._lib import EPI_STORE, EPI_SWIGLU, SJ_BF16
    torch.manual_seed(11)
    rows, E, k, d, f = 4096, 8, 2, 1024, 2816
    _, ids, _ = route(torch.randn(rows, E), k)
    cap, group_rows, pos, row_slot = pack(ids, E)
    a = (0.5 * torch.randn(cap, d)).bfloat16().cuda()
    wgu = (0.02 * torch.randn(E * d, 2 * f)).bfloat16().cuda()
    wd = (0.02 * torch.randn(E * f, d)).bfloat16().cuda()
    gu = torch.empty(cap, 2 * f, dtype=torch.bfloat16, device="cuda")
    h = torch.empty(cap, f, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(cap, d, dtype=torch.bfloat16, device="cuda")
    gp = group_rows.data_ptr()
    call("sj_gemm_grouped", a.data_ptr(), d, 0, wgu.data_ptr(), 2 * f, 0, gu.data_ptr(), 2 * f, SJ_BF16, cap, 2 * f, d,
         EPI_SWIGLU, h.data_ptr(), f, E, gp, 1, d, 0, st())
    call("sj_gemm_grouped", h.data_ptr(), f, 0, wd.data_ptr(), d, 0, out.data_ptr(), d, SJ_BF16, cap, d, f, EPI_STORE,
         0, 0, E, gp, 1, f, 0, st())
    torch.cuda.synchronize()
    gr = group_rows.cpu().numpy()
    for x in range(E):
        lo, hi = int(gr[x]), int(gr[x + 1])
        if hi <= lo:
            continue
        sample = torch.arange(lo, hi, max(1, (hi - lo) // 16)).cuda()
        ref = a[sample].float() @ wgu[x * d:(x + 1) * d].float()
        assert float((gu[sample].float() - ref).norm() / ref.norm()) < 2e-2, x
        refo = h[sample].float() @ wd[x * f:(x + 1) * f].float()
        assert float((out[sample].float() - refo).norm() / refo.norm()) < 2e-2, x


def test_capacity_and_aux_kernels_match_the_restatement():
    """sj_route_capacity drops exactly the slots of oracle.model.apply_capacity; sj_moe_aux adds the
    restated loss to the loss sum and its gradient (closed form) to the router gradient."""
    import math

    from oracle import model as om
    from oracle import ops as oops
    rows, k, E, w = 4096, 2, 8, 0.01
    gen = torch.Generator().manual_seed(5)
    logits = (0.2 * torch.randn(rows, E, generator=gen)).float()
    ld = 8
    dl = logits.cuda().contiguous()
    ids = torch.empty(rows, k, dtype=torch.int32, device="cuda")
    gates = torch.empty(rows, k, dtype=torch.float32, device="cuda")
    call("sj_route_topk", dl.data_ptr(), ld, rows, E, k, ids.data_ptr(), gates.data_ptr(), st())
    cap = (rows * k) // E - 200   # below the balanced load: some experts must drop slots
    call("sj_route_capacity", ids.data_ptr(), rows, k, E, cap, st())
    torch.cuda.synchronize()
    _, ids_ref = oops.route_topk(logits.double(), k)
    want = om.apply_capacity(ids_ref, E, cap)
    got = ids.cpu().long()
    assert torch.equal(got, want)
    assert (got == -1).sum() > 0
    # aux: loss and gradient increments
    dlog = (0.01 * torch.randn(rows, ld, generator=gen)).to(torch.bfloat16).cuda()
    before = dlog.float().cpu()
    loss = torch.zeros(1, dtype=torch.float64, device="cuda")
    ws = torch.empty(lib().sj_moe_aux_workspace(rows, E), device="cuda")
    call("sj_moe_aux", dl.data_ptr(), ld, rows, E, k, w, 0.5, loss.data_ptr(), dlog.data_ptr(), ld, 2.0, ws.data_ptr(),
         st())
    torch.cuda.synchronize()
    lg = logits.double().clone().requires_grad_(True)
    ref = om.aux_loss(lg, ids_ref, E, w)
    ref.backward()
    assert abs(float(loss[0]) - 0.5 * float(ref.detach())) < 1e-6 * float(ref.detach())
    inc = dlog.float().cpu() - before
    want_inc = 2.0 * lg.grad.float()
    assert float((inc[:, :E] - want_inc).abs().max()) < 1e-2 * float(want_inc.abs().max()) + 2e-5
