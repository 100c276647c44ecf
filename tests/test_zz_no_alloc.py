"""sj_rmsnorm_bwd_noalloc (the RMSNorm backward whose dw partials live in a fixed array inside the
library's device image) against sj_rmsnorm_bwd with a caller-owned workspace.

Both run the same kernels in the same order, so the results must agree to the tolerance the
kernel tests use for f32 outputs (1e-4 relative L2); two calls in a row with different inputs show
that nothing left in the fixed array from the first call leaks into the second.  The file name
makes pytest collect it last, so it also runs after every other GPU test in the same process.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def call(name, *args):
    from sejong_b200 import _lib
    return _lib.call(name, *args)


def ptr(t):
    return t.data_ptr()


def stream():
    return torch.cuda.current_stream().cuda_stream


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / max(b.norm(), 1e-30))


def free_bytes():
    free, total = ctypes.c_size_t(0), ctypes.c_size_t(0)
    call("sj_mem_info", ctypes.byref(free), ctypes.byref(total))
    return free.value


def inputs(gen, rows, d, x_f32):
    x = torch.randn(rows, d, generator=gen).to(DEV)
    if not x_f32:
        x = x.to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(d, generator=gen)).float().to(DEV)
    dz = torch.randn(rows, d, generator=gen).to(DEV)
    dres = torch.randn(rows, d, generator=gen).to(DEV)
    inv = torch.rsqrt(x.float().pow(2).mean(1) + 1e-6).contiguous()
    return x, w, inv, dz, dres


def with_workspace(x, xdt, w, inv, dz, dres0, rows, d):
    from sejong_b200 import _lib
    dres, dres_b = dres0.clone(), torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
    dw = torch.full((d,), 0.5, device=DEV)
    partials = torch.empty(_lib.load().sj_rmsnorm_workspace(rows, d), device=DEV)
    call("sj_rmsnorm_bwd", ptr(x), xdt, ptr(w), ptr(inv), ptr(dz), ptr(dres), ptr(dres_b), ptr(dw), ptr(partials),
         rows, d, stream())
    return dres, dres_b, dw


@pytest.mark.parametrize("rows,d,x_f32", [(1000, 768, False), (4096, 256, True), (77, 1024, False)])
def test_noalloc_matches_workspace_twice(rows, d, x_f32):
    from sejong_b200 import _lib
    _lib.load()
    call("sj_device_init", 0)
    gen = torch.Generator().manual_seed(rows * 31 + d)
    xdt = 0 if x_f32 else 4
    for attempt in range(2):
        x, w, inv, dz, dres0 = inputs(gen, rows, d, x_f32)
        ref_dres, ref_dres_b, ref_dw = with_workspace(x, xdt, w, inv, dz, dres0, rows, d)
        dres, dres_b = dres0.clone(), torch.empty(rows, d, dtype=torch.bfloat16, device=DEV)
        dw = torch.full((d,), 0.5, device=DEV)
        torch.cuda.synchronize()
        before, reserved = free_bytes(), torch.cuda.memory_reserved()
        call("sj_rmsnorm_bwd_noalloc", ptr(x), xdt, ptr(w), ptr(inv), ptr(dz), ptr(dres), ptr(dres_b), ptr(dw),
             rows, d, stream())
        torch.cuda.synchronize()
        if attempt == 1:
            # torch's caching allocator was not asked for memory, and the device's free memory did not
            # drop by a cudaMalloc's smallest granule (2 MiB); other processes on a shared GPU may move
            # the device-wide figure a little, so it is not compared exactly
            assert torch.cuda.memory_reserved() == reserved, "torch allocated during the no-allocation call"
            assert before - free_bytes() < (2 << 20), "the no-allocation entry point took device memory"
        assert rel(dres, ref_dres) < 1e-4
        assert rel(dres_b, ref_dres_b) < 1e-2
        assert rel(dw, ref_dw) < 1e-4


def test_noalloc_rejects_shapes_above_the_limit():
    from sejong_b200 import _lib
    lib = _lib.load()
    limit = lib.sj_rmsnorm_noalloc_limit()
    d = 1024
    rows = (limit // d + 1) * 32  # one 32-row group more than the array holds
    assert lib.sj_rmsnorm_workspace(rows, d) > limit
    status = lib.sj_rmsnorm_bwd_noalloc(None, 4, None, None, None, None, None, None, rows, d, None)
    assert status == _lib.SJ_ERR_CAPACITY
    assert b"static limit" in lib.sj_last_error()
