"""The f32 step (BASELINE C1, "one training step in fp32") on the GPU.

* sj_sgemm against an FP64 product for every operand orientation and epilogue (STORE, ACCUM,
  RESIDUAL, ROPE, SWIGLU), ragged shapes included: 1e-5 relative L2 (f32 accumulation).
* sj_attn_f32_fwd / _bwd against the FP64 restatement of hierarchy.py (oracle.ops.grouped_attention,
  pinned to the reference's own kernels): causal GQA with and without a window, a sequence that is
  not a multiple of the 64-row block; O within the reference's 2e-5 absolute attention bar.
* The whole C1 step against the FP64 oracle with no cast (the reference's F32 precision binds the
  f32 weights): loss within 2e-5, every gradient within 1e-4 relative L2, the AdamW update within
  2e-6 of the FP64 transition, and a captured graph replays it.
"""
import numpy as np
import pytest
import torch

from oracle import model as omodel
from oracle import ops
from oracle.corpus import synthetic_corpus
from oracle.rng import Rng

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _rel(a, b):
    a = torch.as_tensor(a, dtype=torch.float64)
    b = torch.as_tensor(b, dtype=torch.float64)
    return float((a - b).norm() / b.norm())


def _rope_table(t, theta=10000.0):
    from sejong_b200._lib import call
    tab = torch.empty(t * 64, device="cuda")
    call("sj_rope_table", tab.data_ptr(), t, 64, 0, theta, _stream())
    return tab


@pytest.mark.parametrize("m,n,k,a_t,b_t", [(300, 200, 100, 0, 0), (128, 256, 64, 1, 0), (77, 130, 257, 0, 1),
                                           (256, 96, 512, 1, 1), (256, 264, 4096, 1, 0), (4096, 512, 256, 0, 0)])
@pytest.mark.parametrize("epi", ["store", "accum", "residual"])
def test_sgemm_orientations_and_epilogues(m, n, k, a_t, b_t, epi):
    from sejong_b200._lib import EPI_ACCUM, EPI_RESIDUAL, EPI_STORE, call
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g, dtype=torch.float64)
    b = torch.randn(k, n, generator=g, dtype=torch.float64)
    ad = (a.t() if a_t else a).contiguous().float().cuda()
    bd = (b.t() if b_t else b).contiguous().float().cuda()
    base = torch.randn(m, n, generator=g, dtype=torch.float64)
    c = base.float().cuda()
    aux = torch.randn(m, n, generator=g, dtype=torch.float64)
    auxd = aux.float().cuda()
    code = {"store": EPI_STORE, "accum": EPI_ACCUM, "residual": EPI_RESIDUAL}[epi]
    call("sj_sgemm", ad.data_ptr(), ad.shape[1], a_t, bd.data_ptr(), bd.shape[1], b_t, c.data_ptr(), n, m, n, k, code,
         auxd.data_ptr() if epi == "residual" else 0, n if epi == "residual" else 0, 0, 0, 0, _stream())
    torch.cuda.synchronize()
    ref = a @ b
    if epi == "accum":
        ref = ref + base
    if epi == "residual":
        ref = ref + aux
    assert _rel(c.cpu(), ref) < 1e-5


def test_sgemm_rope_and_swiglu_epilogues():
    from sejong_b200._lib import EPI_ROPE, EPI_SWIGLU, call
    g = torch.Generator().manual_seed(4)
    m, k, t = 200, 96, 50
    a = torch.randn(m, k, generator=g, dtype=torch.float64)
    b = torch.randn(k, 192, generator=g, dtype=torch.float64)
    tab = _rope_table(t)
    ad, bd = a.float().cuda(), b.float().cuda()  # kept alive until the kernels have run
    c = torch.empty(m, 192, device="cuda")
    call("sj_sgemm", ad.data_ptr(), k, 0, bd.data_ptr(), 192, 0, c.data_ptr(), 192, m, 192, k, EPI_ROPE, 0, 0,
         tab.data_ptr(), 128, t, _stream())
    torch.cuda.synchronize()
    ref = (a @ b).clone()
    tb = tab.cpu().double().reshape(t, 32, 2)
    pos = torch.arange(m) % t
    for h in range(2):
        x = ref[:, h * 64:(h + 1) * 64].reshape(m, 32, 2).clone()
        cs, sn = tb[pos, :, 0], tb[pos, :, 1]
        ref[:, h * 64:(h + 1) * 64] = torch.stack([x[..., 0] * cs - x[..., 1] * sn,
                                                   x[..., 0] * sn + x[..., 1] * cs], -1).reshape(m, 64)
    assert _rel(c.cpu(), ref) < 1e-5
    # SwiGLU: blocks of 16 gate | 16 up columns, h = silu(g) u
    f = 160
    b2 = torch.randn(k, 2 * f, generator=g, dtype=torch.float64)
    b2d = b2.float().cuda()
    gu = torch.empty(m, 2 * f, device="cuda")
    h = torch.empty(m, f, device="cuda")
    call("sj_sgemm", ad.data_ptr(), k, 0, b2d.data_ptr(), 2 * f, 0, gu.data_ptr(), 2 * f, m, 2 * f, k, EPI_SWIGLU,
         h.data_ptr(), f, 0, 0, 0, _stream())
    torch.cuda.synchronize()
    ref = a @ b2
    assert _rel(gu.cpu(), ref) < 1e-5
    blocks = ref.reshape(m, f // 16, 2, 16)
    gate, up = blocks[:, :, 0].reshape(m, f), blocks[:, :, 1].reshape(m, f)
    assert _rel(h.cpu(), torch.nn.functional.silu(gate) * up) < 1e-5


@pytest.mark.parametrize("t,hq,hk,window", [(200, 4, 2, 0), (256, 4, 1, 0), (192, 2, 2, 48)])
def test_attention_f32_against_the_fp64_restatement(t, hq, hk, window):
    from sejong_b200._lib import call
    b, d = 2, 64
    rows = b * t
    g = torch.Generator().manual_seed(t + hq + window)
    q = torch.randn(rows, hq * d, generator=g, dtype=torch.float64, requires_grad=True)
    k = torch.randn(rows, hk * d, generator=g, dtype=torch.float64, requires_grad=True)
    v = torch.randn(rows, hk * d, generator=g, dtype=torch.float64, requires_grad=True)
    o_ref, lse_ref = ops.grouped_attention(q, k, v, t, hq, hk, window or None)
    dout = torch.randn(rows, hq * d, generator=g, dtype=torch.float64)
    (o_ref * dout).sum().backward()
    cq = (hq + 2 * hk) * d
    qkv = torch.cat([q, k, v], 1).detach().float().cuda().contiguous()
    o = torch.empty(rows, hq * d, device="cuda")
    lse = torch.empty(rows * hq, device="cuda")
    s = _stream()
    call("sj_attn_f32_fwd", qkv.data_ptr(), cq, qkv.data_ptr() + hq * d * 4, cq, qkv.data_ptr() + (hq + hk) * d * 4,
         cq, o.data_ptr(), hq * d, lse.data_ptr(), b, t, hq, hk, d, window, s)
    ident = torch.zeros(t, 32, 2, device="cuda")
    ident[..., 0] = 1.0  # cos 1, sin 0: the inverse rotation is the identity
    dqkv = torch.empty(rows, cq, device="cuda")
    from sejong_b200 import _lib
    ws = torch.empty(_lib.load().sj_attn_f32_workspace(b, t, hq), device="cuda")
    dod = dout.float().cuda()
    call("sj_attn_f32_bwd", qkv.data_ptr(), cq, qkv.data_ptr() + hq * d * 4, cq, qkv.data_ptr() + (hq + hk) * d * 4,
         cq, o.data_ptr(), hq * d, lse.data_ptr(), dod.data_ptr(), hq * d, dqkv.data_ptr(), cq,
         dqkv.data_ptr() + hq * d * 4, cq, dqkv.data_ptr() + (hq + hk) * d * 4, cq, ws.data_ptr(), b, t, hq, hk, d,
         window, ident.data_ptr(), s)
    torch.cuda.synchronize()
    assert float((o.cpu().double() - o_ref.detach()).abs().max()) < 2e-5
    assert float((lse.cpu().double() - lse_ref.detach()).abs().max()) < 2e-5
    dq, dk, dv = dqkv.cpu().double().split([hq * d, hk * d, hk * d], 1)
    assert _rel(dq, q.grad) < 1e-5 and _rel(dk, k.grad) < 1e-5 and _rel(dv, v.grad) < 1e-5


def _oracle_config(c):
    return omodel.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                              kv_heads=c.kv_heads, rope_theta=c.rope_theta, norm_epsilon=c.norm_epsilon, seed=c.seed,
                              init_std=c.init_std)


def test_f32_step_matches_the_fp64_oracle():
    from sejong_b200 import model as pm
    from sejong_b200.train import TrainConfig
    from sejong_b200.train_f32 import F32Trainer
    c = pm.config_c1()
    batch, seq = 2, 512
    ids, tg = synthetic_corpus(5, 200000).batch(Rng(77), batch, seq)
    params = pm.initialize(c)
    tc = TrainConfig(sequence=seq, batch=batch, warmup_steps=0, steps=100)
    tr = F32Trainer(c, tc, device=0, params=params)
    tr.stage_batch(ids, tg)
    tr.forward_backward()
    torch.cuda.synchronize()
    assert tr.device_error() == 0
    loss, grads = tr.loss(), tr.gradients()
    ref_loss, ref = omodel.loss_and_grads(params, _oracle_config(c), ids, tg, seq)
    assert abs(loss - ref_loss) < 2e-5, (loss, ref_loss)
    worst = {k: _rel(grads[k], ref[k]) for k in ref if np.any(ref[k] != 0)}
    print("f32 step: loss", loss, ref_loss, "worst", sorted(worst.items(), key=lambda kv: -kv[1])[:4])
    assert max(worst.values()) < 1e-4, sorted(worst.items(), key=lambda kv: -kv[1])[:4]
    tr.optimizer_step()
    torch.cuda.synchronize()
    new = tr.parameters()
    otc = omodel.TrainConfig(sequence=seq, batch=batch, warmup_steps=0, steps=100)
    ref_new, norm = omodel.adam_update(params, {k: v.astype(np.float64) for k, v in grads.items()},
                                       omodel.AdamState(), otc)
    assert abs(float(tr.hyper[4]) - norm) < 1e-5 * max(norm, 1.0)
    for k in params:
        assert float(np.max(np.abs(new[k] - ref_new[k]))) < 2e-6, k
    tr.capture()
    for _ in range(2):
        tr.replay()
    torch.cuda.synchronize()
    assert tr.device_error() == 0 and np.isfinite(tr.loss())
