"""MiniLM encoder forward (BASELINE C2): initialisation and inputs on the CPU; on the GPU each new
kernel (bias / GELU / residual GEMM epilogues, embedding + LayerNorm, LayerNorm, single-tile
attention) against an fp32 or FP64 reference, the whole encoder against the FP64 restatement of
BertEncoder::hidden (oracle/bert.py) at the bf16 bar (2e-2 relative), and at the full C2 size the
property that packing a batch changes nothing: every sequence's rows equal those of the sequence
encoded alone, bit for bit."""
import ctypes

import numpy as np
import pytest

from oracle import bert as obert
from oracle import ops
from oracle.rng import Rng
from sejong_b200 import bert

SMALL = dict(layers=2)


def test_initialize_draws_the_reference_rng():
    c = bert.MiniLMConfig(vocab=1200, max_position=64, **SMALL)
    params = bert.initialize(c)
    rng = Rng(c.seed)
    for name, shape, kind in bert.bert_layout(c):
        if kind == "matrix":
            want = (rng.bulk_normal(int(np.prod(shape))) * np.float32(c.init_std)).astype(np.float32)
            # Box-Muller through the C library's log / cos: equal to the numpy restatement within 1 ulp
            np.testing.assert_allclose(params[name].reshape(-1), want, rtol=2e-6, atol=1e-9, err_msg=name)
        elif kind == "ln_weight":
            assert np.all(params[name] == 1)
        else:
            assert np.all(params[name] == 0)


def test_synthetic_batch_follows_the_c2_spec():
    seqs = bert.synthetic_batch(11, 64)
    rng = Rng(11)
    for s in seqs:
        n = 16 + rng.index(113)
        assert len(s) == n and s[0] == bert.CLS and s[-1] == bert.SEP
        body = np.array([1000 + rng.index(30522 - 1000) for _ in range(n - 2)])
        np.testing.assert_array_equal(s[1:-1], body)
    ids, cu = bert.pack(seqs)
    assert cu[0] == 0 and cu[-1] == len(ids) and np.all(np.diff(cu) >= 16)


def test_oracle_layers_are_layer_normalised():
    c = bert.MiniLMConfig(vocab=1200, max_position=64, **SMALL)
    params = bert.initialize(c)
    x = obert.hidden(params, np.array([101, 1005, 1100, 102]), c.layers, c.heads).numpy()
    np.testing.assert_allclose(x.mean(axis=1), 0, atol=1e-9)
    np.testing.assert_allclose(x.var(axis=1), 1, rtol=1e-6)


# ---------------------------------------------------------------------------------- GPU
def _dev():
    import torch
    return torch.device("cuda", 0)


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k,epi,out", [(200, 1152, 384, 5, "bf16"), (77, 1536, 384, 6, "bf16"),
                                           (300, 384, 1536, 7, "f32"), (130, 200, 64, 5, "f32"),
                                           (129, 264, 128, 6, "f32"), (65, 136, 384, 7, "bf16")])
def test_gemm_bias_epilogues(m, n, k, epi, out):
    import torch
    from sejong_b200._lib import SJ_BF16, SJ_F32, call
    g = torch.Generator().manual_seed(m * n + k)
    x = torch.randn(m, k, generator=g).bfloat16()
    w = (0.05 * torch.randn(n, k, generator=g)).bfloat16()
    b = torch.randn(n, generator=g)
    dt = torch.bfloat16 if out == "bf16" else torch.float32
    res = torch.randn(m, n, generator=g).to(dt)
    xd, wd, bd, rd = x.cuda(), w.cuda(), b.cuda(), res.cuda()
    c = torch.empty(m, n, dtype=dt, device="cuda")
    call("sj_gemm_bias", xd.data_ptr(), k, 0, wd.data_ptr(), k, 1, c.data_ptr(), n, SJ_BF16 if out == "bf16" else SJ_F32,
         m, n, k, epi, 1.0, bd.data_ptr(), rd.data_ptr() if epi == 7 else 0, n if epi == 7 else 0, _stream())
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T + b
    if epi == 6:
        ref = 0.5 * ref * (1 + torch.erf(ref * 0.7071067811865476))
    if epi == 7:
        ref = ref + res.float()
    got = c.float().cpu()
    tol = 2e-2 if out == "bf16" else 1e-4
    assert float((got - ref).norm() / ref.norm()) < tol


@pytest.mark.gpu
def test_gemm_bias_rejects_plain_epilogues():
    from sejong_b200._lib import SejongError, call
    with pytest.raises(SejongError):
        call("sj_gemm", 16, 64, 0, 16, 64, 1, 16, 64, 0, 64, 64, 64, 5, 1.0, 0, 0, 0, 0, 0.0, 0, None)


@pytest.mark.gpu
@pytest.mark.parametrize("d", [128, 384, 768])
def test_layernorm(d):
    import torch
    from sejong_b200._lib import call
    rows = 333
    g = torch.Generator().manual_seed(d)
    x = 3 * torch.randn(rows, d, generator=g) + 0.5
    w, b = 1 + 0.1 * torch.randn(d, generator=g), torch.randn(d, generator=g)
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    y = torch.empty(rows, d, device="cuda")
    yb = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    call("sj_layernorm", xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), 1e-12, y.data_ptr(), yb.data_ptr(), rows, d,
         _stream())
    torch.cuda.synchronize()
    ref = ops.layernorm(x.double(), w.double(), b.double(), 1e-12)
    assert float((y.cpu().double() - ref).abs().max()) < 1e-5
    assert float((yb.cpu().double() - ref).abs().max() / ref.abs().max()) < 1e-2


def _ragged():
    return [np.array(s, dtype=np.int32) for s in
            ([101, 102], [101] + list(range(1000, 1005)) + [102],
             [101] + list(range(2000, 2062)) + [102], [101] + list(range(3000, 3126)) + [102], [101])]


@pytest.mark.gpu
def test_bert_attention_ragged_sequences():
    import torch
    from sejong_b200._lib import call
    heads, hd = 12, 32
    seqs = _ragged()
    ids, cu = bert.pack(seqs)
    rows = len(ids)
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(rows, 3 * heads * hd, generator=g).bfloat16()
    qd = qkv.cuda()
    cud = torch.from_numpy(cu).cuda()
    out = torch.zeros(rows, heads * hd, dtype=torch.bfloat16, device="cuda")
    call("sj_bert_attention", qd.data_ptr(), 3 * heads * hd, cud.data_ptr(), len(seqs), 128, heads, hd,
         out.data_ptr(), heads * hd, _stream())
    torch.cuda.synchronize()
    got = out.float().cpu()
    for s in range(len(seqs)):
        a, e = int(cu[s]), int(cu[s + 1])
        block = qkv[a:e].double()
        q, k, v = block[:, :heads * hd], block[:, heads * hd:2 * heads * hd], block[:, 2 * heads * hd:]
        ref, _ = ops.attention(q, k, v, e - a, heads, causal=False)
        err = float((got[a:e].double() - ref).norm() / ref.norm())
        assert err < 1e-2, (s, e - a, err)


@pytest.mark.gpu
def test_bert_embed_flags_bad_ids():
    import torch
    from sejong_b200._lib import call
    c = bert.MiniLMConfig(vocab=1200, max_position=64, **SMALL)
    m = bert.MiniLM(c, device=0)
    call("sj_device_error", ctypes.byref(ctypes.c_int(0)), 1, None)
    ids = torch.tensor([101, 5000, 102], dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, 3], dtype=torch.int32, device="cuda")
    m.forward(ids, cu)
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    call("sj_device_error", ctypes.byref(code), 1, None)
    assert code.value == 110  # SJ_DEV_BAD_INDEX


@pytest.mark.gpu
def test_encoder_matches_the_fp64_restatement():
    import torch
    c = bert.MiniLMConfig(**SMALL)
    params = bert.initialize(c)
    m = bert.MiniLM(c, params, device=0)
    seqs = _ragged()[:-1] + bert.synthetic_batch(3, 4)
    ids, cu = bert.pack(seqs)
    x = m.forward(torch.from_numpy(ids).cuda(), torch.from_numpy(cu).cuda())
    torch.cuda.synchronize()
    got = x.cpu().double()
    for s, seq in enumerate(seqs):
        ref = obert.hidden(params, seq, c.layers, c.heads, matrix_dtype=torch.bfloat16)
        part = got[int(cu[s]):int(cu[s + 1])]
        err = float((part - ref).norm() / ref.norm())
        assert err < 2e-2, (s, len(seq), err)


@pytest.mark.gpu
def test_full_c2_batch_packing_is_invisible():
    """BASELINE C2 (6 layers, batch 64, lengths 16..128): each sequence's rows in the packed batch
    equal those of the sequence encoded on its own, bit for bit."""
    import torch
    c = bert.MiniLMConfig()
    m = bert.MiniLM(c, device=0)
    seqs = bert.synthetic_batch(21, 64)
    ids, cu = bert.pack(seqs)
    full = m.forward(torch.from_numpy(ids).cuda(), torch.from_numpy(cu).cuda()).clone()
    assert torch.isfinite(full).all()
    for s in (0, 17, 63):
        one_ids, one_cu = bert.pack([seqs[s]])
        alone = m.forward(torch.from_numpy(one_ids).cuda(), torch.from_numpy(one_cu).cuda())
        assert torch.equal(alone, full[int(cu[s]):int(cu[s + 1])]), s
