"""KV-cached inference on the GPU (Model::hidden_cached / forward_cached, architecture.rs:474-533 and
the dense branch of 651-799; runtime generate, crates/sejong-runtime/src/lib.rs:84-126).

* The cached attention kernel against the FP64 restatement of attention_grouped with OFFSET
  (oracle.ops.grouped_attention), GQA, with and without a window.
* A prefill (tcgen05 attention at offset 0, ragged length), single-token decode steps and a
  multi-row chunk at an offset reproduce, row for row, the FP64 forward of the whole sequence at the
  bf16-cast weights (2e-2 relative L2, the bf16 bar).
* The hierarchical model (architecture.rs:534-779): a prefill that ends inside a patch, single bytes
  across patch boundaries, chunks that span boundaries and a start shorter than a patch reproduce
  the FP64 forward of the whole sequence row for row (the global stage sees each patch once it is
  complete, through the running patch sum).
* Greedy generation picks, at every step, a byte whose FP64 logit is within bf16 noise of the FP64
  maximum given the bytes before it; sampling with the cache wrapping around runs to max_bytes.
"""
import numpy as np
import pytest
import torch

from oracle import model as omodel
from oracle import ops

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("offset,rows,hq,hk,window", [(0, 5, 4, 2, 0), (37, 1, 4, 2, 0), (200, 9, 4, 1, 0),
                                                      (300, 3, 2, 2, 64), (1000, 1, 8, 2, 128)])
def test_cached_attention_against_the_restatement(offset, rows, hq, hk, window):
    from sejong_b200._lib import call
    g = torch.Generator().manual_seed(offset + rows)
    total = offset + rows
    q = torch.randn(total, hq * 64, generator=g, dtype=torch.float64)
    k = torch.randn(total, hk * 64, generator=g, dtype=torch.float64)
    v = torch.randn(total, hk * 64, generator=g, dtype=torch.float64)
    q, k, v = (t.bfloat16().double() for t in (q, k, v))
    ref, _ = ops.grouped_attention(q[offset:], k, v, rows, hq, hk, window or None, offset=offset)
    qd = q[offset:].bfloat16().cuda()
    kd, vd = k.bfloat16().cuda(), v.bfloat16().cuda()
    o = torch.empty(rows, hq * 64, dtype=torch.bfloat16, device="cuda")
    call("sj_attn_cached", qd.data_ptr(), hq * 64, kd.data_ptr(), hk * 64, vd.data_ptr(), hk * 64, o.data_ptr(),
         hq * 64, rows, offset, hq, hk, 64, window, _stream())
    torch.cuda.synchronize()
    assert _rel(o.cpu().double(), ref) < 1e-2


def _model():
    from sejong_b200 import model as pm
    return pm.with_(pm.config_c1(), layers=2)


def _oracle_config(c):
    h = c.hierarchy
    return omodel.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                              kv_heads=c.kv_heads, rope_theta=c.rope_theta, norm_epsilon=c.norm_epsilon, seed=c.seed,
                              init_std=c.init_std, hierarchy=None if h is None else omodel.HierarchyConfig(**h.__dict__))


def _oracle_logits(params, c, tokens):
    p = {k: torch.tensor(v, dtype=torch.float64) for k, v in omodel.compute_cast(params, "bf16").items()}
    ids = torch.as_tensor(np.asarray(tokens, dtype=np.int64))
    with torch.no_grad():
        h = omodel.hidden(p, _oracle_config(c), ids, len(tokens))
        return (h @ p["output"]).numpy()


def test_prefill_decode_and_chunks_match_the_full_forward():
    from sejong_b200.generate import Generator
    from sejong_b200.model import initialize
    c = _model()
    params = initialize(c)
    gen = Generator(c, params, device=0, context=512)
    rng = np.random.default_rng(3)
    tokens = [256] + list(rng.integers(0, 256, size=170))
    chunks = [tokens[:101]] + [[t] for t in tokens[101:131]] + [tokens[131:150], tokens[150:171]]
    got = []
    for ch in chunks:
        h = gen.hidden_cached(ch)
        got.append(h.float().cpu().numpy())
    torch.cuda.synchronize()
    got = np.concatenate(got)
    assert gen.length == len(tokens)
    p = {k: torch.tensor(v, dtype=torch.float64) for k, v in omodel.compute_cast(params, "bf16").items()}
    with torch.no_grad():
        ref = omodel.hidden(p, _oracle_config(c), torch.as_tensor(np.asarray(tokens)), len(tokens)).numpy()
    assert _rel(got, ref) < 2e-2
    for a, b in ((0, 101), (101, 131), (131, 171)):  # every part of the sequence, not just on average
        assert _rel(got[a:b], ref[a:b]) < 2e-2, (a, b)
    # the head on the last row of a chunk
    gen.reset()
    logits = gen.forward_cached(tokens[:60]).cpu().numpy()
    assert _rel(logits, _oracle_logits(params, c, tokens[:60])[-1]) < 2e-2


def test_greedy_generation_follows_the_fp64_model_and_wraps_the_cache():
    from sejong_b200.generate import Generator, Sampling
    from sejong_b200.model import initialize
    c = _model()
    params = initialize(c)
    gen = Generator(c, params, device=0, context=128)
    prompt = b"the quick brown fox "
    out, ended = gen.generate(prompt, Sampling(max_bytes=24, temperature=0.0))
    seq = [256] + list(prompt)
    for byte in out:
        ref = _oracle_logits(params, c, seq)[-1][:257]
        assert ref[byte] >= ref.max() - 0.05 * (np.abs(ref).max() + 1e-6), (len(seq), byte, int(ref.argmax()))
        seq.append(byte)
    assert ended or len(out) == 24
    # sampling past the cache: context 128, prompt + 150 bytes forces the restart from the last 128 tokens
    out2, _ = gen.generate(b"x" * 60, Sampling(max_bytes=150, temperature=1.0, top_p=1.0, seed=5))
    assert gen.length <= 128
    torch.cuda.synchronize()


def _full_hidden(params, c, tokens):
    p = {k: torch.tensor(v, dtype=torch.float64) for k, v in omodel.compute_cast(params, "bf16").items()}
    with torch.no_grad():
        return omodel.hidden(p, _oracle_config(c), torch.as_tensor(np.asarray(tokens)), len(tokens)).numpy()


@pytest.mark.parametrize("plan", [[37] + [1] * 30 + [20, 13, 1, 1], [5, 1, 1, 9, 2, 30, 1]])
def test_hierarchical_prefill_and_decode_match_the_full_forward(plan):
    from sejong_b200 import model as pm
    from sejong_b200.generate import Generator
    c = pm.small_hierarchy()
    params = pm.initialize(c)
    gen = Generator(c, params, device=0, context=256)
    rng = np.random.default_rng(len(plan))
    tokens = [256] + list(rng.integers(0, 256, size=sum(plan) - 1))
    got, at = [], 0
    for n in plan:
        got.append(gen.hidden_cached(tokens[at:at + n]).float().cpu().numpy())
        at += n
    torch.cuda.synchronize()
    got = np.concatenate(got)
    ref = _full_hidden(params, c, tokens)
    at = 0
    for n in plan:
        assert _rel(got[at:at + n], ref[at:at + n]) < 2e-2, (at, n, _rel(got[at:at + n], ref[at:at + n]))
        at += n
    assert gen.length == len(tokens)


def test_hierarchical_generation_runs_and_follows_the_model():
    from sejong_b200 import model as pm
    from sejong_b200.generate import Generator, Sampling
    c = pm.small_hierarchy()
    params = pm.initialize(c)
    gen = Generator(c, params, device=0, context=64)
    prompt = b"hierarchy "
    out, ended = gen.generate(prompt, Sampling(max_bytes=12, temperature=0.0))
    seq = [256] + list(prompt)
    for byte in out:
        ref = _oracle_logits(params, c, seq)[-1][:257]
        assert ref[byte] >= ref.max() - 0.05 * (np.abs(ref).max() + 1e-6), (len(seq), byte, int(ref.argmax()))
        seq.append(byte)
    out2, _ = gen.generate(b"y" * 40, Sampling(max_bytes=60, temperature=1.0, top_p=0.9, seed=9))
    assert gen.length <= 64
