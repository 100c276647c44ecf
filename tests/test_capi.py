"""CPU tests of the C-ABI library: it loads, exports every symbol include/sejong.h declares,
and its host-side integer work is bit-exact with the oracle (no GPU compute is called)."""
import ctypes
import os
import re

import numpy as np
import pytest

from oracle import corpus as ocorpus
from oracle import model as omodel
from oracle.rng import Rng

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sejong.h")


@pytest.fixture(scope="module")
def lib():
    from sejong_b200 import _lib, build
    build.build()  # incremental: compiles only what changed (nvcc cross-compiles without a GPU)
    return _lib.load()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sj_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) > 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/sejong.h but not exported"


def test_binding_covers_header():
    from sejong_b200 import _lib
    assert set(declared_functions()) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_rng_bit_exact(lib):
    state = ctypes.c_uint64(987654321)
    ref = Rng(987654321)
    for _ in range(1000):
        assert lib.sj_rng_next_u64(ctypes.byref(state)) == ref.next_u64()
    for size in (1, 2, 3, 7, 255, 1 << 33, (1 << 64) - 5):
        assert lib.sj_rng_index(ctypes.byref(state), size) == ref.index(size)
    assert state.value == ref.state


def test_rng_normal_matches_oracle(lib):
    state = ctypes.c_uint64(42)
    out = np.empty(4096, dtype=np.float32)
    lib.sj_rng_normal_fill(ctypes.byref(state), out.ctypes.data, out.size, ctypes.c_float(1.0))
    ref = Rng(42)
    want = ref.bulk_normal(4096)
    assert state.value == ref.state  # two uniforms per draw, same stream position
    np.testing.assert_allclose(out, want, rtol=2e-6, atol=2e-6)


def test_zipf_bytes_bit_exact(lib):
    out = np.empty(20000, dtype=np.uint8)
    assert lib.sj_zipf_bytes(7, ctypes.c_double(1.1), out.ctypes.data, out.size) == 0
    np.testing.assert_array_equal(out, ocorpus.zipf_bytes(7, 20000, 1.1))
    counts = np.bincount(out, minlength=256)
    assert counts[0] > counts[1] > counts[10] > counts[200]


def test_corpus_batch_bit_exact():
    from sejong_b200.train import corpus_batch, synthetic_corpus_tokens
    toks = synthetic_corpus_tokens(11, 5000)
    corp = ocorpus.synthetic_corpus(11, 5000)
    np.testing.assert_array_equal(toks, corp.token_array())
    st = ctypes.c_uint64(123)
    ref_rng = Rng(123)
    for _ in range(3):
        x, y = corpus_batch(toks, st, 4, 64)
        rx, ry = corp.batch(ref_rng, 4, 64)
        np.testing.assert_array_equal(x, rx)
        np.testing.assert_array_equal(y, ry)
    assert st.value == ref_rng.state
    # EOS at the document start and at the end of the token stream
    assert toks[0] == 256 and toks[-1] == 256
    assert corp.token(0) == 256 and corp.token(corp.tokens - 1) == 256


def test_corpus_batch_rejects_short_corpus(lib):
    from sejong_b200._lib import SejongError
    from sejong_b200.train import corpus_batch
    with pytest.raises(SejongError) as e:
        corpus_batch(np.arange(10, dtype=np.int32), ctypes.c_uint64(1), 1, 16)
    assert e.value.code == 1


def _oracle_config(c):
    h = c.hierarchy
    oh = None if h is None else omodel.HierarchyConfig(**h.__dict__)
    oe = None if c.experts is None else omodel.ExpertConfig(**c.experts.__dict__)
    return omodel.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                              kv_heads=c.kv_heads, context=c.context, rope_theta=c.rope_theta,
                              norm_epsilon=c.norm_epsilon, hierarchy=oh, experts=oe, seed=c.seed,
                              init_std=c.init_std, router_std=c.router_std)


@pytest.mark.parametrize("name", ["config_c1", "config_c3", "config_c5"])
def test_layout_matches_reference_order(name):
    from sejong_b200 import model as pm
    c = getattr(pm, name)()
    ours = [(n, tuple(s), bool(nm)) for n, s, nm in pm.reference_layout(c)]
    ref = [(n, tuple(s), bool(nm)) for n, s, nm in omodel.layout(_oracle_config(c))]
    assert ours == ref


@pytest.mark.parametrize("std", [0.02, 0.0])
def test_initialisation_matches_oracle(std):
    from sejong_b200 import model as pm
    c = pm.with_(pm.small_hierarchy(), init_std=std)
    ours = pm.initialize(c)
    ref = omodel.initialize(_oracle_config(c))
    assert ours.keys() == ref.keys()
    for k in ours:
        np.testing.assert_allclose(ours[k], ref[k], rtol=1e-5, atol=1e-7, err_msg=k)


def test_flat_layout_round_trip():
    from sejong_b200 import model as pm
    c = pm.config_c3()
    lay = pm.FlatLayout(c)
    rng = np.random.default_rng(0)
    params = {n: rng.standard_normal(s).astype(np.float32) for n, s, _ in pm.reference_layout(c)}
    flat = lay.pack(params)
    back = lay.unpack(flat)
    for k, v in params.items():
        np.testing.assert_array_equal(back[k], v)
    # decayed tensors (rank > 1) precede the norm weights
    for e in lay.entries.values():
        assert (e.offset < lay.n_decay) == e.decay
        assert e.offset % pm.ALIGN == 0
    assert lay.total >= pm.parameter_count(c)


def _kernel_bodies():
    """(file, kernel name, body) of every __global__ definition under sejong_b200/csrc."""
    csrc = os.path.join(ROOT, "sejong_b200", "csrc")
    out = []
    for name in sorted(os.listdir(csrc)):
        if not name.endswith(".cu"):
            continue
        text = open(os.path.join(csrc, name)).read()
        for m in re.finditer(r"__global__", text):
            brace, semi = text.index("{", m.start()), text.find(";", m.start())
            if semi != -1 and semi < brace:
                continue  # a declaration
            depth, i = 1, brace + 1
            while depth:
                depth += {"{": 1, "}": -1}.get(text[i], 0)
                i += 1
            header = " ".join(text[m.start():brace].split())
            out.append((name, header[:80], text[brace:i]))
    return out


def test_kernels_order_themselves_after_their_predecessor():
    """Every kernel is launched with programmatic stream serialization, so each must execute
    griddepcontrol.wait (pdl_wait) before touching global memory; pointer parameters carry no
    __restrict__ (read-only loads could be scheduled before the wait), and the library issues no
    memset nodes between its kernels."""
    bodies = _kernel_bodies()
    assert len(bodies) > 30
    for name, header, body in bodies:
        assert "pdl_wait();" in body, f"{name}: {header} does not call pdl_wait()"
    csrc = os.path.join(ROOT, "sejong_b200", "csrc")
    for name in os.listdir(csrc):
        code = re.sub(r"//.*", "", open(os.path.join(csrc, name)).read())
        assert "__restrict__" not in code, f"{name} uses __restrict__"
        assert "<<<" not in code, f"{name} launches without sj::launch"
        assert "cudaMemsetAsync" not in code, f"{name} issues a memset node"
