"""NativeValue host logic on CPU: the request layout of forward_batch (value.rs:117-137), the value
parameters' initialisation (value.rs:39-76) and the request sampler (memory.rs:948-956), each
against the test-side restatement (oracle/value.py, oracle/rng.py), and the sharded layout's
parameter set (body without embedding / output, plus the native parameters)."""
import numpy as np
import pytest

from oracle import model as om
from oracle import value as ov
from oracle.rng import Rng
from sejong_b200 import model as pm
from sejong_b200 import value as pv


def _oracle_config(c):
    h = c.hierarchy
    return om.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width, kv_heads=c.kv_heads,
                          hierarchy=None if h is None else om.HierarchyConfig(**h.__dict__), seed=c.seed,
                          init_std=c.init_std)


def test_request_layout_matches_forward_batch():
    prompts = [b"hello", "hé", b"", b"x" * 40]
    ids, sel, seq = ov.layout_requests(prompts)
    pids, psel = pv.request_batch(prompts)
    assert pids.shape == (4, seq)
    assert np.array_equal(ids, pids.reshape(-1)) and np.array_equal(sel, psel)
    # a longer, fixed sequence keeps every request's rows and SEP position
    qids, qsel = pv.request_batch(prompts, 64)
    assert np.array_equal(qids[:, :seq], pids) and np.all(qids[:, seq:] == 256)
    assert np.array_equal(qsel % 64, psel % seq)
    with pytest.raises(ValueError):
        pv.request_batch(prompts, seq - 1)


def test_value_parameters_follow_the_reference_initialisation():
    c = pm.small_hierarchy()
    a = pv.initialize_value(c, 11)
    b = ov.initialize(_oracle_config(c), 11)
    assert set(a) == set(b)
    for k in a:
        assert a[k].shape == b[k].shape
        np.testing.assert_allclose(a[k], b[k], rtol=3e-6, atol=1e-9, err_msg=k)  # Box-Muller libm: 1 ulp
    assert np.all(a["native_bias"] == 0)


def test_sampler_draws_rng_index():
    st = pv.sampler(99)
    got = pv.sample_requests(st, 50, 37)
    rng = Rng(99 ^ 0x6E6174697665)
    assert np.array_equal(got, [rng.index(37) for _ in range(50)])


def test_value_layout_replaces_the_byte_head():
    c = pm.small_hierarchy()
    lay = pm.FlatLayout(c, values=9)
    names = set(lay.entries)
    assert "embedding" not in names and "output" not in names
    assert {"native_embedding", "native_value", "native_bias"} <= names
    assert lay["native_embedding"].shape == (259, c.width) and lay["native_value"].shape == (c.width, 9)
    # the bias has shape [1, values]: rank 2, so AdamW decays it, as Adam::update does (lib.rs:232)
    assert lay["native_bias"].offset < lay.n_decay


def test_sequence_for_rounds_to_the_patch():
    c = pm.small_hierarchy()
    assert pv.sequence_for(c, [b"a" * 13]) % c.hierarchy.patch_size == 0
    assert pv.sequence_for(c, [b"a" * 13]) >= 15
