"""The runtime's sampling rule (crates/sejong-runtime/src/lib.rs:44-78) on CPU: the product's
`sample` (C Rng) against the test-side restatement (oracle/sampling.py on oracle/rng.py) for
random logits and every option, and its fixed points (temperature 0 and top_k 1 take the argmax,
ties go to the lowest index, invalid options raise)."""
import ctypes

import numpy as np
import pytest

from oracle import sampling as osamp
from oracle.rng import Rng
from sejong_b200.generate import Sampling, sample


@pytest.mark.parametrize("temperature,top_k,top_p", [(0.8, 0, 0.95), (1.0, 0, 1.0), (0.5, 20, 0.9), (2.0, 5, 0.5),
                                                     (1e-3, 0, 0.95)])
def test_sample_matches_the_restatement(temperature, top_k, top_p):
    rng_np = np.random.default_rng(int(temperature * 1000) + top_k)
    state = ctypes.c_uint64(42)
    ref = Rng(42)
    opts = Sampling(temperature=temperature, top_k=top_k, top_p=top_p, seed=42)
    for _ in range(200):
        logits = (rng_np.standard_normal(257) * 3).astype(np.float32)
        assert sample(logits, opts, state) == osamp.sample(logits, temperature, top_k, top_p, ref)


def test_sample_fixed_points():
    logits = np.zeros(257, dtype=np.float32)
    logits[[7, 9]] = 5.0
    state = ctypes.c_uint64(1)
    assert sample(logits, Sampling(temperature=0.0), state) == 7         # ties: the lowest index
    assert sample(logits, Sampling(top_k=1), state) == 7
    with pytest.raises(ValueError):
        sample(logits, Sampling(top_p=0.0), state)
    with pytest.raises(ValueError):
        sample(logits, Sampling(temperature=-1.0), state)
    bad = logits.copy()
    bad[3] = np.inf
    with pytest.raises(ValueError):
        sample(bad, Sampling(), state)
