"""CPU tests of the parameter-VJP host side: the index draw exported by the C ABI and the plan
(which weight gradients are compressed, and when the generator draws) against the oracle and the
reference's golden vectors."""
import os

import numpy as np
import pytest

from oracle import model as om
from oracle import param_vjp as opv
from oracle.corpus import synthetic_corpus
from oracle.rng import Rng
from sejong_b200 import _lib, model, param_vjp

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz"))


@pytest.mark.parametrize("case", ["parameter_indices"] + [f"parameter_indices_{i}" for i in range(4)])
def test_host_indices_match_reference_kernel(case):
    a, b, nb, s, r, group = (int(v) for v in GOLD[f"{case}/shape"])
    columns = np.full(max(r, 1), -7, dtype=np.int32)
    rows = np.full(max(s * group, 1), -7, dtype=np.int32)
    row_map = np.full(max(a, 1), -7, dtype=np.int32)
    _lib.call("sj_param_indices_host", int(GOLD[f"{case}/seed"]), a, b, nb, s, r, group, columns.ctypes.data,
              rows.ctypes.data, row_map.ctypes.data)
    assert list(columns[:r]) == list(GOLD[f"{case}/columns"])
    assert list(rows[:s * group]) == list(GOLD[f"{case}/rows"])
    assert list(row_map[:a]) == list(GOLD[f"{case}/map"])


def test_host_indices_reject_bad_sizes():
    with pytest.raises(_lib.SejongError):
        _lib.call("sj_param_indices_host", 1, 10, 4, 2, 3, 5, 32, None, None, None)  # r > b


def test_cost_model_matches_oracle():
    cfg = param_vjp.VjpConfig()
    ocfg = opv.VjpConfig()
    for n in (64, 128, 256, 1000, 4096, 32768):
        for a in (64, 128, 256, 384, 768, 1024):
            for b in (64, 128, 256, 768, 2048):
                for uses in (1, 2, 3):
                    assert param_vjp.selects_compression(cfg, n, a, b, b, uses) == \
                        opv.selects_compression(ocfg, n, a, b, b, uses), (n, a, b, uses)
                    assert param_vjp.budget(cfg, n, a, b) == opv.budget(ocfg, n, a, b)
    for widths in ([256, 256, 256], [768, 256, 256], [2048, 2048], [5]):
        assert param_vjp.donor_index(widths) == opv.donor_index(widths)
    for n, r in ((128, 16), (32768, 16), (300, 16), (40, 6)):
        assert param_vjp.basis_eps(n, r) == opv.basis_eps(n, r)


def test_full_size_plan():
    """C3 at 8 x 4096 bytes: every QKV and gate/up group is compressed (60 matrices); two draws,
    one per distinct (rows, width) pair, made by the last decoder FFN and the last global FFN."""
    p = param_vjp.plan(model.config_c3(), 8, 4096)
    assert len(p.compressed) == 60
    assert p.draws == 2
    first = p.groups[p.prepare_order[0]]
    assert first.input == "decoder.1.z2" and first.new_basis and first.new_selection and first.k == 64
    glob = p.groups["layers.7.z2"]
    assert glob.draw and glob.k == 192 and glob.rank == 16
    assert p.groups["layers.7.z1"].donor == 0  # the 768-wide query projection


def oracle_config(c):
    h = c.hierarchy
    oh = None if h is None else om.HierarchyConfig(**h.__dict__)
    return om.ModelConfig(width=c.width, layers=c.layers, heads=c.heads, ffn_width=c.ffn_width,
                          kv_heads=c.kv_heads, rope_theta=c.rope_theta, norm_epsilon=c.norm_epsilon,
                          hierarchy=oh, seed=c.seed, init_std=c.init_std, router_std=c.router_std)


@pytest.mark.parametrize("batch,seq", [(1, 256), (1, 2048)])
def test_plan_matches_oracle_tape(batch, seq):
    """The plan's compressed weights and draw count equal what the oracle's tape replay decides."""
    c = model.small_hierarchy()
    oc = oracle_config(c)
    params = om.initialize(oc)
    ids, targets = synthetic_corpus(5, 50000).batch(Rng(11), batch, seq)
    cfg = opv.VjpConfig()
    _, _, info = opv.vjp_gradients(params, oc, ids, targets, seq, cfg, Rng(cfg.seed))
    p = param_vjp.plan(c, batch, seq)
    assert p.compressed, "the case must exercise compression"
    assert p.compressed == info["compressed"]
    assert p.draws == info["draws"]
