"""Host logic of the command line (sejong_b200/cli.py, config.py, checkpoint SGD state), no GPU:
the control-variate budget parses and is validated as TrainConfig::validate does
(crates/sejong-core/src/lib.rs:380-396), unknown fields are refused, the SGD optimizer state round-trips through its 16-bit-word encoding
(crates/sejong-train/src/control_variate.rs:42-64, 208-233), the resume check ignores only
checkpoint_every / log_every, and the NativeValue optimizer settings follow
OptimizerPolicy::configuration (crates/sejong-core/src/native.rs:467-518)."""
import numpy as np
import pytest

from sejong_b200 import checkpoint as ck
from sejong_b200 import cli
from sejong_b200 import config as cfgmod

TINY = """
[model]
id = "tiny"
width = 128
layers = 1
heads = 2
kv_heads = 1
ffn_width = 256
context = 256
seed = 7

[model.hierarchy]
patch_size = 8
encoder_width = 64
encoder_layers = 1
encoder_heads = 1
encoder_ffn_width = 128
decoder_width = 64
decoder_layers = 1
decoder_heads = 1
decoder_ffn_width = 128
local_window = 128

[training]
optimizer = "sgd"
steps = 6
sequence = 128
batch = 2
accumulation = 2
learning_rate = 0.01
warmup_steps = 0
checkpoint_every = 3
log_every = 2
seed = 5

[training.parameter_vjp]
rank = 16
residual_fraction = 0.25
block_rows = 32
seed = 9
"""


def test_tiny_config_parses():
    c = cfgmod.parse(TINY)
    assert c.model.width == 128 and c.model.kv_heads == 1 and c.model.hierarchy.patch_size == 8
    assert c.model.init_std == 0.0 and c.model.norm_epsilon == cfgmod.F32_EPSILON
    t = c.training
    assert (t.optimizer, t.steps, t.accumulation, t.checkpoint_every, t.log_every) == ("sgd", 6, 2, 3, 2)
    assert t.parameter_vjp.seed == 9 and t.parameter_vjp.rank == 16
    j = c.to_json()
    assert j["training"]["accumulation"] == 2 and j["training"]["checkpoint_every"] == 3
    assert j["model"]["id"] == "tiny" and j["model"]["hierarchy"]["local_window"] == 128


def test_unknown_and_unsupported_fields_are_refused():
    with pytest.raises(cfgmod.ConfigError):
        cfgmod.parse(TINY.replace("seed = 7", "seed = 7\nbogus = 1"))
    with pytest.raises(cfgmod.ConfigError):
        cfgmod.parse(TINY.replace('optimizer = "sgd"', 'optimizer = "control_variate_sgd"'))
    with pytest.raises(cfgmod.ConfigError):
        cfgmod.parse(TINY.replace("sequence = 128", "sequence = 130"))  # not a multiple of the patch


CV_TABLE = """
[training.control_variate]
controls = 2
rank = 2
sampling = "stratified"
strata = 2
basis_refresh = 2
predictor_learning_rate = 0.1
"""


def test_control_variate_budget_parses_and_is_validated():
    base = TINY.split("[training.parameter_vjp]")[0].replace('optimizer = "sgd"', 'optimizer = "control_variate_sgd"')
    c = cfgmod.parse(base + CV_TABLE)
    cv = c.training.control_variate
    assert (cv.controls, cv.rank, cv.sampling, cv.strata, cv.basis_refresh) == (2, 2, "stratified", 2, 2)
    j = ck.train_config_json(c.training)
    assert j["optimizer"] == "control_variate_sgd" and j["control_variate"]["predictor_learning_rate"] == 0.1
    for bad in ("controls = 3", "strata = 3", "rank = 0", 'sampling = "random"'):
        key = bad.split(" =")[0]
        line = next(x for x in CV_TABLE.splitlines() if x.startswith(key + " ="))
        with pytest.raises(cfgmod.ConfigError):
            cfgmod.parse(base + CV_TABLE.replace(line, bad))
    with pytest.raises(cfgmod.ConfigError):  # a parameter VJP with control variates: not combined here
        cfgmod.parse(TINY.replace('optimizer = "sgd"', 'optimizer = "control_variate_sgd"') + CV_TABLE)


def test_sgd_state_round_trip():
    state = ck.sgd_state_tensors(123, parameter_rng=0xDEADBEEF12345678)
    assert set(state) == {"sgd.version", "sgd.sampling_rng", "sgd.basis_rng", "sgd.parameter_rng"}
    assert all(v.dtype == np.float32 for v in state.values())
    got = ck.read_sgd_state(state, parameter_vjp=True)
    assert got["sgd.parameter_rng"] == 0xDEADBEEF12345678
    assert got["sgd.sampling_rng"] == 123 ^ ck.SGD_SAMPLING_MIX
    assert got["sgd.basis_rng"] == 123 ^ ck.SGD_BASIS_MIX
    bad = dict(state)
    bad["sgd.version"] = np.array([2.0], np.float32)
    with pytest.raises(ck.ArtifactError):
        ck.read_sgd_state(bad, True)
    bad = dict(state)
    bad["sgd.basis_rng"] = np.array([1.5, 0, 0, 0], np.float32)
    with pytest.raises(ck.ArtifactError):
        ck.read_sgd_state(bad, True)
    with pytest.raises(ck.ArtifactError):  # a parameter-VJP generator where the config has none
        ck.read_sgd_state(state, parameter_vjp=False)


def test_resume_check_ignores_logging_cadence():
    t = cfgmod.parse(TINY).training
    a = ck.train_config_json(t)
    b = dict(a, checkpoint_every=99, log_every=1)
    assert cli._same_training(a, b)
    assert not cli._same_training(a, dict(a, learning_rate=0.5))


def test_value_settings_follow_the_optimizer_policy():
    spec = {"requests": ["a", "b", "c", "d"], "steps": 10, "learning_rate": 1e-3,
            "optimizer": {"weight_decay": 0.01, "clip_norm": 1.0}}
    s = cli._value_settings(spec, batch=2)
    # momentum horizon: the 4 observations in batches of 2 -> h = 2 -> (h-1)/(h+1) = 1/3
    assert abs(s["beta1"] - 1.0 / 3.0) < 1e-7
    # variance horizon: steps * batch = 20 examples -> h = 10 -> 9/11
    assert abs(s["beta2"] - 9.0 / 11.0) < 1e-7
    assert s["min_learning_rate"] == s["learning_rate"] and s["warmup_steps"] == 0
    assert s["clip_enabled"] and s["clip_norm"] == 1.0 and s["epsilon"] == 0.0


def test_value_fingerprint_ignores_resume_and_byte_values():
    spec = {"model": {"width": 128}, "requests": ["x"], "steps": 1, "learning_rate": 1.0, "resume": "/a"}
    assert cli.value_fingerprint(spec) == cli.value_fingerprint(dict(spec, resume="/b"))
    assert cli.value_fingerprint(spec) != cli.value_fingerprint(dict(spec, steps=2))
    assert cli._byte_value({"hex": "00ff"}) == b"\x00\xff" and cli._byte_json(b"\xff") == {"hex": "ff"}
    assert cli._byte_value("ab") == b"ab" and cli._byte_json(b"ab") == "ab"
