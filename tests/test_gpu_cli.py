"""The command line on the GPU (sejong_b200/cli.py): `train` with AdamW and with SGD + parameter VJP
(gradient accumulation over two observations), stopped at a checkpoint and resumed, against the
uninterrupted run; `train-value` (AdamW, AdamW with the parameter VJP, SGD with it) resumed the same
way; `benchmark` writing its report.

Resume bar (crates/sejong-train/examples/control_variate_contract.rs:106-125): weights and optimizer
state of the resumed run within 2e-5 of the uninterrupted run; the data generator, the parameter-VJP
generator and the step counters equal exactly (split-K reductions and attention accumulate in an
order that is not fixed, so floating-point state is compared to a bound, not bit for bit)."""
import json
import os

import numpy as np
import pytest

from sejong_b200 import checkpoint as ck
from sejong_b200 import cli
from sejong_b200 import config as cfgmod
from sejong_b200.corpus import Corpus
from tests.test_cli import TINY

pytestmark = pytest.mark.gpu


def _corpus_dir(path, seed, docs=3, size=6000):
    rng = np.random.default_rng(seed)
    os.makedirs(path, exist_ok=True)
    for i in range(docs):
        text = bytes(rng.integers(32, 127, size=size).astype(np.uint8))
        with open(os.path.join(path, f"doc{i}.txt"), "wb") as fh:
            fh.write(text)
    return path


def _max_diff(a, b):
    assert set(a) == set(b)
    return max(float(np.abs(np.asarray(a[k], np.float64) - np.asarray(b[k], np.float64)).max()) for k in a)


def _resume_case(tmp_path, text):
    corpus = Corpus.open(_corpus_dir(str(tmp_path / "data"), 11))
    cfg = cfgmod.parse(text)
    full = cli.train(cfg, corpus, str(tmp_path / "full"))
    assert full.steps == cfg.training.steps and np.isfinite(full.last_loss)
    records = [json.loads(x) for x in open(tmp_path / "full" / "metrics.jsonl")]
    assert [r["step"] for r in records] == [1, 2, 4, 6]
    for r in records:
        assert r["optimizer"] == cfg.training.optimizer and np.isfinite(r["loss"]) and r["step_seconds"] > 0
        assert r["observed_bytes"] == cfg.training.accumulation * cfg.training.batch * cfg.training.sequence
    mid = tmp_path / "full" / "checkpoints" / "step-00000003"
    assert os.path.isdir(mid)
    cfg2 = cfgmod.parse(text)
    resumed = cli.train(cfg2, corpus, str(tmp_path / "resumed"), resume=str(mid))
    assert resumed.steps == cfg.training.steps
    _, w_full, m_full, o_full = ck.load(full.model_directory)
    _, w_res, m_res, o_res = ck.load(resumed.model_directory)
    assert m_full["step"] == m_res["step"] == cfg.training.steps
    assert m_full["rng_state"] == m_res["rng_state"] and m_full["data_fingerprint"] == corpus.fingerprint
    assert _max_diff(w_full, w_res) < 2e-5
    return o_full, o_res


def test_train_adamw_resume(tmp_path):
    text = TINY.replace('optimizer = "sgd"', 'optimizer = "adamw"').split("[training.parameter_vjp]")[0]
    o_full, o_res = _resume_case(tmp_path, text)
    assert _max_diff(o_full, o_res) < 2e-5


def test_train_sgd_parameter_vjp_resume(tmp_path):
    # 4 x 256 bytes: the local stages' QKV and gate/up gradients are factored (1,024 rows >= 64 features)
    o_full, o_res = _resume_case(tmp_path, TINY.replace("sequence = 128", "sequence = 256").replace("batch = 2",
                                                                                                    "batch = 4"))
    # the SGD state of SgdState::tensors: version, generators as 16-bit words -- equal exactly
    assert set(o_full) == {"sgd.version", "sgd.sampling_rng", "sgd.basis_rng", "sgd.parameter_rng"}
    for k in o_full:
        assert np.array_equal(o_full[k], o_res[k]), k
    # the parameter-VJP generator moved (one draw per new basis / selection and step)
    assert ck.read_sgd_state(o_full, True)["sgd.parameter_rng"] != 9


def _value_spec(kind, vjp):
    rng = np.random.default_rng(4)
    prompts = ["".join(chr(int(c)) for c in rng.integers(97, 123, size=int(rng.integers(4, 30)))) for _ in range(12)]
    model = {"id": "value-tiny", "width": 128, "layers": 1, "heads": 2, "kv_heads": 1, "ffn_width": 256,
             "context": 128, "seed": 3, "norm_epsilon": 1e-6}
    spec = {"optimizer_kind": kind, "optimizer": {"weight_decay": 0.0, "clip_norm": 1.0}, "model": model,
            "requests": [f"r{i}" for i in range(12)], "prompts": prompts, "values": ["yes", "no", "maybe"],
            "labels": [i % 3 for i in range(12)], "steps": 4, "learning_rate": 1e-3, "checkpoint_every": 2,
            "batch": {"max_examples": 8}}
    if vjp:
        spec["parameter_vjp"] = {"rank": 16, "residual_fraction": 0.25, "block_rows": 32, "seed": 21}
    return spec


@pytest.mark.parametrize("kind,vjp", [("adamw", False), ("adamw", True), ("sgd", True)])
def test_train_value_resume(tmp_path, kind, vjp):
    spec = _value_spec(kind, vjp)
    meta = cli.train_value(spec, str(tmp_path / "full"))
    assert meta["steps"] == 4 and np.isfinite(meta["loss"])
    mid = tmp_path / "full" / "checkpoints" / "value-00000002"
    progress = json.load(open(mid / "training.json"))
    assert progress["format"] == "sejong-local-training-v3" and progress["phase"] == "value"
    assert progress["step"] == 2 and progress["batch_size"] == 8
    assert ("parameter_rng" in progress) == vjp
    assert os.path.exists(mid / "original" / "value.json") and os.path.exists(mid / "original" / "body")
    assert os.path.exists(mid / "optimizer.safetensors") == (kind == "adamw")
    cli.train_value(spec, str(tmp_path / "resumed"), resume=str(mid))
    a = ck.read_safetensors(str(tmp_path / "full" / "model" / "native.safetensors"))
    b = ck.read_safetensors(str(tmp_path / "resumed" / "model" / "native.safetensors"))
    assert _max_diff(a, b) < 2e-5
    end_a = json.load(open(tmp_path / "full" / "checkpoints" / "value-00000004" / "training.json"))
    end_b = json.load(open(tmp_path / "resumed" / "checkpoints" / "value-00000004" / "training.json"))
    assert end_a["rng"] == end_b["rng"] and end_a.get("parameter_rng") == end_b.get("parameter_rng")
    assert open(tmp_path / "full" / "model" / "signature").read()


def test_benchmark_report(tmp_path):
    text = TINY.replace('optimizer = "sgd"', 'optimizer = "adamw"').split("[training.parameter_vjp]")[0]
    path = tmp_path / "tiny.toml"
    path.write_text(text)
    train_dir = _corpus_dir(str(tmp_path / "train"), 1)
    val_dir = _corpus_dir(str(tmp_path / "val"), 2)
    reports = cli.benchmark([str(path)], train_dir, val_dir, str(tmp_path / "bench"), 1, 2, 2, 4)
    r = reports[0]
    assert r["measured_steps"] == 2 and len(r["measured_step_records"]) == 2
    assert np.isfinite(r["initial_validation_bits_per_byte_token"]) and np.isfinite(r["final_validation_bits_per_byte_token"])
    assert r["observed_bytes_per_second"] > 0
    inf = r["inference"]
    assert inf["decode_tokens"] == 4 and inf["cached_vs_full_last_logits_max_abs_error"] < 0.25
    top = json.load(open(tmp_path / "bench" / "benchmark.json"))
    assert top["format"] == "sejong-measured-benchmark-v1" and len(top["runs"]) == 1


def test_train_control_variate_resume(tmp_path):
    """control_variate_contract.rs:25-160 on this build: the diagnostic cadence of metrics.jsonl, a run
    resumed from its step-3 checkpoint equal to the uninterrupted one (weights and the SGD /
    control-variate state within 2e-5, generators exactly), a learned predictor and bases that the
    refreshes moved."""
    from tests.test_cli import CV_TABLE
    text = (TINY.split("[training.parameter_vjp]")[0]
            .replace('optimizer = "sgd"', 'optimizer = "control_variate_sgd"')
            .replace("accumulation = 2", "accumulation = 4\ngradient_diagnostics_every = 2\nclip_enabled = false")
            + CV_TABLE)
    o_full, o_res = _resume_case(tmp_path, text)
    assert _max_diff(o_full, o_res) < 2e-5
    for k in ("sgd.version", "sgd.sampling_rng", "sgd.basis_rng"):
        assert np.array_equal(o_full[k], o_res[k]), k
    records = [json.loads(x) for x in open(tmp_path / "full" / "metrics.jsonl")]
    for r in records:
        enabled = r["step"] % 2 == 0
        assert r["gradient_diagnostics"] == enabled
        assert isinstance(r["predictor_mse"], float) == enabled and isinstance(r["diagnostic_seconds"], float) == enabled
        assert r["controls"] == 2 and r["loss_estimator"] == "weighted_control_mean"
        assert r["basis_refreshed"] == enabled and r["basis_source"] == "control_gradient_contrast"
    learned = sum(float((np.asarray(v, np.float64) ** 2).sum()) for k, v in o_full.items() if k.endswith(".predictor"))
    assert learned > 0 and np.isfinite(learned)
    _, _, _, at3 = ck.load(str(tmp_path / "full" / "checkpoints" / "step-00000003"))
    moved = sum(float(((np.asarray(o_full[k], np.float64) - at3[k]) ** 2).sum()) for k in o_full
                if k.endswith(".left") or k.endswith(".right"))
    assert moved > 0 and np.isfinite(moved)
