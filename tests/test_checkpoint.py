"""Artifact layout (crates/sejong-model/src/lib.rs:395-538, crates/sejong-core/src/lib.rs:547-577):
the safetensors container, the manifest, the atomic save and every check of the load path.  The
container is pinned against the `safetensors` serializer (the Rust core the reference links) when
that package is importable; the GPU test resumes a trainer from a checkpoint: the restored state
is bit-identical and the next step agrees to round-off."""
import json
import os

import numpy as np
import pytest

from sejong_b200 import checkpoint as ck
from sejong_b200 import model as pm


def _tensors():
    rng = np.random.default_rng(3)
    return {"b.weight": rng.standard_normal((3, 5)).astype(np.float32), "a": np.ones(7, np.float32),
            "z.f64": rng.standard_normal(4), "embedding": rng.standard_normal((2, 2)).astype(np.float32)}


def test_safetensors_matches_the_reference_serializer(tmp_path):
    st = pytest.importorskip("safetensors.numpy")
    t = _tensors()
    ours, theirs = tmp_path / "ours.safetensors", tmp_path / "theirs.safetensors"
    ck.write_safetensors(ours, t)
    st.save_file(t, str(theirs))
    assert ours.read_bytes() == theirs.read_bytes()
    back = st.load_file(str(ours))
    for k in t:
        np.testing.assert_array_equal(back[k], t[k])


def test_safetensors_round_trip(tmp_path):
    t = _tensors()
    path = tmp_path / "x.safetensors"
    ck.write_safetensors(path, t, metadata={"producer": "test"})
    back = ck.read_safetensors(path)
    assert set(back) == set(t)
    for k in t:
        assert back[k].dtype == t[k].dtype
        np.testing.assert_array_equal(back[k], t[k])


def test_safetensors_rejects_bad_files(tmp_path):
    t = {"x": np.array([1.0, np.nan], np.float32)}
    path = tmp_path / "nan.safetensors"
    ck.write_safetensors(path, t)
    with pytest.raises(ck.ArtifactError, match="nonfinite"):
        ck.read_safetensors(path)
    with pytest.raises(ck.ArtifactError, match="not f32"):
        ck.write_safetensors(tmp_path / "i.safetensors", {"i": np.zeros(2, np.int32)})
    (tmp_path / "short.safetensors").write_bytes(b"\x01\x02")
    with pytest.raises(ck.ArtifactError, match="truncated"):
        ck.read_safetensors(tmp_path / "short.safetensors")


def _config():
    return pm.small_hierarchy()


def _params(c):
    return pm.initialize(c)


def test_save_load_round_trip(tmp_path):
    c = _config()
    params = _params(c)
    rng = np.random.default_rng(1)
    opt = {}
    for name, v in params.items():
        opt[f"m.{name}"] = rng.standard_normal(v.shape).astype(np.float32)
        opt[f"v.{name}"] = np.abs(rng.standard_normal(v.shape)).astype(np.float32)
    from sejong_b200.train import TrainConfig
    tc = TrainConfig(sequence=256, batch=2)
    d = tmp_path / "run" / "model"
    ck.save(d, c, params, 17, opt, ck.train_config_json(tc), "fp-123", 987654321)
    assert sorted(os.listdir(d)) == ["manifest.json", "optimizer.safetensors", "weights.safetensors"]
    assert not [n for n in os.listdir(d.parent) if n.endswith(".tmp")]
    m = json.loads((d / "manifest.json").read_text())
    assert m["format"] == 1 and m["step"] == 17 and m["rng_state"] == 987654321
    assert m["weights"] == "weights.safetensors" and m["optimizer"] == "optimizer.safetensors"
    assert m["model"]["hierarchy"]["patch_size"] == c.hierarchy.patch_size
    assert m["training"]["optimizer"] == "adamw" and m["training"]["accumulation"] == 1
    c2, p2, m2, o2 = ck.load(d)
    assert pm.reference_layout(c2) == pm.reference_layout(c)
    for name in params:
        np.testing.assert_array_equal(p2[name], params[name])
    for name in opt:
        np.testing.assert_array_equal(o2[name], opt[name])
    # the flat layout packs what it unpacked (fused qkv, interleaved gate/up, padded head)
    layout = pm.FlatLayout(c)
    flat = layout.pack(p2)
    again = layout.unpack(flat)
    for name in params:
        np.testing.assert_array_equal(again[name], params[name])


def test_save_is_atomic_and_refuses_an_existing_destination(tmp_path):
    c = _config()
    params = _params(c)
    d = tmp_path / "model"
    ck.save(d, c, params, 0)
    with pytest.raises(ck.ArtifactError, match="already exists"):
        ck.save(d, c, params, 1)
    d2 = tmp_path / "model2"
    with pytest.raises(ck.ArtifactError):
        ck.save(d2, c, params, 0, optimizer={"m.bad": np.zeros(2, np.int64)})
    assert not d2.exists()
    assert not [n for n in os.listdir(tmp_path) if n.endswith(".tmp")]
    missing = dict(params)
    missing.pop("final_norm")
    with pytest.raises(ck.ArtifactError, match="layout"):
        ck.save(tmp_path / "model3", c, missing, 0)


def test_load_checks(tmp_path):
    c = _config()
    params = _params(c)
    d = tmp_path / "model"
    ck.save(d, c, params, 3)
    man = json.loads((d / "manifest.json").read_text())

    def rewrite(**kw):
        m = dict(man)
        m.update(kw)
        (d / "manifest.json").write_text(json.dumps(m))

    rewrite(format=2)
    with pytest.raises(ck.ArtifactError, match="format"):
        ck.load(d)
    rewrite(weights="../weights.safetensors")
    with pytest.raises(ck.ArtifactError, match="basenames"):
        ck.load(d)
    rewrite()
    # a tensor of the wrong shape, then one missing
    bad = dict(params)
    bad["final_norm"] = np.ones(3, np.float32)
    ck.write_safetensors(d / "weights.safetensors", bad)
    with pytest.raises(ck.ArtifactError, match="shape"):
        ck.load(d)
    fewer = dict(params)
    fewer.pop("final_norm")
    ck.write_safetensors(d / "weights.safetensors", fewer)
    with pytest.raises(ck.ArtifactError, match="count"):
        ck.load(d)


def test_config_json_round_trip():
    for c in (pm.config_c1(), pm.config_c3(), pm.config_c5()):
        back = ck.model_config_from_json(json.loads(json.dumps(ck.model_config_json(c))), c.init_std)
        assert pm.reference_layout(back) == pm.reference_layout(c)
        assert (back.kv_heads, back.rope_theta, back.seed) == (c.kv_heads, c.rope_theta, c.seed)


@pytest.mark.gpu
def test_trainer_resumes_from_a_checkpoint(tmp_path):
    import torch

    from oracle.corpus import synthetic_corpus
    from oracle.rng import Rng
    from sejong_b200.train import ByteTrainer, TrainConfig
    c = _config()
    corp = synthetic_corpus(5, 100000)
    batches = [corp.batch(Rng(100 + i), 2, 256) for i in range(3)]
    tc = TrainConfig(sequence=256, batch=2, warmup_steps=0, steps=10)
    a = ByteTrainer(c, tc, device=0, params=_params(c))
    for ids, tg in batches[:2]:
        a.stage_batch(ids, tg)
        a.step()
    a.save_checkpoint(tmp_path / "ckpt", data_fingerprint="synthetic", rng_state=12345)
    b = ByteTrainer(c, tc, device=0, params=_params(pm.with_(c, seed=c.seed + 1)))
    man = b.load_checkpoint(tmp_path / "ckpt")
    assert man["step"] == 2 and man["rng_state"] == 12345
    for name in ("w", "m", "v", "wb"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    ids, tg = batches[2]
    for t in (a, b):
        t.stage_batch(ids, tg)
        t.step()
    torch.cuda.synchronize()
    # the step sums with float atomics (embedding backward, dQ), so equal inputs agree to round-off
    assert float((a.w - b.w).abs().max()) < 1e-5
    assert abs(float(a.loss_sum) - float(b.loss_sum)) <= 1e-6 * abs(float(a.loss_sum))
