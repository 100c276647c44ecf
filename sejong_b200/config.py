"""`Config::load` (crates/sejong-core/src/lib.rs:280-300, 308-434): the TOML file the reference's `train`,
`init` and `benchmark` commands read, with [model] (+ [model.hierarchy], [model.experts]), [training]
(+ [training.parameter_vjp]) and [gpu] tables.

Absent fields take the reference's defaults (ModelConfig::default, TrainConfig::default), unknown
fields are refused as the reference's `deny_unknown_fields` does.  Weights are initialised by the
reference's own rule (fan-in scaled normals, crates/sejong-model/src/lib.rs:82-116), so `init_std`
is 0.  What this build does not implement is refused with a message: the control-variate optimizer.
"""
import tomllib
from dataclasses import dataclass, field, fields
from typing import Optional

from .model import ExpertConfig, HierarchyConfig, ModelConfig
from .param_vjp import VjpConfig
from .train import TrainConfig

F32_EPSILON = 1.1920928955078125e-07

MODEL_DEFAULTS = {"id": "sejong", "width": 512, "layers": 8, "heads": 8, "ffn_width": 1536, "context": 2048,
                  "rope_theta": 10000.0, "norm_epsilon": F32_EPSILON, "precision": "f16", "seed": 42}
HIERARCHY_FIELDS = ("patch_size", "encoder_width", "encoder_layers", "encoder_heads", "encoder_ffn_width",
                    "decoder_width", "decoder_layers", "decoder_heads", "decoder_ffn_width", "local_window")
TRAIN_DEFAULTS = {"optimizer": "adamw", "gradient_diagnostics_every": 0, "activation_checkpointing": False,
                  "steps": 10000, "sequence": 512, "batch": 8, "accumulation": 1, "learning_rate": 3e-4,
                  "min_learning_rate": 3e-5, "warmup_steps": 100, "beta1": 0.9, "beta2": 0.95, "epsilon": 0.0,
                  "weight_decay": 0.1, "clip_norm": 1.0, "clip_enabled": True, "loss_scale": 1.0,
                  "checkpoint_every": 500, "log_every": 10, "seed": 123}
VJP_DEFAULTS = {"rank": 16, "residual_fraction": 0.25, "block_rows": 32, "seed": 124}
CV_FIELDS = ("controls", "rank", "sampling", "strata", "basis_refresh", "predictor_learning_rate")
GPU_DEFAULTS = {"device": 0, "architecture": "", "wavefront": 32, "memory_mb": 0}


class ConfigError(ValueError):
    """A configuration the reference's validation (or this build) refuses."""


def _check_keys(table, allowed, where):
    unknown = set(table) - set(allowed)
    if unknown:
        raise ConfigError(f"unknown field(s) in [{where}]: {', '.join(sorted(unknown))}")


@dataclass
class Config:
    model: ModelConfig
    training: TrainConfig
    model_id: str = "sejong"
    precision: str = "f16"
    gpu: dict = field(default_factory=lambda: dict(GPU_DEFAULTS))
    raw: dict = field(default_factory=dict)   # the parsed file, for config.json

    def to_json(self):
        from .checkpoint import model_config_json, train_config_json
        return {"model": model_config_json(self.model, self.model_id, self.precision),
                "training": train_config_json(self.training), "gpu": dict(self.gpu)}


def model_from_table(m):
    _check_keys(m, list(MODEL_DEFAULTS) + ["kv_heads", "hierarchy", "experts"], "model")
    v = {**MODEL_DEFAULTS, **{k: m[k] for k in m if k not in ("hierarchy", "experts")}}
    hier = None
    if "hierarchy" in m:
        h = m["hierarchy"]
        _check_keys(h, HIERARCHY_FIELDS + ("checkpoint_encoder", "checkpoint_decoder"), "model.hierarchy")
        missing = [k for k in HIERARCHY_FIELDS if k not in h]
        if missing:
            raise ConfigError(f"[model.hierarchy] lacks {', '.join(missing)}")
        if h.get("checkpoint_encoder") or h.get("checkpoint_decoder"):
            raise ConfigError("checkpointing a local stage is not built (the global stage is checkpointed when "
                              "training.activation_checkpointing is set)")
        hier = HierarchyConfig(**{k: int(h[k]) for k in HIERARCHY_FIELDS})
    experts = None
    if "experts" in m:
        e = m["experts"]
        _check_keys(e, ("count", "top_k", "ffn_width"), "model.experts")
        experts = ExpertConfig(int(e["count"]), int(e["top_k"]), int(e["ffn_width"]))
    width, heads = int(v["width"]), int(v["heads"])
    if width <= 0 or heads <= 0 or width % heads or (width // heads) % 2:
        raise ConfigError("width must be divisible by heads, with an even head width")
    c = ModelConfig(width=width, layers=int(v["layers"]), heads=heads, ffn_width=int(v["ffn_width"]),
                    kv_heads=None if "kv_heads" not in m else int(m["kv_heads"]), context=int(v["context"]),
                    rope_theta=float(v["rope_theta"]), norm_epsilon=float(v["norm_epsilon"]), hierarchy=hier,
                    experts=experts, seed=int(v["seed"]), init_std=0.0)
    return c, str(v["id"]), str(v["precision"])


def training_from_table(t):
    _check_keys(t, list(TRAIN_DEFAULTS) + ["parameter_vjp", "control_variate"], "training")
    v = {**TRAIN_DEFAULTS, **{k: t[k] for k in t if k not in ("parameter_vjp", "control_variate")}}
    if v["optimizer"] not in ("adamw", "sgd", "control_variate_sgd"):
        raise ConfigError(f"optimizer {v['optimizer']!r}: adamw, sgd or control_variate_sgd")
    cv = None
    if t.get("control_variate") is not None:
        from .control_variate import ControlVariateConfig
        c = t["control_variate"]
        _check_keys(c, CV_FIELDS, "training.control_variate")
        missing = [k for k in CV_FIELDS if k not in c]
        if missing:
            raise ConfigError(f"[training.control_variate] lacks {', '.join(missing)}")
        cv = ControlVariateConfig(controls=int(c["controls"]), rank=int(c["rank"]), sampling=str(c["sampling"]),
                                  strata=int(c["strata"]), basis_refresh=int(c["basis_refresh"]),
                                  predictor_learning_rate=float(c["predictor_learning_rate"]))
    if v["optimizer"] == "control_variate_sgd":
        # TrainConfig::validate (crates/sejong-core/src/lib.rs:380-396)
        if cv is None:
            raise ConfigError("control_variate_sgd requires an explicit training.control_variate budget")
        try:
            cv.validate(int(v["accumulation"]))
        except ValueError as e:
            raise ConfigError(str(e)) from None
        if "parameter_vjp" in t:
            raise ConfigError("this build's control-variate trainer takes dense gradients (no parameter_vjp)")
    if int(v["accumulation"]) < 1:
        raise ConfigError("accumulation must be positive")
    vjp = None
    if "parameter_vjp" in t:
        p = t["parameter_vjp"]
        _check_keys(p, VJP_DEFAULTS, "training.parameter_vjp")
        p = {**VJP_DEFAULTS, **p}
        vjp = VjpConfig(rank=int(p["rank"]), residual_fraction=float(p["residual_fraction"]),
                        block_rows=int(p["block_rows"]), seed=int(p["seed"]))
        if v["optimizer"] != "sgd":
            raise ConfigError("the parameter VJP of the train command needs optimizer = \"sgd\"")
    names = {f.name for f in fields(TrainConfig)}
    kw = {k: v[k] for k in v if k in names}
    for k in ("steps", "sequence", "batch", "accumulation", "warmup_steps", "checkpoint_every", "log_every", "seed",
              "gradient_diagnostics_every"):
        kw[k] = int(kw[k])
    for k in ("learning_rate", "min_learning_rate", "beta1", "beta2", "epsilon", "weight_decay", "clip_norm",
              "loss_scale"):
        kw[k] = float(kw[k])
    tc = TrainConfig(parameter_vjp=vjp, control_variate=cv, **kw)
    if tc.steps <= 0 or tc.sequence <= 0 or tc.batch <= 0 or tc.log_every <= 0:
        raise ConfigError("steps, sequence, batch and log_every must be positive")
    return tc


def parse(text):
    raw = tomllib.loads(text)
    _check_keys(raw, ("model", "training", "gpu"), "top level")
    model, model_id, precision = model_from_table(raw.get("model", {}))
    training = training_from_table(raw.get("training", {}))
    gpu = {**GPU_DEFAULTS, **raw.get("gpu", {})}
    _check_keys(gpu, GPU_DEFAULTS, "gpu")
    if model.hierarchy is not None and training.sequence % model.hierarchy.patch_size:
        raise ConfigError("training.sequence must be a multiple of the patch size")
    if training.sequence > model.context:
        raise ConfigError("training.sequence exceeds model.context")
    return Config(model=model, training=training, model_id=model_id, precision=precision, gpu=gpu, raw=raw)


def load(path):
    with open(path, "rb") as fh:
        return parse(fh.read().decode())


def device_of(cfg: Optional[Config]):
    return int(cfg.gpu.get("device", 0)) if cfg is not None else 0
